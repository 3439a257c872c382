"""Host-side mirror of StreamingLlamaQuantized (src/streaming_quantized.rs)
over librq's rq_llama_* entry points: every QBlock resident on the GPU.

Mirrored interface: ``forward(input_ids, index_pos)`` (:622-633) returning
last-position logits, ``generate`` greedy (:539-593, temperature 0 ->
argmax), ``truncate_caches`` (:603-609).  Weights are GGML blocks (Q4_K /
Q3_K / Q4_0 linears), f32 RmsNorm weights, F16 embedding and lm_head.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import LlamaConfig, check
from .linear import Context, QWeight

try:
    import torch
except Exception:  # pragma: no cover
    torch = None

LINEARS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def layer_shapes(cfg: dict) -> list[tuple[int, int]]:
    """(out, in) of q, k, v, o, gate, up, down."""
    H, I = cfg["hidden"], cfg["intermediate"]
    nq, nk = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"]
    return [(nq, H), (nk, H), (nk, H), (H, nq), (I, H), (I, H), (H, I)]


class StreamingLlamaQuantized:
    def __init__(self, cfg: dict, device: int = 0):
        self.cfg = dict(cfg)
        self.ctx = Context.get(device)
        c = LlamaConfig(cfg["hidden"], cfg["intermediate"], cfg["n_heads"], cfg["n_kv_heads"],
                        cfg["head_dim"], cfg["n_layers"], cfg["vocab"], cfg.get("max_seq", 512),
                        cfg.get("max_batch_tokens", 64), cfg.get("rms_eps", 1e-5),
                        cfg.get("rope_theta", 10000.0))
        h = ctypes.c_void_p()
        check(_lib.lib().rq_llama_create(self.ctx.handle, ctypes.byref(c), ctypes.byref(h)))
        self.handle = h
        self._keep: list = []  # weights borrowed by the library

    def set_layer(self, layer: int, weights: list, rms1, rms2) -> None:
        assert len(weights) == 7
        arr = (ctypes.c_void_p * 7)(*[w.handle.value for w in weights])
        r1 = np.ascontiguousarray(rms1, dtype=np.float32)
        r2 = np.ascontiguousarray(rms2, dtype=np.float32)
        check(_lib.lib().rq_llama_set_layer(self.handle, layer, arr, r1.ctypes.data, r2.ctypes.data))
        self._keep.append(weights)

    @classmethod
    def from_gguf_dir(cls, cfg: dict, shard_dir, device: int = 0) -> "StreamingLlamaQuantized":
        """The model from a directory of per-layer GGUF shards, laid out as
        StreamingLlamaQuantized::from_pretrained reads them
        (src/streaming_quantized.rs:451-501).  Under tensor parallelism (a
        communicator on the device's context) each rank loads its shards."""
        m = cls(cfg, device)
        check(_lib.lib().rq_llama_load_gguf_dir(m.handle, str(shard_dir).encode()))
        return m

    def layer_weights(self, layer: int) -> list:
        """The QWeights (q, k, v, o, gate, up, down) set for a layer."""
        return self._keep[layer]

    def set_embedding(self, embed_f16) -> None:
        e = np.ascontiguousarray(embed_f16).view(np.uint16)
        check(_lib.lib().rq_llama_set_embedding(self.handle, e.ctypes.data))

    def set_head(self, ln_f, lm_head_f16) -> None:
        n = np.ascontiguousarray(ln_f, dtype=np.float32)
        h = np.ascontiguousarray(lm_head_f16).view(np.uint16)
        check(_lib.lib().rq_llama_set_head(self.handle, n.ctypes.data, h.ctypes.data))

    def forward(self, input_ids, index_pos: int, want_logits: bool = True):
        """Logits (f32 [vocab], single rank only; None when not wanted) of the
        last position and the greedy token."""
        ids = np.ascontiguousarray(input_ids, dtype=np.int32).reshape(-1)
        logits = np.empty(self.cfg["vocab"], dtype=np.float32) if want_logits else None
        nxt = ctypes.c_int32()
        check(_lib.lib().rq_llama_forward(self.handle, ids.ctypes.data, ids.size, index_pos,
                                          logits.ctypes.data if want_logits else None,
                                          ctypes.byref(nxt), None))
        return logits, int(nxt.value)

    def decode_step(self, stream: int = 0) -> None:
        check(_lib.lib().rq_llama_decode_step(self.handle, stream))

    def set_fused(self, enable: bool) -> None:
        """One persistent launch per decode step (one GPU) or the chain of
        per-layer kernels (default); both compute the same bits."""
        check(_lib.lib().rq_llama_set_fused(self.handle, 1 if enable else 0))

    def status(self) -> None:
        """Raises RqError if a wait inside a one-launch decode step timed out."""
        check(_lib.lib().rq_llama_status(self.handle))

    def tokens(self) -> tuple[list, int]:
        cap = self.cfg.get("max_seq", 512)
        buf = np.empty(cap, dtype=np.int32)
        n, p = ctypes.c_int64(), ctypes.c_int64()
        check(_lib.lib().rq_llama_tokens(self.handle, buf.ctypes.data, cap, ctypes.byref(n),
                                         ctypes.byref(p)))
        return buf[:min(n.value, cap)].tolist(), p.value

    def forward_all(self, input_ids, index_pos: int, want_logits: bool = False):
        """The verify forward (forward_all, src/streaming_quantized.rs:611-620):
        greedy token at every position, and [T, vocab] logits when wanted."""
        ids = np.ascontiguousarray(input_ids, dtype=np.int32).reshape(-1)
        logits = np.empty((ids.size, self.cfg["vocab"]), dtype=np.float32) if want_logits else None
        amax = np.empty(ids.size, dtype=np.int32)
        check(_lib.lib().rq_llama_forward_all(self.handle, ids.ctypes.data, ids.size, index_pos,
                                              logits.ctypes.data if want_logits else None,
                                              amax.ctypes.data, None))
        return logits, amax.tolist()

    def truncate_caches(self, new_len: int) -> None:
        check(_lib.lib().rq_llama_truncate(self.handle, new_len))

    def generate(self, prompt_ids, max_new_tokens: int) -> list:
        """Greedy generation (generate with temperature 0): the prompt in one
        forward, then device-side decode steps."""
        check(_lib.lib().rq_llama_reset_tokens(self.handle))
        self.forward(prompt_ids, 0, want_logits=False)
        for _ in range(max_new_tokens - 1):
            self.decode_step()
        if torch is not None:
            torch.cuda.synchronize(self.ctx.device)
        self.status()
        toks, _ = self.tokens()
        return toks[:max_new_tokens]

    def close(self) -> None:
        if self.handle:
            _lib.lib().rq_llama_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def random_model(cfg: dict, qtype: int, seed: int, device: int = 0, host_blocks: bool = False,
                 tp: tuple[int, int] = (1, 0), host_tensors: bool = False):
    """Random-init weights of the configured architecture, N(0, 0.02), on the
    device; linears quantized on the GPU.  With tp = (world, rank) every rank
    draws the same full tensors and keeps its shard, so any world size holds
    the same model.  Returns (model, host dict of the GGML bytes and F16/f32
    tensors when host_blocks; with host_tensors the same dict without the
    block bytes -- layers hold (None, rms1, rms2) and the device weights of
    layer l stay reachable as model.layer_weights(l))."""
    from .tp import LINEAR_SPLIT, shard
    world, rank = tp
    g = torch.Generator(device=f"cuda:{device}").manual_seed(seed)
    m = StreamingLlamaQuantized(cfg, device)
    host = {"layers": []} if (host_blocks or host_tensors) else None
    for l in range(cfg["n_layers"]):
        ws = []
        for k, (o, i) in enumerate(layer_shapes(cfg)):
            wf = torch.randn(o, i, device=f"cuda:{device}", generator=g) * 0.02
            ws.append(QWeight.quantize(m.ctx, qtype, shard(LINEAR_SPLIT[k], wf, world, rank)))
            del wf
        r1 = (1.0 + 0.1 * torch.randn(cfg["hidden"], device=f"cuda:{device}", generator=g)).cpu().numpy()
        r2 = (1.0 + 0.1 * torch.randn(cfg["hidden"], device=f"cuda:{device}", generator=g)).cpu().numpy()
        m.set_layer(l, ws, r1, r2)
        if host_blocks:
            host["layers"].append(([w.download() for w in ws], r1, r2))
        elif host_tensors:
            host["layers"].append((None, r1, r2))
    emb = (torch.randn(cfg["vocab"], cfg["hidden"], device=f"cuda:{device}", generator=g) * 0.02
           ).half().cpu().numpy()
    lnf = (1.0 + 0.1 * torch.randn(cfg["hidden"], device=f"cuda:{device}", generator=g)).cpu().numpy()
    head = (torch.randn(cfg["vocab"], cfg["hidden"], device=f"cuda:{device}", generator=g) * 0.02
            ).half()
    head = shard("col", head, world, rank).cpu().numpy()
    m.set_embedding(emb)
    m.set_head(lnf, head)
    if host is not None:
        host.update(embed=emb, ln_f=lnf, lm_head=head)
    return m, host
