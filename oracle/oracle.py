"""ctypes wrapper over the CPU oracle (``rq_oracle.c``).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
module; the product library never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

F16, Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 1, 2, 8, 10, 11, 12, 13, 14
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q2_K: 84, Q3_K: 110, Q4_K: 144, Q5_K: 176, Q6_K: 210}
BLOCK_ELEMS = {Q4_0: 32, Q8_0: 32, Q2_K: 256, Q3_K: 256, Q4_K: 256, Q5_K: 256, Q6_K: 256}

_lib = None


def build() -> str:
    """Compile the oracle in place (make); returns the library path."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.rqo_quantize.argtypes = [I, P, I64, I64, P]
        L.rqo_dequantize.argtypes = [I, P, I64, I64, P]
        L.rqo_matmul_ref.argtypes = [I, P, I64, I64, P, I64, P, I]
        L.rqo_linear_threaded.argtypes = [I, P, I64, I64, P, I64, P, I]
        L.rqo_linear_rows.argtypes = [I, P, I64, I64, P, I64, P, I]
        L.rqo_parallel_linear_f16.argtypes = [P, I64, I64, P, I64, P, I, I]
        L.rqo_dot_q4_0_scalar.argtypes = [P, P, I64]
        L.rqo_dot_q4_0_scalar.restype = F
        L.rqo_dot_q4_0_avx2order.argtypes = [P, P, I64]
        L.rqo_dot_q4_0_avx2order.restype = F
        L.rqo_f32_to_f16_n.argtypes = [P, P, I64]
        L.rqo_f16_to_f32_n.argtypes = [P, P, I64]
        L.rqo_router_logits.argtypes = [P, I64, I64, P, I, P]
        L.rqo_route_topk.argtypes = [P, I64, I, I, P, P]
        L.rqo_permute.argtypes = [P, P, I64, I, I, P, P, P]
        L.rqo_moe_forward.argtypes = [P, I64, I64, I64, I, I, P, I, P, P, P, P, P, P, P, I]
        L.rqo_silu.argtypes = [F]
        L.rqo_silu.restype = F
        for fn in ("rqo_quantize", "rqo_dequantize", "rqo_matmul_ref", "rqo_linear_threaded",
                   "rqo_linear_rows", "rqo_parallel_linear_f16", "rqo_moe_forward"):
            getattr(L, fn).restype = I
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def row_bytes(qtype: int, n_in: int) -> int:
    return n_in // BLOCK_ELEMS[qtype] * BLOCK_BYTES[qtype]


def quantize(qtype: int, w: np.ndarray) -> np.ndarray:
    """f32 [rows, in] -> GGML block bytes uint8 [rows, row_bytes]."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, n_in = w.shape
    out = np.zeros((rows, row_bytes(qtype, n_in)), dtype=np.uint8)
    rc = lib().rqo_quantize(qtype, _p(w), rows, n_in, _p(out))
    if rc != 0:
        raise ValueError(f"rqo_quantize failed ({rc})")
    return out


def dequantize(qtype: int, blocks: np.ndarray, rows: int, n_in: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    assert blocks.size == rows * row_bytes(qtype, n_in)
    out = np.empty((rows, n_in), dtype=np.float32)
    rc = lib().rqo_dequantize(qtype, _p(blocks), rows, n_in, _p(out))
    if rc != 0:
        raise ValueError(f"rqo_dequantize failed ({rc})")
    return out


def matmul_ref(qtype: int, blocks: np.ndarray, n_out: int, n_in: int, x: np.ndarray,
               acc64: bool = False) -> np.ndarray:
    """y = x @ deq(W).T, dequantize then dot (f32 or f64 accumulation)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, n_in)
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    y = np.empty((x.shape[0], n_out), dtype=np.float32)
    rc = lib().rqo_matmul_ref(qtype, _p(blocks), n_out, n_in, _p(x), x.shape[0], _p(y), int(acc64))
    if rc != 0:
        raise ValueError(f"rqo_matmul_ref failed ({rc})")
    return y


def linear_threaded(qtype: int, blocks: np.ndarray, n_out: int, n_in: int, x: np.ndarray,
                    nthreads: int = 0, y: np.ndarray | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, n_in)
    if y is None:
        y = np.empty((x.shape[0], n_out), dtype=np.float32)
    rc = lib().rqo_linear_threaded(qtype, _p(blocks), n_out, n_in, _p(x), x.shape[0], _p(y),
                                   nthreads)
    if rc != 0:
        raise ValueError(f"rqo_linear_threaded failed ({rc})")
    return y


def linear_rows(qtype: int, blocks: np.ndarray, n_out: int, n_in: int, x: np.ndarray,
                nthreads: int = 0) -> np.ndarray:
    """rqo_linear_threaded's products, each weight row dequantized once."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, n_in)
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    y = np.empty((x.shape[0], n_out), dtype=np.float32)
    rc = lib().rqo_linear_rows(qtype, _p(blocks), n_out, n_in, _p(x), x.shape[0], _p(y), nthreads)
    if rc != 0:
        raise ValueError(f"rqo_linear_rows failed ({rc})")
    return y


def parallel_linear_f16(w16: np.ndarray, x: np.ndarray, avx2: bool = True, nthreads: int = 0,
                        y: np.ndarray | None = None) -> np.ndarray:
    """ParallelLinear::forward (parallel_linear.rs:191-295): w16 [out, in]
    float16 (or its uint16 bits), x f32 [n, in]."""
    w = np.ascontiguousarray(w16).view(np.uint16)
    out, n_in = w.shape
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, n_in)
    if y is None:
        y = np.empty((x.shape[0], out), dtype=np.float32)
    rc = lib().rqo_parallel_linear_f16(_p(w), out, n_in, _p(x), x.shape[0], _p(y), int(avx2), nthreads)
    if rc != 0:
        raise ValueError(f"rqo_parallel_linear_f16 failed ({rc})")
    return y


def router_f16(wr: np.ndarray) -> np.ndarray:
    """The router weight as the reference holds it: ParallelLinear::new
    converts it to F16 (round to nearest even), as uint16 bits."""
    if wr.dtype == np.float16:
        return np.ascontiguousarray(wr).view(np.uint16)
    if wr.dtype == np.uint16:
        return np.ascontiguousarray(wr)
    return f32_to_f16_bits(np.ascontiguousarray(wr, dtype=np.float32))


def dot_q4_0_scalar(w_row: np.ndarray, x_row: np.ndarray) -> float:
    nb = x_row.size // 32
    return float(lib().rqo_dot_q4_0_scalar(_p(w_row), _p(x_row), nb))


def dot_q4_0_avx2order(w_row: np.ndarray, x_row: np.ndarray) -> float:
    nb = x_row.size // 32
    return float(lib().rqo_dot_q4_0_avx2order(_p(w_row), _p(x_row), nb))


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    h = np.empty(x.shape, dtype=np.uint16)
    lib().rqo_f32_to_f16_n(_p(x), _p(h), x.size)
    return h


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    x = np.empty(h.shape, dtype=np.float32)
    lib().rqo_f16_to_f32_n(_p(h), _p(x), h.size)
    return x


def router_logits(x: np.ndarray, wr: np.ndarray) -> np.ndarray:
    """Gate logits: ParallelLinear over the F16 router weight (wr f32, f16
    or f16 bits)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    wr = router_f16(wr)
    T, H = x.shape
    E = wr.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    lib().rqo_router_logits(_p(x), T, H, _p(wr), E, _p(out))
    return out


def route_topk(logits: np.ndarray, k: int):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = logits.shape
    ids = np.empty((T, k), dtype=np.int32)
    w = np.empty((T, k), dtype=np.float32)
    lib().rqo_route_topk(_p(logits), T, E, k, _p(ids), _p(w))
    return ids, w


def permute(ids: np.ndarray, weights: np.ndarray, E: int):
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    weights = np.ascontiguousarray(weights, dtype=np.float32)
    T, k = ids.shape
    offs = np.empty(E + 1, dtype=np.int32)
    rows = np.empty(T * k, dtype=np.int32)
    sw = np.empty(T * k, dtype=np.float32)
    lib().rqo_permute(_p(ids), _p(weights), T, E, k, _p(offs), _p(rows), _p(sw))
    return offs, rows, sw


def moe_forward(x: np.ndarray, wr: np.ndarray, qtype: int, w1: list, w3: list, w2: list,
                F: int, k: int = 2, nthreads: int = 0):
    """Full SparseMoe layer on the CPU; returns (y, ids, perm, offsets).
    qtype F16: w1/w3/w2 are float16 [out, in] arrays (the reference's
    ParallelLinear experts); otherwise GGML block bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    wr = router_f16(wr)
    T, H = x.shape
    E = wr.shape[0]
    arr_t = ctypes.c_void_p * E
    if qtype == F16:
        keep = [np.ascontiguousarray(a).view(np.uint16) for a in (*w1, *w3, *w2)]
    else:
        keep = [np.ascontiguousarray(a, dtype=np.uint8) for a in (*w1, *w3, *w2)]
    p1 = arr_t(*[_p(a) for a in keep[:E]])
    p3 = arr_t(*[_p(a) for a in keep[E:2 * E]])
    p2 = arr_t(*[_p(a) for a in keep[2 * E:]])
    y = np.empty((T, H), dtype=np.float32)
    ids = np.empty((T, k), dtype=np.int32)
    perm = np.empty(T * k, dtype=np.int32)
    offs = np.empty(E + 1, dtype=np.int32)
    rc = lib().rqo_moe_forward(_p(x), T, H, F, E, k, _p(wr), qtype, ctypes.cast(p1, ctypes.c_void_p),
                               ctypes.cast(p3, ctypes.c_void_p), ctypes.cast(p2, ctypes.c_void_p),
                               _p(y), _p(ids), _p(perm), _p(offs), nthreads)
    if rc != 0:
        raise ValueError(f"rqo_moe_forward failed ({rc})")
    return y, ids, perm, offs


class OracleLlama:
    """CPU restatement of the quantized Llama forward (rqo_llama_*)."""

    def __init__(self, cfg: dict, qtype: int):
        L = lib()
        L.rqo_llama_create.restype = ctypes.c_void_p
        L.rqo_llama_create.argtypes = [ctypes.c_int64] * 8 + [ctypes.c_float, ctypes.c_float, ctypes.c_int]
        L.rqo_llama_free.argtypes = [ctypes.c_void_p]
        L.rqo_llama_set_layer.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p]
        L.rqo_llama_set_embedding.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        L.rqo_llama_set_head.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.rqo_llama_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                        ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.rqo_llama_embed.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        L.rqo_llama_layer.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int]
        L.rqo_llama_head.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                     ctypes.c_void_p, ctypes.c_int]
        self.cfg = cfg
        self.h = L.rqo_llama_create(cfg["hidden"], cfg["intermediate"], cfg["n_heads"],
                                    cfg["n_kv_heads"], cfg["head_dim"], cfg["n_layers"],
                                    cfg["vocab"], cfg.get("max_seq", 512), cfg.get("rms_eps", 1e-5),
                                    cfg.get("rope_theta", 10000.0), qtype)
        self.keep = []

    def set_layer(self, l, blocks7, rms1, rms2):
        bl = [np.ascontiguousarray(b, dtype=np.uint8) for b in blocks7]
        r1 = np.ascontiguousarray(rms1, dtype=np.float32)
        r2 = np.ascontiguousarray(rms2, dtype=np.float32)
        arr = (ctypes.c_void_p * 7)(*[_p(b) for b in bl])
        self.keep += [bl, r1, r2, arr]
        lib().rqo_llama_set_layer(self.h, l, ctypes.cast(arr, ctypes.c_void_p), _p(r1), _p(r2))

    def stream_layer(self, l, blocks7, rms1, rms2, x: np.ndarray, index_pos: int, nthreads=0) -> None:
        """Run layer l over x in place with weights given for this call only
        (not kept: a model larger than host memory runs a layer at a time)."""
        bl = [np.ascontiguousarray(b, dtype=np.uint8) for b in blocks7]
        r1 = np.ascontiguousarray(rms1, dtype=np.float32)
        r2 = np.ascontiguousarray(rms2, dtype=np.float32)
        arr = (ctypes.c_void_p * 7)(*[_p(b) for b in bl])
        lib().rqo_llama_set_layer(self.h, l, ctypes.cast(arr, ctypes.c_void_p), _p(r1), _p(r2))
        try:
            self.layer(l, x, index_pos, nthreads)
        finally:
            null = (ctypes.c_void_p * 7)()
            lib().rqo_llama_set_layer(self.h, l, ctypes.cast(null, ctypes.c_void_p), _p(r1), _p(r2))

    def set_embedding(self, emb_f16):
        e = np.ascontiguousarray(emb_f16).view(np.uint16)
        self.keep.append(e)
        lib().rqo_llama_set_embedding(self.h, _p(e))

    def set_head(self, ln_f, head_f16):
        n = np.ascontiguousarray(ln_f, dtype=np.float32)
        h = np.ascontiguousarray(head_f16).view(np.uint16)
        self.keep += [n, h]
        lib().rqo_llama_set_head(self.h, _p(n), _p(h))

    def forward(self, tokens, index_pos, nthreads=0):
        ids = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        logits = np.empty(self.cfg["vocab"], dtype=np.float32)
        nxt = ctypes.c_int32()
        rc = lib().rqo_llama_forward(self.h, _p(ids), ids.size, index_pos, _p(logits),
                                     ctypes.addressof(nxt), nthreads)
        if rc != 0:
            raise ValueError(f"rqo_llama_forward failed ({rc})")
        return logits, int(nxt.value)

    def embed(self, tokens) -> np.ndarray:
        ids = np.ascontiguousarray(tokens, dtype=np.int32).reshape(-1)
        x = np.empty((ids.size, self.cfg["hidden"]), dtype=np.float32)
        lib().rqo_llama_embed(self.h, _p(ids), ids.size, _p(x))
        return x

    def layer(self, l, x: np.ndarray, index_pos: int, nthreads=0) -> None:
        """QBlock l over the hidden rows x [T, hidden] in place."""
        assert x.dtype == np.float32 and x.flags["C_CONTIGUOUS"]
        rc = lib().rqo_llama_layer(self.h, l, _p(x), x.shape[0], index_pos, nthreads)
        if rc != 0:
            raise ValueError(f"rqo_llama_layer failed ({rc})")

    def head(self, x: np.ndarray, nthreads=0):
        """(logits [T, vocab], argmax [T]) of every row of x."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        T = x.shape[0]
        logits = np.empty((T, self.cfg["vocab"]), dtype=np.float32)
        amax = np.empty(T, dtype=np.int32)
        rc = lib().rqo_llama_head(self.h, _p(x), T, _p(logits), _p(amax), nthreads)
        if rc != 0:
            raise ValueError(f"rqo_llama_head failed ({rc})")
        return logits, amax

    def forward_all(self, tokens, index_pos, nthreads=0):
        """forward_all (src/streaming_quantized.rs:611-620): logits and the
        greedy token of every position.  Fed the prompt plus the tokens a
        greedy decode produced, position p's argmax is the token that decode
        step p emitted (every position's arithmetic is that of the
        incremental step)."""
        x = self.embed(tokens)
        for l in range(self.cfg["n_layers"]):
            self.layer(l, x, index_pos, nthreads)
        return self.head(x, nthreads)

    def generate(self, prompt, max_new_tokens, nthreads=0):
        toks = []
        _, nxt = self.forward(prompt, 0, nthreads)
        toks.append(nxt)
        pos = len(prompt)
        for _ in range(max_new_tokens - 1):
            _, nxt = self.forward([nxt], pos, nthreads)
            pos += 1
            toks.append(nxt)
        return toks

    def __del__(self):
        try:
            lib().rqo_llama_free(self.h)
        except Exception:
            pass
