"""Host-side mirror of Mixtral's SparseMoe (src/streaming_mixtral.rs:259-319)
over librq's rq_moe_* entry points, with quantized experts.

``SparseMoe(router_w, experts, top_k).forward(xs)`` takes xs [..., hidden]
(numpy or torch) and returns the mixed expert outputs of the same shape;
``forward_with_routing`` also returns the expert ids [T, k] and the
permutation (tokens of expert 0, expert 1, ...).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import check
from .linear import Context, QWeight

try:
    import torch
except Exception:  # pragma: no cover
    torch = None


class SparseMoe:
    def __init__(self, router_w, experts: list, top_k: int = 2, device: int = 0,
                 expert_parallel: bool = False):
        """experts: [(w1 gate, w2 down, w3 up) QWeight triples], as Expert.
        With expert_parallel (after rustyllm_b200.tp.init_from_torch), expert
        e lives on rank e % world and the entries of other ranks are None;
        forward takes this rank's tokens."""
        self.ctx = Context.get(device)
        self.expert_parallel = expert_parallel
        r = np.ascontiguousarray(router_w, dtype=np.float32)
        E, H = r.shape
        F = next(e for e in experts if e is not None)[0].out
        arr = lambda ws: (ctypes.c_void_p * E)(*[w.handle.value if w is not None else None  # noqa: E731
                                                   for w in ws])
        experts = [e if e is not None else (None, None, None) for e in experts]
        h = ctypes.c_void_p()
        check(_lib.lib().rq_moe_create(self.ctx.handle, E, top_k, H, F, r.ctypes.data,
                                       arr([e[0] for e in experts]), arr([e[2] for e in experts]),
                                       arr([e[1] for e in experts]), ctypes.byref(h)))
        self.handle, self.E, self.k, self.H, self.F = h, E, top_k, H, F
        self._keep = experts

    def forward_with_routing(self, xs, routing: bool = True):
        torch_in = torch is not None and isinstance(xs, torch.Tensor)
        shape = tuple(xs.shape)
        if torch_in:
            x2 = xs.reshape(-1, self.H).float().contiguous()
            T = x2.shape[0]
            y = torch.empty_like(x2)
            xp, yp = x2.data_ptr(), y.data_ptr()
            stream = torch.cuda.current_stream(x2.device).cuda_stream if x2.is_cuda else 0
        else:
            x2 = np.ascontiguousarray(np.asarray(xs, dtype=np.float32).reshape(-1, self.H))
            T = x2.shape[0]
            y = np.empty_like(x2)
            xp, yp, stream = x2.ctypes.data, y.ctypes.data, 0
        ids = np.empty((T, self.k), dtype=np.int32) if routing else None
        perm = np.empty(T * self.k, dtype=np.int32) if routing else None
        fwd = _lib.lib().rq_moe_forward_ep if self.expert_parallel else _lib.lib().rq_moe_forward
        check(fwd(self.ctx.handle, self.handle, xp, yp, T, ids.ctypes.data if routing else None,
                  perm.ctypes.data if routing else None, stream))
        return y.reshape(shape), ids, perm

    def forward(self, xs):
        """The layer output.  With CUDA tensors and fewer than four tokens the
        call stays on the device (no host synchronisation) and can be captured
        in a CUDA graph once a first call at that token count has run."""
        return self.forward_with_routing(xs, routing=False)[0]

    __call__ = forward

    def set_device_plan(self, max_tokens: int) -> None:
        """Forwards of up to max_tokens tokens plan on the device (no host
        synchronisation, graph-capturable; slower from about 4 tokens)."""
        check(_lib.lib().rq_moe_set_device_plan(self.handle, int(max_tokens)))

    def close(self):
        if self.handle:
            _lib.lib().rq_moe_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
