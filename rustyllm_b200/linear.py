"""Host-side mirror of rustyllm's quantized-linear API over librq's C ABI.

Reference interfaces mirrored here (same names, argument meaning and error
behaviour):

* ``ParallelQ4Linear`` -- src/q4_kernel.rs:78-257 (``from_qtensor``,
  ``forward``, ``in_features``, ``out_features``).
* ``QMatMul`` -- the candle ``QMatMul`` held by ``QAttn``/``QMlp``
  (src/streaming_quantized.rs:160-169,260-264), built by
  ``GgufLayer::qmatmul`` (:63-70) from raw GGUF block bytes.
* ``QTensor`` -- the (dtype, shape, block bytes) triple candle hands over.

Activations may be numpy arrays (host memory; the library stages them) or
torch tensors (CUDA tensors run asynchronously on torch's current stream).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import BLOCK_BYTES, BLOCK_ELEMS, Q3_K, Q4_0, Q4_K, TYPE_NAMES, RqError, check

try:  # torch is plumbing only (device memory, streams)
    import torch
except Exception:  # pragma: no cover
    torch = None

__all__ = ["Context", "QTensor", "QMatMul", "ParallelQ4Linear", "RqError", "Q4_0", "Q3_K", "Q4_K"]


class Context:
    """One librq context per CUDA device (``rq_init``/``rq_destroy``)."""

    _per_device: dict[int, "Context"] = {}

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(_lib.lib().rq_init(int(device), ctypes.byref(h)))
        self.handle = h
        self.device = int(device)

    @classmethod
    def get(cls, device: int = 0) -> "Context":
        ctx = cls._per_device.get(device)
        if ctx is None:
            ctx = cls._per_device[device] = Context(device)
        return ctx

    def close(self) -> None:
        if self.handle:
            _lib.lib().rq_destroy(self.handle)
            self.handle = None
            if Context._per_device.get(self.device) is self:
                del Context._per_device[self.device]


def _stream_of(t) -> int:
    if torch is not None and isinstance(t, torch.Tensor) and t.is_cuda:
        return torch.cuda.current_stream(t.device).cuda_stream
    return 0


@dataclass
class QTensor:
    """GGML block bytes of a 2-D weight [out, in] (row-major blocks)."""

    ggml_type: int
    shape: tuple
    blocks: np.ndarray  # uint8, out * in / block * block_bytes

    def dtype(self) -> int:
        return self.ggml_type

    def dims(self) -> tuple:
        return tuple(self.shape)

    @staticmethod
    def nbytes_for(ggml_type: int, out: int, n_in: int) -> int:
        return out * (n_in // BLOCK_ELEMS[ggml_type]) * BLOCK_BYTES[ggml_type]

    @classmethod
    def quantize(cls, w, ggml_type: int, device: int = 0) -> "QTensor":
        """Quantize an f32 [out, in] matrix on the GPU (rq_weight_quantize) and
        return its GGML bytes -- the counterpart of QTensor::quantize
        (src/quantize.rs:131)."""
        if torch is None:
            raise RqError(1, "QTensor.quantize needs torch for device memory")
        wt = torch.as_tensor(w, dtype=torch.float32).to(f"cuda:{device}").contiguous()
        qw = QWeight.quantize(Context.get(device), ggml_type, wt)
        torch.cuda.synchronize(device)
        blocks = qw.download()
        return cls(ggml_type, tuple(wt.shape), blocks)


class QWeight:
    """A device-resident quantized weight owned by librq."""

    def __init__(self, ctx: Context, handle: ctypes.c_void_p, ggml_type: int, out: int, n_in: int):
        self.ctx, self.handle = ctx, handle
        self.ggml_type, self.out, self.n_in = ggml_type, out, n_in

    @classmethod
    def upload(cls, ctx: Context, ggml_type: int, blocks, out: int, n_in: int) -> "QWeight":
        if torch is not None and isinstance(blocks, torch.Tensor):
            ptr, nbytes = blocks.data_ptr(), blocks.numel() * blocks.element_size()
            keep = blocks
        else:
            keep = np.ascontiguousarray(blocks, dtype=np.uint8)
            ptr, nbytes = keep.ctypes.data, keep.nbytes
        h = ctypes.c_void_p()
        check(_lib.lib().rq_weight_upload(ctx.handle, ggml_type, ptr, nbytes, out, n_in,
                                          ctypes.byref(h)))
        del keep
        return cls(ctx, h, ggml_type, out, n_in)

    @classmethod
    def quantize(cls, ctx: Context, ggml_type: int, w_dev) -> "QWeight":
        out, n_in = w_dev.shape
        h = ctypes.c_void_p()
        check(_lib.lib().rq_weight_quantize(ctx.handle, ggml_type, w_dev.data_ptr(), out, n_in,
                                            ctypes.byref(h), _stream_of(w_dev)))
        return cls(ctx, h, ggml_type, out, n_in)

    def download(self) -> np.ndarray:
        n = QTensor.nbytes_for(self.ggml_type, self.out, self.n_in)
        buf = np.empty(n, dtype=np.uint8)
        check(_lib.lib().rq_weight_download(self.ctx.handle, self.handle, buf.ctypes.data, n))
        return buf.reshape(self.out, -1)

    def dequantize(self, into=None):
        """f32 [out, in]: numpy (host) unless `into` is a CUDA tensor."""
        y = into if into is not None else np.empty((self.out, self.n_in), dtype=np.float32)
        ptr = y.data_ptr() if (torch is not None and isinstance(y, torch.Tensor)) else y.ctypes.data
        check(_lib.lib().rq_dequantize(self.ctx.handle, self.handle, ptr, _stream_of(y)))
        return y

    def device_bytes(self) -> int:
        n = ctypes.c_size_t()
        check(_lib.lib().rq_weight_info(self.handle, None, None, None, ctypes.byref(n)))
        return n.value

    def free(self) -> None:
        if self.handle:
            _lib.lib().rq_weight_free(self.ctx.handle, self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _linear(w: QWeight, x):
    """y = x W^T through rq_linear; x numpy / torch (host or CUDA)."""
    L = _lib.lib()
    if torch is not None and isinstance(x, torch.Tensor):
        lead = tuple(x.shape[:-1])
        xin = x.reshape(-1, w.n_in)
        if xin.dtype != torch.float32:
            xin = xin.float()
        xin = xin.contiguous()
        M = xin.shape[0]
        y = torch.empty((M, w.out), dtype=torch.float32, device=xin.device)
        check(L.rq_linear(w.ctx.handle, w.handle, xin.data_ptr(), y.data_ptr(), M, _stream_of(xin)))
        y = y.reshape(*lead, w.out)
        return y if x.dtype == torch.float32 else y.to(x.dtype)
    xa = np.asarray(x)
    lead = xa.shape[:-1]
    xin = np.ascontiguousarray(xa.reshape(-1, w.n_in), dtype=np.float32)
    M = xin.shape[0]
    y = np.empty((M, w.out), dtype=np.float32)
    check(L.rq_linear(w.ctx.handle, w.handle, xin.ctypes.data, y.ctypes.data, M, 0))
    y = y.reshape(*lead, w.out)
    return y if xa.dtype == np.float32 else y.astype(xa.dtype)


class QMatMul:
    """Drop-in for candle's QMatMul over Q4_0 / Q4_K / Q3_K GGUF tensors."""

    def __init__(self, weight: QWeight):
        self.weight = weight

    @classmethod
    def from_qtensor(cls, qt: QTensor, device: int = 0) -> "QMatMul":
        if qt.ggml_type not in TYPE_NAMES:
            raise RqError(3, f"QMatMul: unsupported dtype {qt.ggml_type}")
        if len(qt.shape) != 2:
            raise RqError(1, f"QMatMul: expected 2D weight, got {list(qt.shape)}")
        out, n_in = qt.shape
        return cls(QWeight.upload(Context.get(device), qt.ggml_type, qt.blocks, out, n_in))

    def forward(self, x):
        n_in = self.weight.n_in
        if tuple(x.shape)[-1] != n_in:
            raise RqError(1, f"QMatMul: last dim {tuple(x.shape)[-1]} != in_features {n_in}")
        return _linear(self.weight, x)

    __call__ = forward


class ParallelQ4Linear:
    """Mirror of src/q4_kernel.rs:78-257 on the GPU."""

    QK4_0 = 32
    BLOCK_SIZE = 18

    def __init__(self, weight: QWeight):
        self.weight = weight

    @classmethod
    def from_qtensor(cls, qt: QTensor, device: int = 0) -> "ParallelQ4Linear":
        # argument checks and messages follow q4_kernel.rs:90-108
        if qt.ggml_type != Q4_0:
            raise RqError(1, f"ParallelQ4Linear: expected Q4_0, got {TYPE_NAMES.get(qt.ggml_type, qt.ggml_type)}")
        if len(qt.shape) != 2:
            raise RqError(1, f"ParallelQ4Linear: expected 2D weight, got {list(qt.shape)}")
        out, n_in = qt.shape
        if n_in % cls.QK4_0 != 0:
            raise RqError(1, f"ParallelQ4Linear: in_features {n_in} not divisible by {cls.QK4_0}")
        ctx = Context.get(device)
        # q4_kernel.rs:120-163 round-trips through an f32 dequantize and
        # re-packs with its own rule; do the same on the device.
        src = QWeight.upload(ctx, Q4_0, qt.blocks, out, n_in)
        deq = torch.empty((out, n_in), dtype=torch.float32, device=f"cuda:{device}")
        src.dequantize(into=deq)
        w = QWeight.quantize(ctx, Q4_0, deq)
        torch.cuda.synchronize(device)
        src.free()
        return cls(w)

    def in_features(self) -> int:
        return self.weight.n_in

    def out_features(self) -> int:
        return self.weight.out

    def forward(self, x):
        last = tuple(x.shape)[-1] if len(x.shape) else 0
        if last != self.weight.n_in:
            raise RqError(1, f"ParallelQ4Linear: last dim {last} != in_features {self.weight.n_in}")
        return _linear(self.weight, x)

    __call__ = forward
