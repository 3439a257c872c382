"""GGUF files through librq (rq_gguf_* in include/rq.h): the counterpart of
the reference's per-layer shard reader GgufLayer
(src/streaming_quantized.rs:42-91) -- open, list tensors, read F16/F32
norms, upload Q4_0 / Q4_K / Q3_K matrices (optionally a tensor-parallel
slice) straight to the GPU."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import check


class GGUFFile:
    """A GGUF file read into host memory once and parsed by the library."""

    def __init__(self, source):
        h = ctypes.c_void_p()
        if isinstance(source, (bytes, bytearray, memoryview)):
            buf = bytes(source)
            check(_lib.lib().rq_gguf_open_memory(buf, len(buf), ctypes.byref(h)))
        else:
            check(_lib.lib().rq_gguf_open(str(source).encode(), ctypes.byref(h)))
        self.handle = h

    def close(self) -> None:
        if self.handle:
            _lib.lib().rq_gguf_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        n = ctypes.c_int64()
        check(_lib.lib().rq_gguf_tensor_count(self.handle, ctypes.byref(n)))
        return n.value

    def info(self, index: int) -> dict:
        """name, ggml type, shape (outermost first, like numpy), file offset
        and byte size of tensor `index`."""
        name = ctypes.create_string_buffer(512)
        t, nd = ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_int64 * 4)()
        off, nb = ctypes.c_uint64(), ctypes.c_uint64()
        check(_lib.lib().rq_gguf_tensor_info(self.handle, index, name, len(name), ctypes.byref(t),
                                             ctypes.byref(nd), dims, ctypes.byref(off), ctypes.byref(nb)))
        shape = tuple(int(dims[d]) for d in range(nd.value))[::-1]
        return {"name": name.value.decode(), "type": t.value, "shape": shape,
                "offset": off.value, "nbytes": nb.value}

    def names(self) -> list[str]:
        return [self.info(i)["name"] for i in range(len(self))]

    def index(self, name: str) -> int:
        i = ctypes.c_int64()
        check(_lib.lib().rq_gguf_find(self.handle, name.encode(), ctypes.byref(i)))
        return i.value

    def raw(self, name: str) -> np.ndarray:
        """A copy of the tensor's bytes."""
        p, nb = ctypes.c_void_p(), ctypes.c_uint64()
        check(_lib.lib().rq_gguf_tensor_data(self.handle, self.index(name), ctypes.byref(p), ctypes.byref(nb)))
        return np.ctypeslib.as_array((ctypes.c_uint8 * nb.value).from_address(p.value)).copy()

    def read_f32(self, name: str) -> np.ndarray:
        """An F32 / F16 / BF16 tensor as f32 (GgufLayer::tensor)."""
        info = self.info(self.index(name))
        n = int(np.prod(info["shape"]))
        out = np.empty(n, dtype=np.float32)
        check(_lib.lib().rq_gguf_read_f32(self.handle, name.encode(), out.ctypes.data, n))
        return out.reshape(info["shape"])

    def upload(self, ctx, name: str, rows: tuple[int, int] | None = None, cols: tuple[int, int] | None = None):
        """QWeight of a 2-D block-quantized tensor, or of rows [r0, r1) x
        columns [c0, c1) of it (GgufLayer::qmatmul)."""
        from .linear import QWeight
        r0, r1 = rows if rows else (0, -1)
        c0, c1 = cols if cols else (0, -1)
        h = ctypes.c_void_p()
        check(_lib.lib().rq_weight_upload_gguf(ctx.handle, self.handle, name.encode(), r0,
                                               r1 - r0 if r1 >= 0 else -1, c0, c1 - c0 if c1 >= 0 else -1,
                                               ctypes.byref(h)))
        info = self.info(self.index(name))
        out = (r1 if r1 >= 0 else info["shape"][0]) - r0
        n_in = (c1 if c1 >= 0 else info["shape"][1]) - c0
        return QWeight(ctx, h, info["type"], out, n_in)
