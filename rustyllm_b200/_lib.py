"""ctypes binding of librq.so (the C ABI declared in include/rq.h).

The library is built in place (``rustyllm_b200/librq.so``).  Loading fails
loudly when it is missing: there is no CPU fallback behind this package.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "librq.so")
HEADERS = [os.path.join(os.path.dirname(HERE), "include", h) for h in ("rq.h",)]

RQ_OK = 0
Q4_0, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 2, 8, 10, 11, 12, 13, 14
TYPE_NAMES = {Q4_0: "Q4_0", Q8_0: "Q8_0", Q2_K: "Q2_K", Q3_K: "Q3_K", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q2_K: 84, Q3_K: 110, Q4_K: 144, Q5_K: 176, Q6_K: 210}
BLOCK_ELEMS = {Q4_0: 32, Q8_0: 32, Q2_K: 256, Q3_K: 256, Q4_K: 256, Q5_K: 256, Q6_K: 256}


class RqError(RuntimeError):
    """A non-zero status from librq; the message is rq_last_error()
    (the counterpart of the reference's ``Error::Msg``)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"rq: {msg} (status {code})")
        self.code = code


P, I64, I, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
PP = ctypes.POINTER(ctypes.c_void_p)

# name -> (restype, argtypes)
SIGNATURES = {
    "rq_init": (I, [I, PP]),
    "rq_destroy": (I, [P]),
    "rq_last_error": (I, [ctypes.c_char_p, SZ]),
    "rq_version": (ctypes.c_char_p, []),
    "rq_block_bytes": (SZ, [I]),
    "rq_block_elems": (I, [I]),
    "rq_weight_upload": (I, [P, I, P, SZ, I64, I64, PP]),
    "rq_weight_quantize": (I, [P, I, P, I64, I64, PP, P]),
    "rq_weight_download": (I, [P, P, P, SZ]),
    "rq_weight_free": (I, [P, P]),
    "rq_weight_info": (I, [P, ctypes.POINTER(I), ctypes.POINTER(I64), ctypes.POINTER(I64),
                           ctypes.POINTER(SZ)]),
    "rq_dequantize": (I, [P, P, P, P]),
    "rq_linear": (I, [P, P, P, P, I64, P]),
    "rq_linear_noalloc": (I, [P, P, P, I64, P]),
    "rq_ctx_status": (I, [P]),
    "rq_linear_allreduce": (I, [P, P, P, P, I64, P]),
    "rq_linear_batch": (I, [P, I, PP, PP, PP, P]),
    "rq_linear_prefetch_hint": (I, [P, I, PP]),
}

class LlamaConfig(ctypes.Structure):
    """rq_llama_config of include/rq.h."""
    _fields_ = [("hidden", ctypes.c_int64), ("intermediate", ctypes.c_int64),
                ("n_heads", ctypes.c_int64), ("n_kv_heads", ctypes.c_int64),
                ("head_dim", ctypes.c_int64), ("n_layers", ctypes.c_int64),
                ("vocab", ctypes.c_int64), ("max_seq", ctypes.c_int64),
                ("max_batch_tokens", ctypes.c_int64), ("rms_eps", ctypes.c_float),
                ("rope_theta", ctypes.c_float)]


SIGNATURES.update({
    "rq_llama_create": (I, [P, ctypes.POINTER(LlamaConfig), PP]),
    "rq_llama_free": (I, [P]),
    "rq_llama_set_layer": (I, [P, I64, PP, P, P]),
    "rq_llama_set_embedding": (I, [P, P]),
    "rq_llama_set_head": (I, [P, P, P]),
    "rq_llama_forward": (I, [P, P, I64, I64, P, P, P]),
    "rq_llama_decode_step": (I, [P, P]),
    "rq_llama_forward_all": (I, [P, P, I64, I64, P, P, P]),
    "rq_llama_set_fused": (I, [P, I]),
    "rq_llama_status": (I, [P]),
    "rq_llama_tokens": (I, [P, P, I64, ctypes.POINTER(I64), ctypes.POINTER(I64)]),
    "rq_llama_reset_tokens": (I, [P]),
    "rq_llama_truncate": (I, [P, I64]),
    "rq_tp_unique_id": (I, [P, SZ]),
    "rq_tp_init": (I, [P, I, I, P, I]),
    "rq_tp_allreduce_f32": (I, [P, P, P, I64, P]),
    "rq_tp_status": (I, [P]),
    "rq_tp_finalize": (I, [P]),
    "rq_moe_create": (I, [P, I, I, I64, I64, P, PP, PP, PP, PP]),
    "rq_moe_free": (I, [P]),
    "rq_moe_forward": (I, [P, P, P, P, I64, P, P, P]),
    "rq_moe_set_device_plan": (I, [P, I64]),
    "rq_moe_forward_ep": (I, [P, P, P, P, I64, P, P, P]),
    "rq_gguf_open": (I, [ctypes.c_char_p, PP]),
    "rq_gguf_open_memory": (I, [P, SZ, PP]),
    "rq_gguf_free": (I, [P]),
    "rq_gguf_tensor_count": (I, [P, ctypes.POINTER(I64)]),
    "rq_gguf_find": (I, [P, ctypes.c_char_p, ctypes.POINTER(I64)]),
    "rq_gguf_tensor_info": (I, [P, I64, ctypes.c_char_p, SZ, ctypes.POINTER(I), ctypes.POINTER(I),
                                ctypes.POINTER(I64), ctypes.POINTER(ctypes.c_uint64),
                                ctypes.POINTER(ctypes.c_uint64)]),
    "rq_gguf_tensor_data": (I, [P, I64, PP, ctypes.POINTER(ctypes.c_uint64)]),
    "rq_gguf_read_f32": (I, [P, ctypes.c_char_p, P, I64]),
    "rq_weight_upload_gguf": (I, [P, P, ctypes.c_char_p, I64, I64, I64, I64, PP]),
    "rq_llama_load_gguf_dir": (I, [P, ctypes.c_char_p]),
})

_lib = None


def declared_symbols() -> list[str]:
    """Entry points declared in include/*.h (parsed from the headers)."""
    names = []
    for h in HEADERS:
        with open(h) as f:
            txt = f.read()
        names += re.findall(r"^RQ_API\s+[\w\s\*]+?\b(rq_\w+)\s*\(", txt, flags=re.M)
    return names


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"librq.so not built at {LIB_PATH}; run __graft_entry__.build() "
                          "(make -C rustyllm_b200/csrc)")
    L = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().rq_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != RQ_OK:
        raise RqError(rc, last_error())
