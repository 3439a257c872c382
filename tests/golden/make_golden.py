"""Generate golden vectors for the oracle from gguf-py 0.19.0.

gguf-py is the published GGML reference dequantizer (the same block formats
candle-core 0.10.2 reads through QMatMul in src/streaming_quantized.rs:63-70).
This script runs in the development container only; its output
(golden_gguf.npz) is committed and is what the tests read.

    python tests/golden/make_golden.py
"""
import os

import numpy as np
from gguf import GGMLQuantizationType as GT
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))


def finite_blocks(rng, nb, bb, f16_offsets):
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    for off in f16_offsets:        # keep every f16 field finite and moderate
        raw[:, off + 1] &= 0x3F
    return raw


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    specs = {"q4_0": (GT.Q4_0, 18, [0]), "q4_k": (GT.Q4_K, 144, [0, 2]),
             "q3_k": (GT.Q3_K, 110, [108]), "q8_0": (GT.Q8_0, 34, [0]),
             "q6_k": (GT.Q6_K, 210, [208])}
    for name, (gt, bb, offs) in specs.items():
        raw = finite_blocks(rng, 96, bb, offs)
        out[f"{name}_blocks"] = raw
        out[f"{name}_dequant"] = quants.dequantize(raw.reshape(-1), gt).reshape(96, -1).astype(np.float32)
    # Q4_0 quantizer (same rule as src/q4_kernel.rs:137-163)
    w = (rng.standard_normal((8, 256)) * 0.1).astype(np.float32)
    w[0, :32] = 0.0                                  # all-zero block: d = 0, id = 0
    w[1, 5] = -3.0                                   # negative max
    out["q4_0_quant_in"] = w
    out["q4_0_quant_out"] = quants.quantize(w, GT.Q4_0).reshape(8, -1)
    # Q8_0 quantizer (GGML quantize_row_q8_0_ref; random data has no rounding
    # ties, where gguf-py's half-to-even and candle's half-away would differ)
    w8 = (rng.standard_normal((8, 256)) * 0.1).astype(np.float32)
    w8[0, :32] = 0.0
    out["q8_0_quant_in"] = w8
    out["q8_0_quant_out"] = quants.quantize(w8, GT.Q8_0).reshape(8, -1)
    # Q5_K and Q2_K blocks (a separate stream, so the vectors above keep
    # their values)
    rng2 = np.random.default_rng(20261202)
    for name, (gt, bb, offs) in {"q5_k": (GT.Q5_K, 176, [0, 2]), "q2_k": (GT.Q2_K, 84, [80, 82])}.items():
        raw = finite_blocks(rng2, 96, bb, offs)
        out[f"{name}_blocks"] = raw
        out[f"{name}_dequant"] = quants.dequantize(raw.reshape(-1), gt).reshape(96, -1).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "golden_gguf.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
