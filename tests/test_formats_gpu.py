"""The other GGML formats of the reference's quantizer (src/quantize.rs:
29-37) on the M=1 pipeline: Q8_0 (blocks of 32: f16 d, 32 int8), Q6_K
(super-blocks of 256: 6-bit q from ql / qh, int8 scale per 16, f16 d), Q5_K
(Q4_K's 6-bit scale/min pairs per 32 with a fifth q bit from qh) and Q2_K
(2-bit q, 4-bit scale and min per 16, f16 d and dmin).
Bytes survive the device layout, GPU dequantization is bit-identical to the
oracle (pinned to gguf-py) including on arbitrary block bytes, the GPU
quantizer writes the oracle's bytes, and matvec outputs are within relative
L2 1e-4 of the f64 reference at partial slices and 70B shapes."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-4
Q8_0, Q6_K, Q5_K, Q2_K = 8, 14, 13, 10
ALL = [Q8_0, Q6_K, Q5_K, Q2_K]
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_gguf.npz")


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("qtype,name,n_in", [(Q8_0, "q8_0", 256), (Q6_K, "q6_k", 1024), (Q5_K, "q5_k", 1024),
                                              (Q2_K, "q2_k", 1024)])
def test_golden_blocks_roundtrip_and_dequant(oracle, rq_ctx, qtype, name, n_in):
    from rustyllm_b200 import QWeight
    g = np.load(GOLDEN)
    blocks = g[f"{name}_blocks"]
    per_row = n_in // oracle.BLOCK_ELEMS[qtype]
    out = blocks.shape[0] // per_row
    blocks = blocks.reshape(out, -1)
    w = QWeight.upload(rq_ctx, qtype, blocks, out, n_in)
    assert np.array_equal(w.download(), blocks)
    got = w.dequantize()
    want = g[f"{name}_dequant"].reshape(out, n_in)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("qtype", ALL)
def test_gpu_quantizer_matches_oracle(oracle, rq_ctx, qtype):
    import torch
    from rustyllm_b200 import QWeight
    rng = np.random.default_rng(qtype)
    w = (rng.standard_normal((40, 2048)) * 0.02).astype(np.float32)
    w[0, :256] = 0.0
    w[1, 7] = -0.7
    qw = QWeight.quantize(rq_ctx, qtype, torch.from_numpy(w).cuda())
    torch.cuda.synchronize()
    assert np.array_equal(qw.download(), oracle.quantize(qtype, w).reshape(40, -1))


@pytest.mark.parametrize("qtype", ALL)
@pytest.mark.parametrize("out,n_in,M", [(64, 1024, 1), (200, 3072, 1), (48, 5120, 3), (1024, 8192, 1),
                                        (256, 28672, 2)])
def test_matvec_matches_oracle(oracle, rq_ctx, qtype, out, n_in, M):
    """Partial K-slices (1024, 3072, 5120 are not multiples of 2048), several
    rows per call, and the 70B K of 8192 / 28672."""
    from rustyllm_b200 import QWeight
    from rustyllm_b200.linear import _linear
    rng = np.random.default_rng(out + n_in + qtype)
    w = (rng.standard_normal((out, n_in)) * 0.02).astype(np.float32)
    blocks = oracle.quantize(qtype, w)
    qw = QWeight.upload(rq_ctx, qtype, blocks, out, n_in)
    x = rng.standard_normal((M, n_in)).astype(np.float32)
    y = _linear(qw, x)
    ref = oracle.matmul_ref(qtype, blocks, out, n_in, x, acc64=True)
    assert np.isfinite(y).all()
    for m in range(M):
        assert rel_l2(y[m], ref[m]) <= REL_L2_TOL


@pytest.mark.parametrize("qtype", [Q6_K, Q2_K])
def test_20_byte_headers_need_whole_kilo_rows(oracle, rq_ctx, qtype):
    """Q6_K and Q2_K rows must be a multiple of 1024 elements for the
    pipeline (their 20-byte headers); other sizes are refused with a
    message, not run."""
    from rustyllm_b200 import QWeight
    from rustyllm_b200._lib import RqError
    from rustyllm_b200.linear import _linear
    blocks = oracle.quantize(qtype, np.zeros((8, 768), np.float32))
    qw = QWeight.upload(rq_ctx, qtype, blocks, 8, 768)
    with pytest.raises(RqError, match="multiple of 1024"):
        _linear(qw, np.ones((1, 768), np.float32))


@pytest.mark.parametrize("n_in", [256, 768, 1280])
def test_q5_k_short_rows(oracle, rq_ctx, n_in):
    """Q5_K's 160 + 16 bytes per super-block keep every row a 16-byte
    multiple, so rows of any whole number of super-blocks run (one, three,
    five of them: a partial K-slice with lanes past the row end)."""
    from rustyllm_b200 import QWeight
    from rustyllm_b200.linear import _linear
    rng = np.random.default_rng(n_in)
    w = (rng.standard_normal((96, n_in)) * 0.02).astype(np.float32)
    blocks = oracle.quantize(Q5_K, w)
    qw = QWeight.upload(rq_ctx, Q5_K, blocks, 96, n_in)
    x = rng.standard_normal((2, n_in)).astype(np.float32)
    y = _linear(qw, x)
    ref = oracle.matmul_ref(Q5_K, blocks, 96, n_in, x, acc64=True)
    for m in range(2):
        assert rel_l2(y[m], ref[m]) <= REL_L2_TOL
