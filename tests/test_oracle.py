"""CPU tests of the oracle itself: pinned against gguf-py golden vectors and
against the reference's own Q4_0 tests (src/q4_kernel.rs:362-432)."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_gguf.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_f16_conversion_matches_numpy(oracle):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(200_000) * np.exp(rng.uniform(-30, 12, 200_000))).astype(np.float32)
    edge = np.array([65519.0, 65520.0, 6.1e-5, 5.96e-8, 2.98e-8, 2.9802322e-08, 0.0, -0.0,
                     1e-10, -65504.0, np.inf, -np.inf], dtype=np.float32)
    x = np.concatenate([x, edge])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(oracle.f32_to_f16_bits(x), want)
    allh = np.arange(65536, dtype=np.uint16)
    got = oracle.f16_bits_to_f32(allh)
    ref = allh.view(np.float16).astype(np.float32)
    ok = np.isnan(ref) | (got.view(np.uint32) == ref.view(np.uint32))
    assert ok.all()


@pytest.mark.parametrize("name,qtype", [("q4_0", 2), ("q4_k", 12), ("q3_k", 11), ("q8_0", 8), ("q6_k", 14),
                                        ("q5_k", 13), ("q2_k", 10)])
def test_dequant_matches_gguf_golden(oracle, golden, name, qtype):
    blocks = golden[f"{name}_blocks"]
    want = golden[f"{name}_dequant"]
    got = oracle.dequantize(qtype, blocks, blocks.shape[0], want.shape[1])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_q8_0_quantizer_matches_gguf_golden(oracle, golden):
    got = oracle.quantize(oracle.Q8_0, golden["q8_0_quant_in"])
    assert np.array_equal(got, golden["q8_0_quant_out"])


def test_q6_k_quantizer_roundtrip(oracle):
    """The Q6_K quantizer is this project's own rule (unpinned, like Q4_K /
    Q3_K): its blocks dequantize close to the input and re-quantize to the
    same bytes."""
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((6, 512)) * 0.02).astype(np.float32)
    w[0, :256] = 0.0
    b = oracle.quantize(oracle.Q6_K, w)
    d = oracle.dequantize(oracle.Q6_K, b, 6, 512)
    assert np.all(d[0, :256] == 0.0)
    assert np.linalg.norm(d - w) / np.linalg.norm(w) < 0.03
    assert np.array_equal(oracle.quantize(oracle.Q6_K, d), b)


@pytest.mark.parametrize("qtype,tol", [(13, 0.05), (10, 0.4)])
def test_k_quantizers_roundtrip(oracle, qtype, tol):
    """The Q5_K / Q2_K quantizers are this project's own rules (unpinned):
    an all-zero super-block stays zero, blocks dequantize within the
    format's expected error (5-bit vs 2-bit levels), and the packed fields
    decode back to the levels the quantizer chose."""
    rng = np.random.default_rng(qtype)
    w = (rng.standard_normal((6, 512)) * 0.02).astype(np.float32)
    w[0, :256] = 0.0
    b = oracle.quantize(qtype, w)
    assert b.shape == (6, 2 * oracle.BLOCK_BYTES[qtype])
    d = oracle.dequantize(qtype, b, 6, 512)
    assert np.all(d[0, :256] == 0.0)
    assert np.linalg.norm(d - w) / np.linalg.norm(w) < tol


def test_q4_0_quantizer_matches_gguf_golden(oracle, golden):
    got = oracle.quantize(oracle.Q4_0, golden["q4_0_quant_in"])
    assert np.array_equal(got, golden["q4_0_quant_out"])


def test_q4_0_repack_is_idempotent(oracle):
    # from_qtensor (q4_kernel.rs:120-163) dequantizes then re-packs; a second
    # pass must reproduce the same bytes
    rng = np.random.default_rng(2)
    w = (rng.standard_normal((64, 256)) * 0.1).astype(np.float32)
    b1 = oracle.quantize(oracle.Q4_0, w)
    b2 = oracle.quantize(oracle.Q4_0, oracle.dequantize(oracle.Q4_0, b1, 64, 256))
    assert np.array_equal(b1, b2)


def test_scalar_and_avx2_agree(oracle):
    # q4_kernel.rs:406-431: 32x128, |diff| < 1e-4
    rng = np.random.default_rng(3)
    w = oracle.quantize(oracle.Q4_0, (rng.standard_normal((32, 128)) * 0.1).astype(np.float32))
    x = rng.standard_normal(128).astype(np.float32)
    for r in range(32):
        a = oracle.dot_q4_0_avx2order(w[r], x)
        s = oracle.dot_q4_0_scalar(w[r], x)
        assert abs(a - s) < 1e-4


@pytest.mark.parametrize("qtype,tol", [(2, 0.10), (12, 0.09), (11, 0.18)])
def test_quantizer_round_trip_error(oracle, qtype, tol):
    rng = np.random.default_rng(4)
    w = (rng.standard_normal((32, 1024)) * 0.02).astype(np.float32)
    d = oracle.dequantize(qtype, oracle.quantize(qtype, w), 32, 1024)
    assert np.linalg.norm(d - w) / np.linalg.norm(w) < tol


@pytest.mark.parametrize("qtype", [2, 12, 11])
def test_threaded_forward_matches_reference(oracle, qtype):
    rng = np.random.default_rng(5)
    out, n_in = 37, 512
    b = oracle.quantize(qtype, (rng.standard_normal((out, n_in)) * 0.02).astype(np.float32))
    x = rng.standard_normal((3, n_in)).astype(np.float32)
    ref = oracle.matmul_ref(qtype, b, out, n_in, x, acc64=True)
    for nt in (1, 4):
        y = oracle.linear_threaded(qtype, b, out, n_in, x, nthreads=nt)
        assert np.linalg.norm(y - ref) / np.linalg.norm(ref) < 1e-5


def test_quantized_zero_rows(oracle):
    z = np.zeros((2, 256), dtype=np.float32)
    for qtype in (2, 12, 11):
        b = oracle.quantize(qtype, z)
        assert not oracle.dequantize(qtype, b, 2, 256).any()


def test_route_topk_semantics(oracle):
    # streaming_mixtral.rs:292-303: stable descending order, ties to the lower
    # index, weights renormalised over the selected experts
    logits = np.array([[0.0, 1.0, 1.0, -1.0, 0.5, 1.0, -2.0, 0.0],
                       [3.0, 3.0, 3.0, 3.0, 3.0, 3.0, 3.0, 3.0]], dtype=np.float32)
    ids, w = oracle.route_topk(logits, 2)
    assert ids.tolist() == [[1, 2], [0, 1]]
    np.testing.assert_allclose(w, [[0.5, 0.5], [0.5, 0.5]], rtol=1e-6)
    offs, rows, sw = oracle.permute(ids, w, 8)
    assert offs.tolist() == [0, 1, 3, 4, 4, 4, 4, 4, 4]
    assert rows.tolist() == [1, 0, 1, 0]


def test_router_logits_close_to_f64(oracle):
    rng = np.random.default_rng(6)
    x = rng.standard_normal((5, 4096)).astype(np.float32)
    wr = (rng.standard_normal((8, 4096)) * 0.02).astype(np.float32)
    got = oracle.router_logits(x, wr)
    ref = x.astype(np.float64) @ wr.astype(np.float64).T
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)
