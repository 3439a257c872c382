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
    """The gate holds its weight in F16 (ParallelLinear::new,
    parallel_linear.rs:128-131)."""
    rng = np.random.default_rng(6)
    x = rng.standard_normal((5, 4096)).astype(np.float32)
    wr = (rng.standard_normal((8, 4096)) * 0.02).astype(np.float32)
    got = oracle.router_logits(x, wr)
    ref = x.astype(np.float64) @ wr.astype(np.float16).astype(np.float64).T
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)


def _f32_nearest(v):
    """The float32 nearest to the rational v, ties to even."""
    from fractions import Fraction
    f = np.float32(float(v))
    best = None
    for c in (np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))):
        d = abs(Fraction(float(c)) - v)
        key = (d, int(np.array(c, np.float32).view(np.uint32)) & 1)
        if best is None or key < best[0]:
            best = (key, c)
    return np.float32(best[1])


def _parallel_linear_exact(w16, x, avx2):
    """parallel_linear.rs:33-94 with every rounding done exactly: fused
    multiply-adds round once, the scalar and tail products twice."""
    from fractions import Fraction
    w = w16.astype(np.float32)
    out, n_in = w.shape
    y = np.empty((x.shape[0], out), np.float32)
    for b in range(x.shape[0]):
        for j in range(out):
            if avx2:
                acc = [np.float32(0.0)] * 8
                for i in range(n_in // 8):
                    for c in range(8):
                        k = 8 * i + c
                        acc[c] = _f32_nearest(Fraction(float(x[b, k])) * Fraction(float(w[j, k]))
                                              + Fraction(float(acc[c])))
                s = np.float32(-0.0)
                for c in range(8):
                    s = np.float32(s + acc[c])
                for k in range(n_in // 8 * 8, n_in):
                    s = np.float32(s + np.float32(x[b, k] * w[j, k]))
            else:
                s = np.float32(0.0)
                for k in range(n_in):
                    s = np.float32(s + np.float32(x[b, k] * w[j, k]))
            y[b, j] = s
    return y


@pytest.mark.parametrize("avx2", [True, False])
def test_parallel_linear_restates_reference_exactly(oracle, avx2):
    """The ParallelLinear restatement (a row of F16 weights converted to f32,
    then dot_f32_avx2_fma or the scalar loop) against an exact-rounding
    Python model of parallel_linear.rs:33-94, bit for bit; in = 44 exercises
    the scalar tail."""
    rng = np.random.default_rng(11)
    for n_in in (40, 44):
        w16 = (rng.standard_normal((5, n_in)) * 0.1).astype(np.float16)
        x = rng.standard_normal((3, n_in)).astype(np.float32)
        got = oracle.parallel_linear_f16(w16, x, avx2=avx2, nthreads=2)
        want = _parallel_linear_exact(w16, x, avx2)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_parallel_linear_matches_f32_linear(oracle):
    """parallel_linear.rs:304-328 matches_candle_linear_on_random_input:
    within 1e-2 of the plain f32 linear on the F16 weight; and the bias-free
    ones test of :330-343 (64 x 32 ones -> 32)."""
    rng = np.random.default_rng(12)
    w16 = (rng.standard_normal((128, 256)) * 0.1).astype(np.float16)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    ref = x.astype(np.float64) @ w16.astype(np.float64).T
    for avx2 in (True, False):
        for nt in (1, 5):
            got = oracle.parallel_linear_f16(w16, x, avx2=avx2, nthreads=nt)
            assert np.abs(got - ref).max() < 1e-2
    ones = oracle.parallel_linear_f16(np.ones((64, 32), np.float16), np.ones((1, 32), np.float32))
    assert np.all(ones == 32.0)


@pytest.mark.parametrize("qtype", [2, 8, 10, 11, 12, 13, 14])
def test_linear_rows_bits_equal_threaded(oracle, qtype):
    """The oracle's dequantize-once fast path gives rqo_linear_threaded's
    bits for every type and several M."""
    rng = np.random.default_rng(13 + qtype)
    out, n_in = 41, 1024
    b = oracle.quantize(qtype, (rng.standard_normal((out, n_in)) * 0.02).astype(np.float32))
    for M in (1, 3, 8):
        x = rng.standard_normal((M, n_in)).astype(np.float32)
        a = oracle.linear_threaded(qtype, b, out, n_in, x, nthreads=3)
        r = oracle.linear_rows(qtype, b, out, n_in, x, nthreads=4)
        assert np.array_equal(a.view(np.uint32), r.view(np.uint32))


def test_moe_f16_experts_close_to_f64(oracle):
    """The reference's own Mixtral layer (ParallelLinear F16 experts and
    gate) against a float64 restatement of SparseMoe::forward."""
    rng = np.random.default_rng(14)
    E, H, F, T, k = 4, 64, 96, 7, 2
    wr = (rng.standard_normal((E, H)) * 0.3).astype(np.float32)
    w1 = [(rng.standard_normal((F, H)) * 0.1).astype(np.float16) for _ in range(E)]
    w3 = [(rng.standard_normal((F, H)) * 0.1).astype(np.float16) for _ in range(E)]
    w2 = [(rng.standard_normal((H, F)) * 0.1).astype(np.float16) for _ in range(E)]
    x = rng.standard_normal((T, H)).astype(np.float32)
    y, ids, perm, offs = oracle.moe_forward(x, wr, oracle.F16, w1, w3, w2, F, k=k)
    lg = x.astype(np.float64) @ wr.astype(np.float16).astype(np.float64).T
    p = np.exp(lg - lg.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    want = np.zeros((T, H))
    for t in range(T):
        top = sorted(range(E), key=lambda e: -p[t, e])[:k]
        assert list(ids[t]) == top
        for e in sorted(top):
            g = w1[e].astype(np.float64) @ x[t]
            u = w3[e].astype(np.float64) @ x[t]
            want[t] += (p[t, e] / p[t, top].sum()) * (w2[e].astype(np.float64) @ (g / (1 + np.exp(-g)) * u))
    assert np.abs(y - want).max() < 1e-4 * np.abs(want).max() + 1e-6


def test_llama_teacher_forced_equals_incremental(oracle):
    """forward_all over prompt + generated tokens reproduces, position by
    position, the tokens and logits of the incremental greedy decode (the
    check the 70B bench applies to its tokens)."""
    rng = np.random.default_rng(15)
    cfg = dict(hidden=256, intermediate=512, n_heads=4, n_kv_heads=2, head_dim=64, n_layers=2,
               vocab=300, max_seq=40)
    ref = oracle.OracleLlama(cfg, 12)
    H, I = cfg["hidden"], cfg["intermediate"]
    shapes = [(256, H), (128, H), (128, H), (H, 256), (I, H), (I, H), (H, I)]
    for l in range(2):
        bl = [oracle.quantize(12, (rng.standard_normal(s) * 0.05).astype(np.float32)) for s in shapes]
        ref.set_layer(l, bl, (1 + 0.1 * rng.standard_normal(H)).astype(np.float32),
                      (1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    ref.set_embedding((rng.standard_normal((cfg["vocab"], H)) * 0.5).astype(np.float16))
    ref.set_head((1 + 0.1 * rng.standard_normal(H)).astype(np.float32),
                 (rng.standard_normal((cfg["vocab"], H)) * 0.1).astype(np.float16))
    prompt = rng.integers(0, cfg["vocab"], 9).astype(np.int32)
    gen = ref.generate(prompt, 6)
    last_logits, _ = ref.forward(np.array([gen[-1]], np.int32), len(prompt) + 5)
    logits, amax = ref.forward_all(np.concatenate([prompt, gen]).astype(np.int32), 0)
    assert amax[len(prompt) - 1:len(prompt) + 5].tolist() == gen
    assert np.array_equal(logits[-1].view(np.uint32), last_logits.view(np.uint32))
