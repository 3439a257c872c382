"""rq_linear_noalloc: the quantized linear for callers that cannot allocate.

Serving engines that reserve nearly all device memory up front, or host
frameworks whose allocator owns every device buffer, cannot let librq grow a
workspace with cudaMalloc.  rq_linear_noalloc stages activations in a static
device array instead.  These tests call it through the C ABI and compare it
with rq_linear, on two calls in a row (the array keeps the previous call's
contents, so a second call with a different shape would expose stale data).

The file sorts last so that a run stopping at the first failure has run
every other test first; it also passes on its own in a fresh process.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-4  # the tolerance the linear parity tests use


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _weight(oracle, rq_ctx, qtype, out, n_in, seed):
    from rustyllm_b200 import QWeight
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((out, n_in)) * 0.02).astype(np.float32)
    return QWeight.upload(rq_ctx, qtype, oracle.quantize(qtype, w), out, n_in)


# (type, out, in, M): consecutive calls differ in every size, a larger one
# before a smaller one, so a call reading stale staging would show.  M = 16
# is where rq_linear itself runs a tensor-core kernel; the no-alloc path runs
# the M=1 matvec on each of its rows.
CASES = [
    (12, 1000, 4096, 16),
    (12, 1000, 4096, 1),
    (11, 512, 8192, 3),
    (12, 768, 28672, 20),   # the largest M the array holds at in = 28672
    (12, 96, 8192, 5),
]


def test_noalloc_matches_rq_linear_and_oracle_on_two_calls(oracle, rq_ctx):
    import torch
    from rustyllm_b200._lib import check, lib
    L = lib()
    for rnd in range(2):
        for k, (qtype, out, n_in, M) in enumerate(CASES):
            qw = _weight(oracle, rq_ctx, qtype, out, n_in, seed=10 * k + 1)
            xn = np.random.default_rng(k + 7 * rnd).standard_normal((M, n_in)).astype(np.float32)
            x = torch.from_numpy(xn).cuda()
            y_ref = torch.empty(M, out, device="cuda")
            y_na = torch.full((M, out), float("nan"), device="cuda")
            st = torch.cuda.current_stream().cuda_stream
            check(L.rq_linear(rq_ctx.handle, qw.handle, x.data_ptr(), y_ref.data_ptr(), M, st))
            check(L.rq_linear_noalloc(qw.handle, x.data_ptr(), y_na.data_ptr(), M, st))
            torch.cuda.synchronize()
            got = y_na.cpu().numpy()
            assert rel_l2(got, y_ref.cpu().numpy()) <= REL_L2_TOL
            want = oracle.matmul_ref(qtype, qw.download(), out, n_in, xn)
            assert rel_l2(got, want) <= REL_L2_TOL
            qw.free()
    check(L.rq_ctx_status(rq_ctx.handle))  # no kernel wait gave up


def test_noalloc_allocates_nothing(oracle, rq_ctx):
    """After the shapes have run once (the library's kernels and the static
    array are loaded by then), repeated calls at every shape, the largest M
    the array holds included, leave the device's free memory unchanged."""
    import torch
    from rustyllm_b200._lib import check, lib
    L = lib()
    st = torch.cuda.current_stream().cuda_stream
    bufs = []
    for k, (qtype, out, n_in, M) in enumerate(CASES):
        qw = _weight(oracle, rq_ctx, qtype, out, n_in, seed=50 + k)
        x = torch.randn(M, n_in, device="cuda")
        y = torch.empty(M, out, device="cuda")
        bufs.append((qw, x, y, M))

    def run():
        for qw, x, y, M in bufs:
            check(L.rq_linear_noalloc(qw.handle, x.data_ptr(), y.data_ptr(), M, st))
        torch.cuda.synchronize()

    run()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        run()
    assert torch.cuda.mem_get_info()[0] == free0
    for qw, *_ in bufs:
        qw.free()


def test_noalloc_rejects_oversize_and_host_pointers(oracle, rq_ctx):
    import torch
    from rustyllm_b200._lib import last_error, lib
    L = lib()
    qw = _weight(oracle, rq_ctx, 12, 64, 28672, seed=3)
    M = 64  # 64 x 28672 x 3.5 bytes > 2 MiB
    x = torch.zeros(M, 28672, device="cuda")
    y = torch.zeros(M, 64, device="cuda")
    rc = L.rq_linear_noalloc(qw.handle, x.data_ptr(), y.data_ptr(), M, None)
    assert rc == 1 and "static scratch" in last_error()
    xh = np.zeros((1, 28672), np.float32)
    rc = L.rq_linear_noalloc(qw.handle, xh.ctypes.data, y.data_ptr(), 1, None)
    assert rc == 1 and "device memory" in last_error()
    assert L.rq_linear_noalloc(qw.handle, x.data_ptr(), y.data_ptr(), 0, None) == 0
    assert L.rq_linear_noalloc(None, x.data_ptr(), y.data_ptr(), 1, None) == 1
