"""Two-GPU tensor parallelism of the Llama decode loop: greedy tokens of the
TP=2 model (column/row-parallel shards, all-reduces, vocab-parallel argmax)
equal the single-GPU model's with the all-reduce fused into the row-parallel
matvec kernel (the decode default), as a separate peer-memory kernel
(RQ_TP_FUSED=0) and with NCCL.
The peer-memory all-reduce itself: every rank gets the same bits, the sum
in rank order, over both buffer parities, in place and out of place, at
sizes below and above its NCCL cut-over.  Skipped with fewer than two
GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(hidden=512, intermediate=1024, n_heads=8, n_kv_heads=2, head_dim=64, n_layers=2,
           vocab=1000, max_seq=64, max_batch_tokens=32, rms_eps=1e-5, rope_theta=10000.0)
# shards whole heads and whole super-blocks at 4 and 8 ranks: 8 KV heads,
# o_proj's 2048 inputs and down_proj's 4096 split on 256-element boundaries
CFG8 = dict(hidden=2048, intermediate=4096, n_heads=16, n_kv_heads=8, head_dim=128, n_layers=2,
            vocab=1024, max_seq=64, max_batch_tokens=32, rms_eps=1e-5, rope_theta=10000.0)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_rank(rank, world, port, out_dir, mode="p2p", cfg=CFG):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    if mode == "nccl":
        os.environ["RQ_TP_ALLREDUCE"] = "nccl"
    if mode == "unfused":
        os.environ["RQ_TP_FUSED"] = "0"
    if mode == "fused":
        os.environ["RQ_TP_FUSED"] = "1"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from rustyllm_b200 import Context
    from rustyllm_b200 import tp as tpmod
    from rustyllm_b200.llama import random_model
    ctx = Context.get(rank)
    tpmod.init_from_torch(ctx, timeout_ms=60000)
    model, _ = random_model(cfg, 12, seed=11, device=rank, tp=(world, rank))
    prompt = np.random.default_rng(4).integers(0, cfg["vocab"], size=16).astype(np.int32)
    toks = model.generate(prompt, 12)
    np.save(os.path.join(out_dir, f"tp{mode}{world}_{rank}.npy"), np.array(toks))
    model.close()
    from rustyllm_b200 import _lib
    _lib.check(_lib.lib().rq_tp_status(ctx.handle))   # no peer wait timed out
    tpmod.finalize(ctx)
    dist.destroy_process_group()


def test_tp2_decode_matches_single_gpu(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from rustyllm_b200.llama import random_model
    model, _ = random_model(CFG, 12, seed=11, device=0)
    prompt = np.random.default_rng(4).integers(0, CFG["vocab"], size=16).astype(np.int32)
    want = model.generate(prompt, 12)
    model.close()
    for mode in ("p2p", "unfused", "nccl"):
        mp.spawn(_tp_rank, args=(2, _free_port(), str(tmp_path), mode), nprocs=2, join=True)
        for r in range(2):
            assert np.load(tmp_path / f"tp{mode}2_{r}.npy").tolist() == want


@pytest.mark.parametrize("world", [4, 8])
def test_tp_decode_matches_single_gpu_at_4_and_8(tmp_path, world):
    """Tensor parallelism at 4 and 8 ranks: the fused matvec + all-reduce
    epilogue, the separate peer-memory all-reduce kernel and NCCL all give
    the single-GPU tokens."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    from rustyllm_b200.llama import random_model
    model, _ = random_model(CFG8, 12, seed=11, device=0)
    prompt = np.random.default_rng(4).integers(0, CFG8["vocab"], size=16).astype(np.int32)
    want = model.generate(prompt, 12)
    model.close()
    for mode in ("fused", "unfused", "nccl"):
        mp.spawn(_tp_rank, args=(world, _free_port(), str(tmp_path), mode, CFG8), nprocs=world, join=True)
        for r in range(world):
            assert np.load(tmp_path / f"tp{mode}{world}_{r}.npy").tolist() == want, (mode, r)


SIZES = [1, 8192, 163840, 600000]  # the last one exceeds the peer buffer: NCCL


def _allreduce_rank(rank, world, port, out_dir):
    import ctypes
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from rustyllm_b200 import Context
    from rustyllm_b200 import _lib
    from rustyllm_b200 import tp as tpmod
    ctx = Context.get(rank)
    tpmod.init_from_torch(ctx, timeout_ms=60000)
    L = _lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    outs = {}
    for it in range(3):                     # both buffer parities, reused
        for n in SIZES:
            g = torch.Generator(device="cuda").manual_seed(1000 * it + 10 * rank + n % 7)
            x = torch.randn(n, device="cuda", generator=g)
            y = torch.empty_like(x)
            _lib.check(L.rq_tp_allreduce_f32(ctx.handle, x.data_ptr(), y.data_ptr(), n, s))
            z = x.clone()
            _lib.check(L.rq_tp_allreduce_f32(ctx.handle, z.data_ptr(), z.data_ptr(), n, s))   # in place
            torch.cuda.synchronize()
            outs[f"in{it}_{n}"] = x.cpu().numpy()
            outs[f"out{it}_{n}"] = y.cpu().numpy()
            outs[f"inplace{it}_{n}"] = z.cpu().numpy()
    _lib.check(L.rq_tp_status(ctx.handle))
    np.savez(os.path.join(out_dir, f"ar{rank}.npz"), **outs)
    tpmod.finalize(ctx)
    dist.destroy_process_group()


def test_peer_allreduce_two_gpus(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_allreduce_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    a = [np.load(tmp_path / f"ar{r}.npz") for r in range(2)]
    for it in range(3):
        for n in SIZES:
            want = a[0][f"in{it}_{n}"] + a[1][f"in{it}_{n}"]      # f32, rank order
            for r in range(2):
                assert np.array_equal(a[r][f"out{it}_{n}"], want)
                assert np.array_equal(a[r][f"inplace{it}_{n}"], want)


def _timeout_rank(rank, world, port, out_dir):
    """Rank 1 skips one all-reduce (it leaves between steps, nothing in
    flight); rank 0's bounded wait for rank 1's flag must give up (~1 s) and
    rq_tp_status must report it, with no GPU fault."""
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from rustyllm_b200 import Context
    from rustyllm_b200 import _lib
    from rustyllm_b200 import tp as tpmod
    ctx = Context.get(rank)
    tpmod.init_from_torch(ctx, timeout_ms=60000)
    L = _lib.lib()
    s = torch.cuda.current_stream().cuda_stream
    x = torch.ones(8192, device="cuda")
    y = torch.empty_like(x)
    _lib.check(L.rq_tp_allreduce_f32(ctx.handle, x.data_ptr(), y.data_ptr(), 8192, s))
    torch.cuda.synchronize()
    _lib.check(L.rq_tp_status(ctx.handle))
    result = {"first": float(y[0].item())}
    if rank == 0:
        _lib.check(L.rq_tp_allreduce_f32(ctx.handle, x.data_ptr(), y.data_ptr(), 8192, s))
        torch.cuda.synchronize()
        result["rc"] = L.rq_tp_status(ctx.handle)
        result["msg"] = _lib.last_error()
    dist.barrier()
    np.save(os.path.join(out_dir, f"to{rank}.npy"), np.array([result], dtype=object), allow_pickle=True)
    tpmod.finalize(ctx)
    dist.destroy_process_group()


def test_peer_allreduce_wait_gives_up_when_a_rank_skips(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_timeout_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    r0 = np.load(tmp_path / "to0.npy", allow_pickle=True)[0]
    r1 = np.load(tmp_path / "to1.npy", allow_pickle=True)[0]
    assert r0["first"] == 2.0 and r1["first"] == 2.0
    assert r0["rc"] == 5 and "did not signal" in r0["msg"]  # RQ_ERR_TIMEOUT


def _lonely_init(q):
    import ctypes
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from rustyllm_b200 import Context
    from rustyllm_b200 import _lib
    ctx = Context.get(0)
    L = _lib.lib()
    uid = ctypes.create_string_buffer(256)
    _lib.check(L.rq_tp_unique_id(uid, 256))
    rc = L.rq_tp_init(ctx.handle, 2, 0, uid, 3000)
    q.put((rc, _lib.last_error()))


def test_tp_init_times_out_when_a_rank_never_joins():
    """rq_tp_init on rank 0 of 2 while rank 1 never calls: the bounded
    initialisation returns RQ_ERR_TIMEOUT (communicator aborted), no hang.
    Host-side only; the child process is bounded by a join timeout."""
    import multiprocessing as mpc

    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = mpc.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_init, args=(q,))
    p.start()
    p.join(timeout=120)
    if p.is_alive():
        p.kill()
        pytest.fail("rq_tp_init did not return")
    rc, msg = q.get(timeout=5)
    assert rc == 5 and "no progress" in msg
