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


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_rank(rank, world, port, out_dir, mode="p2p"):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    if mode == "nccl":
        os.environ["RQ_TP_ALLREDUCE"] = "nccl"
    if mode == "unfused":
        os.environ["RQ_TP_FUSED"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from rustyllm_b200 import Context
    from rustyllm_b200 import tp as tpmod
    from rustyllm_b200.llama import random_model
    ctx = Context.get(rank)
    tpmod.init_from_torch(ctx, timeout_ms=60000)
    model, _ = random_model(CFG, 12, seed=11, device=rank, tp=(world, rank))
    prompt = np.random.default_rng(4).integers(0, CFG["vocab"], size=16).astype(np.int32)
    toks = model.generate(prompt, 12)
    np.save(os.path.join(out_dir, f"tp{mode}{rank}.npy"), np.array(toks))
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
            assert np.load(tmp_path / f"tp{mode}{r}.npy").tolist() == want


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
