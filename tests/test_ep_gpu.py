"""Two-GPU expert parallelism of the sparse-MoE layer (rq_moe_forward_ep):
expert e on rank e % 2, each rank routes its own tokens, rows travel to their
experts' ranks and back through NCCL all-to-alls.  Every rank's outputs and
routing equal the single-GPU layer's on the same tokens bit for bit, also
with uneven and empty token counts.  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

E, H, F = 8, 512, 1024
SPLITS = [(0, 7, 7, 40), (7, 40, 0, 0)]  # per rank: forward 1 token range, forward 2 token range


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _layer(seed=21):
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    wr = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    blocks = []
    for _ in range(E):
        blocks.append(tuple(O.quantize(12, (rng.standard_normal((o, i)) * 0.02).astype(np.float32))
                            for o, i in ((F, H), (H, F), (F, H))))
    x = np.random.default_rng(seed + 1).standard_normal((40, H)).astype(np.float32)
    return wr, blocks, x


def _upload(ctx, blocks, owned):
    from rustyllm_b200 import QWeight
    out = []
    for e, (b1, b2, b3) in enumerate(blocks):
        if not owned(e):
            out.append(None)
            continue
        out.append((QWeight.upload(ctx, 12, b1, F, H), QWeight.upload(ctx, 12, b2, H, F),
                    QWeight.upload(ctx, 12, b3, F, H)))
    return out


def _ep_rank(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from rustyllm_b200 import Context
    from rustyllm_b200 import tp as tpmod
    from rustyllm_b200.mixtral import SparseMoe
    ctx = Context.get(rank)
    tpmod.init_from_torch(ctx, timeout_ms=60000)
    wr, blocks, x = _layer()
    experts = _upload(ctx, blocks, lambda e: e % world == rank)
    moe = SparseMoe(wr, experts, top_k=2, device=rank, expert_parallel=True)
    a0, a1, b0, b1 = SPLITS[rank]
    for tag, (lo, hi) in (("a", (a0, a1)), ("b", (b0, b1))):
        y, ids, perm = moe.forward_with_routing(torch.from_numpy(x[lo:hi].copy()).cuda(rank))
        np.save(os.path.join(out_dir, f"{tag}{rank}_y.npy"), y.cpu().numpy())
        np.save(os.path.join(out_dir, f"{tag}{rank}_ids.npy"), ids)
    moe.close()
    tpmod.finalize(ctx)
    dist.destroy_process_group()


def test_ep2_moe_matches_single_gpu(tmp_path, oracle):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from rustyllm_b200 import Context
    from rustyllm_b200.mixtral import SparseMoe
    wr, blocks, x = _layer()
    ctx = Context.get(0)
    moe = SparseMoe(wr, _upload(ctx, blocks, lambda e: True), top_k=2)
    mp.spawn(_ep_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for rank in range(2):
        a0, a1, b0, b1 = SPLITS[rank]
        for tag, (lo, hi) in (("a", (a0, a1)), ("b", (b0, b1))):
            y = np.load(tmp_path / f"{tag}{rank}_y.npy")
            ids = np.load(tmp_path / f"{tag}{rank}_ids.npy")
            if hi == lo:
                assert y.shape[0] == 0
                continue
            y1, ids1, _ = moe.forward_with_routing(x[lo:hi])
            assert np.array_equal(ids, ids1)
            assert np.array_equal(y.view(np.uint32), y1.view(np.uint32))
            y_ref, ids_ref, _, _ = oracle.moe_forward(x[lo:hi], wr, 12, [b[0] for b in blocks],
                                                      [b[2] for b in blocks], [b[1] for b in blocks], F, k=2)
            assert np.array_equal(ids, ids_ref)
            err = np.linalg.norm(y.astype(np.float64) - y_ref) / np.linalg.norm(y_ref)
            assert err <= 1e-4
