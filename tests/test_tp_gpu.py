"""Two-GPU tensor parallelism of the Llama decode loop: greedy tokens of the
TP=2 model (column/row-parallel shards, NCCL all-reduces, vocab-parallel
argmax) equal the single-GPU model's.  Skipped with fewer than two GPUs."""
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


def _tp_rank(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
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
    np.save(os.path.join(out_dir, f"tp{rank}.npy"), np.array(toks))
    model.close()
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
    mp.spawn(_tp_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        assert np.load(tmp_path / f"tp{r}.npy").tolist() == want
