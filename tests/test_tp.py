"""Tensor-parallel host logic on CPU: the shard rule, and the row-parallel
all-reduce / column-parallel gather reproduced by world-size-2 gloo ranks on
the oracle; a rank that fails before the collective must surface as an
error on the other rank within the timeout, not a hang."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rustyllm_b200.tp import LINEAR_SPLIT, shard


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_blocks_equal_full_blocks(oracle):
    """Quantizing a shard gives exactly the blocks of the full matrix: the
    row-parallel split falls on super-block boundaries."""
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((64, 2048)) * 0.02).astype(np.float32)
    for qtype in (12, 11, 2):
        full = oracle.quantize(qtype, w)
        for world in (2, 4, 8):
            rb = full.shape[1] // world
            for r in range(world):
                col = oracle.quantize(qtype, shard("row", torch.from_numpy(w), world, r).numpy())
                assert np.array_equal(col, full[:, r * rb:(r + 1) * rb])
                row = oracle.quantize(qtype, shard("col", torch.from_numpy(w), world, r).numpy())
                assert np.array_equal(row, full[r * 64 // world:(r + 1) * 64 // world])
    assert LINEAR_SPLIT == ("col", "col", "col", "row", "col", "col", "row")


def _rank_main(rank, world, port, out_dir, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    from oracle import oracle as O
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 1024)).astype(np.float32)
    w = (rng.standard_normal((96, 1024)) * 0.02).astype(np.float32)
    try:
        if rank == fail_rank:
            raise RuntimeError("rank failed before the collective")
        # row-parallel: partial products over this rank's input columns
        ws = shard("row", torch.from_numpy(w), world, rank).numpy()
        n = 1024 // world
        part = O.matmul_ref(12, O.quantize(12, ws), 96, n, x[:, rank * n:(rank + 1) * n], acc64=True)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        # column-parallel: this rank's output rows, gathered
        wc = shard("col", torch.from_numpy(w), world, rank).numpy()
        yc = torch.from_numpy(O.matmul_ref(12, O.quantize(12, wc), 96 // world, 1024, x, acc64=True))
        gathered = [torch.empty_like(yc) for _ in range(world)]
        dist.all_gather(gathered, yc)
        full = O.matmul_ref(12, O.quantize(12, w), 96, 1024, x, acc64=True)
        np.save(os.path.join(out_dir, f"r{rank}.npy"),
                np.stack([t.numpy(), torch.cat(gathered, 1).numpy(), full]))
    except RuntimeError as e:
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(str(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_row_and_column_parallel_on_gloo_ranks(tmp_path):
    mp.spawn(_rank_main, args=(2, free_port(), str(tmp_path), -1), nprocs=2, join=True)
    for r in range(2):
        red, gat, full = np.load(tmp_path / f"r{r}.npy")
        np.testing.assert_allclose(red, full, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(gat, full, rtol=1e-6, atol=1e-7)


def test_failed_rank_surfaces_as_error(tmp_path):
    """Rank 1 fails before the all-reduce; rank 0 must get an error from the
    collective within the process-group timeout instead of hanging."""
    mp.spawn(_rank_main, args=(2, free_port(), str(tmp_path), 1), nprocs=2, join=True)
    assert (tmp_path / "err1.txt").exists()
    assert (tmp_path / "err0.txt").exists() or not (tmp_path / "r0.npy").exists()
