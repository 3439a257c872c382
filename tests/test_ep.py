"""Expert-parallel dispatch and combine on CPU with world-size-2 gloo ranks:
each rank routes its own tokens with the oracle, sends every token row to
the rank owning its expert (e % world), the owners run the experts, the rows
come back and each rank combines in ascending expert order.  The result
equals the single-process oracle layer on the same tokens (routing bit for
bit, outputs to 1e-6), also with a rank that holds no tokens."""
import os
import socket

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp

E, H, F, K = 8, 256, 512, 2


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def layer():
    from oracle import oracle as O
    rng = np.random.default_rng(3)
    wr = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    w = [[O.quantize(12, (rng.standard_normal((o, i)) * 0.02).astype(np.float32)) for o, i in ((F, H), (F, H), (H, F))]
         for _ in range(E)]
    x = np.random.default_rng(4).standard_normal((19, H)).astype(np.float32)
    return wr, w, x


def expert(O, w, rows):
    g = O.linear_threaded(12, w[0], F, H, rows)
    u = O.linear_threaded(12, w[1], F, H, rows)
    h = (g / (1.0 + np.exp(-g.astype(np.float64))).astype(np.float32) * u).astype(np.float32)
    return O.linear_threaded(12, w[2], H, F, h)


def _rank(rank, world, port, out_dir, splits):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from oracle import oracle as O
    wr, w, x = layer()
    lo, hi = splits[rank]
    xl = x[lo:hi]
    T = xl.shape[0]
    if T:
        ids, wts = O.route_topk(O.router_logits(xl, wr), K)
        offs, perm, sw = O.permute(ids, wts, E)
    else:
        ids, perm, offs = np.zeros((0, K), np.int32), np.zeros(0, np.int32), np.zeros(E + 1, np.int32)
    # dispatch: rows of expert e go to rank e % world, in expert order
    out = {d: [] for d in range(world)}
    for e in range(E):
        rows = [int(t) for t in perm[offs[e]:offs[e + 1]]] if T else []
        out[e % world].append((e, xl[rows] if rows else np.zeros((0, H), np.float32)))
    got = [None] * world
    dist.all_gather_object(got, out)
    # owners run their experts on the rows of every source rank
    results = {}
    for src in range(world):
        for e, rows in got[src][rank]:
            results[(src, e)] = expert(O, w[e], rows) if len(rows) else np.zeros((0, H), np.float32)
    back = [None] * world
    dist.all_gather_object(back, results)
    # combine this rank's tokens in ascending expert order
    y = np.zeros((T, H), np.float32)
    for e in range(E):
        o = back[e % world][(rank, e)]
        for i, t in enumerate(perm[offs[e]:offs[e + 1]] if T else []):
            wv = sw[offs[e] + i]
            y[t] = y[t] + o[i] * wv
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    np.save(os.path.join(out_dir, f"ids{rank}.npy"), ids)
    dist.destroy_process_group()


def test_ep_dispatch_combine_matches_oracle(tmp_path, oracle):
    wr, w, x = layer()
    for splits in ([(0, 6), (6, 19)], [(0, 19), (19, 19)]):
        mp.spawn(_rank, args=(2, free_port(), str(tmp_path), splits), nprocs=2, join=True)
        for rank, (lo, hi) in enumerate(splits):
            y = np.load(tmp_path / f"y{rank}.npy")
            ids = np.load(tmp_path / f"ids{rank}.npy")
            if hi == lo:
                assert y.shape == (0, H)
                continue
            y_ref, ids_ref, _, _ = oracle.moe_forward(x[lo:hi], wr, 12, [a[0] for a in w], [a[1] for a in w],
                                                      [a[2] for a in w], F, k=K)
            assert np.array_equal(ids, ids_ref)
            err = np.linalg.norm(y.astype(np.float64) - y_ref) / np.linalg.norm(y_ref)
            assert err <= 1e-6
