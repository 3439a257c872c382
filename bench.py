#!/usr/bin/env python
"""Benchmark: Q4_K matvec (M=1) at Llama-2-70B layer shapes on B200.

A step is one pass of the decode hot path over one 70B layer's seven
quantized linears (q, k, v, o: 8192->8192/1024/1024/8192; gate, up:
8192->28672; down: 28672->8192) through librq's public entry points with
device-resident activations, grouped as a decoder issues them: q/k/v in one
rq_linear_batch call on their shared x, o, gate/up in one batch call, down.  Weights are random
N(0, 0.02) f32 quantized to Q4_K on the device; x ~ N(0, 1).  Steps rotate
over 4 distinct layer copies (1.93 GB > 126 MB L2), so every weight byte
comes from HBM.  value = algorithmic bytes (weights + x + y) per step / time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

With --gpus N > 1 (under torchrun) every rank runs the same workload on its
own GPU (independent replicas, weak scaling): the layer matvecs have no
cross-GPU exchange when each GPU decodes its own stream.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# Llama-2-70B layer shapes (examples/bench_q4_kernel.rs:11-19): (name, in, out)
SHAPES = [("q_proj", 8192, 8192), ("k_proj", 8192, 1024), ("v_proj", 8192, 1024),
          ("o_proj", 8192, 8192), ("gate_proj", 8192, 28672), ("up_proj", 8192, 28672),
          ("down_proj", 28672, 8192)]
Q4_K = 12
Q4K_BYTES = lambda n_in, n_out: n_out * (n_in // 256) * 144  # noqa: E731
N_COPIES = 4
METRIC = "Q4_K matvec HBM GB/s at Llama-2-70B layer shapes (M=1)"
WORKLOAD = ("Q4_K matvec M=1 over one Llama-2-70B layer's 7 linears "
            "(q,k,v,o 8192->8192/1024/1024/8192; gate,up 8192->28672; down 28672->8192)")


def step_bytes() -> int:
    return sum(Q4K_BYTES(i, o) + 4 * (i + o) for _, i, o in SHAPES)


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.rows: list[list[str]] = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            if len(r) < 9:
                continue
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_baseline(blocks: dict, seconds: float = 6.0) -> dict:
    """The oracle's threaded CPU restatement over the same seven shapes
    (one layer), all host cores; bounded to ~`seconds` of work."""
    from oracle import oracle as O
    nthreads = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    xs = {n: rng.standard_normal((1, i)).astype(np.float32) for n, i, _ in SHAPES}
    ys = {n: np.empty((1, o), np.float32) for n, _, o in SHAPES}
    O.lib()
    passes, t0 = 0, time.perf_counter()
    while True:
        for n, i, o in SHAPES:
            O.linear_threaded(Q4_K, blocks[n], o, i, xs[n], nthreads=nthreads, y=ys[n])
        passes += 1
        el = time.perf_counter() - t0
        if el >= seconds or passes >= 200:
            break
    gbs = step_bytes() * passes / el / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
            "sample": f"{passes} passes over the 7 Q4_K layer shapes (one layer copy), "
                      f"{el:.1f} s, oracle rqo_linear_threaded"}


def host_blocks_for_cpu(seed: int = 1234) -> dict:
    """Seeded Q4_K blocks of the seven shapes for the CPU-only reference arm,
    quantized by the oracle (no GPU needed)."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    out = {}
    for n, i, o in SHAPES:
        w = (rng.standard_normal((o, i), dtype=np.float32) * np.float32(0.02))
        out[n] = O.quantize(Q4_K, w)
    return out


def run_reference(args) -> None:
    world, rank, _ = dist_env()
    if rank != 0:
        return
    blocks = host_blocks_for_cpu()
    from oracle import oracle as O
    nthreads = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    xs = {n: rng.standard_normal((1, i)).astype(np.float32) for n, i, _ in SHAPES}
    ys = {n: np.empty((1, o), np.float32) for n, _, o in SHAPES}

    def one_step():
        for n, i, o in SHAPES:
            O.linear_threaded(Q4_K, blocks[n], o, i, xs[n], nthreads=nthreads, y=ys[n])

    for _ in range(args.warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    el = time.perf_counter() - t0
    ms = el / args.steps * 1e3
    gbs = step_bytes() / (ms / 1e3) / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: W ~ N(0,0.02) f32 quantized to Q4_K (seeded), x ~ N(0,1)",
        "config": {"workload": WORKLOAD, "l2": "CPU path", "batch_m": 1},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": nthreads, "kind": "port",
                         "sample": f"{args.steps} timed passes over the 7 shapes, "
                                   "oracle rqo_linear_threaded (dequant-fused f32, "
                                   "q4_kernel.rs:207-243 chunking)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


Q4_0, Q3_K = 2, 11
Q3K_BYTES = lambda n_in, n_out: n_out * (n_in // 256) * 110  # noqa: E731
Q40_BYTES = lambda n_in, n_out: n_out * (n_in // 32) * 18  # noqa: E731


def other_formats(L, ctx, stream, timed, capture, dev, g) -> dict:
    """Config 1: the 4096x4096 Q4_0 matvec (M=1) over 16 rotating copies
    (151 MB > L2); config 2's Q3_K sweep and the same sweep in Q8_0, Q6_K,
    Q5_K and Q2_K:
    the seven 70B shapes, each over 4 rotating copies.  GB/s = GGML weight
    bytes + 4 (in + out) per call."""
    import torch
    from rustyllm_b200 import QWeight
    from rustyllm_b200._lib import check
    res = {}

    def sweep(qtype, shapes, copies, nbytes):
        out = {}
        for name, i, o in shapes:
            ws = []
            for _ in range(copies):
                wf = torch.randn(o, i, device=dev, generator=g) * 0.02
                ws.append(QWeight.quantize(ctx, qtype, wf))
                del wf
            x = torch.randn(1, i, device=dev, generator=g)
            y = torch.empty(1, o, device=dev)

            def run(st, ws=ws, x=x, y=y):
                for w in ws:
                    check(L.rq_linear(ctx.handle, w.handle, x.data_ptr(), y.data_ptr(), 1, st))
            with torch.cuda.stream(stream):
                run(stream.cuda_stream)
            stream.synchronize()
            gr = capture(run)
            with torch.cuda.stream(stream):
                gr.replay()
            reps = 10
            ms = timed(lambda r: gr.replay(), reps) / (reps * copies)
            out[name] = round((nbytes(i, o) + 4 * (i + o)) / (ms / 1e3) / 1e9, 1)
            del gr
            for w in ws:
                w.free()
        return out

    res["q4_0_4096x4096_gbs"] = sweep(Q4_0, [("q4_0", 4096, 4096)], 16, Q40_BYTES)["q4_0"]
    res["q3_k_per_shape_gbs"] = sweep(Q3_K, SHAPES, 4, Q3K_BYTES)
    # the other formats of the reference's quantizer (src/quantize.rs:29-37)
    res["q8_0_per_shape_gbs"] = sweep(8, SHAPES, 4, lambda i, o: o * (i // 32) * 34)
    res["q6_k_per_shape_gbs"] = sweep(14, SHAPES, 4, lambda i, o: o * (i // 256) * 210)
    res["q5_k_per_shape_gbs"] = sweep(13, SHAPES, 4, lambda i, o: o * (i // 256) * 176)
    res["q2_k_per_shape_gbs"] = sweep(10, SHAPES, 4, lambda i, o: o * (i // 256) * 84)
    res["note"] = ("single rq_linear calls (activation staging + M=1 pipeline), graph-replayed over "
                   "rotating weight copies larger than L2")
    return res


SMALL_M = (2, 3, 4, 8, 16, 24, 128, 512)


def small_m_sweep(L, ctx, weights, stream, timed, capture, dev, g) -> dict:
    """Small-M Q4_K matmul at the seven 70B layer shapes (M = 2, 3, 4, 8
    for speculative verify; 16, 24, 128, 512 for prefill): one rq_linear
    call per linear with [M, in] device activations, graph-replayed over the
    rotating layer copies.  GB/s = (Q4_K weight bytes + 4 M (in + out)) per
    layer / time, weight bytes counted once; TFLOP/s = 2 M sum(in * out) /
    time."""
    import torch
    from rustyllm_b200._lib import check
    res = {}
    for M in SMALL_M:
        xs = [torch.randn(M, i, device=dev, generator=g) for _, i, _ in SHAPES]
        ys = [torch.empty(M, o, device=dev) for _, _, o in SHAPES]

        def layer(c, st, xs=xs, ys=ys, M=M):
            for k in range(len(SHAPES)):
                check(L.rq_linear(ctx.handle, weights[c][k].handle, xs[k].data_ptr(), ys[k].data_ptr(),
                                  M, st))

        with torch.cuda.stream(stream):
            for c in range(N_COPIES):
                layer(c, stream.cuda_stream)
        stream.synchronize()
        gr = capture(lambda st: [layer(c, st) for c in range(N_COPIES)])
        with torch.cuda.stream(stream):
            gr.replay()
        reps = 10
        ms = timed(lambda r: gr.replay(), reps) / (reps * N_COPIES)
        nbytes = sum(Q4K_BYTES(i, o) + 4 * M * (i + o) for _, i, o in SHAPES)
        flops = 2 * M * sum(i * o for _, i, o in SHAPES)
        res[str(M)] = {"ms_per_layer": round(ms, 4), "gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
                       "tflops": round(flops / (ms / 1e3) / 1e12, 1),
                       "tok_per_s_layer_equiv": round(M / (ms / 1e3), 1)}
        del gr
    res["note"] = ("7 rq_linear calls per layer, 4 rotating layer copies. M <= 3: activation staging + "
                   "one M=1 pipeline pass per row; M = 4..23: f16 hi/lo staging + the mma.sync "
                   "tensor-core kernel, weights read once per 8-row tile; M >= 24: the tcgen05 kernel "
                   "(exact sc*q weights in TMEM, 128 rows x up to 112 tokens per tile)")
    return res


MIXTRAL = dict(E=8, H=4096, F=14336, k=2)
MOE_T = (1, 16, 512)


def moe_sweep(device: int, seed: int = 4321) -> dict:
    """Mixtral-8x7B sparse-MoE layer: router [8, 4096] f32 N(0, 0.02), 8
    experts of Q4_K SwiGLU weights (4096 -> 14336 -> 4096) quantized on the
    device from N(0, 0.02), hidden states N(0, 1) for T = 1, 16, 512 tokens,
    device-resident.  One forward = route, permute, expert products,
    combine (with its one host sync after routing).  GB/s counts the Q4_K
    bytes of the experts the tokens touch, once; T=512 also reports
    TFLOP/s of the 2*T*k*3*H*F expert flops."""
    import torch
    from rustyllm_b200 import Context, QWeight
    from rustyllm_b200.mixtral import SparseMoe
    E, H, F, k = MIXTRAL["E"], MIXTRAL["H"], MIXTRAL["F"], MIXTRAL["k"]
    dev = torch.device("cuda", device)
    ctx = Context.get(device)
    g = torch.Generator(device=dev).manual_seed(seed)
    router = (torch.randn(E, H, device=dev, generator=g) * 0.02).cpu().numpy()
    experts = []
    for _ in range(E):
        trip = []
        for o, i in ((F, H), (H, F), (F, H)):
            wf = torch.randn(o, i, device=dev, generator=g) * 0.02
            trip.append(QWeight.quantize(ctx, Q4_K, wf))
            del wf
        experts.append(tuple(trip))
    moe = SparseMoe(router, experts, top_k=k, device=device)
    mat_bytes = Q4K_BYTES(H, F)
    res = {}
    for T in MOE_T:
        x = torch.randn(T, H, device=dev, generator=g)
        _, ids, _ = moe.forward_with_routing(x)
        touched = len(set(ids.reshape(-1).tolist()))
        for _ in range(2):
            moe.forward(x)
        torch.cuda.synchronize()
        reps = 20 if T < 512 else 5
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            moe.forward(x)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        r = {"ms": round(ms, 4), "tok_per_s": round(T / (ms / 1e3), 1), "experts_touched": touched,
             "weight_gbs": round(touched * 3 * mat_bytes / (ms / 1e3) / 1e9, 1)}
        if T == 512:
            r["tflops"] = round(2 * T * k * 3 * H * F / (ms / 1e3) / 1e12, 2)
        res[str(T)] = r
    res["config"] = "Mixtral-8x7B MoE layer: E=8, top-2, H=4096, F=14336, Q4_K experts, 1 GPU"
    moe.close()
    for trip in experts:
        for w in trip:
            w.free()
    return res


def moe_ep_sweep(device: int, pg, seed: int = 4321) -> dict:
    """The Mixtral layer expert-parallel over the ranks (rq_moe_forward_ep):
    expert e on rank e % world, every rank with its own T tokens (weak
    scaling), NCCL all-to-all dispatch and return.  tok/s = world * T / the
    slowest rank's time per forward."""
    import torch
    from rustyllm_b200 import Context, QWeight
    from rustyllm_b200 import tp as tpmod
    from rustyllm_b200.mixtral import SparseMoe
    E, H, F, k = MIXTRAL["E"], MIXTRAL["H"], MIXTRAL["F"], MIXTRAL["k"]
    dev = torch.device("cuda", device)
    ctx = Context.get(device)
    world, rank = tpmod.init_from_torch(ctx)
    g = torch.Generator(device=dev).manual_seed(seed)
    router = (torch.randn(E, H, device=dev, generator=g) * 0.02).cpu().numpy()
    experts = []
    for e in range(E):
        ge = torch.Generator(device=dev).manual_seed(seed + 1 + e)
        if e % world != rank:
            experts.append(None)
            continue
        trip = []
        for o, i in ((F, H), (H, F), (F, H)):
            wf = torch.randn(o, i, device=dev, generator=ge) * 0.02
            trip.append(QWeight.quantize(ctx, Q4_K, wf))
            del wf
        experts.append(tuple(trip))
    moe = SparseMoe(router, experts, top_k=k, device=device, expert_parallel=True)
    res = {}
    for T in MOE_T:
        x = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(99 + rank))
        for _ in range(2):
            moe.forward(x)
        torch.cuda.synchronize()
        pg.barrier()
        reps = 20 if T < 512 else 5
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            moe.forward(x)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
        res[str(T)] = {"ms": round(ms, 4), "tokens_per_rank": T, "tok_per_s": round(world * T / (ms / 1e3), 1)}
    res["config"] = (f"Mixtral-8x7B MoE layer expert-parallel over {world} GPUs (expert e on rank e % {world}), "
                     "T tokens per rank, NCCL all-to-all")
    moe.close()
    for trip in experts:
        if trip:
            for w in trip:
                w.free()
    tpmod.finalize(ctx)
    torch.cuda.empty_cache()
    return res


LLAMA70B = dict(hidden=8192, intermediate=28672, n_heads=64, n_kv_heads=8, head_dim=128,
                n_layers=80, vocab=32000, max_seq=64, max_batch_tokens=32, rms_eps=1e-5,
                rope_theta=10000.0)


def decode_70b(device: int, new_tokens: int = 16, prompt_len: int = 20, pg=None,
               n_layers: int | None = None) -> dict:
    """Config 5: the full 80-layer Llama-2-70B shape (Platypus2-70B), random
    N(0, 0.02) weights quantized to Q4_K and resident on the GPUs, F16
    embedding / lm_head; 20 seeded uniform prompt ids, greedy decode of 16
    tokens.  Decode steps are device-side and replayed from one CUDA graph.
    Under torch.distributed the model is tensor-parallel over the ranks
    (column/row-parallel linears joined by NCCL all-reduces over NVLink)."""
    import torch
    from rustyllm_b200 import Context
    from rustyllm_b200._lib import check, lib
    from rustyllm_b200.llama import random_model
    cfg = dict(LLAMA70B)
    if n_layers:
        cfg["n_layers"] = n_layers
    world, rank = 1, 0
    if pg is not None:
        from rustyllm_b200 import tp as tpmod
        world, rank = tpmod.init_from_torch(Context.get(device))
    t0 = time.perf_counter()
    model, _ = random_model(cfg, Q4_K, seed=7070, device=device, tp=(world, rank))
    build_s = time.perf_counter() - t0
    prompt = np.random.default_rng(20).integers(0, cfg["vocab"], size=prompt_len).astype(np.int32)
    L = lib()
    stream = torch.cuda.Stream(device=device)
    # warm-up: one prompt pass and one step (kernel attributes), then capture
    model.forward(prompt, 0, want_logits=False)
    model.decode_step(stream.cuda_stream)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        model.decode_step(torch.cuda.current_stream().cuda_stream)
    # timed generate: prompt forward + (new_tokens - 1) graph-replayed steps
    check(L.rq_llama_reset_tokens(model.handle))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    model.forward(prompt, 0, want_logits=False)
    prefill_s = time.perf_counter() - t0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(new_tokens - 1):
            g.replay()
        e1.record(stream)
    stream.synchronize()
    gen_s = time.perf_counter() - t0
    step_ms = e0.elapsed_time(e1) / (new_tokens - 1)
    if pg is not None:  # the slowest rank sets the pace
        t = torch.tensor([step_ms, gen_s, prefill_s], device=f"cuda:{device}")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        step_ms, gen_s, prefill_s = (float(v) for v in t.tolist())
    toks, pos = model.tokens()
    # speculative-decoding verify forwards (forward_all over K+1 tokens at
    # the current position, cache rolled back after each): their cost next
    # to one decode step sets the acceptance a draft model must reach
    verify_ms = {}
    for kp1 in (2, 5, 9):
        ids = np.array(toks[:kp1] + [0] * max(0, kp1 - len(toks)), dtype=np.int32)[:kp1]
        model.forward_all(ids, pos)
        model.truncate_caches(pos)
        torch.cuda.synchronize()
        reps = 5
        t1 = time.perf_counter()
        for _ in range(reps):
            model.forward_all(ids, pos)
            model.truncate_caches(pos)
        ms = (time.perf_counter() - t1) * 1e3 / reps
        if pg is not None:
            t = torch.tensor([ms], device=f"cuda:{device}")
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms = float(t.item())
        verify_ms[str(kp1)] = round(ms, 3)
    del g
    model.close()
    if pg is not None:
        from rustyllm_b200 import tp as tpmod
        tpmod.finalize(Context.get(device))
    torch.cuda.empty_cache()
    layer_bytes = sum(Q4K_BYTES(i, o) for (o, i) in [(8192, 8192), (1024, 8192), (1024, 8192),
                                                        (8192, 8192), (28672, 8192), (28672, 8192),
                                                        (8192, 28672)])
    tok_bytes = cfg["n_layers"] * layer_bytes + cfg["vocab"] * cfg["hidden"] * 2
    return {"config": f"Llama-2-70B shape, {cfg['n_layers']} layers, Q4_K resident, F16 lm_head, "
                      f"tensor-parallel over {world} GPU(s)",
            "tp": world,
            "prompt_tokens": prompt_len, "new_tokens": new_tokens,
            "decode_tok_s": round(1e3 / step_ms, 2), "ms_per_token": round(step_ms, 3),
            "prefill_ms": round(prefill_s * 1e3, 2),
            "generate_tok_s": round(new_tokens / gen_s, 2),
            "weight_bytes_per_token": tok_bytes,
            "decode_hbm_gbs": round(tok_bytes / (step_ms / 1e3) / 1e9, 1),
            "tokens": toks[:new_tokens], "final_position": pos,
            "verify_forward_ms": verify_ms,
            "verify_note": "rq_llama_forward_all over K+1 tokens (host call incl. argmax copy), "
                           "keys = K+1; a draft that gets accepted tokens cheaper than "
                           "decode ms_per_token * (accepted+1) - verify pays off",
            "model_build_s": round(build_s, 2)}


def run_gpu(args) -> None:
    import ctypes

    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
        pg = dist
    if args.only_decode:
        dec = decode_70b(local, pg=pg, n_layers=args.decode_layers)
        if rank == 0:
            print(json.dumps({"metric": "70B Q4_K greedy decode tok/s", "value": dec["decode_tok_s"],
                              "unit": "tok/s", "n_gpus": world, "decode_70b": dec}), flush=True)
        if pg is not None:
            pg.barrier()
            pg.destroy_process_group()
        return
    from rustyllm_b200 import Context, QWeight
    from rustyllm_b200._lib import check, lib
    L = lib()
    ctx = Context.get(local)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    weights = []  # [copy][shape] -> QWeight
    for c in range(N_COPIES):
        layer = []
        for n, i, o in SHAPES:
            wf = torch.randn(o, i, device=dev, generator=g) * 0.02
            layer.append(QWeight.quantize(ctx, Q4_K, wf))
            del wf
        weights.append(layer)
    torch.cuda.synchronize()
    # activations: q/k/v share one x, gate/up share one x (as QAttn / QMlp do)
    x_attn = torch.randn(1, 8192, device=dev, generator=g)
    x_o = torch.randn(1, 8192, device=dev, generator=g)
    x_mlp = torch.randn(1, 8192, device=dev, generator=g)
    x_down = torch.randn(1, 28672, device=dev, generator=g)
    xs = [x_attn, x_attn, x_attn, x_o, x_mlp, x_mlp, x_down]
    ys = [torch.empty(1, o, device=dev) for _, _, o in SHAPES]
    stream = torch.cuda.Stream(device=dev)
    arr = lambda vals: (ctypes.c_void_p * len(vals))(*vals)  # noqa: E731
    groups = [(0, 1, 2), (3,), (4, 5), (6,)]  # q/k/v batched, o, gate/up batched, down

    def launch_group(c, grp, st):
        if len(grp) == 1:
            k = grp[0]
            check(L.rq_linear(ctx.handle, weights[c][k].handle, xs[k].data_ptr(),
                              ys[k].data_ptr(), 1, st))
        else:
            check(L.rq_linear_batch(ctx.handle, len(grp),
                                    arr([weights[c][k].handle.value for k in grp]),
                                    arr([xs[k].data_ptr() for k in grp]),
                                    arr([ys[k].data_ptr() for k in grp]), st))

    def launch_layer(c, st):
        for grp in groups:
            launch_group(c, grp, st)

    def capture(fn):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=stream):
            fn(torch.cuda.current_stream().cuda_stream)
        return gr

    # warm the workspace and kernel attributes outside capture
    with torch.cuda.stream(stream):
        for c in range(N_COPIES):
            launch_layer(c, stream.cuda_stream)
            for k in range(len(SHAPES)):
                launch_group(c, (k,), stream.cuda_stream)
    stream.synchronize()
    graphs = [capture(lambda st, c=c: launch_layer(c, st)) for c in range(N_COPIES)]
    # per-shape single calls and the dominant launch (gate+up batched), each
    # over the rotating copies
    shape_graphs = [capture(lambda st, k=k: [launch_group(c, (k,), st) for c in range(N_COPIES)])
                    for k in range(len(SHAPES))]
    dom = capture(lambda st: [launch_group(c, (4, 5), st) for c in range(N_COPIES)])

    def timed(fn, reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for r in range(reps):
                fn(r)
            e1.record(stream)
        stream.synchronize()
        return e0.elapsed_time(e1)

    with torch.cuda.stream(stream):
        for s in range(max(args.warmup, 3)):
            graphs[s % N_COPIES].replay()
        for gr in shape_graphs + [dom]:
            gr.replay()
    stream.synchronize()

    def barrier():
        if pg is not None:
            pg.barrier()

    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    ms_total = timed(lambda s: graphs[s % N_COPIES].replay(), args.steps)
    reps = max(10, args.steps // 4)
    dom_ms = timed(lambda r: dom.replay(), reps) / (reps * N_COPIES)
    per_shape = {}
    for k, (n, i, o) in enumerate(SHAPES):
        t = timed(lambda r, k=k: shape_graphs[k].replay(), reps) / (reps * N_COPIES)
        per_shape[n] = round((Q4K_BYTES(i, o) + 4 * (i + o)) / (t / 1e3) / 1e9, 1)
    small_m = None
    if not args.no_small_m:
        small_m = small_m_sweep(L, ctx, weights, stream, timed, capture, dev, g)
    formats = None
    if not args.no_small_m:
        formats = other_formats(L, ctx, stream, timed, capture, dev, g)
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()

    ms_step = ms_total / args.steps
    if pg is not None:
        t = torch.tensor([ms_step], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms_step = float(t.item())

    # e2e: the seven linears through the public call with HOST buffers
    # (pinned), host->device of x and device->host of y inside the timed region
    xh = [torch.randn(1, i, generator=torch.Generator().manual_seed(7)).pin_memory()
          for _, i, _ in SHAPES]
    yh = [torch.empty(1, o).pin_memory() for _, _, o in SHAPES]

    def e2e_step(c):
        for k in range(len(SHAPES)):
            check(L.rq_linear(ctx.handle, weights[c][k].handle, xh[k].data_ptr(), yh[k].data_ptr(),
                              1, stream.cuda_stream))

    for c in range(3):
        e2e_step(c % N_COPIES)
    barrier()
    torch.cuda.synchronize()
    e2e_steps = max(5, min(args.steps, 50))
    t0 = time.perf_counter()
    for s in range(e2e_steps):
        e2e_step(s % N_COPIES)
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) / e2e_steps * 1e3
    if pg is not None:
        t = torch.tensor([e2e_ms], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_ms = float(t.item())

    sb = step_bytes()
    value = sb * world / (ms_step / 1e3) / 1e9
    e2e_val = sb * world / (e2e_ms / 1e3) / 1e9
    pk = peaks()
    dom_bytes = 2 * Q4K_BYTES(8192, 28672) + 4 * (8192 + 2 * 28672)
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        host = {n: weights[0][k].download() for k, (n, _, _) in enumerate(SHAPES)}
        cpu = cpu_baseline(host, seconds=args.cpu_seconds)
    moe = None
    if not args.no_moe:
        moe = moe_sweep(local) if world == 1 else moe_ep_sweep(local, pg)
    dec = None
    if not args.no_decode:
        del graphs, shape_graphs, dom
        graphs = shape_graphs = dom = None
        for layer in weights:
            for w in layer:
                w.free()
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        dec = decode_70b(local, pg=pg)
    if rank == 0:
        traffic = None
        tp = os.path.join(ROOT, "profiles", "traffic_q4k_gate_up.json")
        if os.path.exists(tp):
            with open(tp) as f:
                traffic = json.load(f).get("bytes_per_launch")
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8x3 dp4a + f32 (4-bit weights)",
            "data": "synthetic: W ~ N(0,0.02) f32 quantized to Q4_K on device (seeded), x ~ N(0,1)",
            "config": {"workload": WORKLOAD, "batch_m": 1, "weight_format": "GGML Q4_K",
                       "bytes_per_step": sb,
                       "launch_grouping": "q/k/v batched on their shared x, o, gate/up batched "
                                          "on their shared x, down (4 rq_linear[_batch] calls)",
                       "l2": f"inputs larger than L2: {N_COPIES} rotating layer copies, "
                             f"{N_COPIES * sb / 1e9:.2f} GB per rotation vs 126 MB L2",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "pct_of_hbm_peak": round(100 * value / world / pk["hbm_gbs"], 1),
                       "per_shape_single_call_gbs": per_shape},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                         "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                         "traffic": traffic,
                         "kernel": "rq_linear_batch gate+up 2x(8192->28672): xquant + mv_pipe, "
                                   f"peak {pk['source']}"},
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": sum(4 * i for _, i, _ in SHAPES),
                    "d2h_bytes_per_step": sum(4 * o for _, _, o in SHAPES)},
            "gpu_launches": args.steps * 2 * len(groups),
            "clocks": clk,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if dec is not None:
            line["decode_70b"] = dec
        if small_m is not None:
            line["small_m_q4k"] = small_m
        if moe is not None:
            line["mixtral_moe"] = moe
        if formats is not None:
            line["other_formats"] = formats
        print(json.dumps(line), flush=True)
    del graphs, shape_graphs, dom
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()


def run_case(name: str) -> None:
    """A few launches of one kernel for an ncu capture: 'pipe_gate_up' (the
    gate+up rq_linear_batch of one 70B layer, M=1), 'mm_gate_m8' (gate_proj
    8192 -> 28672 at M=8 on the mma.sync kernel), 'sk_gate_m16' (the same at
    M=16 on the split-K tcgen05 kernel) or 'tc_gate_m128' (M=128 on the tiled
    tcgen05 kernel).  Prints the per-call time measured
    without the profiler."""
    import ctypes

    import torch
    from rustyllm_b200 import Context, QWeight
    from rustyllm_b200._lib import check, lib
    L = lib()
    ctx = Context.get(0)
    g = torch.Generator(device="cuda").manual_seed(5)
    ws = [QWeight.quantize(ctx, Q4_K, torch.randn(28672, 8192, device="cuda", generator=g) * 0.02)
          for _ in range(2)]
    s = torch.cuda.current_stream().cuda_stream
    arr = lambda v: (ctypes.c_void_p * len(v))(*v)  # noqa: E731
    if name == "pipe_gate_up":
        x = torch.randn(1, 8192, device="cuda", generator=g)
        ys = [torch.empty(1, 28672, device="cuda") for _ in range(2)]

        def call():
            check(L.rq_linear_batch(ctx.handle, 2, arr([w.handle.value for w in ws]), arr([x.data_ptr()] * 2),
                                    arr([y.data_ptr() for y in ys]), s))
        nbytes = 2 * Q4K_BYTES(8192, 28672)
    else:
        M = {"mm_gate_m8": 8, "sk_gate_m16": 16}.get(name, 128)
        x = torch.randn(M, 8192, device="cuda", generator=g)
        y = torch.empty(M, 28672, device="cuda")

        def call():
            check(L.rq_linear(ctx.handle, ws[0].handle, x.data_ptr(), y.data_ptr(), M, s))
        nbytes = Q4K_BYTES(8192, 28672)
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        call()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 10
    out = {"case": name, "us_per_call": round(ms * 1e3, 2), "weight_gbs": round(nbytes / (ms / 1e3) / 1e9, 1)}
    if name in ("tc_gate_m128", "sk_gate_m16"):
        out["tflops"] = round(2 * M * 8192 * 28672 / (ms / 1e3) / 1e12, 1)
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=6.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the 80-layer 70B decode run")
    ap.add_argument("--only-decode", action="store_true", help="run only the 70B decode")
    ap.add_argument("--no-small-m", action="store_true", help="skip the small-M Q4_K matmul sweep")
    ap.add_argument("--no-moe", action="store_true", help="skip the Mixtral MoE layer sweep")
    ap.add_argument("--decode-layers", type=int, default=None,
                    help="layers of the decode model (default 80; fewer for profiling)")
    ap.add_argument("--case", choices=["pipe_gate_up", "mm_gate_m8", "sk_gate_m16", "tc_gate_m128"], default=None,
                    help="run a few launches of one kernel (for profiling) and exit")
    args = ap.parse_args()
    if args.case:
        run_case(args.case)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
