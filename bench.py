#!/usr/bin/env python
"""Benchmark: Q4_K matvec (M=1) at Llama-2-70B layer shapes on B200.

A step is one pass of the decode hot path over one 70B layer's seven
quantized linears (q, k, v, o: 8192->8192/1024/1024/8192; gate, up:
8192->28672; down: 28672->8192) through librq's public entry points with
device-resident activations, grouped as a decoder issues them: q/k/v in one
rq_linear_batch call on their shared x, o, gate/up in one batch call, down.
Weights are random N(0, 0.02) f32 quantized to Q4_K on the device; x ~
N(0, 1).  Steps rotate over 4 distinct layer copies (1.93 GB > 126 MB L2), so
every weight byte comes from HBM.  value = algorithmic bytes (weights + x +
y) of the full layer per step / time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

With --gpus N > 1 (under torchrun) the same layer runs tensor-parallel over
the N GPUs (strong scaling): q/k/v/gate/up are split by output rows, o/down
by input columns, and o/down end in an all-reduce over NVLink that runs
inside the matvec kernel (rq_linear_allreduce).  value = the full layer's
bytes / the slowest rank's time per step.  The line also carries the
tensor-parallel 80-layer 70B decode (config 5) and the expert-parallel
Mixtral layer at that N.

Beside each GPU figure at N = 1 sits the reference's CPU path, restated in
the oracle and timed on the host's cores (`cpu_baseline`), and the roofline
of the kernel that dominates it (`roofline`).
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
SPLIT = ("col", "col", "col", "row", "col", "col", "row")  # tensor-parallel split per linear
Q4_K, Q4_0, Q3_K = 12, 2, 11
Q4K_BYTES = lambda n_in, n_out: n_out * (n_in // 256) * 144  # noqa: E731
Q3K_BYTES = lambda n_in, n_out: n_out * (n_in // 256) * 110  # noqa: E731
Q40_BYTES = lambda n_in, n_out: n_out * (n_in // 32) * 18  # noqa: E731
N_COPIES = 4
METRIC = "Q4_K matvec HBM GB/s at Llama-2-70B layer shapes (M=1)"
WORKLOAD = ("Q4_K matvec M=1 over one Llama-2-70B layer's 7 linears "
            "(q,k,v,o 8192->8192/1024/1024/8192; gate,up 8192->28672; down 28672->8192)")


def step_bytes() -> int:
    return sum(Q4K_BYTES(i, o) + 4 * (i + o) for _, i, o in SHAPES)


def layer_weight_bytes() -> int:
    return sum(Q4K_BYTES(i, o) for _, i, o in SHAPES)


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def traffic(name: str):
    """Per-launch DRAM bytes of an ncu capture summarised under profiles/."""
    p = os.path.join(ROOT, "profiles", f"traffic_{name}.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("bytes_per_launch")
    return None


def roofline_hbm(nbytes: float, ms: float, pk: dict, kernel: str, traffic_name: str | None = None) -> dict:
    a = nbytes / (ms / 1e3) / 1e9
    return {"bound": "hbm", "achieved": round(a, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": round(a / pk["hbm_gbs"], 4), "traffic": traffic(traffic_name) if traffic_name else None,
            "kernel": kernel, "peak_source": pk["source"]}


def roofline_tensor(flops: float, ms: float, pk: dict, kernel: str, traffic_name: str | None = None) -> dict:
    a = flops / (ms / 1e3) / 1e12
    return {"bound": "tensor", "achieved": round(a, 1), "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(a / pk["bf16_tflops"], 4), "traffic": traffic(traffic_name) if traffic_name else None,
            "kernel": kernel, "peak_source": pk["source"] + " (bf16 dense, burst)"}


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


def nthreads_host() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def cpu_desc() -> str:
    """Host CPU model and NUMA layout, for the baselines' record."""
    model, nodes = "unknown", None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except Exception:
        pass
    try:
        nodes = len([d for d in os.listdir("/sys/devices/system/node") if d.startswith("node")])
    except Exception:
        pass
    return f"{model}; {nthreads_host()} usable threads; {nodes} NUMA node(s); threads not pinned"


def _timed_loop(fn, seconds: float, max_iters: int = 1000, warm: bool = True) -> tuple[float, int]:
    if warm:
        fn()  # page faults, thread start-up
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or n >= max_iters:
            return el / n, n


def cpu_layer_q4k(blocks: dict, seconds: float = 6.0) -> dict:
    """Config 2 on the CPU: the oracle's threaded restatement of the
    reference's path (q4_kernel.rs:207-243 chunking over a dequant-fused f32
    dot) over the seven shapes of one layer, all host cores."""
    from oracle import oracle as O
    nt = nthreads_host()
    rng = np.random.default_rng(1)
    xs = {n: rng.standard_normal((1, i)).astype(np.float32) for n, i, _ in SHAPES}
    ys = {n: np.empty((1, o), np.float32) for n, _, o in SHAPES}

    def one():
        for n, i, o in SHAPES:
            O.linear_threaded(Q4_K, blocks[n], o, i, xs[n], nthreads=nt, y=ys[n])

    t, n = _timed_loop(one, seconds, 200)
    return {"value": round(step_bytes() / t / 1e9, 3), "unit": "GB/s", "cores": nt, "kind": "port",
            "sample": f"{n} passes over the 7 Q4_K layer shapes (one layer copy), oracle rqo_linear_threaded "
                      f"(dequant-fused f32, q4_kernel.rs:207-243 chunking); {cpu_desc()}"}


def cpu_q4_0(blocks: np.ndarray, seconds: float = 2.0) -> dict:
    """Config 1 on the CPU: ParallelQ4Linear::forward (q4_kernel.rs:183-256)
    with the AVX2-order dot (:300-360), restated in the oracle."""
    from oracle import oracle as O
    nt = nthreads_host()
    x = np.random.default_rng(2).standard_normal((1, 4096)).astype(np.float32)
    y = np.empty((1, 4096), np.float32)
    t, n = _timed_loop(lambda: O.linear_threaded(Q4_0, blocks, 4096, 4096, x, nthreads=nt, y=y), seconds)
    nbytes = Q40_BYTES(4096, 4096) + 4 * (4096 + 4096)
    return {"value": round(nbytes / t / 1e9, 3), "unit": "GB/s", "cores": nt, "kind": "port",
            "sample": f"{n} calls of the 4096x4096 Q4_0 forward, oracle rqo_linear_threaded "
                      "(AVX2-order dot q4_kernel.rs:300-360, chunking :207-243)"}


def cpu_small_m(blocks: dict, ms_list=None) -> dict:
    """Config 3 on the CPU: the threaded restatement at each M over the
    seven shapes; at large M over a leading fraction f = min(1, 8/M) of each
    weight's rows, scaled by 1/f (the work per row is the same)."""
    from oracle import oracle as O
    nt = nthreads_host()
    rng = np.random.default_rng(3)
    out = {}
    for M in (ms_list or SMALL_M):
        f = min(1.0, 8.0 / M)
        xs = {n: rng.standard_normal((M, i)).astype(np.float32) for n, i, _ in SHAPES}
        rows = {n: max(1, int(o * f)) for n, _, o in SHAPES}

        def one():
            for n, i, o in SHAPES:
                O.linear_threaded(Q4_K, blocks[n][:rows[n]], rows[n], i, xs[n], nthreads=nt)

        t, _ = _timed_loop(one, 0.5, 3)
        frac = sum(rows[n] * i for n, i, _ in SHAPES) / sum(o * i for _, i, o in SHAPES)
        ms = t / frac * 1e3
        nbytes = sum(Q4K_BYTES(i, o) + 4 * M * (i + o) for _, i, o in SHAPES)
        out[str(M)] = {"ms_per_layer": round(ms, 2), "gbs": round(nbytes / (ms / 1e3) / 1e9, 3),
                       "tok_per_s_layer_equiv": round(M / (ms / 1e3), 2)}
    return {"value_by_M": out, "unit": "ms per layer", "cores": nt, "kind": "port",
            "sample": "oracle rqo_linear_threaded over the 7 shapes at each M; rows scaled by "
                      "f = min(1, 8/M) (M=512: 1/64 of each weight's rows), time / f"}


def cpu_moe_f16(router: np.ndarray, xs: dict, seconds_cap: float = 30.0) -> dict:
    """Config 4 on the CPU: the reference's own Mixtral layer
    (SparseMoe::forward, streaming_mixtral.rs:280-319, with ParallelLinear
    F16 gate and experts, parallel_linear.rs:191-295), restated in the
    oracle.  One expert's F16 weights (352 MB, far above the host caches)
    serve all eight experts; T = 512 is timed on its first 32 tokens."""
    from oracle import oracle as O
    nt = nthreads_host()
    H, F, E = MIXTRAL["H"], MIXTRAL["F"], MIXTRAL["E"]
    rng = np.random.default_rng(8)
    w1 = (rng.standard_normal((F, H), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    w3 = (rng.standard_normal((F, H), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    w2 = (rng.standard_normal((H, F), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    res = {}
    for T, x in xs.items():
        xt = x if T < 512 else x[:32]
        t, n = _timed_loop(lambda: O.moe_forward(xt, router, O.F16, [w1] * E, [w3] * E, [w2] * E, F,
                                                 k=MIXTRAL["k"], nthreads=nt), 1.0, 5, warm=T == 1)
        res[str(T)] = {"ms": round(t * 1e3 * (T / xt.shape[0]), 2),
                       "tok_per_s": round(xt.shape[0] / t, 2),
                       "sample": f"T={xt.shape[0]}" + (" of 512, ms scaled by 16" if T == 512 else "")}
    return {"value_by_T": res, "unit": "tok/s", "cores": nt, "kind": "port",
            "sample": "oracle rqo_moe_forward with F16 experts (ParallelLinear restatement, AVX2 lane order) and "
                      "the F16 gate; 8 experts share one F16 weight set"}


def cpu_decode(blocks7: list, head_f16: np.ndarray, n_layers: int, seconds: float = 3.0) -> dict:
    """Config 5 on the CPU, extrapolated: one layer's seven Q4_K linears at
    M = 1 (the threaded restatement) times the layer count, plus the F16
    lm_head through the ParallelLinear restatement (the reference's
    parallel-cpu F16 path).  Attention over <= 36 positions is negligible."""
    from oracle import oracle as O
    nt = nthreads_host()
    rng = np.random.default_rng(9)
    xs = [rng.standard_normal((1, i)).astype(np.float32) for _, i, _ in SHAPES]

    def layer():
        for k, (_, i, o) in enumerate(SHAPES):
            O.linear_threaded(Q4_K, blocks7[k], o, i, xs[k], nthreads=nt)

    tl, _ = _timed_loop(layer, seconds, 50)
    xh = rng.standard_normal((1, head_f16.shape[1])).astype(np.float32)
    th, _ = _timed_loop(lambda: O.parallel_linear_f16(head_f16, xh, nthreads=nt), 1.0, 20)
    ms = (n_layers * tl + th) * 1e3
    return {"value": round(1e3 / ms, 4), "unit": "tok/s", "cores": nt, "kind": "port",
            "ms_per_token": round(ms, 1),
            "sample": f"one 70B layer's 7 linears at M=1 ({tl * 1e3:.1f} ms, oracle rqo_linear_threaded) x "
                      f"{n_layers} + the 32000x8192 F16 lm_head ({th * 1e3:.1f} ms, ParallelLinear "
                      "restatement); extrapolated per token"}


def headline_config(world: int) -> dict:
    """The config of the headline line, shared by both arms (the reference
    arm replaces only the l2 field)."""
    par = "single GPU" if world == 1 else (
        f"tensor parallel x{world}: q/k/v/gate/up split by rows, o/down by columns + all-reduce "
        "(rq_linear_allreduce)")
    return {"workload": WORKLOAD, "batch_m": 1, "weight_format": "GGML Q4_K",
            "bytes_per_step": step_bytes(),
            "launch_grouping": "q/k/v batched on their shared x, o, gate/up batched on their shared x, down "
                               "(4 rq_linear[_batch|_allreduce] calls)",
            "l2": f"inputs larger than L2: {N_COPIES} rotating layer copies, "
                  f"{N_COPIES * step_bytes() / 1e9:.2f} GB per rotation vs 126 MB L2",
            "parallelism": par}


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
    """The reference arm: the reference's CPU path for this workload (the
    oracle's threaded restatement, all host cores), same metric and config.
    Under torchrun only rank 0 runs."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    blocks = host_blocks_for_cpu()
    from oracle import oracle as O
    nt = nthreads_host()
    rng = np.random.default_rng(1)
    xs = {n: rng.standard_normal((1, i)).astype(np.float32) for n, i, _ in SHAPES}
    ys = {n: np.empty((1, o), np.float32) for n, _, o in SHAPES}

    def one_step():
        for n, i, o in SHAPES:
            O.linear_threaded(Q4_K, blocks[n], o, i, xs[n], nthreads=nt, y=ys[n])

    for _ in range(args.warmup):
        one_step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_step()
    el = time.perf_counter() - t0
    ms = el / args.steps * 1e3
    gbs = step_bytes() / (ms / 1e3) / 1e9
    cfg = headline_config(world)
    cfg["l2"] = "CPU path: one layer copy (481 MB, far above the host caches)"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak" if world == 1 else "strong", "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: W ~ N(0,0.02) f32 quantized to Q4_K (seeded), x ~ N(0,1)",
        "config": cfg,
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": nt, "kind": "port",
                         "sample": f"{args.steps} timed passes over the 7 shapes, "
                                   "oracle rqo_linear_threaded (dequant-fused f32, "
                                   f"q4_kernel.rs:207-243 chunking); {cpu_desc()}"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def other_formats(L, ctx, stream, timed, capture, dev, g, pk, with_cpu: bool) -> dict:
    """Config 1: the 4096x4096 Q4_0 matvec (M=1) over 16 rotating copies
    (151 MB > L2); config 2's Q3_K sweep and the same sweep in Q8_0, Q6_K,
    Q5_K and Q2_K: the seven 70B shapes, each over 4 rotating copies.  GB/s =
    GGML weight bytes + 4 (in + out) per call; each format's roofline is its
    gate_proj call (the M=1 pipeline kernel)."""
    import torch
    from rustyllm_b200 import QWeight
    from rustyllm_b200._lib import check
    res = {}
    host0 = {}

    def sweep(qtype, shapes, copies, nbytes, keep_host=False):
        out = {}
        for name, i, o in shapes:
            ws = []
            for _ in range(copies):
                wf = torch.randn(o, i, device=dev, generator=g) * 0.02
                ws.append(QWeight.quantize(ctx, qtype, wf))
                del wf
            if keep_host:
                host0[name] = ws[0].download()
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
            out[name] = {"gbs": round((nbytes(i, o) + 4 * (i + o)) / (ms / 1e3) / 1e9, 1), "ms": ms}
            del gr
            for w in ws:
                w.free()
        return out

    def fmt(qtype, name, nb):
        r = sweep(qtype, SHAPES, 4, nb)
        gate = r["gate_proj"]
        res[f"{name}_per_shape_gbs"] = {k: v["gbs"] for k, v in r.items()}
        res[f"{name}_roofline"] = roofline_hbm(nb(8192, 28672) + 4 * (8192 + 28672), gate["ms"], pk,
                                               f"xquant + mv_pipe_kernel<{name.upper()}> gate_proj 8192->28672",
                                               f"{name}_gate" if name == "q3_k" else None)

    q40 = sweep(Q4_0, [("q4_0", 4096, 4096)], 16, Q40_BYTES, keep_host=with_cpu)["q4_0"]
    res["q4_0_4096x4096_gbs"] = q40["gbs"]
    res["q4_0_roofline"] = roofline_hbm(Q40_BYTES(4096, 4096) + 4 * 8192, q40["ms"], pk,
                                        "xquant + mv_pipe_kernel<Q4_0> 4096x4096 (9.4 MB: launch-latency bound)")
    if with_cpu:
        res["q4_0_cpu_baseline"] = cpu_q4_0(host0["q4_0"])
    res["q4_0_small_m"] = q40_small_m(L, ctx, stream, timed, capture, dev, g)
    fmt(Q3_K, "q3_k", Q3K_BYTES)
    res["q3_k_small_m"] = q3k_small_m(L, ctx, stream, timed, capture, dev, g, pk)
    # the other formats of the reference's quantizer (src/quantize.rs:29-37)
    fmt(8, "q8_0", lambda i, o: o * (i // 32) * 34)
    fmt(14, "q6_k", lambda i, o: o * (i // 256) * 210)
    fmt(13, "q5_k", lambda i, o: o * (i // 256) * 176)
    fmt(10, "q2_k", lambda i, o: o * (i // 256) * 84)
    res["note"] = ("single rq_linear calls (activation staging + M=1 pipeline), graph-replayed over "
                   "rotating weight copies larger than L2")
    return res


SMALL_M = (2, 3, 4, 8, 16, 24, 128, 512)
Q3K_SMALL_M = (2, 3, 4, 8, 16, 128)
Q40_SMALL_M = (1, 2, 3, 4, 8, 16)


def q40_small_m(L, ctx, stream, timed, capture, dev, g) -> dict:
    """The 4096x4096 Q4_0 linear (config 1's weight) at M rows: one
    rq_linear call, graph-replayed over 16 rotating copies (151 MB).
    M = 2..8 run the int8 tensor-core kernels in one weight pass, larger M
    one int8 launch per group of up to 8 rows.  GB/s counts the weight
    bytes once per call."""
    import torch
    from rustyllm_b200 import QWeight
    from rustyllm_b200._lib import check
    ws = []
    for _ in range(16):
        wf = torch.randn(4096, 4096, device=dev, generator=g) * 0.02
        ws.append(QWeight.quantize(ctx, Q4_0, wf))
        del wf
    res = {}
    for M in Q40_SMALL_M:
        x = torch.randn(M, 4096, device=dev, generator=g)
        y = torch.empty(M, 4096, device=dev)

        def run(st, x=x, y=y, M=M):
            for w in ws:
                check(L.rq_linear(ctx.handle, w.handle, x.data_ptr(), y.data_ptr(), M, st))
        with torch.cuda.stream(stream):
            run(stream.cuda_stream)
        stream.synchronize()
        gr = capture(run)
        with torch.cuda.stream(stream):
            gr.replay()
        reps = 10
        ms = timed(lambda r: gr.replay(), reps) / (reps * len(ws))
        res[str(M)] = {"us_per_call": round(ms * 1e3, 2),
                       "gbs": round((Q40_BYTES(4096, 4096) + 4 * M * 8192) / (ms / 1e3) / 1e9, 1)}
        del gr
    for w in ws:
        w.free()
    res["note"] = ("rq_linear on the 4096x4096 Q4_0 weight, 16 rotating copies; M=1 the pipeline, "
                   "M = 2..8 the int8 tensor-core kernels, larger M one int8 launch per group of up to 8 rows")
    return res


def q3k_small_m(L, ctx, stream, timed, capture, dev, g, pk) -> dict:
    """Q3_K matmul at the seven 70B layer shapes for a few M: one rq_linear
    call per linear, graph-replayed over 4 rotating layer copies (1.5 GB).
    M = 2..8 runs the int8 tensor-core kernels, larger M the tcgen05
    kernel, each in one weight pass.  GB/s counts the GGML weight bytes
    once."""
    import torch
    from rustyllm_b200 import QWeight
    from rustyllm_b200._lib import check
    layers = []
    for _ in range(N_COPIES):
        row = []
        for _, i, o in SHAPES:
            wf = torch.randn(o, i, device=dev, generator=g) * 0.02
            row.append(QWeight.quantize(ctx, Q3_K, wf))
            del wf
        layers.append(row)
    nbytes_w = sum(Q3K_BYTES(i, o) for _, i, o in SHAPES)
    res = {}
    for M in Q3K_SMALL_M:
        xs = [torch.randn(M, i, device=dev, generator=g) for _, i, _ in SHAPES]
        ys = [torch.empty(M, o, device=dev) for _, _, o in SHAPES]

        def layer(c, st, xs=xs, ys=ys, M=M):
            for k in range(len(SHAPES)):
                check(L.rq_linear(ctx.handle, layers[c][k].handle, xs[k].data_ptr(), ys[k].data_ptr(), M, st))

        with torch.cuda.stream(stream):
            for c in range(N_COPIES):
                layer(c, stream.cuda_stream)
        stream.synchronize()
        gr = capture(lambda st: [layer(c, st) for c in range(N_COPIES)])
        with torch.cuda.stream(stream):
            gr.replay()
        reps = 10
        ms = timed(lambda r: gr.replay(), reps) / (reps * N_COPIES)
        flops = 2 * M * sum(i * o for _, i, o in SHAPES)
        kern = ("xq2_stage + mm_i8 kernels<Q3_K> (int8 mma.sync k16, one weight pass)" if M <= 8 else
                "xh_stage + mm_tc_kernel<Q3_K> (tcgen05, one weight pass)")
        res[str(M)] = {"ms_per_layer": round(ms, 4),
                       "gbs": round((nbytes_w + 4 * M * sum(i + o for _, i, o in SHAPES)) / (ms / 1e3) / 1e9, 1),
                       "tflops": round(flops / (ms / 1e3) / 1e12, 1), "kernel": kern}
        del gr
    for row in layers:
        for w in row:
            w.free()
    res["note"] = ("7 rq_linear calls per 70B layer (Q3_K weights), 4 rotating layer copies; "
                   "ms per layer")
    return res


def small_m_sweep(L, ctx, weights, stream, timed, capture, dev, g, pk, host_blocks) -> dict:
    """Small-M Q4_K matmul at the seven 70B layer shapes (M = 2, 3, 4, 8
    for speculative verify; 16, 24, 128, 512 for prefill): one rq_linear
    call per linear with [M, in] device activations, graph-replayed over the
    rotating layer copies.  GB/s = (Q4_K weight bytes + 4 M (in + out)) per
    layer / time, weight bytes counted once; TFLOP/s = 2 M sum(in * out) /
    time.  Roofline per M: HBM up to M = 8, the tensor cores from 16."""
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
        kern = ("xq2_stage + mm_i8_kernel (int8 mma.sync, one weight pass; down_proj K split 4 ways)" if M == 2 else
                "xq2_stage + mm_i8x4_kernel (int8 mma.sync, B in TMEM, one weight pass; down_proj K split 4 ways)"
                if M <= 4 else
                "xq2_stage + mm_i8x8_kernel (int8 mma.sync, B in TMEM, one weight pass; down_proj K split 4 ways)"
                if M <= 8 else
                "xh_stage + mm_skinny_kernel (split-K tcgen05)" if M <= 16 else
                "xh_stage + mm_q4k_kernel (mma.sync)" if M < 24 else "xh_stage + mm_tc_kernel (tcgen05)")
        r = {"ms_per_layer": round(ms, 4), "gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
             "tflops": round(flops / (ms / 1e3) / 1e12, 1),
             "tok_per_s_layer_equiv": round(M / (ms / 1e3), 1)}
        r["roofline"] = (roofline_hbm(nbytes, ms, pk, kern + ", 7 linears of a layer") if M <= 8 else
                         roofline_tensor(flops, ms, pk, kern + ", 7 linears of a layer"))
        res[str(M)] = r
        del gr
    res["note"] = ("7 rq_linear calls per layer, 4 rotating layer copies. M = 2..8: 24-bit int8-plane "
                   "staging + the int8 mma.sync kernels, weights read once; M = 17..23: f16 hi/lo staging + the mma.sync "
                   "tensor-core kernel, weights read once per 8-row tile; M = 9..16: split-K tcgen05; "
                   "M >= 24: the tiled tcgen05 kernel (exact sc*q weights in TMEM)")
    if host_blocks is not None:
        res["cpu_baseline"] = cpu_small_m(host_blocks)
    return res


MIXTRAL = dict(E=8, H=4096, F=14336, k=2)
MOE_T = (1, 16, 512)


def moe_sweep(device: int, pk, with_cpu: bool, seed: int = 4321) -> dict:
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
    xs_host = {}
    for T in MOE_T:
        x = torch.randn(T, H, device=dev, generator=g)
        xs_host[T] = x.cpu().numpy()
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
        wb = touched * 3 * mat_bytes
        r = {"ms": round(ms, 4), "tok_per_s": round(T / (ms / 1e3), 1), "experts_touched": touched,
             "weight_gbs": round(wb / (ms / 1e3) / 1e9, 1)}
        flops = 2 * T * k * 3 * H * F
        if T == 512:
            r["tflops"] = round(flops / (ms / 1e3) / 1e12, 2)
            r["roofline"] = roofline_tensor(flops, ms, pk, "route + permute + expert tiles (mm_tc_kernel) + combine")
        else:
            what = ("router (stages x) + gate/up matvec of the routed slots (SwiGLU staging epilogue) + down "
                    "matvec (combine epilogue), planned on the device" if T < 4 else
                    "route + permute + expert products (M=1 pipeline / mma.sync) + combine, planned on the host")
            r["roofline"] = roofline_hbm(wb + 4 * T * H * 2, ms, pk, what, f"moe_t{T}")
        res[str(T)] = r
    res["config"] = "Mixtral-8x7B MoE layer: E=8, top-2, H=4096, F=14336, Q4_K experts, 1 GPU"
    moe.close()
    for trip in experts:
        for w in trip:
            w.free()
    if with_cpu:
        res["cpu_baseline"] = cpu_moe_f16(router, xs_host)
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
    world, rank = tpmod.world_rank(ctx)
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
    torch.cuda.empty_cache()
    return res


LLAMA70B = dict(hidden=8192, intermediate=28672, n_heads=64, n_kv_heads=8, head_dim=128,
                n_layers=80, vocab=32000, max_seq=64, max_batch_tokens=32, rms_eps=1e-5,
                rope_theta=10000.0)


def verify_decode(model, host: dict, cfg: dict, prompt: np.ndarray, toks: list) -> dict:
    """Replay the decode through the oracle, one layer at a time (the
    layer's Q4_K blocks downloaded from the device, run, dropped): the
    prompt plus the first 15 generated tokens teacher-forced, so position p's
    greedy token is the one decode step p emitted, with the arithmetic of
    the incremental step.  Also the top-1 / top-2 logit margin per step."""
    from oracle import oracle as O
    t0 = time.perf_counter()
    ref = O.OracleLlama(cfg, Q4_K)
    ref.set_embedding(host["embed"])
    ref.set_head(host["ln_f"], host["lm_head"])
    seq = np.concatenate([prompt, np.array(toks[:-1], np.int32)]).astype(np.int32)
    x = ref.embed(seq)
    layer0 = None
    for l in range(cfg["n_layers"]):
        blocks = [w.download() for w in model.layer_weights(l)]
        _, r1, r2 = host["layers"][l]
        ref.stream_layer(l, blocks, r1, r2, x, 0)
        if l == 0:
            layer0 = blocks
    logits, amax = ref.head(x)
    p0 = len(prompt) - 1
    want = amax[p0:].tolist()
    top2 = np.sort(logits[p0:], axis=1)[:, -2:]
    margins = (top2[:, 1] - top2[:, 0]).tolist()
    return {"tokens_match_oracle": want == list(toks), "oracle_tokens": want,
            "top1_top2_margins": [round(float(m), 5) for m in margins],
            "min_margin": round(float(min(margins)), 5),
            "logit_std": round(float(logits[p0:].std()), 4),
            "oracle_check_s": round(time.perf_counter() - t0, 1),
            "oracle_check_note": "oracle rqo_llama_layer per layer on the downloaded blocks, prompt + generated "
                                 "tokens teacher-forced (positions 19..34); logits of the F16 lm_head"}, layer0


def decode_70b(device: int, pk, new_tokens: int = 16, prompt_len: int = 20, pg=None,
               n_layers: int | None = None, verify: bool = True, with_cpu: bool = True) -> dict:
    """Config 5: the full 80-layer Llama-2-70B shape (Platypus2-70B), random
    N(0, 0.02) weights quantized to Q4_K and resident on the GPUs, F16
    embedding / lm_head; 20 seeded uniform prompt ids, greedy decode of 16
    tokens.  Decode steps are device-side and replayed from one CUDA graph.
    Under torch.distributed the model is tensor-parallel over the ranks
    (column/row-parallel linears joined by all-reduces over NVLink).  On one
    GPU the tokens are checked against the oracle."""
    import torch
    from rustyllm_b200 import Context
    from rustyllm_b200 import tp as tpmod
    from rustyllm_b200._lib import check, lib
    from rustyllm_b200.llama import random_model
    cfg = dict(LLAMA70B)
    if n_layers:
        cfg["n_layers"] = n_layers
    world, rank = tpmod.world_rank(Context.get(device))
    verify = verify and world == 1
    t0 = time.perf_counter()
    model, host = random_model(cfg, Q4_K, seed=7070, device=device, tp=(world, rank), host_tensors=verify)
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
    model.status()
    step_ms = e0.elapsed_time(e1) / (new_tokens - 1)
    if pg is not None:  # the slowest rank sets the pace
        t = torch.tensor([step_ms, gen_s, prefill_s], device=f"cuda:{device}")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        step_ms, gen_s, prefill_s = (float(v) for v in t.tolist())
    toks, pos = model.tokens()
    toks = toks[:new_tokens]
    # speculative-decoding verify forwards (forward_all over K+1 tokens at
    # the current position, cache rolled back after each): their cost next
    # to one decode step sets the acceptance a draft model must reach
    verify_ms = {}
    for kp1 in (2, 3, 4, 5, 8, 9):
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
    tok_bytes = cfg["n_layers"] * layer_weight_bytes() + cfg["vocab"] * cfg["hidden"] * 2
    out = {"config": f"Llama-2-70B shape, {cfg['n_layers']} layers, Q4_K resident, F16 lm_head, "
                     f"tensor-parallel over {world} GPU(s)",
           "tp": world,
           "prompt_tokens": prompt_len, "new_tokens": new_tokens,
           "decode_tok_s": round(1e3 / step_ms, 2), "ms_per_token": round(step_ms, 3),
           "prefill_ms": round(prefill_s * 1e3, 2),
           "generate_tok_s": round(new_tokens / gen_s, 2),
           "weight_bytes_per_token": tok_bytes,
           "decode_hbm_gbs": round(tok_bytes / (step_ms / 1e3) / 1e9, 1),
           "roofline": roofline_hbm(tok_bytes / world, step_ms, pk,
                                    "one graph-replayed decode step (per layer: rmsnorm staging, q/k/v, attention, "
                                    "o, staging, gate/up, swiglu staging, down; lm_head + argmax); bytes per rank"),
           "tokens": toks, "final_position": pos,
           "verify_forward_ms": verify_ms,
           "verify_note": "rq_llama_forward_all over K+1 tokens (host call incl. argmax copy), keys = K+1; a draft "
                          "that gets accepted tokens cheaper than decode ms_per_token * (accepted+1) - verify pays "
                          "off",
           "model_build_s": round(build_s, 2)}
    if verify:
        chk, layer0 = verify_decode(model, host, cfg, prompt, toks)
        out.update(chk)
        if with_cpu:
            out["cpu_baseline"] = cpu_decode(layer0, host["lm_head"], cfg["n_layers"])
    model.close()
    torch.cuda.empty_cache()
    return out


def run_gpu(args) -> None:
    import ctypes

    import torch
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    from rustyllm_b200 import Context, QWeight
    from rustyllm_b200 import tp as tpmod
    from rustyllm_b200._lib import check, lib
    L = lib()
    ctx = Context.get(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist
        tpmod.init_from_torch(ctx)
    pk = peaks()
    if args.only_decode:
        dec = decode_70b(local, pk, pg=pg, n_layers=args.decode_layers, verify=not args.no_verify,
                         with_cpu=False)
        if rank == 0:
            print(json.dumps({"metric": "70B Q4_K greedy decode tok/s", "value": dec["decode_tok_s"],
                              "unit": "tok/s", "n_gpus": world, "decode_70b": dec}), flush=True)
        if pg is not None:
            pg.barrier()
            tpmod.finalize(ctx)
            pg.destroy_process_group()
        return
    # every rank draws the same full tensors and keeps its shard (the whole
    # layer at one GPU)
    from rustyllm_b200.tp import shard
    g = torch.Generator(device=dev).manual_seed(1234)
    weights = []  # [copy][shape] -> QWeight
    for c in range(N_COPIES):
        layer = []
        for k, (n, i, o) in enumerate(SHAPES):
            wf = torch.randn(o, i, device=dev, generator=g) * 0.02
            layer.append(QWeight.quantize(ctx, Q4_K, shard(SPLIT[k], wf, world, rank).contiguous()))
            del wf
        weights.append(layer)
    torch.cuda.synchronize()
    # activations: q/k/v share one x, gate/up share one x (as QAttn / QMlp do);
    # o and down take this rank's slice of their input
    x_attn = torch.randn(1, 8192, device=dev, generator=g)
    x_o = torch.randn(1, 8192 // world, device=dev, generator=g)
    x_mlp = torch.randn(1, 8192, device=dev, generator=g)
    x_down = torch.randn(1, 28672 // world, device=dev, generator=g)
    xs = [x_attn, x_attn, x_attn, x_o, x_mlp, x_mlp, x_down]
    ys = [torch.empty(1, w.out, device=dev) for w in weights[0]]
    stream = torch.cuda.Stream(device=dev)
    arr = lambda vals: (ctypes.c_void_p * len(vals))(*vals)  # noqa: E731
    groups = [(0, 1, 2), (3,), (4, 5), (6,)]  # q/k/v batched, o, gate/up batched, down

    def launch_group(c, grp, st, xs=xs, ys=ys):
        if len(grp) == 1:
            k = grp[0]
            if world > 1 and SPLIT[k] == "row":
                check(L.rq_linear_allreduce(ctx.handle, weights[c][k].handle, xs[k].data_ptr(),
                                            ys[k].data_ptr(), 1, st))
            else:
                check(L.rq_linear(ctx.handle, weights[c][k].handle, xs[k].data_ptr(),
                                  ys[k].data_ptr(), 1, st))
        else:
            check(L.rq_linear_batch(ctx.handle, len(grp),
                                    arr([weights[c][k].handle.value for k in grp]),
                                    arr([xs[k].data_ptr() for k in grp]),
                                    arr([ys[k].data_ptr() for k in grp]), st))

    def hint(c, gi):
        # the weights of the next group (after down: the next layer copy's q/k/v)
        c2, g2 = (c, gi + 1) if gi + 1 < len(groups) else ((c + 1) % N_COPIES, 0)
        ws2 = [weights[c2][k].handle.value for k in groups[g2]]
        check(L.rq_linear_prefetch_hint(ctx.handle, len(ws2), arr(ws2)))

    def launch_layer(c, st, xs=xs, ys=ys):
        # the layer loop knows its next weights: each call prefetches the next
        # call's first rows into L2 in its tail (rq_linear_prefetch_hint)
        for gi, grp in enumerate(groups):
            hint(c, gi)
            launch_group(c, grp, st, xs, ys)

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

    def max_over_ranks(v: float) -> float:
        if pg is None:
            return v
        t = torch.tensor([v], device=dev)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    ms_total = timed(lambda s: graphs[s % N_COPIES].replay(), args.steps)
    clk = clocks.stop()
    reps = max(10, args.steps // 4)
    barrier()
    dom_ms = max_over_ranks(timed(lambda r: dom.replay(), reps) / (reps * N_COPIES))
    per_shape = {}
    for k, (n, i, o) in enumerate(SHAPES):
        barrier()
        t = max_over_ranks(timed(lambda r, k=k: shape_graphs[k].replay(), reps) / (reps * N_COPIES))
        per_shape[n] = round((Q4K_BYTES(i, o) + 4 * (i + o)) / world / (t / 1e3) / 1e9, 1)
    ms_step = max_over_ranks(ms_total / args.steps)

    # e2e: the public calls with host buffers -- every step copies its four
    # activation rows (one packed page-locked host buffer) to the device,
    # runs the four calls (each after the prefetch hint naming the next
    # call's weights, as in the device-timed step), copies the seven outputs
    # back to one page-locked host buffer and synchronises once.  The step (two copies, four calls)
    # is captured in a CUDA graph per layer copy, as a decoder would.
    nx = [8192, 8192 // world, 8192, 28672 // world]
    hxin = torch.randn(sum(nx), generator=torch.Generator().manual_seed(7)).pin_memory()
    dxin = torch.empty(sum(nx), device=dev)
    xv = [dxin[sum(nx[:i]):sum(nx[:i + 1])].view(1, -1) for i in range(4)]
    xs_e = [xv[0], xv[0], xv[0], xv[1], xv[2], xv[2], xv[3]]
    ny = [y.shape[1] for y in ys]
    dyout = torch.empty(sum(ny), device=dev)
    ys_e = [dyout[sum(ny[:i]):sum(ny[:i + 1])].view(1, -1) for i in range(len(ny))]
    hyout = torch.empty(sum(ny)).pin_memory()
    h2d, d2h = hxin.numel() * 4, hyout.numel() * 4

    # copies overlap the calls: the first call's row goes first, the other
    # rows follow on a copy stream while it runs, and each call's outputs go
    # back on the copy stream while the next call runs
    copy_stream = torch.cuda.Stream(device=dev)
    yk = [sum(ny[:k]) for k in range(len(ny) + 1)]

    def e2e_body(c, st):
        main = torch.cuda.current_stream()
        dxin[:nx[0]].copy_(hxin[:nx[0]], non_blocking=True)
        copy_stream.wait_stream(main)
        with torch.cuda.stream(copy_stream):
            dxin[nx[0]:].copy_(hxin[nx[0]:], non_blocking=True)
        rows_in = torch.cuda.Event()
        rows_in.record(copy_stream)
        for gi, grp in enumerate(groups):
            if gi == 1:
                main.wait_event(rows_in)
            hint(c, gi)
            launch_group(c, grp, main.cuda_stream, xs_e, ys_e)
            copy_stream.wait_stream(main)
            with torch.cuda.stream(copy_stream):
                lo, hi = yk[grp[0]], yk[grp[-1] + 1]
                hyout[lo:hi].copy_(dyout[lo:hi], non_blocking=True)
        main.wait_stream(copy_stream)

    with torch.cuda.stream(stream):
        for c in range(N_COPIES):
            e2e_body(c, stream.cuda_stream)
    stream.synchronize()
    e2e_graphs = [capture(lambda st, c=c: e2e_body(c, st)) for c in range(N_COPIES)]

    def e2e_step(c):
        with torch.cuda.stream(stream):
            e2e_graphs[c].replay()
        stream.synchronize()

    for c in range(3):
        e2e_step(c % N_COPIES)
    barrier()
    torch.cuda.synchronize()
    e2e_steps = max(5, min(args.steps, 100))
    t0 = time.perf_counter()
    for s in range(e2e_steps):
        e2e_step(s % N_COPIES)
    e2e_ms = max_over_ranks((time.perf_counter() - t0) / e2e_steps * 1e3)
    del e2e_graphs

    sb = step_bytes()
    value = sb / (ms_step / 1e3) / 1e9
    e2e_val = sb / (e2e_ms / 1e3) / 1e9
    dom_bytes = (2 * Q4K_BYTES(8192, 28672)) // world + 4 * (8192 + 2 * 28672 // world)
    cpu = None
    host_layer = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        host_layer = {n: weights[0][k].download() for k, (n, _, _) in enumerate(SHAPES)}
        cpu = cpu_layer_q4k(host_layer, seconds=args.cpu_seconds)
    small_m = formats = None
    if world == 1 and not args.no_small_m:
        small_m = small_m_sweep(L, ctx, weights, stream, timed, capture, dev, g, pk, host_layer)
        formats = other_formats(L, ctx, stream, timed, capture, dev, g, pk, host_layer is not None)
    del graphs, shape_graphs, dom
    graphs = shape_graphs = dom = None
    for layer in weights:
        for w in layer:
            w.free()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    moe = None
    if not args.no_moe:
        moe = (moe_sweep(local, pk, with_cpu=host_layer is not None) if world == 1
               else moe_ep_sweep(local, pg))
    dec = None
    if not args.no_decode:
        dec = decode_70b(local, pk, pg=pg, verify=not args.no_verify, with_cpu=host_layer is not None)
    if rank == 0:
        launches = 2 * len(groups)  # staging + matvec per call (the all-reduce runs inside the matvec)
        if world > 1 and not fused_allreduce_default(world):
            launches += 2           # a separate all-reduce kernel after o and down
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "weak" if world == 1 else "strong", "vs_baseline": None,
            "dtype": "int8x3 dp4a + f32 (4-bit weights)",
            "data": "synthetic: W ~ N(0,0.02) f32 quantized to Q4_K on device (seeded), x ~ N(0,1)",
            "config": headline_config(world),
            "method": ("value: each of the 4 calls after rq_linear_prefetch_hint naming the next call's weights "
                       "(the next layer copy's q/k/v after down); e2e: the same calls and hints on host buffers"),
            "pct_of_hbm_peak_per_gpu": round(100 * value / world / pk["hbm_gbs"], 1),
            "per_shape_single_call_gbs": per_shape,
            "roofline": roofline_hbm(dom_bytes, dom_ms, pk,
                                     "rq_linear_batch gate+up 2x(8192->28672" +
                                     (f"/{world}" if world > 1 else "") + "): xquant + mv_pipe_kernel<Q4_K>",
                                     "q4k_gate_up" if world == 1 else None),
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "how": "per step, timed on the host: the activation rows copied from page-locked host "
                           "memory, the 4 public calls, the 7 outputs copied back to page-locked host memory "
                           "(copies on a second stream overlapping the calls: the first row before the first "
                           "call, the others during it; each call's outputs during the next call; copies and "
                           "calls captured in one CUDA graph per layer copy), one stream synchronisation"},
            "gpu_launches": args.steps * launches,
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
    if pg is not None:
        pg.barrier()
        tpmod.finalize(ctx)
        pg.destroy_process_group()


def fused_allreduce_default(world: int) -> bool:
    """Mirrors librq's rule for the in-kernel all-reduce (RQ_TP_FUSED)."""
    return os.environ.get("RQ_TP_FUSED") != "0" and world >= 2


CASES = ("pipe_gate_up", "i8_gate_m2", "i8_gate_m4", "i8_gate_m8", "mm_gate_m20", "sk_gate_m16", "tc_gate_m128", "q3k_gate", "tc_q3k_gate_m128", "moe_t1", "moe_t16",
         "attn_decode")


def run_case(name: str) -> None:
    """A few launches of one kernel or layer for an ncu capture, at the
    bench's shapes: 'pipe_gate_up' (the gate+up rq_linear_batch of one 70B
    layer, M=1), 'i8_gate_m2' / 'i8_gate_m4' / 'i8_gate_m8' (gate_proj
    8192 -> 28672 at M=2 / 4 / 8, the int8 tensor-core kernels),
    'mm_gate_m20' (M=20, the mma.sync kernel in 8-row tiles),
    'sk_gate_m16' (M=16, split-K tcgen05), 'tc_gate_m128' (M=128, tiled
    tcgen05), 'q3k_gate' (the Q3_K gate_proj matvec), 'tc_q3k_gate_m128'
    (Q3_K gate_proj at M=128 on tcgen05), 'moe_t1' / 'moe_t16'
    (the Mixtral layer at T = 1 / 16), 'attn_decode' (a 4-layer 70B-shape
    model's decode steps: attention at head_dim 128).  Prints the per-call
    time measured without the profiler."""
    import ctypes

    import torch
    from rustyllm_b200 import Context, QWeight
    from rustyllm_b200._lib import check, lib
    L = lib()
    ctx = Context.get(0)
    g = torch.Generator(device="cuda").manual_seed(5)
    s = torch.cuda.current_stream().cuda_stream
    if name in ("moe_t1", "moe_t16"):
        from rustyllm_b200.mixtral import SparseMoe
        E, H, F = MIXTRAL["E"], MIXTRAL["H"], MIXTRAL["F"]
        router = (torch.randn(E, H, device="cuda", generator=g) * 0.02).cpu().numpy()
        experts = [tuple(QWeight.quantize(ctx, Q4_K, torch.randn(o, i, device="cuda", generator=g) * 0.02)
                         for o, i in ((F, H), (H, F), (F, H))) for _ in range(E)]
        moe = SparseMoe(router, experts, top_k=2)
        T = 1 if name == "moe_t1" else 16
        x = torch.randn(T, H, device="cuda", generator=g)

        def call():
            moe.forward(x)
        nbytes = 0
    elif name == "attn_decode":
        from rustyllm_b200.llama import random_model
        cfg = dict(LLAMA70B, n_layers=4)
        model, _ = random_model(cfg, Q4_K, seed=3)
        model.forward(np.arange(20, dtype=np.int32), 0, want_logits=False)

        def call():
            model.decode_step(s)
        nbytes = 0
    else:
        qt = Q3_K if name in ("q3k_gate", "tc_q3k_gate_m128") else Q4_K
        ws = [QWeight.quantize(ctx, qt, torch.randn(28672, 8192, device="cuda", generator=g) * 0.02)
              for _ in range(2)]
        arr = lambda v: (ctypes.c_void_p * len(v))(*v)  # noqa: E731
        if name == "pipe_gate_up":
            x = torch.randn(1, 8192, device="cuda", generator=g)
            ys = [torch.empty(1, 28672, device="cuda") for _ in range(2)]

            def call():
                check(L.rq_linear_batch(ctx.handle, 2, arr([w.handle.value for w in ws]),
                                        arr([x.data_ptr()] * 2), arr([y.data_ptr() for y in ys]), s))
            nbytes = 2 * Q4K_BYTES(8192, 28672)
        else:
            M = {"i8_gate_m2": 2, "i8_gate_m4": 4, "i8_gate_m8": 8, "mm_gate_m20": 20, "sk_gate_m16": 16,
                 "q3k_gate": 1}.get(name, 128)
            x = torch.randn(M, 8192, device="cuda", generator=g)
            y = torch.empty(M, 28672, device="cuda")

            def call():
                check(L.rq_linear(ctx.handle, ws[0].handle, x.data_ptr(), y.data_ptr(), M, s))
            nbytes = (Q3K_BYTES if qt == Q3_K else Q4K_BYTES)(8192, 28672)
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
    out = {"case": name, "us_per_call": round(ms * 1e3, 2)}
    if nbytes:
        out["weight_gbs"] = round(nbytes / (ms / 1e3) / 1e9, 1)
    if name in ("tc_gate_m128", "tc_q3k_gate_m128", "sk_gate_m16"):
        M = 16 if name == "sk_gate_m16" else 128
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
    ap.add_argument("--no-verify", action="store_true", help="skip the oracle replay of the decode tokens")
    ap.add_argument("--only-decode", action="store_true", help="run only the 70B decode")
    ap.add_argument("--no-small-m", action="store_true", help="skip the small-M and other-format sweeps")
    ap.add_argument("--no-moe", action="store_true", help="skip the Mixtral MoE layer sweep")
    ap.add_argument("--decode-layers", type=int, default=None,
                    help="layers of the decode model (default 80; fewer for profiling)")
    ap.add_argument("--case", choices=CASES, default=None,
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
