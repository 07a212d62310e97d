"""Benchmark of the B200 AWQ W4A16 path (one JSON line on rank 0).

Workload: the Llama-3-8B-shaped AWQ projection set
QKV 4096->6144, O 4096->4096, gate_up 4096->28672, down 14336->4096, group 128,
bf16 activations N(0,1) at M in {1, 8, 32, 64}. One step = the 4 projections at
each of the 4 batch sizes (16 GEMMs), weights resident in HBM (453 MB streamed
per step, larger than the 126 MB L2, so no flush is needed between steps).
With N > 1 ranks the same projections are tensor-parallel (QKV / gate_up split
by output columns, O / down by input rows followed by an NCCL all-reduce of the
[M, 4096] output), strong scaling. Inputs are seeded synthetic data.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

G = 128
SHAPES = {"qkv": (4096, 6144), "o": (4096, 4096), "gate_up": (4096, 28672), "down": (14336, 4096)}
ROW_PARALLEL = ("o", "down")
MS = (1, 8, 32, 64)
DTYPE = torch.bfloat16
METRIC = "W4A16 GEMM weight GB/s, Llama-3-8B decode projections (QKV/O/gate_up/down) at M=1,8,32,64"


def awq_bytes(K: int, N: int) -> int:
    """Weight + scale + zero bytes of one AWQ projection (algorithmic)."""
    return K * N // 2 + (K // G) * N * 2 + (K // G) * N // 2


def algo_bytes(M: int, K: int, N: int) -> int:
    return awq_bytes(K, N) + M * K * 2 + M * N * 2


def local_shape(name: str, tp: int):
    K, N = SHAPES[name]
    return (K // tp, N) if name in ROW_PARALLEL else (K, N // tp)


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def make_weights(K: int, N: int, device, seed: int):
    """Random AWQ tensors on the device: uniformly random int32 words are
    uniformly random nibbles (q and z in [0, 15]); scales uniform in [1e-3, 1e-2]."""
    g = torch.Generator(device=device).manual_seed(seed)
    qw = torch.randint(-2**31, 2**31 - 1, (K, N // 8), generator=g, device=device, dtype=torch.int64).to(torch.int32)
    qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), generator=g, device=device, dtype=torch.int64).to(torch.int32)
    sc = (torch.rand((K // G, N), generator=g, device=device) * 9e-3 + 1e-3).to(DTYPE)
    return qw, qz, sc


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak_hbm():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profiled_traffic():
    """DRAM bytes per step of the GEMM kernel from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "gemm_decode_llama8b_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


# --------------------------------------------------------------- CPU baseline
def cpu_baseline(sample_seconds: float = 15.0):
    """The reference's math (dequantise every call, then matmul) restated in
    PyTorch on the host with all cores, on a bounded sample of the step."""
    from oracle.awq_ref import cpu_awq_linear

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    done_bytes = 0
    t_total = 0.0
    order = [(n, M) for M in MS for n in SHAPES]
    weights = {}
    for j, (name, (K, N)) in enumerate(SHAPES.items()):
        g = torch.Generator().manual_seed(j)
        weights[name] = (torch.randint(-2**31, 2**31 - 1, (K, N // 8), generator=g, dtype=torch.int64).to(torch.int32),
                         torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), generator=g, dtype=torch.int64).to(torch.int32),
                         (torch.rand((K // G, N), generator=g) * 9e-3 + 1e-3).to(DTYPE))
    i = 0
    while t_total < sample_seconds and i < 64 * len(order):
        name, M = order[i % len(order)]
        K, N = SHAPES[name]
        x = torch.randn((M, K), generator=torch.Generator().manual_seed(i)).to(DTYPE)
        t0 = time.perf_counter()
        cpu_awq_linear(x, *weights[name], G, compute_dtype=torch.float32)
        t_total += time.perf_counter() - t0
        done_bytes += awq_bytes(K, N)
        i += 1
    return {"value": done_bytes / t_total / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{i} of the step's 16 projection GEMMs, dequantise + fp32 matmul per call, {t_total:.1f} s"}


def bench_config(world: int) -> dict:
    return {"workload": "llama3_8b_awq_decode_projections", "group_size": G,
            "batch_sizes": list(MS), "projections": {k: list(v) for k, v in SHAPES.items()},
            "parallelism": f"tp{world}", "l2": "working set 453 MB > 126 MB L2, no flush"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    torch.manual_seed(0)
    steps, warm = args.steps, args.warmup
    from oracle.awq_ref import cpu_awq_linear

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # one bounded sample per step: the O projection at each M (dequant + matmul)
    K, N = SHAPES["o"]
    g = torch.Generator().manual_seed(1)
    qw = torch.randint(-2**31, 2**31 - 1, (K, N // 8), generator=g, dtype=torch.int64).to(torch.int32)
    qz = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), generator=g, dtype=torch.int64).to(torch.int32)
    sc = (torch.rand((K // G, N), generator=g) * 9e-3 + 1e-3).to(DTYPE)
    xs = [torch.randn((M, K), generator=g).to(DTYPE) for M in MS]
    for _ in range(warm):
        cpu_awq_linear(xs[0], qw, qz, sc, G)
    t0 = time.perf_counter()
    for _ in range(steps):
        for x in xs:
            cpu_awq_linear(x, qw, qz, sc, G)
    dt = time.perf_counter() - t0
    b = awq_bytes(K, N) * len(xs) * steps
    v = b / dt / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": dt / steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": dict(bench_config(world), sample="O projection at M=1,8,32,64 per step"),
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "O projection (K=N=4096) at M=1,8,32,64 per step, dequantise + fp32 matmul"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# --------------------------------------------------------------- our arm
def run_ours(args):
    import torch.distributed as dist

    from sglite_b200 import ops
    from sglite_b200.quantization import AWQB200Config

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = ex = None
    if world > 1:
        from datetime import timedelta

        from sglite_b200.distributed import init_nccl, init_peer_exchange

        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
        max_bytes = max(MS) * 4096 * 2
        comm = init_nccl(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                         max_size_bytes=max_bytes)
        if args.allreduce == "fused":
            ex = init_peer_exchange(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                                    max_rows=max(MS), max_n=4096)
            ex.set_mode(args.tp_mode)

    cfg = AWQB200Config(4, G, True)
    method = cfg.get_linear_method()
    layers = {}
    for i, name in enumerate(SHAPES):
        K, N = local_shape(name, world)
        w = method.create_weights(K, N)
        qw, qz, sc = make_weights(K, N, dev, seed=1000 * rank + i)
        w["qweight"], w["qzeros"], w["scales"] = qw, qz, sc
        layers[name] = method.process_weights_after_loading(w)
        del qw, qz, sc
    torch.cuda.synchronize()
    gx = torch.Generator(device=dev).manual_seed(7 + rank)
    xs = {(n, M): torch.randn((M, local_shape(n, world)[0]), generator=gx, device=dev).to(DTYPE)
          for M in MS for n in SHAPES}
    ys = {(n, M): torch.empty((M, local_shape(n, world)[1]), device=dev, dtype=DTYPE) for M in MS for n in SHAPES}
    order = [(n, M) for M in MS for n in SHAPES]

    def step():
        for (n, M) in order:
            w = layers[n]
            if ex is not None and n in ROW_PARALLEL:  # GEMM + all-reduce in one kernel over peer memory
                ex.gemm_allreduce(xs[(n, M)], w["qweight"], w["_input_size"], w["_output_size"], G,
                                  out=ys[(n, M)])
                continue
            ops.gemm(xs[(n, M)], w["qweight"], w["_input_size"], w["_output_size"], G, out=ys[(n, M)])
            if comm is not None and n in ROW_PARALLEL:
                comm.all_reduce(ys[(n, M)])

    def gemms_only():
        for (n, M) in order:
            w = layers[n]
            ops.gemm(xs[(n, M)], w["qweight"], w["_input_size"], w["_output_size"], G, out=ys[(n, M)])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # The reference replays decode steps from captured CUDA graphs
    # (model_executor/cuda_graph.py:153-177); the timed step is one replay.
    for _ in range(args.warmup):
        step()
    barrier()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph_g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph_g):
        gemms_only()
    barrier()
    for _ in range(args.warmup):
        graph.replay()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        start.record()
        for _ in range(args.steps):
            graph.replay()
        end.record()
        barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # GEMM kernels alone (same launches, no all-reduce): the roofline figure
    for _ in range(args.warmup):
        graph_g.replay()
    torch.cuda.synchronize()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record()
    for _ in range(args.steps):
        graph_g.replay()
    g1.record()
    torch.cuda.synchronize()
    gemm_ms = g0.elapsed_time(g1)

    # e2e through the linear-method API: pinned host activations in, outputs
    # back to the host, every step. The inputs of one batch size (four
    # projections) sit contiguously in pinned host memory and go in with one
    # copy; their outputs are written into one contiguous device buffer
    # (apply_weights(out=...)) and leave with one copy. Copies run on their own
    # streams (one per direction) and both sides are double-buffered across
    # steps, so PCIe transfers of one step overlap the GEMMs of the next.
    groups = [(M, [(n, M) for n in SHAPES]) for M in MS]
    nbuf = 2
    hx_g, hy_g, dx_g, dy_g, dx, dy = {}, {}, {}, {}, [{} for _ in range(nbuf)], [{} for _ in range(nbuf)]
    for M, keys in groups:
        nin = sum(xs[k].numel() for k in keys)
        nout = sum(ys[k].numel() for k in keys)
        src = torch.cat([xs[k].reshape(-1) for k in keys]).cpu()
        for b in range(nbuf):
            hx_g[(b, M)] = src.clone().pin_memory()
            hy_g[(b, M)] = torch.empty(nout, dtype=DTYPE).pin_memory()
            dx_g[(b, M)] = torch.empty(nin, dtype=DTYPE, device=dev)
            dy_g[(b, M)] = torch.empty(nout, dtype=DTYPE, device=dev)
            oi = oo = 0
            for k in keys:
                dx[b][k] = dx_g[(b, M)][oi:oi + xs[k].numel()].view(xs[k].shape)
                dy[b][k] = dy_g[(b, M)][oo:oo + ys[k].numel()].view(ys[k].shape)
                oi += xs[k].numel()
                oo += ys[k].numel()
    h2d = sum(hx_g[(0, M)].numel() * 2 for M, _ in groups)
    d2h = sum(hy_g[(0, M)].numel() * 2 for M, _ in groups)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = {(b, M): torch.cuda.Event() for b in range(nbuf) for M, _ in groups}
    ev_used = {(b, M): torch.cuda.Event() for b in range(nbuf) for M, _ in groups}
    ev_done = {(b, M): torch.cuda.Event() for b in range(nbuf) for M, _ in groups}
    ev_out = {(b, M): torch.cuda.Event() for b in range(nbuf) for M, _ in groups}
    fresh = set(ev_used)
    step_no = [0]

    def e2e_step():
        b = step_no[0] % nbuf
        step_no[0] += 1
        compute = torch.cuda.current_stream(dev)
        with torch.cuda.stream(s_in):
            for M, _ in groups:
                if (b, M) not in fresh:
                    s_in.wait_event(ev_used[(b, M)])  # GEMMs two steps back are done with this buffer
                dx_g[(b, M)].copy_(hx_g[(b, M)], non_blocking=True)
                ev_in[(b, M)].record(s_in)
        for M, keys in groups:
            compute.wait_event(ev_in[(b, M)])
            if (b, M) not in fresh:
                compute.wait_event(ev_out[(b, M)])  # its outputs two steps back have left
            for (n, _) in keys:
                k = (n, M)
                if ex is not None and n in ROW_PARALLEL:
                    w = layers[n]
                    ex.gemm_allreduce(dx[b][k], w["qweight"], w["_input_size"], w["_output_size"], G,
                                      out=dy[b][k])
                else:
                    method.apply_weights(layers[n], dx[b][k], out=dy[b][k])
                    if comm is not None and n in ROW_PARALLEL:
                        comm.all_reduce(dy[b][k])
            ev_used[(b, M)].record(compute)
            ev_done[(b, M)].record(compute)
            s_out.wait_event(ev_done[(b, M)])
            with torch.cuda.stream(s_out):
                hy_g[(b, M)].copy_(dy_g[(b, M)], non_blocking=True)
                ev_out[(b, M)].record(s_out)
            fresh.discard((b, M))

    def e2e_drain():
        torch.cuda.current_stream(dev).wait_stream(s_in)
        torch.cuda.current_stream(dev).wait_stream(s_out)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_drain()
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e2e_drain()  # the timed region ends when the last output is on the host
    e1.record()
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    step_bytes_full = sum(awq_bytes(*SHAPES[n]) for n in SHAPES) * len(MS)  # whole job (all ranks)
    value = step_bytes_full * args.steps / (ms / 1e3) / 1e9
    e2e_value = step_bytes_full * args.steps / (e2e_ms / 1e3) / 1e9
    # roofline of the GEMM kernel: algorithmic bytes per launch / mean launch time
    algo = sum(algo_bytes(M, *local_shape(n, world)) for (n, M) in order)
    achieved = algo * args.steps / (gemm_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak_hbm()
    traffic = profiled_traffic()
    err = ops.device_error()
    result = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random AWQ weights and N(0,1) activations)",
        "config": bench_config(world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": (traffic["dram_bytes_per_step"] / traffic["launches_per_step"]
                                 if traffic and world == 1 else None),
                     "traffic_source": "profiles/gemm_decode_llama8b_traffic.json (ncu, mean per launch)",
                     "algorithmic_bytes_per_launch": algo / len(order),
                     "algorithmic_bytes_per_step": algo,
                     "mean_gemm_us": gemm_ms * 1e3 / (args.steps * len(order))},
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": len(order) * args.steps,
        "graph": "one CUDA-graph replay per step (16 GEMM launches)",
        "allreduce": ("none" if world == 1 else
                      "fused into the row-parallel GEMM over peer memory" if ex is not None else "NCCL"),
        "clocks": clk.summary(),
        "device_error": err,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(result), flush=True)
    del graph, graph_g
    torch.cuda.synchronize()
    if ex is not None:
        ex.destroy()
    if comm is not None:
        comm.destroy()
    if world > 1:
        dist.destroy_process_group()


# --------------------------------------------------------------- other configs
def _graph_us(fn, warm, steps, reps=4):
    """Time of one fn() from graph replays of reps back-to-back calls (the graph
    launch itself is amortised over reps)."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    for _ in range(warm):
        g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        g.replay()
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / (steps * reps)
    del g
    return us


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def _linear(K, N, dev, dtype, seed):
    from sglite_b200.quantization import AWQB200Config

    m = AWQB200Config(4, G, True).get_linear_method()
    w = m.create_weights(K, N)
    g = torch.Generator(device=dev).manual_seed(seed)
    w["qweight"] = torch.randint(-2**31, 2**31 - 1, (K, N // 8), generator=g, device=dev, dtype=torch.int64).to(torch.int32)
    w["qzeros"] = torch.randint(-2**31, 2**31 - 1, (K // G, N // 8), generator=g, device=dev, dtype=torch.int64).to(torch.int32)
    w["scales"] = (torch.rand((K // G, N), generator=g, device=dev) * 9e-3 + 1e-3).to(dtype)
    return m, m.process_weights_after_loading(w)


def run_prefill(args):
    """Config 2: Qwen3-4B AWQ projections at M = 512, 2048, 8192 (fp16)."""
    from sglite_b200 import ops

    dev = torch.device("cuda", 0)
    shapes = {"qkv": (2560, 6144), "o": (4096, 2560), "gate_up": (2560, 19456), "down": (9728, 2560)}
    hbm, tflops_peak, kind = _peaks()
    rows = {}
    tot_flop = tot_us = 0.0
    clk = ClockSampler(0)  # clocks over all timed regions: long tensor-bound runs meet the power cap
    clk.__enter__()
    try:
        for i, (n, (K, N)) in enumerate(shapes.items()):
            _, w = _linear(K, N, dev, torch.float16, i)
            for M in (512, 2048, 8192):
                x = torch.randn((M, K), device=dev).to(torch.float16)
                y = torch.empty((M, N), device=dev, dtype=torch.float16)
                us = _graph_us(lambda: ops.gemm(x, w["qweight"], K, N, G, out=y), args.warmup, args.steps)
                fl = 2.0 * M * N * K
                rows[f"{n}@M{M}"] = {"us": round(us, 2), "tflops": round(fl / us / 1e6, 1),
                                     "frac": round(fl / us / 1e6 / tflops_peak, 3)}
                tot_flop += fl
                tot_us += us
    finally:
        clk.__exit__(None, None, None)
    sustained = None
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            sustained = float(json.load(f)["bf16_tflops_sustained"])
    except (OSError, KeyError, ValueError):
        pass
    value = tot_flop / tot_us / 1e6
    print(json.dumps({"workload": "qwen3_4b_awq_prefill (config 2)", "metric": "W4A16 GEMM TFLOP/s",
                      "value": value, "unit": "TFLOP/s", "peak": tflops_peak, "peak_kind": kind,
                      "frac": value / tflops_peak,
                      "peak_sustained": sustained, "frac_sustained": value / sustained if sustained else None,
                      "per_gemm": rows, "dtype": "fp16", "clocks": clk.summary()}), flush=True)


def run_single(args):
    """Config 0: one K=N=4096 projection at M=16 (fp16)."""
    from sglite_b200 import ops

    dev = torch.device("cuda", 0)
    K = N = 4096
    M = 16
    _, w = _linear(K, N, dev, torch.float16, 0)
    x = torch.randn((M, K), device=dev).to(torch.float16)
    y = torch.empty((M, N), device=dev, dtype=torch.float16)
    us = _graph_us(lambda: ops.gemm(x, w["qweight"], K, N, G, out=y), args.warmup, args.steps)
    hbm, _, kind = _peaks()
    b = algo_bytes(M, K, N)
    print(json.dumps({"workload": "single K=N=4096 M=16 (config 0)", "metric": "GEMM us", "value": us,
                      "unit": "us", "weight_GBps": awq_bytes(K, N) / us / 1e3, "algo_GBps": b / us / 1e3,
                      "frac_hbm": b / us / 1e3 / hbm, "peak_kind": kind}), flush=True)


def run_gemm(args):
    """One projection, plain launches (no graph): the case the ncu captures profile."""
    from sglite_b200 import ops

    K, N, M = (int(v) for v in args.shape.split("x"))
    dtype = torch.float16 if args.fp16 else DTYPE
    dev = torch.device("cuda", 0)
    _, w = _linear(K, N, dev, dtype, 0)
    x = torch.randn((M, K), device=dev).to(dtype)
    y = torch.empty((M, N), device=dev, dtype=dtype)
    for _ in range(args.warmup + args.steps):
        ops.gemm(x, w["qweight"], K, N, G, out=y)
    torch.cuda.synchronize()
    print(json.dumps({"workload": f"gemm K={K} N={N} M={M}", "launches": args.warmup + args.steps,
                      "dtype": str(dtype), "device_error": ops.device_error()}), flush=True)


def run_tp70b(args):
    """Config 3: Llama-3.1-70B layer projections under TP=N, all-reduce after O and down."""
    import torch.distributed as dist

    from sglite_b200 import ops

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = ex = None
    if world > 1:
        from datetime import timedelta

        from sglite_b200.distributed import init_nccl, init_peer_exchange

        dist.init_process_group("gloo", timeout=timedelta(seconds=120))
        comm = init_nccl(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                         max_size_bytes=256 * 8192 * 2)
        if args.allreduce == "fused":
            ex = init_peer_exchange(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                                    max_rows=64, max_n=8192)
            ex.set_mode(args.tp_mode)
    full = {"qkv": (8192, 10240), "o": (8192, 8192), "gate_up": (8192, 57344), "down": (28672, 8192)}
    loc = {n: ((K // world, N) if n in ROW_PARALLEL else (K, N // world)) for n, (K, N) in full.items()}
    ws = {}
    for i, (n, (K, N)) in enumerate(loc.items()):
        _, ws[n] = _linear(K, N, dev, DTYPE, 100 * rank + i)
    hbm, tflops_peak, kind = _peaks()
    out = {}
    for M in (1, 32, 256, 4096):
        xs = {n: torch.randn((M, K), device=dev).to(DTYPE) for n, (K, N) in loc.items()}
        ys = {n: torch.empty((M, N), device=dev, dtype=DTYPE) for n, (K, N) in loc.items()}

        def layer():
            for n, (K, N) in loc.items():
                if ex is not None and n in ROW_PARALLEL and M <= ex.max_rows:
                    ex.gemm_allreduce(xs[n], ws[n]["qweight"], K, N, G, out=ys[n])
                    continue
                ops.gemm(xs[n], ws[n]["qweight"], K, N, G, out=ys[n])
                if comm is not None and n in ROW_PARALLEL:
                    comm.all_reduce(ys[n])

        if world > 1:
            dist.barrier()
        us = _graph_us(layer, args.warmup, args.steps)
        if world > 1:
            t = torch.tensor([us], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            us = float(t.item())
        wbytes = sum(awq_bytes(K, N) for K, N in loc.values())
        flops = sum(2.0 * M * K * N for K, N in loc.values())
        ring = 2 * (world - 1) / world * M * 8192 * 2 if world > 1 else 0.0
        roof_us = max(wbytes / hbm / 1e3, flops / tflops_peak / 1e6) + 2 * ring / 770e3
        out[f"M{M}"] = {"layer_us": round(us, 2), "roofline_us": round(roof_us, 2), "ratio": round(us / roof_us, 2)}
    if rank == 0:
        print(json.dumps({"workload": f"llama3.1_70b_awq_layer_tp{world} (config 3)", "metric": "TP-layer us",
                          "unit": "us", "n_gpus": world, "per_m": out,
                          "roofline": "max(weight bytes / measured HBM, flops / measured bf16 peak) + 2 ring all-reduces at 770 GB/s",
                          "allreduce": (f"fused GEMM + all-reduce over peer memory for M <= 64 ({args.tp_mode}), "
                                        "NCCL above" if ex is not None else "NCCL"),
                          "peak_kind": kind}), flush=True)
    if ex is not None:
        ex.destroy()
    if comm is not None:
        comm.destroy()
    if world > 1:
        dist.destroy_process_group()


def run_moe(args):
    """Config 4: Qwen3-30B-A3B AWQ MoE layer at M = 16, 256, 4096."""
    from sglite_b200.moe import AWQB200MoeBackend, AWQExpertWeights

    dev = torch.device("cuda", 0)
    E, k, H, I = 128, 8, 2048, 768
    g = torch.Generator(device=dev).manual_seed(0)

    def experts(K, N, gate_up=False):
        qw = torch.randint(-2**31, 2**31 - 1, (E, K, N // 8), generator=g, device=dev, dtype=torch.int64).to(torch.int32)
        qz = torch.randint(-2**31, 2**31 - 1, (E, K // G, N // 8), generator=g, device=dev, dtype=torch.int64).to(torch.int32)
        sc = (torch.rand((E, K // G, N), generator=g, device=dev) * 9e-3 + 1e-3).to(DTYPE)
        return AWQExpertWeights.from_awq(qw, qz, sc, G, gate_up=gate_up)

    w1, w2 = experts(H, 2 * I, gate_up=True), experts(I, H)
    backend = AWQB200MoeBackend()
    hbm, tflops_peak, kind = _peaks()
    per = {}
    for M in (16, 256, 4096):
        x = torch.randn((M, H), device=dev).to(DTYPE)
        lg = torch.randn((M, E), device=dev)
        buf = x.clone()
        us = _graph_us(lambda: backend.forward(buf, w1, w2, lg, k, True), args.warmup, args.steps)
        _, ids = torch.topk(lg, k, dim=-1)
        touched = int(torch.unique(ids).numel())
        wbytes = touched * (awq_bytes(H, 2 * I) + awq_bytes(I, H))
        flops = 2.0 * M * k * (H * 2 * I + I * H)
        per[f"M{M}"] = {"us": round(us, 2), "experts_touched": touched, "weight_GBps": round(wbytes / us / 1e3, 1),
                        "tflops": round(flops / us / 1e6, 1)}
    print(json.dumps({"workload": "qwen3_30b_a3b_awq_moe (config 4)", "metric": "MoE layer us", "unit": "us",
                      "per_m": per, "peak_hbm_GBps": hbm, "peak_tflops": tflops_peak, "peak_kind": kind}), flush=True)


def run_norm(args):
    """Residual-add RMSNorm after the row-parallel projections (the reference's
    RMSNormFused, layers/norm.py:28-47), hidden 8192 (config 3), bf16. HBM-bound:
    algorithmic bytes = 4 * M * N * 2 (read x and residual, write both) + N * 2."""
    from sglite_b200 import ops

    dev = torch.device("cuda", 0)
    N = 8192
    hbm, _, kind = _peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    per = {}
    for M in (1, 32, 256, 4096, 32768):
        x = torch.randn((M, N), generator=g, device=dev).to(DTYPE)
        r = torch.randn((M, N), generator=g, device=dev).to(DTYPE)
        w = (torch.rand(N, generator=g, device=dev) + 0.5).to(DTYPE)
        us = _graph_us(lambda: ops.fused_add_rmsnorm(x, r, w, 1e-6), args.warmup, args.steps, reps=16)
        nbytes = 4 * M * N * 2 + N * 2
        per[f"M{M}"] = {"us": round(us, 3), "GBps": round(nbytes / us / 1e3, 1),
                        "frac_hbm": round(nbytes / us / 1e3 / hbm, 3)}
    print(json.dumps({"workload": "fused_add_rmsnorm hidden 8192 (after the row-parallel all-reduce)",
                      "metric": "us per call", "unit": "us", "per_m": per, "peak_hbm_GBps": hbm,
                      "peak_kind": kind, "l2": "M <= 4096 fits in L2 between calls; M = 32768 (1 GB) does not"}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "single", "tp70b", "moe", "gemm", "norm"],
                    help="decode (default, the contract line) or another BASELINE config")
    ap.add_argument("--allreduce", default="fused", choices=["fused", "nccl"],
                    help="row-parallel all-reduce at N > 1: fused into the GEMM over peer memory, or NCCL")
    ap.add_argument("--tp-mode", default="auto", choices=["auto", "all_to_all", "reduce_scatter"],
                    help="exchange pattern of the fused all-reduce")
    ap.add_argument("--shape", default="4096x28672x1", help="KxNxM for --workload gemm")
    ap.add_argument("--fp16", action="store_true", help="fp16 activations for --workload gemm")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "single":
        run_single(args)
    elif args.workload == "tp70b":
        run_tp70b(args)
    elif args.workload == "moe":
        run_moe(args)
    elif args.workload == "norm":
        run_norm(args)
    elif args.workload == "gemm":
        run_gemm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
