"""Benchmark of the B200 AWQ W4A16 path (one JSON line on rank 0).

Workload: the Llama-3-8B-shaped AWQ projection set
QKV 4096->6144, O 4096->4096, gate_up 4096->28672, down 14336->4096, group 128,
bf16 activations N(0,1) at M in {1, 8, 32, 64}. One step = the 4 projections at
each of the 4 batch sizes (16 GEMMs). Every batch size has its own copy of the
weights, so each GEMM of a step streams weights no other GEMM of the step
touches (453 MB of distinct weights per step, 3.6x the 126 MB L2: nothing is
re-read from L2 between uses, no flush needed). With N > 1 ranks the same
projections are tensor-parallel (QKV / gate_up split by output columns, O /
down by input rows followed by the all-reduce of the [M, 4096] output), strong
scaling. Before timing, every projection's output is checked against a PyTorch
fp32 dequantise-then-matmul of the unsharded weights on a column slice, and at
N > 1 every rank must hold identical bits; the result is the line's "parity"
object and a failure exits non-zero. The line also carries the other BASELINE
configurations measured in the same run ("extra"): config 3 (Llama-3.1-70B
layer at TP = N), config 4 (Qwen3-30B-A3B MoE layer, experts split over the N
ranks) and, at N = 1, config 2 (Qwen3-4B prefill). Inputs are seeded synthetic
data with the benchmark's shapes and value distributions.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

from __future__ import annotations

import argparse
import hashlib
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
PARITY_TOL = 1e-2  # max |y - ref| <= 1e-2 * max |ref| (the task's GEMM contract)

LLAMA70B = {"qkv": (8192, 10240), "o": (8192, 8192), "gate_up": (8192, 57344), "down": (28672, 8192)}
QWEN3_4B = {"qkv": (2560, 6144), "o": (4096, 2560), "gate_up": (2560, 19456), "down": (9728, 2560)}


def awq_bytes(K: int, N: int) -> int:
    """Weight + scale + zero bytes of one AWQ projection (algorithmic)."""
    return K * N // 2 + (K // G) * N * 2 + (K // G) * N // 2


def algo_bytes(M: int, K: int, N: int) -> int:
    return awq_bytes(K, N) + M * K * 2 + M * N * 2


def local_shape(name: str, tp: int, shapes=SHAPES):
    K, N = shapes[name]
    return (K // tp, N) if name in ROW_PARALLEL else (K, N // tp)


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def full_awq(K: int, N: int, device, seed: int, dtype=DTYPE, lead=()):
    """Random AWQ tensors of the whole (unsharded) projection, the same on
    every rank for a given seed: uniformly random int32 words are uniformly
    random nibbles (q and z in [0, 15]); scales uniform in [1e-3, 1e-2]."""
    g = torch.Generator(device=device).manual_seed(seed)
    qw = torch.randint(-2**31, 2**31 - 1, (*lead, K, N // 8), generator=g, device=device,
                       dtype=torch.int64).to(torch.int32)
    qz = torch.randint(-2**31, 2**31 - 1, (*lead, K // G, N // 8), generator=g, device=device,
                       dtype=torch.int64).to(torch.int32)
    sc = (torch.rand((*lead, K // G, N), generator=g, device=device) * 9e-3 + 1e-3).to(dtype)
    return {"qweight": qw, "qzeros": qz, "scales": sc}


def shard(full, name: str, rank: int, world: int):
    from sglite_b200.tp import shard_awq

    if world == 1:
        return dict(full)
    return shard_awq(full, "row" if name in ROW_PARALLEL else "column", rank, world)


_SHIFTS = (0, 16, 4, 20, 8, 24, 12, 28)  # AWQ bit offset of logical column i of a packed word


def torch_ref_cols(x: torch.Tensor, full, c0: int, c1: int) -> torch.Tensor:
    """PyTorch fp32 reference of x @ dequant(W)[:, c0:c1] (on x's device):
    unpack the AWQ nibbles, W = (q - z) * s rounded to the activation dtype
    (layers/quantization/awq_triton.py:53-62,119-122), fp32 matmul."""
    sh = torch.tensor(_SHIFTS, dtype=torch.int32, device=x.device)

    def unpack(p):
        return ((p.unsqueeze(-1) >> sh) & 0xF).reshape(*p.shape[:-1], p.shape[-1] * 8)

    q = unpack(full["qweight"][:, c0 // 8:c1 // 8])
    z = unpack(full["qzeros"][:, c0 // 8:c1 // 8])
    s = full["scales"][:, c0:c1]
    w = ((q - z.repeat_interleave(G, 0)).to(s.dtype) * s.repeat_interleave(G, 0)).float()
    return x.float() @ w


def rel_err(y: torch.Tensor, ref: torch.Tensor) -> float:
    return float((y.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

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


def _peaks_file():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def measured_peak_hbm():
    d = _peaks_file()
    try:
        return float(d["hbm_gbs"]), "measured"
    except (TypeError, KeyError, ValueError):
        return 6650.0, "fallback"


def _peaks():
    d = _peaks_file()
    try:
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    except (TypeError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


def profiled_traffic():
    """DRAM bytes per step of the GEMM kernels from the committed ncu summary."""
    path = os.path.join(REPO, "profiles", "gemm_decode_llama8b_traffic.json")
    try:
        with open(path) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for ln in f:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# --------------------------------------------------------------- CPU baseline
def _cpu_weights():
    out = {}
    for j, (name, (K, N)) in enumerate(SHAPES.items()):
        out[name] = tuple(full_awq(K, N, "cpu", seed=j).values())
    return out


def _cpu_sample(weights, compute_dtype, seconds: float, max_gemms: int):
    from oracle.awq_ref import cpu_awq_linear

    order = [(n, M) for M in MS for n in SHAPES]
    done = 0
    t_total = 0.0
    i = 0
    while t_total < seconds and i < max_gemms:
        name, M = order[i % len(order)]
        K, N = SHAPES[name]
        x = torch.randn((M, K), generator=torch.Generator().manual_seed(i)).to(DTYPE)
        t0 = time.perf_counter()
        cpu_awq_linear(x, *weights[name], G, compute_dtype=compute_dtype)
        t_total += time.perf_counter() - t0
        done += awq_bytes(K, N)
        i += 1
    return done / t_total / 1e9, i, t_total


def cpu_baseline(sample_seconds: float = 8.0):
    """The reference's math (dequantise every call, then matmul) restated in
    PyTorch on the host with all cores, on a bounded sample of the step: once
    computing in fp32 and once in the activation dtype."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    weights = _cpu_weights()
    v32, n32, t32 = _cpu_sample(weights, torch.float32, sample_seconds, 64)
    v16, n16, t16 = _cpu_sample(weights, DTYPE, sample_seconds, 64)
    return {"value": v32, "unit": "GB/s", "cores": threads, "kind": "port", "cpu": cpu_model(),
            "value_act_dtype": v16,
            "sample": (f"{n32} of the step's 16 projection GEMMs in order, dequantise + fp32 matmul per call, "
                       f"{t32:.1f} s; value_act_dtype: {n16} GEMMs dequantised and multiplied in bf16, {t16:.1f} s")}


def bench_config(world: int) -> dict:
    return {"workload": "llama3_8b_awq_decode_projections", "group_size": G,
            "batch_sizes": list(MS), "projections": {k: list(v) for k, v in SHAPES.items()},
            "parallelism": f"tp{world}",
            "l2": "one weight copy per batch size: 453 MB of distinct weights per step > 126 MB L2, no flush"}


def run_reference(args):
    """The reference's own math for this path (dequantise + matmul, the oracle
    port) on the host cores, timed on the same 16-GEMM step."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle.awq_ref import cpu_awq_linear

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    weights = _cpu_weights()
    order = [(n, M) for M in MS for n in SHAPES]
    gx = torch.Generator().manual_seed(7)
    xs = {(n, M): torch.randn((M, SHAPES[n][0]), generator=gx).to(DTYPE) for (n, M) in order}

    def step():
        for (n, M) in order:
            cpu_awq_linear(xs[(n, M)], *weights[n], G)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    b = sum(awq_bytes(*SHAPES[n]) for (n, _) in order) * args.steps
    v = b / dt / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": dict(bench_config(world), same_config=True),
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port", "cpu": cpu_model(),
                         "sample": "the whole 16-GEMM step per timed step, dequantise + fp32 matmul per GEMM"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# --------------------------------------------------------------- helpers on the GPU
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


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _same_on_all_ranks(y: torch.Tensor, world: int) -> bool:
    if world == 1:
        return True
    import torch.distributed as dist

    h = hashlib.sha1(y.contiguous().view(torch.uint8).cpu().numpy().tobytes()).hexdigest()
    got = [None] * world
    dist.all_gather_object(got, h)
    return all(g == got[0] for g in got)


class _Parity:
    def __init__(self):
        self.cases = []
        self.ok = True

    def add(self, name: str, err: float, identical: bool = True):
        good = err <= PARITY_TOL and identical
        self.ok &= good
        self.cases.append({"case": name, "rel_err": round(err, 6), "ranks_identical": identical, "ok": good})

    def summary(self):
        return {"pass": self.ok, "tol": PARITY_TOL, "cases": len(self.cases),
                "max_rel_err": max((c["rel_err"] for c in self.cases), default=None),
                "failed": [c for c in self.cases if not c["ok"]],
                "reference": "PyTorch fp32 dequantise-then-matmul of the unsharded weights, 256-column slices"}


def _row_parallel_paths(ex, comm, world):
    """Exchange paths a row-parallel projection is checked on at N > 1."""
    paths = []
    if ex is not None:
        paths += [("fused_all_to_all", "all_to_all"), ("fused_reduce_scatter", "reduce_scatter")]
    if comm is not None:
        paths.append(("nccl", None))
    return paths if world > 1 else [("local", None)]


def _run_projection(name, x, w, ex, comm, path, out=None, row_parallel=ROW_PARALLEL):
    from sglite_b200 import ops

    K, N = w["_input_size"], w["_output_size"]
    if name in row_parallel and path is not None and path.startswith("fused"):
        return ex.gemm_allreduce(x, w["qweight"], K, N, G, out=out)
    y = ops.gemm(x, w["qweight"], K, N, G, out=out)
    if name in row_parallel and comm is not None:
        comm.all_reduce(y)
    return y


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

        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
        comm = init_nccl(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                         max_size_bytes=256 * 8192 * 2)
        if args.allreduce == "fused":
            ex = init_peer_exchange(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                                    max_rows=max(MS), max_n=8192)

    cfg = AWQB200Config(4, G, True)
    method = cfg.get_linear_method()
    # one weight copy per batch size (same full tensors on every rank, then sharded)
    layers = {}
    full0 = {}
    for ci, M in enumerate(MS):
        for i, name in enumerate(SHAPES):
            K, N = SHAPES[name]
            full = full_awq(K, N, dev, seed=100 * ci + i)
            w = method.create_weights(*local_shape(name, world))
            w.update(shard(full, name, rank, world))
            layers[(name, M)] = method.process_weights_after_loading(w)
            if ci == 0:
                full0[name] = full
            del full
    torch.cuda.synchronize()

    # ---- parity before timing: every projection at M = 1 and 64 on every path
    par = _Parity()
    for name in SHAPES:
        K, N = SHAPES[name]
        Kl, Nl = local_shape(name, world)
        for M in (1, 64):
            gx = torch.Generator(device=dev).manual_seed(1000 + M)
            xf = torch.randn((M, K), generator=gx, device=dev).to(DTYPE)
            w = layers[(name, MS[0])]
            if name in ROW_PARALLEL:
                xl = xf[:, rank * Kl:(rank + 1) * Kl].contiguous()
                ref = torch_ref_cols(xf, full0[name], N - 256, N)
                for pname, mode in _row_parallel_paths(ex, comm, world):
                    if mode is not None:
                        ex.set_mode(mode)
                    y = _run_projection(name, xl, w, ex, comm, pname)
                    par.add(f"{name}@M{M}/{pname}", rel_err(y[:, N - 256:], ref), _same_on_all_ranks(y, world))
            else:
                c0 = rank * Nl
                ref = torch_ref_cols(xf, full0[name], c0, c0 + 256)
                y = _run_projection(name, xf, w, ex, comm, None)
                par.add(f"{name}@M{M}/rank{rank}", _max_over_ranks(rel_err(y[:, :256], ref), world))
    if ex is not None:
        ex.set_mode(args.tp_mode)
    del full0
    torch.cuda.synchronize()

    gx = torch.Generator(device=dev).manual_seed(7 + rank)
    order = [(n, M) for M in MS for n in SHAPES]
    xs = {(n, M): torch.randn((M, local_shape(n, world)[0]), generator=gx, device=dev).to(DTYPE) for (n, M) in order}
    ys = {(n, M): torch.empty((M, local_shape(n, world)[1]), device=dev, dtype=DTYPE) for (n, M) in order}
    path = "fused" if ex is not None else None

    def step():
        for key in order:
            _run_projection(key[0], xs[key], layers[key], ex, comm, path, out=ys[key])

    def gemms_only():
        for key in order:
            w = layers[key]
            ops.gemm(xs[key], w["qweight"], w["_input_size"], w["_output_size"], G, out=ys[key])

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
    ms = _max_over_ranks(start.elapsed_time(end), world)
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

    e2e_ms, h2d, d2h = _e2e(args, world, dev, method, layers, xs, ys, ex, comm, barrier)

    step_bytes_full = sum(awq_bytes(*SHAPES[n]) for n in SHAPES) * len(MS)  # whole job (all ranks)
    value = step_bytes_full * args.steps / (ms / 1e3) / 1e9
    e2e_value = step_bytes_full * args.steps / (e2e_ms / 1e3) / 1e9
    # roofline of the GEMM kernels: algorithmic bytes per launch / mean launch time
    algo = sum(algo_bytes(M, *local_shape(n, world)) for (n, M) in order)
    achieved = algo * args.steps / (gemm_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak_hbm()
    traffic = profiled_traffic()
    extra = {}
    if not args.no_extras:
        extra = run_extras(args, rank, world, dev, comm, ex)
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
        "parity": par.summary(),
        "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "AWQB200LinearMethod.apply_weights (fused GEMM + all-reduce at N > 1) captured in a "
                        "CUDA graph over static buffers; one pinned H2D copy of the 16 activations, replay, "
                        "one D2H copy of the 16 outputs per step, double-buffered on copy streams"},
        "gpu_launches": len(order) * args.steps,
        "graph": "one CUDA-graph replay per step (16 GEMM launches)",
        "allreduce": ("none" if world == 1 else
                      f"fused into the row-parallel GEMM over peer memory ({args.tp_mode})" if ex is not None
                      else "NCCL"),
        "clocks": clk.summary(),
        "extra": extra,
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
    if not par.ok or err:
        sys.exit(3)


def _e2e(args, world, dev, method, layers, xs, ys, ex, comm, barrier):
    """e2e through the linear-method API: pinned host activations in, outputs
    back to the host, every step. The step's 16 calls (apply_weights, or the
    fused GEMM + all-reduce for the row-parallel projections at N > 1) are
    captured once per input buffer into a CUDA graph over static device
    buffers, as the reference's decode runner does (model_executor/
    cuda_graph.py:119-177: static inputs, copy in, replay). Every step copies
    all 16 activations from one pinned host buffer into the static inputs (one
    copy), replays the graph, and copies all 16 outputs back into one pinned
    host buffer (one copy). Copies run on their own streams (one per direction)
    and both sides are double-buffered across steps, so the PCIe transfers of
    one step overlap the GEMMs of the next."""
    keys = [(n, M) for M in MS for n in SHAPES]
    nbuf = 2
    nin = sum(xs[k].numel() for k in keys)
    nout = sum(ys[k].numel() for k in keys)
    src = torch.cat([xs[k].reshape(-1) for k in keys]).cpu()
    hx = [src.clone().pin_memory() for _ in range(nbuf)]
    hy = [torch.empty(nout, dtype=DTYPE).pin_memory() for _ in range(nbuf)]
    dxg = [torch.empty(nin, dtype=DTYPE, device=dev) for _ in range(nbuf)]
    dyg = [torch.empty(nout, dtype=DTYPE, device=dev) for _ in range(nbuf)]
    dx, dy = [{} for _ in range(nbuf)], [{} for _ in range(nbuf)]
    for b in range(nbuf):
        oi = oo = 0
        for k in keys:
            dx[b][k] = dxg[b][oi:oi + xs[k].numel()].view(xs[k].shape)
            dy[b][k] = dyg[b][oo:oo + ys[k].numel()].view(ys[k].shape)
            oi += xs[k].numel()
            oo += ys[k].numel()
    h2d, d2h = nin * 2, nout * 2

    def calls(b):
        for k in keys:
            n = k[0]
            if ex is not None and n in ROW_PARALLEL:
                w = layers[k]
                ex.gemm_allreduce(dx[b][k], w["qweight"], w["_input_size"], w["_output_size"], G, out=dy[b][k])
            else:
                method.apply_weights(layers[k], dx[b][k], out=dy[b][k])
                if comm is not None and n in ROW_PARALLEL:
                    comm.all_reduce(dy[b][k])

    for b in range(nbuf):  # eager once: workspaces sized, kernels loaded
        dxg[b].copy_(hx[b])
        calls(b)
    torch.cuda.synchronize(dev)
    barrier()
    graphs = []
    for b in range(nbuf):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            calls(b)
        graphs.append(g)
    torch.cuda.synchronize(dev)
    barrier()
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]
    ev_used = [torch.cuda.Event() for _ in range(nbuf)]
    ev_out = [torch.cuda.Event() for _ in range(nbuf)]
    fresh = [True] * nbuf
    step_no = [0]

    def e2e_step():
        b = step_no[0] % nbuf
        step_no[0] += 1
        compute = torch.cuda.current_stream(dev)
        with torch.cuda.stream(s_in):
            if not fresh[b]:
                s_in.wait_event(ev_used[b])  # the replay two steps back is done with this buffer
            dxg[b].copy_(hx[b], non_blocking=True)
            ev_in[b].record(s_in)
        compute.wait_event(ev_in[b])
        if not fresh[b]:
            compute.wait_event(ev_out[b])  # its outputs two steps back have left
        graphs[b].replay()
        ev_used[b].record(compute)
        s_out.wait_event(ev_used[b])
        with torch.cuda.stream(s_out):
            hy[b].copy_(dyg[b], non_blocking=True)
            ev_out[b].record(s_out)
        fresh[b] = False

    def e2e_drain():
        torch.cuda.current_stream(dev).wait_stream(s_in)
        torch.cuda.current_stream(dev).wait_stream(s_out)

    for _ in range(args.warmup):
        e2e_step()
    e2e_drain()
    torch.cuda.synchronize(dev)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e2e_drain()  # the timed region ends when the last output is on the host
    e1.record()
    torch.cuda.synchronize(dev)
    barrier()
    del graphs  # graphs that hold collectives go before the process group
    torch.cuda.synchronize(dev)
    return _max_over_ranks(e0.elapsed_time(e1), world), h2d, d2h


# --------------------------------------------------------------- other configs
def _linear(K, N, dev, dtype, seed, full=None):
    from sglite_b200.quantization import AWQB200Config

    m = AWQB200Config(4, G, True).get_linear_method()
    w = m.create_weights(K, N)
    w.update(full if full is not None else full_awq(K, N, dev, seed, dtype))
    return m, m.process_weights_after_loading(w)


def tp70b_layer(args, rank, world, dev, comm, ex, par=None):
    """Config 3: Llama-3.1-70B layer projections under TP = world; the O and
    down outputs are all-reduced (fused over peer memory up to the exchange's
    rows, NCCL above). Returns per-M layer time and its ratio to the roofline
    max(weight bytes / HBM, flops / sustained bf16 peak) + 2 ring all-reduces
    at the measured 770 GB/s peer bandwidth."""
    hbm, _, tflops_sus, kind = _peaks()
    loc = {n: local_shape(n, world, LLAMA70B) for n in LLAMA70B}
    ws = {}
    for i, n in enumerate(LLAMA70B):
        K, N = LLAMA70B[n]
        full = full_awq(K, N, dev, seed=500 + i)
        Kl, Nl = loc[n]
        _, ws[n] = _linear(Kl, Nl, dev, DTYPE, 0, full=shard(full, n, rank, world))
        if par is not None and n == "o":
            # the row-parallel projection against the unsharded weights: fused at
            # M = 1 (if there is an exchange), NCCL at M = 256
            for M in (1, 256):
                gx = torch.Generator(device=dev).manual_seed(2000 + M)
                xf = torch.randn((M, K), generator=gx, device=dev).to(DTYPE)
                xl = xf[:, rank * Kl:(rank + 1) * Kl].contiguous()
                use_fused = ex is not None and M <= ex.max_rows
                y = _run_projection(n, xl, ws[n], ex, comm, "fused" if use_fused else None)
                ref = torch_ref_cols(xf, full, N - 256, N)
                par.add(f"llama70b_o@M{M}/{'fused' if use_fused else ('nccl' if world > 1 else 'local')}",
                        rel_err(y[:, N - 256:], ref), _same_on_all_ranks(y, world))
        del full
    out = {}
    clk = ClockSampler(dev.index)
    clk.__enter__()
    try:
        for M in (1, 32, 256, 4096):
            xs = {n: torch.randn((M, K), device=dev).to(DTYPE) for n, (K, N) in loc.items()}
            ys = {n: torch.empty((M, N), device=dev, dtype=DTYPE) for n, (K, N) in loc.items()}
            use_fused = ex is not None and M <= ex.max_rows

            def layer():
                for n in loc:
                    _run_projection(n, xs[n], ws[n], ex, comm, "fused" if use_fused else None, out=ys[n])

            if world > 1:
                import torch.distributed as dist

                dist.barrier()
            us = _max_over_ranks(_graph_us(layer, args.warmup, args.steps), world)
            wbytes = sum(awq_bytes(K, N) for K, N in loc.values())
            flops = sum(2.0 * M * K * N for K, N in loc.values())
            ring = 2 * (world - 1) / world * M * 8192 * 2 if world > 1 else 0.0
            roof_us = max(wbytes / hbm / 1e3, flops / tflops_sus / 1e6) + 2 * ring / 770e3
            out[f"M{M}"] = {"layer_us": round(us, 2), "roofline_us": round(roof_us, 2),
                            "ratio": round(us / roof_us, 2),
                            "allreduce": "fused" if use_fused else ("nccl" if world > 1 else "none")}
    finally:
        clk.__exit__(None, None, None)
    return {"workload": f"llama3.1_70b_awq_layer_tp{world} (config 3)", "unit": "us", "per_m": out,
            "roofline": "max(weight bytes / measured HBM, flops / measured sustained bf16) + 2 ring all-reduces "
                        "at 770 GB/s", "peak_kind": kind, "clocks": clk.summary()}


def prefill_set(args, dev):
    """Config 2: Qwen3-4B AWQ projections at M = 512, 2048, 8192 (fp16)."""
    from sglite_b200 import ops

    _, tflops_peak, tflops_sus, kind = _peaks()
    rows = {}
    tot_flop = tot_us = 0.0
    clk = ClockSampler(dev.index)
    clk.__enter__()
    try:
        for i, (n, (K, N)) in enumerate(QWEN3_4B.items()):
            _, w = _linear(K, N, dev, torch.float16, 700 + i)
            for M in (512, 2048, 8192):
                x = torch.randn((M, K), device=dev).to(torch.float16)
                y = torch.empty((M, N), device=dev, dtype=torch.float16)
                us = _graph_us(lambda: ops.gemm(x, w["qweight"], K, N, G, out=y), args.warmup, args.steps)
                fl = 2.0 * M * N * K
                rows[f"{n}@M{M}"] = {"us": round(us, 2), "tflops": round(fl / us / 1e6, 1),
                                     "frac_sustained": round(fl / us / 1e6 / tflops_sus, 3)}
                tot_flop += fl
                tot_us += us
    finally:
        clk.__exit__(None, None, None)
    value = tot_flop / tot_us / 1e6
    return {"workload": "qwen3_4b_awq_prefill (config 2)", "metric": "W4A16 GEMM TFLOP/s", "value": value,
            "unit": "TFLOP/s", "peak_sustained": tflops_sus, "frac_sustained": value / tflops_sus,
            "peak_burst": tflops_peak, "frac_burst": value / tflops_peak, "peak_kind": kind,
            "per_gemm": rows, "dtype": "fp16", "clocks": clk.summary()}


def moe_layer(args, rank, world, dev, comm, par=None):
    """Config 4: Qwen3-30B-A3B AWQ MoE layer at M = 16, 256, 4096; with N > 1
    ranks each rank holds E / N experts (expert parallelism) and the [M, 2048]
    output is all-reduced over NCCL (layers/moe_layer.py:62-63)."""
    from sglite_b200.moe import AWQB200MoeBackend, AWQExpertWeights

    E, k, H, I = 128, 8, 2048, 768
    el = E // world
    e0 = rank * el
    f1 = full_awq(H, 2 * I, dev, 900, lead=(E,))
    f2 = full_awq(I, H, dev, 901, lead=(E,))
    w1 = AWQExpertWeights.from_awq(*(f1[key][e0:e0 + el].contiguous() for key in ("qweight", "qzeros", "scales")),
                                   G, e_begin=e0, num_global_experts=E, gate_up=True)
    w2 = AWQExpertWeights.from_awq(*(f2[key][e0:e0 + el].contiguous() for key in ("qweight", "qzeros", "scales")),
                                   G, e_begin=e0, num_global_experts=E)
    backend = AWQB200MoeBackend()
    hbm, tflops_peak, tflops_sus, kind = _peaks()

    def layer(buf, lg):
        backend.forward(buf, w1, w2, lg, k, True)
        if comm is not None:
            comm.all_reduce(buf)

    if par is not None:
        # 4 tokens of an M = 16 batch against a PyTorch fp32 reference of the
        # full (all-expert) layer
        M = 16
        x = torch.randn((M, H), generator=torch.Generator(device=dev).manual_seed(3), device=dev).to(DTYPE)
        lg = torch.randn((M, E), generator=torch.Generator(device=dev).manual_seed(4), device=dev)
        buf = x.clone()
        layer(buf, lg)
        p = torch.softmax(lg.float(), dim=-1)
        tw, ti = torch.topk(p, k, dim=-1)
        tw = tw / tw.sum(-1, keepdim=True)
        tw = tw / (tw.sum(-1, keepdim=True) + 1e-8)
        ref = torch.zeros((4, H), dtype=torch.float32, device=dev)
        for t in range(4):
            for j in range(k):
                e = int(ti[t, j])
                sel1 = {key: f1[key][e] for key in ("qweight", "qzeros", "scales")}
                sel2 = {key: f2[key][e] for key in ("qweight", "qzeros", "scales")}
                h1 = torch_ref_cols(x[t:t + 1], sel1, 0, 2 * I)
                a = (torch.nn.functional.silu(h1[:, :I]) * h1[:, I:]).to(DTYPE)
                ref[t] += (torch_ref_cols(a, sel2, 0, H) * tw[t, j])[0]
        par.add(f"moe@M16/ep{world}", rel_err(buf[:4], ref), _same_on_all_ranks(buf, world))
    del f1, f2
    per = {}
    clk = ClockSampler(dev.index)
    clk.__enter__()
    try:
        for M in (16, 256, 4096):
            x = torch.randn((M, H), device=dev).to(DTYPE)
            lg = torch.randn((M, E), device=dev)
            buf = x.clone()
            if world > 1:
                import torch.distributed as dist

                dist.barrier()
            us = _max_over_ranks(_graph_us(lambda: layer(buf, lg), args.warmup, args.steps), world)
            _, ids = torch.topk(lg, k, dim=-1)
            touched = int(torch.unique(ids).numel())
            wbytes = touched * (awq_bytes(H, 2 * I) + awq_bytes(I, H))
            flops = 2.0 * M * k * (H * 2 * I + I * H)
            per[f"M{M}"] = {"us": round(us, 2), "experts_touched": touched,
                            "weight_GBps": round(wbytes / us / 1e3, 1), "tflops": round(flops / us / 1e6, 1)}
    finally:
        clk.__exit__(None, None, None)
    return {"workload": f"qwen3_30b_a3b_awq_moe (config 4), {el} experts per rank x {world}", "unit": "us",
            "per_m": per, "allreduce": "nccl" if comm is not None else "none", "peak_hbm_GBps": hbm,
            "peak_kind": kind, "clocks": clk.summary()}


def run_extras(args, rank, world, dev, comm, ex):
    par = _Parity()
    out = {"config3": tp70b_layer(args, rank, world, dev, comm, ex, par)}
    torch.cuda.empty_cache()
    out["config4"] = moe_layer(args, rank, world, dev, comm, par)
    torch.cuda.empty_cache()
    if world == 1:
        out["config2"] = prefill_set(args, dev)
    out["parity"] = par.summary()
    return out


def run_prefill(args):
    print(json.dumps(prefill_set(args, torch.device("cuda", 0))), flush=True)


def run_single(args):
    """Config 0: one K=N=4096 projection at M=16 (fp16)."""
    from sglite_b200 import ops

    dev = torch.device("cuda", 0)
    K = N = 4096
    M = 16
    copies = [_linear(K, N, dev, torch.float16, s)[1] for s in range(32)]  # 290 MB: no L2 reuse
    x = torch.randn((M, K), device=dev).to(torch.float16)
    y = torch.empty((M, N), device=dev, dtype=torch.float16)
    us = _graph_us(lambda: [ops.gemm(x, w["qweight"], K, N, G, out=y) for w in copies], args.warmup, args.steps,
                   reps=1) / len(copies)
    hbm, _, _, kind = _peaks()
    b = algo_bytes(M, K, N)
    print(json.dumps({"workload": "single K=N=4096 M=16 (config 0)", "metric": "GEMM us", "value": us,
                      "unit": "us", "weight_GBps": awq_bytes(K, N) / us / 1e3, "algo_GBps": b / us / 1e3,
                      "frac_hbm": b / us / 1e3 / hbm, "peak_kind": kind}), flush=True)


def run_shapes(args):
    """Each decode projection alone at each M, graph-replayed over rotating
    weight copies that total more than twice the L2 (so every launch streams
    its weights from DRAM): per-launch us, weight GB/s and the fraction of the
    measured HBM bandwidth."""
    from sglite_b200 import ops

    dev = torch.device("cuda", 0)
    hbm, _, _, kind = _peaks()
    out = {}
    for i, (name, (K, N)) in enumerate(SHAPES.items()):
        n_copies = max(2, (300 << 20) // awq_bytes(K, N) + 1)
        copies = [_linear(K, N, dev, DTYPE, 10 * i + c)[1] for c in range(n_copies)]
        for M in MS:
            x = torch.randn((M, K), device=dev).to(DTYPE)
            y = torch.empty((M, N), device=dev, dtype=DTYPE)
            us = _graph_us(lambda: [ops.gemm(x, w["qweight"], K, N, G, out=y) for w in copies], args.warmup,
                           args.steps, reps=1) / n_copies
            out[f"{name}@M{M}"] = {"us": round(us, 2), "weight_GBps": round(awq_bytes(K, N) / us / 1e3, 1),
                                   "frac_hbm": round(algo_bytes(M, K, N) / us / 1e3 / hbm, 3),
                                   "plan": ops.gemm_plan(M, K, N, G)}
        del copies
        torch.cuda.empty_cache()
    print(json.dumps({"workload": "llama3_8b decode projections, one at a time", "unit": "us", "per_gemm": out,
                      "peak_hbm_GBps": hbm, "peak_kind": kind}), flush=True)


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


def _dist_setup(args, max_rows=64):
    import torch.distributed as dist

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = ex = None
    if world > 1:
        from datetime import timedelta

        from sglite_b200.distributed import init_nccl, init_peer_exchange

        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
        comm = init_nccl(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                         max_size_bytes=256 * 8192 * 2)
        if args.allreduce == "fused":
            ex = init_peer_exchange(tp_rank=rank, tp_size=world, tp_cpu_group=dist.group.WORLD, device=dev,
                                    max_rows=max_rows, max_n=8192)
            ex.set_mode(args.tp_mode)
    return rank, world, dev, comm, ex


def _dist_teardown(world, comm, ex):
    if ex is not None:
        ex.destroy()
    if comm is not None:
        comm.destroy()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


def run_tp70b(args):
    rank, world, dev, comm, ex = _dist_setup(args)
    par = _Parity()
    r = tp70b_layer(args, rank, world, dev, comm, ex, par)
    r["parity"] = par.summary()
    if rank == 0:
        print(json.dumps(r), flush=True)
    _dist_teardown(world, comm, ex)


def run_moe(args):
    rank, world, dev, comm, ex = _dist_setup(args)
    par = _Parity()
    r = moe_layer(args, rank, world, dev, comm, par)
    r["parity"] = par.summary()
    if rank == 0:
        print(json.dumps(r), flush=True)
    _dist_teardown(world, comm, ex)


def run_norm(args):
    """Residual-add RMSNorm after the row-parallel projections (the reference's
    RMSNormFused, layers/norm.py:28-47), hidden 8192 (config 3), bf16. HBM-bound:
    algorithmic bytes = 4 * M * N * 2 (read x and residual, write both) + N * 2."""
    from sglite_b200 import ops

    dev = torch.device("cuda", 0)
    N = 8192
    hbm, _, _, kind = _peaks()
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
    ap.add_argument("--no-extras", action="store_true", help="skip configs 2-4 in the default line")
    ap.add_argument("--workload", default="decode",
                    choices=["decode", "prefill", "single", "tp70b", "moe", "gemm", "norm", "shapes"],
                    help="decode (default, the contract line) or another BASELINE config alone")
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
    elif args.workload == "shapes":
        run_shapes(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
