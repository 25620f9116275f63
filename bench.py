"""Benchmark of the ConvRot INT8 linear hot path on B200.

Metric: "ConvRot int8 linear TOPS @M=2048,K=1280,N=10240;
rotate+quant HBM GB/s".  One step is one INT8 ConvRot linear forward over one
batch: rotate+quantize bf16 x [2048,1280] -> int8, then the tcgen05 int8 GEMM
against the pre-rotated int8 weight [10240,1280] with the dequant epilogue
fused -> bf16 [2048,10240] (the SDXL GEGLU up-projection shape, config C3/W1).

Timing: the K = --steps steps of a timed region are replayed from CUDA graphs
of exactly those launches (a graph of min(K, 600) steps, replayed, plus a graph
of the remainder); the region is repeated R times back to back on the stream,
each repetition timed by its own CUDA events, R chosen so the repetitions
cover about 2.5 s (the clock sampler's window); ``ms_per_step`` is the median
repetition / K, max over ranks.  ``value`` = 2*M*N*K ops x ranks / that time,
in TOPS; inputs resident in HBM, six rotating buffer sets (x, weight, scales,
output: 378 MB in all, three times the 126 MB L2) so no step reads the
L2-resident leftovers of the previous one.

Also reported on the same line:
* ``roofline``: the GEMM kernel alone (its average launch time by CUDA
  events), achieved int8 TOPS against the int8 dense peak (2x the measured
  bf16 cuBLAS burst of MEASURED_PEAKS.json) and against cuBLASLt's int8 GEMM
  measured here at 8192^3, with the DRAM traffic of one launch from the
  committed ncu summary;
* ``rotate_quant``: the rotate+quantize kernel at config C5 (x [65536,4096],
  3*M*K + 4*M = 805.6 MB per launch) in HBM GB/s against the measured copy
  bandwidth -- the metric's second half;
* ``c5_mshard``: config C5 (x [65536,4096]) M-sharded over the ranks with the
  [4096,4096] and [14336,4096] weights replicated: whole-job TOPS, strong
  scaling (no collective on the data path);
* ``c5_nshard`` (N > 1): config C5's N-sharded variant, the [14336,4096]
  weight split by output channels with the output all-gather fused into the
  GEMM epilogue (peer stores over NVLink), and the NCCL form;
* ``e2e``: the same step through the public API ``xpu_kernels.linear`` with x
  copied from pinned host memory and the bf16 result copied back each step;
* ``cpu_baseline``: the reference's own CPU path (reference/convrot_linear.py's
  op sequence with torch._int_mm, the Hadamard in place of its identity
  placeholder), restated in oracle/convrot_torch_cpu.py, on the full workload;
* ``other_configs`` (one GPU): the other BASELINE configs through the public
  API, device time per call from CUDA graphs -- C1 and one C2 linear, the C3
  GEGLU FFN, C4's int8 dx and dW.

``--impl reference`` times that same CPU path on the host cores (the
reference's device library is SYCL for Intel GPUs and does not build here) on
the same metric, unit and workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "oko-xpu-kernels_b200"))
sys.path.insert(0, ROOT)

M, K, N = 2048, 1280, 10240
OPS = 2.0 * M * N * K
METRIC = "ConvRot int8 linear TOPS @M=2048,K=1280,N=10240; rotate+quant HBM GB/s"
NSETS = 6
C5_M, C5_K = 65536, 4096
C5_BYTES = 3 * C5_M * C5_K + 4 * C5_M
WORKLOAD = ("linear(x bf16 [2048,1280]) -> rotate+quantize -> tcgen05 int8 GEMM with fused "
            "dequant -> bf16 [2048,10240] (config C3 W1, SDXL GEGLU up-projection)")


class _stdout_to_stderr:
    """File descriptor 1 pointed at stderr for the duration (C libraries included)."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _committed_traffic():
    """DRAM bytes per GEMM launch from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "gemm_i8_dequant_C3W1.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
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
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------------------- CPU arms

REF_SAMPLE = ("the reference's CPU path: reference/convrot_linear.py:5-23's op sequence "
              "(bf16 group matmul with the Hadamard, row abs-max scale, round/clamp, "
              "torch._int_mm against the transposed int8 weight, bf16 dequant), restated in "
              "torch in oracle/convrot_torch_cpu.py, on the full M=2048 x K=1280 x N=10240 "
              "workload per step")


def _cpu_inputs(rows, seed=2):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, K, generator=g)
    x[:, :13] *= 10
    x = x.to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
    return x, w, bias


def _cpu_reference_setup():
    """The workload for the reference's CPU path: x, the prepared int8 weight
    (prepare_weight's format, made by the numpy oracle once, untimed)."""
    from oracle import convrot_oracle as O
    from oracle import convrot_torch_cpu as T
    x, w, bias = _cpu_inputs(M)
    w8, ws = O.prepare_weight(w.view(torch.int16).numpy().view(np.uint16))
    return x, torch.from_numpy(w8), torch.from_numpy(ws), bias, T.hadamard_bf16(), T


def cpu_reference_rate(budget_s: float):
    """TOPS of the reference's CPU path on the full workload, repeated for
    about `budget_s` seconds with every host thread."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    x, w8, ws, bias, h, T = _cpu_reference_setup()
    T.convrot_int8_linear_cpu(x, w8, ws, bias, h=h)  # warm the thread pool
    reps, t0 = 0, time.perf_counter()
    while True:
        T.convrot_int8_linear_cpu(x, w8, ws, bias, h=h)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return OPS * reps / el / 1e12, reps, el, cores


def cpu_numpy_oracle_rate(rows: int, budget_s: float):
    """TOPS of the numpy oracle's forward (the bit-exact restatement of the
    kernels' arithmetic) on `rows` rows of the workload, for context."""
    from oracle import convrot_oracle as O
    x, w, _ = _cpu_inputs(rows)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    w8, ws = O.prepare_weight(w.view(torch.int16).numpy().view(np.uint16))
    O.linear(xb[:8], w8, ws)
    reps, t0 = 0, time.perf_counter()
    while True:
        O.linear(xb, w8, ws)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return 2.0 * rows * N * K * reps / el / 1e12, reps, el


def run_reference(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return 0
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    x, w8, wsc, bias, h, T = _cpu_reference_setup()
    for _ in range(max(1, args.warmup)):
        T.convrot_int8_linear_cpu(x, w8, wsc, bias, h=h)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        T.convrot_int8_linear_cpu(x, w8, wsc, bias, h=h)
    el = time.perf_counter() - t0
    value = OPS * args.steps / el / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TOPS",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,1) x with 1% outlier channels x10, N(0,0.02) W)",
        "config": {"workload": WORKLOAD, "M": M, "K": K, "N": N},
        "cpu_baseline": {"value": value, "unit": "TOPS", "cores": cores, "kind": "port",
                         "sample": REF_SAMPLE},
        "e2e": {"value": value, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference's device library is SYCL for Intel Xe2 and cannot be built or "
                 "run here; its plain-PyTorch CPU path is timed (the op sequence of "
                 "reference/convrot_linear.py, restated because the reference tree does not "
                 "travel to the GPU box)"),
    }
    print(json.dumps(line))
    return 0


# --------------------------------------------------------------------------- GPU arm

def run_gpu(args):
    import xpu_kernels
    from xpu_kernels.int8 import _lib as L

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        # NCCL may print its version on stdout while it sets up the
        # communicator; stdout carries only the result line
        with _stdout_to_stderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=dev)
            dist.barrier()
    lib = L._lib()
    stream = torch.cuda.current_stream(dev)

    # inputs: six buffer sets, each its own x, weight, scales and output
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    sets = []
    for i in range(NSETS):
        x = torch.randn(M, K, generator=g, device=dev)
        x[:, :13] *= 10  # 1 % outlier channels, as config C2 specifies
        x = x.to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w8, wsc = xpu_kernels.prepare_weight(w)
        bias = torch.randn(N, generator=g, device=dev) * 0.01
        sets.append(dict(x=x, w8=w8, ws=wsc, bias=bias,
                         out=torch.empty(M, N, dtype=torch.bfloat16, device=dev),
                         xq=torch.empty(M, K, dtype=torch.int8, device=dev),
                         xs=torch.empty(M, dtype=torch.float32, device=dev)))
    sptr = L._stream(dev)

    def step(s):
        rc = lib.xpuint8_linear_stream(sptr, L._ptr(s["x"]), L._ptr(s["w8"]), L._ptr(s["ws"]),
                                       L._ptr(s["bias"]), L._ptr(s["out"]), L._ptr(s["xq"]),
                                       L._ptr(s["xs"]), M, N, K, 0)
        if rc != 0:
            raise RuntimeError(lib.xpuint8_last_error())

    # correctness guard on the bench's own data: sampled rows against the oracle
    step(sets[0])
    torch.cuda.synchronize()
    if rank == 0:
        from oracle import convrot_oracle as O
        rows = torch.arange(0, M, 341, device=dev)
        xb = sets[0]["x"][rows].cpu().view(torch.int16).numpy().view(np.uint16)
        ref = O.linear(xb, sets[0]["w8"].cpu().numpy(), sets[0]["ws"].cpu().numpy(),
                       sets[0]["bias"].cpu().numpy())
        got = sets[0]["out"][rows].cpu().view(torch.int16).numpy().view(np.uint16)
        if not np.array_equal(got, ref):
            raise RuntimeError("bench output differs from the oracle on sampled rows")

    # CUDA graphs of exactly the timed launches (captured on a side stream):
    # one of min(K, 600) steps, replayed, and one of the remainder
    per_graph = min(args.steps, 600)
    full_reps, rest = divmod(args.steps, per_graph)
    capture_stream = torch.cuda.Stream(dev)

    def capture(nsteps):
        graph = torch.cuda.CUDAGraph()
        capture_stream.wait_stream(stream)
        with torch.cuda.stream(capture_stream):
            csptr = L._stream(dev)
            with torch.cuda.graph(graph, stream=capture_stream):
                for j in range(nsteps):
                    s = sets[j % NSETS]
                    rc = lib.xpuint8_linear_stream(csptr, L._ptr(s["x"]), L._ptr(s["w8"]),
                                                   L._ptr(s["ws"]), L._ptr(s["bias"]),
                                                   L._ptr(s["out"]), L._ptr(s["xq"]),
                                                   L._ptr(s["xs"]), M, N, K, 0)
                    if rc != 0:
                        raise RuntimeError(lib.xpuint8_last_error())
        stream.wait_stream(capture_stream)
        return graph

    graphs = [capture(per_graph)] + ([capture(rest)] if rest else [])
    torch.cuda.synchronize()

    def run_region():
        """exactly K steps: the main graph full_reps times, then the remainder"""
        for _ in range(full_reps):
            graphs[0].replay()
        if rest:
            graphs[1].replay()

    def barrier():
        if ws > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(max(3, args.warmup)):  # warm-up steps (untimed)
        step(sets[_ % NSETS])
    run_region()
    barrier()
    # R repetitions of the K-step region, sized on rank 0's first region and
    # agreed over the ranks (every rank runs the same number)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run_region()
    e1.record(stream)
    e1.synchronize()
    first_ms = e0.elapsed_time(e1)
    reps = int(min(5000, max(3, 2500.0 / max(first_ms, 1e-3))))
    if ws > 1:
        import torch.distributed as dist
        rt = torch.tensor([reps], device=dev, dtype=torch.int64)
        dist.all_reduce(rt, op=dist.ReduceOp.MAX)
        reps = int(rt.item())
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    with ClockSampler(local) as clk:
        barrier()
        for r in range(reps):
            starts[r].record(stream)
            run_region()
            ends[r].record(stream)
        ends[-1].synchronize()
        barrier()
    region_ms = torch.tensor([starts[r].elapsed_time(ends[r]) for r in range(reps)],
                             dtype=torch.float64, device=dev)
    if ws > 1:
        import torch.distributed as dist
        dist.all_reduce(region_ms, op=dist.ReduceOp.MAX)  # per repetition, the slowest rank
    region_ms = region_ms.cpu()
    t_ms = float(region_ms.median().item())
    value = OPS * args.steps * ws / (t_ms * 1e-3) / 1e12
    clocks = clk.summary()

    # eager launches (no graph) for context
    torch.cuda.synchronize()
    n_eager = min(args.steps, 600)
    e0.record(stream)
    for j in range(n_eager):
        step(sets[j % NSETS])
    e1.record(stream)
    e1.synchronize()
    eager_ms = e0.elapsed_time(e1) / n_eager

    result = {
        "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded N(0,1) x with 1% outlier channels x10, N(0,0.02) W, "
                "random-init weights prepared with prepare_weight)",
        "config": {"workload": WORKLOAD, "M": M, "K": K, "N": N, "per_rank_rows": M,
                   "parallelism": f"M-shard x{ws} (replicated weights, no collective)",
                   "l2": f"{NSETS} rotating buffer sets, "
                         f"{NSETS * (M * K * 3 + N * K + M * N * 2) / 1e6:.0f} MB > 126 MB L2",
                   "timing": (f"each timed region is exactly {args.steps} steps replayed from CUDA "
                              f"graphs of those launches; {reps} regions back to back, each timed "
                              f"by CUDA events (max over ranks); ms_per_step = median region / "
                              f"steps; eager launches in eager_ms_per_step")},
        "repeats": reps,
        "region_ms": {"median": t_ms, "min": float(region_ms.min().item()),
                      "max": float(region_ms.max().item())},
        "eager_ms_per_step": eager_ms,
        "gpu_launches": 2 * args.steps * reps,
        "clocks": clocks,
    }
    del graphs

    if rank == 0:
        result.update(_rank0_extras(args, lib, L, dev, sets, stream))
    del sets
    if rank == 0 and ws == 1:
        torch.cuda.empty_cache()
        result["other_configs"] = _other_configs(dev)
    torch.cuda.empty_cache()
    # config C5 at N ranks: M-sharded (every rank), then the N-sharded all-gather
    result["c5_mshard"] = _c5_mshard(args, dev, stream, ws, rank)
    if ws > 1:
        result["c5_nshard"] = _c5_nshard(args, dev, stream, ws, rank)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(result))
    return 0


def _timed_max(fn, steps, stream, ws, dev):
    """Device time of `steps` calls (ms), max over ranks, after a barrier."""
    import torch.distributed as dist
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        fn(i)
    e1.record(stream)
    e1.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _c5_mshard(args, dev, stream, ws, rank):
    """Config C5 M-sharded: 65536 rows of x [., 4096] split over the ranks, the
    [4096,4096] and [14336,4096] weights replicated; whole-job TOPS =
    2 * 65536 * N * 4096 / the slowest rank's time (strong scaling)."""
    import xpu_kernels
    from xpu_kernels.int8 import shard
    r0, r1 = shard.row_range(C5_M, ws, rank)
    g = torch.Generator(device=dev).manual_seed(40 + rank)
    x = torch.randn(r1 - r0, C5_K, generator=g, device=dev)
    x[:, :20] *= 20
    x = x.to(torch.bfloat16)
    out = {}
    steps = max(3, min(args.steps, 50))
    for n in (4096, 14336):
        gw = torch.Generator(device=dev).manual_seed(n)
        w = (torch.randn(n, C5_K, generator=gw, device=dev) * 0.02).to(torch.bfloat16)
        w8, wsc = xpu_kernels.prepare_weight(w)
        del w
        y = torch.empty(r1 - r0, n, dtype=torch.bfloat16, device=dev)
        xq = torch.empty(r1 - r0, C5_K, dtype=torch.int8, device=dev)
        xs = torch.empty(r1 - r0, dtype=torch.float32, device=dev)
        from xpu_kernels.int8 import _lib as L
        lib = L._lib()
        sp = L._stream(dev)

        def fn(_):
            rc = lib.xpuint8_linear_stream(sp, L._ptr(x), L._ptr(w8), L._ptr(wsc), None, L._ptr(y),
                                           L._ptr(xq), L._ptr(xs), r1 - r0, n, C5_K, 0)
            if rc != 0:
                raise RuntimeError(lib.xpuint8_last_error())
        for i in range(3):
            fn(i)
        t = _timed_max(fn, steps, stream, ws, dev) / steps
        out[f"w{n}"] = {"ms_per_step": t, "tops": 2.0 * C5_M * n * C5_K / (t * 1e-3) / 1e12,
                        "rows_per_rank": r1 - r0}
        del w8, wsc, y, xq, xs
    out["shape"] = (f"x bf16 [{C5_M},{C5_K}] split over {ws} rank(s) by rows; weights "
                    f"[4096,4096] and [14336,4096] replicated; {steps} steps timed, max over ranks")
    del x
    torch.cuda.empty_cache()
    return out


def _c5_nshard(args, dev, stream, ws, rank):
    """Config C5's N-sharded variant at N ranks: x [65536,4096] on every rank,
    [14336,4096] split by output channels; the fused form stores every output
    tile into every rank's buffer over NVLink (no multicast), the NCCL form
    all-gathers the blocks.  Whole-job TOPS, strong scaling."""
    import xpu_kernels
    from xpu_kernels.int8 import shard
    m, n = C5_M, 14336
    g = torch.Generator(device=dev).manual_seed(4)
    x = torch.randn(m, C5_K, generator=g, device=dev)
    x[:, :20] *= 20
    x = x.to(torch.bfloat16)
    w = (torch.randn(n, C5_K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w8, wsc = xpu_kernels.prepare_weight(w)
    del w
    w8l, wsl, _ = shard.shard_weight(w8, wsc, ws, rank)
    del w8, wsc
    peer = shard.PeerOutput(m, n)
    steps = max(3, min(args.steps, 20))
    try:
        y_f = shard.linear_nshard_fused(x, w8l, wsl, None, peer).clone()
        y_n = shard.linear_nshard(x, w8l, wsl, None, n_total=n)
        same = bool(torch.equal(y_f.view(torch.int16), y_n.view(torch.int16)))
        del y_f, y_n
        t_f = _timed_max(lambda i: shard.linear_nshard_fused(x, w8l, wsl, None, peer), steps,
                         stream, ws, dev) / steps
        t_n = _timed_max(lambda i: shard.linear_nshard(x, w8l, wsl, None, n_total=n), steps,
                         stream, ws, dev) / steps
    finally:
        peer.close()
    ops_ = 2.0 * m * n * C5_K
    return {"fused_allgather_ms": t_f, "fused_tops": ops_ / (t_f * 1e-3) / 1e12,
            "nccl_allgather_ms": t_n, "nccl_tops": ops_ / (t_n * 1e-3) / 1e12,
            "forms_bit_identical": same,
            "output_bytes_sent_per_rank": m * (n // ws) * 2 * (ws - 1),
            "shape": f"x bf16 [{m},{C5_K}] on every rank, W [{n},{C5_K}] split over {ws} ranks"}


def _graph_us(fn, n, reps=5):
    """Device time per call (us) of n calls captured in one CUDA graph, the
    graph replayed `reps` times between CUDA events (after eager warm-up)."""
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for i in range(n):
                fn(i)
    torch.cuda.current_stream().wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (reps * n)
    del graph
    return us


def _other_configs(dev):
    """The other BASELINE configs on one GPU through the public API (device
    time per call from CUDA graphs, warm, two rotating input sets; synthetic
    seeded inputs of the configs' shapes and distributions): C1 linear, one
    C2 projection, the C3 GEGLU FFN, and C4's int8 dx and dW."""
    import xpu_kernels as xk
    g = torch.Generator(device=dev).manual_seed(7)

    def bf(*shape, s=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * s).to(torch.bfloat16)

    out = {}
    for name, (m, k, n) in {"C1_linear": (256, 1024, 1024), "C2_linear": (2048, 1280, 1280)}.items():
        xs_ = [bf(m, k) for _ in range(2)]
        w8, wsc = xk.prepare_weight(bf(n, k, s=0.02))
        b = bf(n, s=0.01).float()
        us = _graph_us(lambda i: xk.linear(xs_[i % 2], w8, wsc, b), 20)
        out[name] = {"us": us, "tops": 2.0 * m * n * k / (us * 1e-6) / 1e12, "shape": [m, k, n]}
    m, k, inner = 2048, 1280, 5120
    xs_ = [bf(m, k) for _ in range(2)]
    up8, ups = xk.prepare_weight(bf(2 * inner, k, s=0.02))
    dn8, dns = xk.prepare_weight(bf(k, inner, s=0.02))
    us = _graph_us(lambda i: xk.ffn(xs_[i % 2], up8, ups, dn8, dns, act="geglu_erf"), 10)
    out["C3_ffn_geglu"] = {"us": us, "tops": (2.0 * m * 2 * inner * k + 2.0 * m * k * inner) / (us * 1e-6) / 1e12,
                           "shape": [m, k, inner]}
    m, k, n = 4096, 1280, 5120
    w8, wsc = xk.prepare_weight(bf(n, k, s=0.02))
    dys = [bf(m, n, s=1e-3) for _ in range(2)]
    xq, xsc = xk.quantize(bf(m, k))
    us = _graph_us(lambda i: xk.linear_dx_int8(dys[i % 2], w8, wsc), 10)
    out["C4_dx_int8"] = {"us": us, "tops": 2.0 * m * n * k / (us * 1e-6) / 1e12, "shape": [m, k, n]}
    us = _graph_us(lambda i: xk.linear_dw_int8(dys[i % 2], xq, xsc), 10)
    out["C4_dw_int8"] = {"us": us, "tops": 2.0 * m * n * k / (us * 1e-6) / 1e12, "shape": [m, k, n]}
    out["timing"] = ("device time per call: calls captured in a CUDA graph, replayed between CUDA "
                     "events, two rotating input sets; shapes [M, K, N] (C3: [M, K, inner])")
    return out


def _time_launches(fn, n, stream):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for i in range(n):
        fn(i)
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / n


def _rank0_extras(args, lib, L, dev, sets, stream):
    import xpu_kernels
    peaks, src = _peaks()
    sptr = L._stream(dev)
    out = {}

    # the GEMM alone: the dominant kernel (inputs already quantized)
    for s in sets:
        lib.xpuint8_convrot_quantize_stream(sptr, L._ptr(s["x"]), L._ptr(s["xq"]), L._ptr(s["xs"]),
                                            M, K)

    def gemm(i):
        s = sets[i % NSETS]
        lib.xpuint8_int_mm_dequant_stream(sptr, L._ptr(s["xq"]), L._ptr(s["w8"]), L._ptr(s["out"]),
                                          L._ptr(s["xs"]), L._ptr(s["ws"]), L._ptr(s["bias"]),
                                          M, N, K, 0, N)

    for i in range(12):
        gemm(i)
    t_gemm = _time_launches(gemm, 300, stream)
    achieved = OPS / (t_gemm * 1e-3) / 1e12
    int8_peak = 2.0 * peaks["bf16_tflops"]
    traffic = _committed_traffic()
    out["roofline"] = {
        "bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s",
        "frac": achieved / int8_peak, "traffic": traffic,
        "kernel": "gemm_i8_kernel<dequant> (tcgen05.mma.kind::i8 128x256x32, TMA, TMEM x2)",
        "ms_per_launch": t_gemm,
        "peak_source": (f"int8 dense = 2 x the {src} bf16 cuBLAS burst "
                        f"({peaks['bf16_tflops']} TFLOP/s); unit is int8 TOPS"),
        "algorithmic": "2*M*N*K = 53.69 GOP per launch",
    }
    # cuBLASLt int8 (torch._int_mm) on the same operands, as a library comparison
    try:
        def cublas(i):
            s = sets[i % NSETS]
            torch._int_mm(s["xq"], s["w8"].t())
        for i in range(6):
            cublas(i)
        t_cub = _time_launches(cublas, 100, stream)
        out["roofline"]["cublaslt_int_mm_tops"] = OPS / (t_cub * 1e-3) / 1e12
    except Exception as exc:  # noqa: BLE001 - context only
        out["roofline"]["cublaslt_int_mm_tops"] = f"unavailable: {exc}"
    # a measured int8 dense peak: cuBLASLt's int8 GEMM at 8192^3 (burst, best of
    # 20 launches), the denominator of `frac_of_measured_int8`
    try:
        g8 = torch.Generator(device=dev).manual_seed(8)
        a8 = torch.randint(-127, 128, (8192, 8192), generator=g8, device=dev, dtype=torch.int8)
        b8 = torch.randint(-127, 128, (8192, 8192), generator=g8, device=dev, dtype=torch.int8)
        bt = b8.t()
        for _ in range(3):
            torch._int_mm(a8, bt)
        best = None
        for _ in range(20):
            t = _time_launches(lambda i: torch._int_mm(a8, bt), 1, stream)
            best = t if best is None else min(best, t)
        peak8 = 2.0 * 8192 ** 3 / (best * 1e-3) / 1e12
        out["roofline"]["int8_measured_peak"] = {
            "tops": peak8, "how": "cuBLASLt int8 GEMM (torch._int_mm) 8192^3, best of 20"}
        out["roofline"]["frac_of_measured_int8"] = achieved / peak8
        del a8, b8, bt
    except Exception as exc:  # noqa: BLE001 - context only
        out["roofline"]["int8_measured_peak"] = f"unavailable: {exc}"

    # rotate+quantize at config C5, the HBM-bound half of the metric
    del_sets = []
    try:
        g = torch.Generator(device=dev).manual_seed(4)
        big = []
        for i in range(2):
            x = torch.randn(C5_M, C5_K, generator=g, device=dev).to(torch.bfloat16)
            big.append((x, torch.empty(C5_M, C5_K, dtype=torch.int8, device=dev),
                        torch.empty(C5_M, dtype=torch.float32, device=dev)))
        del_sets = big

        def rq(i):
            x, q, s = big[i % 2]
            lib.xpuint8_convrot_quantize_stream(sptr, L._ptr(x), L._ptr(q), L._ptr(s), C5_M, C5_K)

        for i in range(4):
            rq(i)
        t_rq = _time_launches(rq, 40, stream)
        gbs = C5_BYTES / (t_rq * 1e-3) / 1e9
        out["rotate_quant"] = {
            "shape": "x bf16 [65536,4096] (config C5)", "ms_per_launch": t_rq, "gbs": gbs,
            "peak_gbs": peaks["hbm_gbs"], "frac": gbs / peaks["hbm_gbs"],
            "algorithmic_bytes": C5_BYTES, "peak_source": f"{src} copy bandwidth",
        }
    finally:
        del del_sets
        torch.cuda.empty_cache()

    # end to end through the public API with host buffers, pipelined as a
    # server would run it: step i's input copy (host->device stream), its
    # linear (compute stream) and its result copy (device->host stream) are
    # ordered by events, so one step's result copy overlaps the next step's
    # input copy and compute (PCIe is full duplex); two device buffers each
    # for x and y, reused only after the step that last used them is done
    x_host = [s["x"].cpu().pin_memory() for s in sets[:2]]
    y_host = [torch.empty(M, N, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    s0 = sets[0]
    h2d_s, cmp_s, d2h_s = (torch.cuda.Stream(dev) for _ in range(3))
    x_dev = [torch.empty(M, K, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    y_dev = [None, None]
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("in", "done", "out")}
    used = [False, False]

    def e2e(i):
        b = i % 2
        with torch.cuda.stream(h2d_s):
            if used[b]:
                h2d_s.wait_event(ev["done"][b])     # the linear that read x_dev[b]
            x_dev[b].copy_(x_host[b], non_blocking=True)
            ev["in"][b].record(h2d_s)
        with torch.cuda.stream(cmp_s):
            cmp_s.wait_event(ev["in"][b])
            if used[b]:
                cmp_s.wait_event(ev["out"][b])      # the copy that read y_dev[b]
            y_dev[b] = xpu_kernels.linear(x_dev[b], s0["w8"], s0["ws"], s0["bias"])
            ev["done"][b].record(cmp_s)
        with torch.cuda.stream(d2h_s):
            d2h_s.wait_event(ev["done"][b])
            y_host[b].copy_(y_dev[b], non_blocking=True)
            ev["out"][b].record(d2h_s)
        used[b] = True

    for i in range(4):
        e2e(i)
    torch.cuda.synchronize()
    n_e2e = 60
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for st in (h2d_s, cmp_s, d2h_s):
        st.wait_event(e0)
    for i in range(n_e2e):
        e2e(i)
    for st in (h2d_s, cmp_s, d2h_s):
        stream.wait_stream(st)
    e1.record(stream)
    e1.synchronize()
    t_e2e = e0.elapsed_time(e1) / n_e2e
    ok = torch.equal(y_host[(n_e2e - 1) % 2].view(torch.int16),
                     xpu_kernels.linear(sets[(n_e2e - 1) % 2]["x"], s0["w8"], s0["ws"],
                                        s0["bias"]).cpu().view(torch.int16))
    out["e2e"] = {"value": OPS / (t_e2e * 1e-3) / 1e12, "unit": "TOPS",
                  "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N * 2,
                  "ms_per_step": t_e2e, "result_checked": bool(ok),
                  "api": ("xpu_kernels.linear (pinned host in/out; host->device copy, linear "
                          "and device->host copy on three streams, consecutive steps overlapped)")}

    # the CPU baseline: the reference's CPU path on the full workload, and the
    # numpy oracle on a row sample for context
    budget = float(os.environ.get("CPU_BASELINE_S", "10"))
    rate, reps, el, cores = cpu_reference_rate(budget)
    nrate, nreps, nel = cpu_numpy_oracle_rate(128, budget_s=min(5.0, budget))
    out["cpu_baseline"] = {
        "value": rate, "unit": "TOPS", "cores": cores, "kind": "port",
        "sample": f"{REF_SAMPLE}; {reps} steps in {el:.1f} s",
        "numpy_oracle": {"value": nrate, "unit": "TOPS",
                         "sample": (f"128 of the 2048 rows x {nreps} repetitions ({nel:.1f} s): "
                                    f"the bit-exact numpy restatement, float64 BLAS GEMM")}}
    return out


def run_nshard(args):
    """Config C5's N-sharded variant (not the headline): x [M, 4096] on every
    rank, W [14336, 4096] split by output channels, the output all-gathered to
    every rank.  Times the fused form (the GEMM stores its tiles into every
    rank's buffer over NVLink) and the NCCL form (GEMM, all-gather, strided
    copy); whole-job TOPS = 2*M*N*K / time (max over ranks): strong scaling."""
    import datetime
    import torch.distributed as dist
    import xpu_kernels
    from xpu_kernels.int8 import shard

    ws_, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws_ > 1:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        with _stdout_to_stderr():
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
            dist.barrier()
    m, k, n = args.nshard_m, 4096, 14336
    g = torch.Generator(device=dev).manual_seed(4)
    x = torch.randn(m, k, generator=g, device=dev)
    x[:, :20] *= 20
    x = x.to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w8, wsc = xpu_kernels.prepare_weight(w)
    del w
    w8l, wsl, _ = shard.shard_weight(w8, wsc, ws_, rank)
    out = shard.PeerOutput(m, n) if ws_ > 1 else None
    stream = torch.cuda.current_stream(dev)

    def fused():
        if out is None:
            return xpu_kernels.linear(x, w8l, wsl)
        return shard.linear_nshard_fused(x, w8l, wsl, None, out)

    def nccl():
        if ws_ == 1:
            return xpu_kernels.linear(x, w8l, wsl)
        return shard.linear_nshard(x, w8l, wsl, None, n_total=n)

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        if ws_ > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fn()
        e1.record(stream)
        e1.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=dev, dtype=torch.float64)
        if ws_ > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # the two forms agree bit for bit
    y_f = fused().clone()
    y_n = nccl()
    same = bool(torch.equal(y_f.view(torch.int16), y_n.view(torch.int16)))
    t_f = timed(fused)
    t_n = timed(nccl)
    ops_ = 2.0 * m * n * k
    if out is not None:
        out.close()
    if rank == 0:
        print(json.dumps({
            "metric": f"ConvRot int8 linear N-sharded TOPS @M={m},K={k},N={n}",
            "value": ops_ / (t_f * 1e-3) / 1e12, "unit": "TOPS", "n_gpus": ws_,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_f,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic", "config": {"workload": "config C5 N-sharded variant", "M": m,
                                            "K": k, "N": n, "parallelism": f"N-shard x{ws_}"},
            "fused_allgather_ms": t_f, "nccl_allgather_ms": t_n,
            "nccl_tops": ops_ / (t_n * 1e-3) / 1e12, "forms_bit_identical": same,
            "output_bytes_per_rank_sent": m * (n // ws_) * 2 * (ws_ - 1)}))
    if ws_ > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--mode", choices=("linear", "nshard"), default="linear",
                    help="linear: the headline (config C3 W1, M-sharded); nshard: config C5's "
                         "N-sharded variant with the output all-gather")
    ap.add_argument("--nshard-m", type=int, default=65536)
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.mode == "nshard":
        return run_nshard(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
