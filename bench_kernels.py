"""Per-kernel benchmark harness: one kernel of the library on one shape.

    python bench_kernels.py gemm --M 2048 --N 10240 --K 1280 --iters 20
    python bench_kernels.py rotate_quant --M 65536 --K 4096
    python bench_kernels.py linear | ffn | dx | dw | quantize_row | dequant | ...
    python bench_kernels.py suite [--iters N]   (every shape of SUITE, timing only)

Inputs are seeded and generated on the device; each case launches its kernel
`--iters` times over `--sets` rotating buffer sets and prints the average
device time per launch (CUDA events) with the algorithmic throughput.  The
ncu summaries under profiles/ each name the single-case command they came
from, captured one kernel at a time (``ncu -k regex:<kernel> -s <skip> -c 1``)
on a small case.  ``bench.py`` is the headline benchmark; this file is for the
individual kernels.
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "oko-xpu-kernels_b200"))

from xpu_kernels.int8 import ops  # noqa: E402
from xpu_kernels.int8._lib import _lib, _ptr, _stream  # noqa: E402


def _time(fn, iters, stream):
    """Device time per call (ms): the `iters` calls captured in a CUDA graph
    (after eager warm-up calls), the graph replayed three times between CUDA
    events.  Host-side launch overhead is not in the number."""
    for i in range(min(3, iters)):
        fn(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        with torch.cuda.graph(graph, stream=side):
            for i in range(iters):
                fn(i)
    stream.wait_stream(side)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(3):
        graph.replay()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / (3 * iters)


# The shapes of the BASELINE configs (C3 W1, C3 GEGLU, C4 backward, C5), run by
# ``suite`` in one process for timing.  Profile one case at a time, never the
# suite (it holds up to a few GB and runs every kernel).
SUITE = [
    ["gemm", "--M", "2048", "--N", "10240", "--K", "1280", "--sets", "6"],
    ["geglu", "--M", "2048", "--N", "5120", "--K", "1280", "--sets", "6"],
    ["gemm", "--M", "8192", "--N", "14336", "--K", "4096", "--sets", "1"],
    ["gemm_nn", "--M", "4096", "--N", "1280", "--K", "5120", "--sets", "2"],
    ["gemm_tn", "--M", "5120", "--N", "1280", "--K", "4096", "--sets", "2"],
    ["rotate_quant", "--M", "65536", "--K", "4096", "--sets", "1"],
    ["rotate_quant", "--M", "2048", "--K", "1280", "--sets", "8"],
    ["rotate", "--M", "65536", "--K", "4096", "--sets", "1"],
    ["quantize_row", "--M", "4096", "--K", "5120", "--sets", "2"],
    ["dequant", "--M", "16384", "--N", "14336", "--sets", "1"],
    ["dequant_act", "--M", "2048", "--K", "5120", "--sets", "2"],
    ["dw", "--M", "4096", "--N", "5120", "--K", "1280"],
]


def main(argv=None):
    import sys
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "suite":
        iters = argv[argv.index("--iters") + 1] if "--iters" in argv else "2"
        for case in SUITE:
            main(case + ["--iters", iters])
        return
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "gemm_raw", "gemm_nn", "gemm_tn", "geglu",
                                     "rotate_quant", "rotate", "linear", "ffn", "dx", "dw",
                                     "quantize_row", "colquant", "rope", "dequant", "dequant_act"])
    ap.add_argument("--M", type=int, default=2048)
    ap.add_argument("--N", type=int, default=10240)
    ap.add_argument("--K", type=int, default=1280)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--sets", type=int, default=2)
    ap.add_argument("--colscale", action="store_true",
                    help="quantize_row: with a column scale (the form linear_dx_int8 runs)")
    ap.add_argument("--act", type=int, default=4,
                    help="dequant_act / ffn: 3 situ, 4 GEGLU (paired), 5 GELU-erf (unpaired)")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", torch.cuda.current_device())
    lib = _lib()
    st = torch.cuda.current_stream(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    M, N, K = a.M, a.N, a.K

    def i8(*shape):
        return torch.randint(-127, 128, shape, generator=g, device=dev, dtype=torch.int8)

    def bf(*shape, s=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * s).to(torch.bfloat16)

    def f32(*shape):
        return torch.rand(*shape, generator=g, device=dev) * 1e-3 + 1e-5

    S = a.sets
    if a.case in ("gemm", "gemm_raw", "gemm_nn", "gemm_tn", "geglu"):
        lay = {"gemm": 0, "gemm_raw": 0, "gemm_nn": 1, "gemm_tn": 2, "geglu": 0}[a.case]
        nb = 2 * N if a.case == "geglu" else N
        A = [i8(M, K) if lay < 2 else i8(K, M) for _ in range(S)]
        B = [i8(nb, K) if lay == 0 else i8(K, N) for _ in range(S)]
        xs, ws, bias = f32(M), f32(nb), f32(N)
        if a.case == "gemm_raw":
            O = [torch.empty(M, N, dtype=torch.int32, device=dev) for _ in range(S)]
        else:
            O = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(S)]

        def fn(i):
            j = i % S
            if a.case == "gemm_raw":
                rc = lib.xpuint8_int_mm_stream(_stream(dev), _ptr(A[j]), _ptr(B[j]), _ptr(O[j]), M, N, K, 0, N)
            elif a.case == "geglu":
                rc = lib.xpuint8_int_mm_geglu_stream(_stream(dev), _ptr(A[j]), _ptr(B[j]), _ptr(O[j]),
                                                     _ptr(xs), _ptr(ws), M, N, K)
            else:
                rc = lib.xpuint8_int_mm_dequant_stream(_stream(dev), _ptr(A[j]), _ptr(B[j]), _ptr(O[j]),
                                                       _ptr(xs), _ptr(ws), _ptr(bias), M, N, K,
                                                       lay, N)
            assert rc == 0, lib.xpuint8_last_error()
        ops_ = 2.0 * M * (2 * N if a.case == "geglu" else N) * K
        t = _time(fn, a.iters, st)
        res = {"case": a.case, "ms": t, "TOPS": ops_ / (t * 1e-3) / 1e12}
    elif a.case in ("rotate_quant", "rotate", "quantize_row"):
        X = [bf(M, K) for _ in range(S)]
        Q = [torch.empty(M, K, dtype=torch.bfloat16 if a.case == "rotate" else torch.int8,
                         device=dev) for _ in range(S)]
        sc = [torch.empty(M, dtype=torch.float32, device=dev) for _ in range(S)]
        # --colscale: the column-scaled form linear_dx_int8 runs (x * bf16(col_scale))
        cs = f32(K) if a.colscale else None
        cs_ptr = _ptr(cs) if a.colscale else None

        def fn(i):
            j = i % S
            if a.case == "rotate_quant":
                rc = lib.xpuint8_convrot_quantize_stream(_stream(dev), _ptr(X[j]), _ptr(Q[j]), _ptr(sc[j]), M, K)
            elif a.case == "rotate":
                rc = lib.xpuint8_convrot_rotate_bf16_stream(_stream(dev), _ptr(X[j]), _ptr(Q[j]), M, K)
            else:
                rc = lib.xpuint8_quantize_row_stream(_stream(dev), _ptr(X[j]), cs_ptr, _ptr(Q[j]), _ptr(sc[j]), M, K)
            assert rc == 0, lib.xpuint8_last_error()
        nbytes = (4 * M * K) if a.case == "rotate" else (3 * M * K + 4 * M)
        t = _time(fn, a.iters, st)
        res = {"case": a.case, "ms": t, "GBps": nbytes / (t * 1e-3) / 1e9, "bytes": nbytes}
    elif a.case == "colquant":
        DY = [bf(M, N, s=1e-3) for _ in range(S)]
        GQ = [torch.empty(M, N, dtype=torch.int8, device=dev) for _ in range(S)]
        TG = [torch.empty(N, dtype=torch.float32, device=dev) for _ in range(S)]
        xs = f32(M)

        def fn(i):
            j = i % S
            rc = lib.xpuint8_colquant_stream(_stream(dev), _ptr(DY[j]), _ptr(xs), _ptr(GQ[j]),
                                             _ptr(TG[j]), M, N)
            assert rc == 0, lib.xpuint8_last_error()
        nbytes = 3 * M * N + 4 * M + 4 * N
        t = _time(fn, a.iters, st)
        res = {"case": a.case, "ms": t, "GBps": nbytes / (t * 1e-3) / 1e9, "bytes": nbytes}
    elif a.case == "rope":
        # M rows (B=1, S=M) of N // 128 heads of D=128 from an int32 [M, 3N] qkv accumulator
        H, D = N // 128, 128
        ACC = [torch.randint(-2 ** 20, 2 ** 20, (M, 3 * N), generator=g, device=dev, dtype=torch.int32)
               for _ in range(S)]
        xs, ws, wt = f32(M), f32(3 * N), torch.ones(D, device=dev)
        ang = torch.rand(1, M, 1, D // 2, generator=g, device=dev) * 3.0
        pe = torch.stack([torch.stack([ang.cos(), -ang.sin()], -1),
                          torch.stack([ang.sin(), ang.cos()], -1)], -2)

        def fn(i):
            a3 = ACC[i % S].view(1, M, 3 * N)
            ops.rms_rope_split_half_dequant(a3[:, :, :N].unflatten(-1, (H, D)),
                                            a3[:, :, N:2 * N].unflatten(-1, (H, D)), pe,
                                            ws[:N], ws[N:2 * N], xs, wt)
        nbytes = 2 * (4 * M * N + 2 * M * N)
        t = _time(fn, a.iters, st)
        res = {"case": a.case, "ms": t, "GBps": nbytes / (t * 1e-3) / 1e9, "bytes": nbytes}
    elif a.case == "dequant":
        ACC = [torch.randint(-2 ** 20, 2 ** 20, (M, N), generator=g, device=dev, dtype=torch.int32)
               for _ in range(S)]
        O = [torch.empty(M, N, dtype=torch.bfloat16, device=dev) for _ in range(S)]
        xs, ws, bias = f32(M), f32(N), f32(N)

        def fn(i):
            j = i % S
            rc = lib.xpuint8_dequant_epilogue_stream(_stream(dev), _ptr(ACC[j]), _ptr(O[j]), _ptr(xs), _ptr(ws),
                                                     _ptr(bias), M, N)
            assert rc == 0, lib.xpuint8_last_error()
        nbytes = 6 * M * N + 4 * M + 12 * N
        t = _time(fn, a.iters, st)
        res = {"case": a.case, "ms": t, "GBps": nbytes / (t * 1e-3) / 1e9}
    elif a.case == "dequant_act":
        halves = 1 if a.act == 5 else 2
        ACC = [torch.randint(-2 ** 20, 2 ** 20, (M, halves * K), generator=g, device=dev,
                             dtype=torch.int32) for _ in range(S)]
        Q = [torch.empty(M, K, dtype=torch.int8, device=dev) for _ in range(S)]
        sc = [torch.empty(M, dtype=torch.float32, device=dev) for _ in range(S)]
        xs, ws = f32(M), f32(halves * K)

        def fn(i):
            j = i % S
            rc = lib.xpuint8_dequant_act_quantize_stream(_stream(dev), _ptr(ACC[j]), _ptr(Q[j]), _ptr(sc[j]),
                                                         _ptr(xs), _ptr(ws), M, K, a.act)
            assert rc == 0, lib.xpuint8_last_error()
        nbytes = halves * (4 * M * K + 4 * K) + M * K + 8 * M
        t = _time(fn, a.iters, st)
        res = {"case": a.case, "act": a.act, "ms": t, "GBps": nbytes / (t * 1e-3) / 1e9}
    elif a.case == "linear":
        X = [bf(M, K) for _ in range(S)]
        w8, ws = ops.prepare_weight(bf(N, K, s=0.02))

        def fn(i):
            ops.linear(X[i % S], w8, ws)
        t = _time(fn, a.iters, st)
        res = {"case": a.case, "ms": t, "TOPS": 2.0 * M * N * K / (t * 1e-3) / 1e12}
    elif a.case == "ffn":
        # N: the up-projection's rows for a paired activation ([hidden | gate])
        inner = N // 2
        act = {3: "situ", 4: "geglu_erf", 5: "gelu_erf"}[a.act]
        n_up = inner if act == "gelu_erf" else N
        X = [bf(M, K) for _ in range(S)]
        up8, ups = ops.prepare_weight(bf(n_up, K, s=0.02))
        dn8, dns = ops.prepare_weight(bf(K, inner, s=0.02))

        def fn(i):
            ops.ffn(X[i % S], up8, ups, dn8, dns, act=act)
        t = _time(fn, a.iters, st)
        res = {"case": a.case, "act": act, "ms": t,
               "TOPS": (2.0 * M * n_up * K + 2.0 * M * inner * K) / (t * 1e-3) / 1e12}
    elif a.case in ("dx", "dw"):
        x = bf(M, K)
        w8, ws = ops.prepare_weight(bf(N, K, s=0.02))
        dy = bf(M, N, s=1e-3)
        xq, xs = ops.quantize(x)

        def fn(i):
            if a.case == "dx":
                ops.linear_dx_int8(dy, w8, ws)
            else:
                ops.linear_dw_int8(dy, xq, xs)
        t = _time(fn, a.iters, st)
        res = {"case": a.case, "ms": t, "TOPS": 2.0 * M * N * K / (t * 1e-3) / 1e12}
    res.update({"M": M, "N": N, "K": K})
    print(json.dumps(res))


if __name__ == "__main__":
    main()
