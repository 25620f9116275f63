"""``python -m xpu_kernels``: does the library work on this machine?

A table of named checks, each run through this build's C entry points on the
current CUDA device and judged against a stated gate.  The seeded problem
(x [512, 1024], W [512, 1024], a 1024-wide FFN) and the pass thresholds are the
reference self-test's contract (python/xpu_kernels/int8/selftest.py:52-56 for
the shapes and scales, :157-163 for the thresholds); the checks marked "new"
cover what this build adds (the exact int8 GEMM, the fused qkv split, the int8
weight gradient, the bounded-wait fault word).  ``run_checks`` returns one
record per check; ``selftest`` prints them and returns True when all pass.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List

import torch

from . import _lib as L
from . import ops


@dataclass
class Check:
    name: str
    gate: str                       # the pass condition, in words
    source: str                     # the reference line whose gate it keeps, or "new"
    run: Callable[["_Problem"], tuple]   # -> (measured value, passed)


def _rel(a, b) -> float:
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


def _bits_equal(a, b) -> bool:
    return bool(a.view(torch.int16).equal(b.view(torch.int16)))


class _Problem:
    """The seeded inputs of the self-test and the results several checks share,
    computed once on first use."""

    M, K, N, FF = 512, 1024, 512, 1024

    def __init__(self, dev):
        self.dev = dev
        g = torch.Generator(device=dev).manual_seed(0)

        def randn(*shape, scale):
            return (torch.randn(*shape, generator=g, device=dev) * scale).to(torch.bfloat16)

        self.x = randn(self.M, self.K, scale=0.5)
        self.w = randn(self.N, self.K, scale=0.05)
        self.bias = torch.randn(self.N, generator=g, device=dev) * 0.1
        self.w_up = randn(2 * self.FF, self.K, scale=0.05)
        self.x_up = randn(self.M, self.K, scale=0.5)
        self.w_down = randn(self.K, self.FF, scale=0.05)
        self.dy = randn(self.M, self.N, scale=0.5)
        self.w8, self.ws = ops.prepare_weight(self.w)
        self.up8, self.up_s = ops.prepare_weight(self.w_up)
        self.down8, self.down_s = ops.prepare_weight(self.w_down)
        self.y = ops.linear(self.x, self.w8, self.ws, self.bias)
        self.xq, self.xs = ops.quantize(self.x)
        self.w_deq = ops.dequant_weight(self.w8, self.ws)
        xr = self.x.detach().clone().requires_grad_(True)
        torch.nn.functional.linear(xr, self.w).backward(self.dy)
        self.dx_autograd = xr.grad
        # dW of the dequantized weight by autograd
        xa = self.x.detach().clone().requires_grad_(True)
        wa = self.w_deq.detach().clone().requires_grad_(True)
        torch.nn.functional.linear(xa, wa).backward(self.dy)
        self.dw_autograd = wa.grad


# ---------------------------------------------------------------- the checks

def _linear_vs_bf16(p):
    ref = (p.x.float() @ p.w.float().t() + p.bias).to(torch.bfloat16)
    r = _rel(p.y, ref)
    return r, r < 0.02


def _acc_path_is_linear(p):
    acc, xs = ops.linear_acc(p.x, p.w8, p.ws)
    same = _bits_equal(ops.dequant(acc, xs, p.ws, p.bias), p.y)
    return same, same


def _gemm_exact(p):
    acc = ops.int_mm(p.xq, p.w8)
    exact = bool(acc.equal((p.xq.double() @ p.w8.double().t()).to(torch.int32)))
    return exact, exact


def _strided_slice(p):
    acc2, xs2 = ops.linear_acc(p.x, torch.cat([p.w8, p.w8]), torch.cat([p.ws, p.ws]))
    left = acc2[:, :p.N]
    same = _bits_equal(ops.dequant_slice(left, xs2, p.ws, p.bias),
                       ops.dequant(left.contiguous(), xs2, p.ws, p.bias))
    return same, same


def _split_projection(p):
    w3 = torch.cat([p.w8, p.w8, p.w8])
    s3 = torch.cat([p.ws, p.ws, p.ws])
    b3 = torch.cat([p.bias, p.bias * 2, p.bias * 3])
    parts = ops.linear_split(p.x, w3, s3, b3, parts=3)
    same = all(_bits_equal(t, ops.linear(p.x, p.w8, p.ws, p.bias * (i + 1)))
               for i, t in enumerate(parts))
    return same, same


def _situ_epilogue(p):
    acc, xs = ops.linear_acc(p.x_up, p.up8, p.up_s)
    q, s = ops.dequant_act_quantize(acc, xs, p.up_s, "situ")
    q_ref, s_ref = ops.quantize_act(ops.dequant(acc, xs, p.up_s), "situ")
    code = int((q.to(torch.int16) - q_ref.to(torch.int16)).abs().max())
    srel = float(((s - s_ref).abs() / s_ref.clamp_min(1e-20)).max())
    return (code, round(srel, 5)), code <= 1 and srel < 0.05


def _geglu_ffn(p):
    fused = ops.ffn(p.x_up, p.up8, p.up_s, p.down8, p.down_s, act="geglu_erf")
    acc, xs = ops.linear_acc(p.x_up, p.up8, p.up_s)
    hidden, gate = ops.dequant(acc, xs, p.up_s).chunk(2, dim=-1)
    q2, xs2 = ops.quantize(hidden * torch.nn.functional.gelu(gate))
    chain = ops.dequant(ops.int_mm(q2, p.down8), xs2, p.down_s)
    differ = int((fused.view(torch.int16) != chain.view(torch.int16)).sum())
    return differ, differ == 0


def _dx_dense(p):
    r = _rel(ops.linear_dx(p.dy, p.w), p.dx_autograd)
    return r, r < 1e-6


def _dequant_weight(p):
    same = _bits_equal(p.w_deq, ops.dequant_weight_torch(p.w8, p.ws))
    r = _rel(p.w_deq, p.w)
    return (same, round(r, 5)), same and r < 0.02


def _dx_int8_weight(p):
    r = _rel(ops.linear_dx(p.dy, p.w_deq), p.dx_autograd)
    return r, r < 0.03


def _dx_int8_gemm(p):
    r = _rel(ops.linear_dx_int8(p.dy, p.w8, p.ws), p.dx_autograd)
    return r, r < 0.04


def _row_quantizer(p):
    q, s = ops.quantize_row(p.dy)
    qt, st = ops.quantize_row_torch(p.dy)
    differ = int((q != qt).sum())
    scales = bool(s.view(torch.int32).equal(st.view(torch.int32)))
    return (differ, scales), differ == 0 and scales


def _autograd_op(p):
    xi = p.x.detach().clone().requires_grad_(True)
    ops.int8_linear(xi, p.w8, p.ws, None, mode="dense").backward(p.dy)
    r_dx = _rel(xi.grad, p.dy @ p.w_deq)
    r_dw = _rel(ops.linear_dw(p.dy, p.x), p.dw_autograd)
    return (r_dx, r_dw), r_dx < 1e-6 and r_dw < 1e-6


def _dw_int8(p):
    r = _rel(ops.linear_dw_int8(p.dy, p.xq, p.xs), p.dw_autograd)
    return r, r < 0.04


def _trainable(p):
    mod = ops.TrainableInt8Linear(p.w, p.bias)
    y = mod(p.x)
    w8f, wsf = ops.prepare_weight_fused(p.w)
    fwd = _bits_equal(y, ops.linear(p.x, w8f, wsf, mod.bias.detach()))
    y.backward(p.dy)
    dw = _bits_equal(mod.weight.grad, ops.linear_dw(p.dy, p.x))
    return (fwd, dw), fwd and dw


def _fault_word(p):
    torch.cuda.synchronize(p.dev)
    word = L.load().xpuint8_fault_status(0)
    return word, word == 0


CHECKS: List[Check] = [
    Check("linear vs bf16 matmul", "relative error < 0.02", "selftest.py:157", _linear_vs_bf16),
    Check("accumulator path", "dequant(linear_acc(x)) == linear(x), bit for bit",
          "selftest.py:157", _acc_path_is_linear),
    Check("int8 GEMM", "int32 result == the fp64 product exactly", "new", _gemm_exact),
    Check("strided dequant slice", "== the contiguous copy's dequant, bit for bit",
          "selftest.py:157", _strided_slice),
    Check("fused qkv split", "each part == linear() of that part, bit for bit", "new",
          _split_projection),
    Check("fused situ epilogue", "codes within 1 and scales within 5 % of the unfused chain",
          "selftest.py:157-158", _situ_epilogue),
    Check("fused GEGLU FFN", "0 bf16 values differ from quantize(hidden * gelu(gate)) chain",
          "selftest.py:162", _geglu_ffn),
    Check("dense dx", "relative error vs autograd < 1e-6", "selftest.py:159", _dx_dense),
    Check("dequant_weight", "== its torch chain bit for bit; within 0.02 of W",
          "selftest.py:159-161", _dequant_weight),
    Check("dx through the int8 weight", "relative error < 0.03", "selftest.py:159",
          _dx_int8_weight),
    Check("dx with the int8 GEMM", "relative error < 0.04", "selftest.py:160", _dx_int8_gemm),
    Check("row quantizer", "codes == quantize_row_torch's; scales bit-identical",
          "selftest.py:161", _row_quantizer),
    Check("autograd op", "dx vs the same GEMM and dW vs autograd < 1e-6",
          "selftest.py:162", _autograd_op),
    Check("int8 dW", "relative error vs the bf16 dW < 0.04", "new", _dw_int8),
    Check("trainable linear", "forward == the INT8 model's; dW == the bf16 model's",
          "selftest.py:162-163", _trainable),
    Check("device fault word", "no bounded wait gave up", "new", _fault_word),
]


def run_checks() -> List[dict]:
    """Run every check on the current CUDA device; one record per check:
    ``{"name", "gate", "source", "measured", "ok"}`` (``ok`` False with the
    exception text as ``measured`` when a check raises)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    problem = _Problem(dev)
    out = []
    for c in CHECKS:
        try:
            measured, ok = c.run(problem)
        except Exception as exc:  # noqa: BLE001 - reported as a failed check
            measured, ok = f"{type(exc).__name__}: {exc}", False
        out.append({"name": c.name, "gate": c.gate, "source": c.source,
                    "measured": measured, "ok": bool(ok)})
    torch.cuda.synchronize(dev)
    return out


def selftest(verbose: bool = True) -> bool:
    """Quick end-to-end check on this machine.  Returns True when every check passes."""
    if not L.available():
        if verbose:
            print(f"libxpuint8 unavailable: {L._ERR}")
        return False
    records = run_checks()
    ok = all(r["ok"] for r in records)
    if verbose:
        print(f"device: {L.device_name()}")
        width = max(len(r["name"]) for r in records)
        for r in records:
            print(f"  {'ok  ' if r['ok'] else 'FAIL'} {r['name']:<{width}}  {r['measured']!s:<28} "
                  f"[{r['gate']}; {r['source']}]")
        print("PASS" if ok else "FAIL")
    return ok
