"""``python -m xpu_kernels``: does the library work on this machine?

The B200 build of the reference's self-test (python/xpu_kernels/int8/selftest.py)
with the same checks and pass thresholds (:157-163), plus the int32 GEMM
against an exact reference and the int8 weight gradient:

* INT8 linear vs the bf16 matmul: relative error < 0.02
* ``dequant(linear_acc(x))`` == ``linear(x)`` bit for bit; strided slice == contiguous
* fused situ epilogue vs the unfused chain: codes within 1
* fused GEGLU FFN == the unfused chain ``quantize(hidden * gelu(gate))`` bit for bit
* backward: dx conventions exact, dequant_weight == its torch chain, dx_int8 < 0.04,
  quantize_row == quantize_row_torch with exact scales, autograd dx/dW < 1e-6
* trainable linear: forward == the INT8 model, dW == the bf16 model
* int8 GEMM == an fp64 reference exactly; int8 dW within 0.04 of the bf16 dW
"""

from __future__ import annotations

import torch

from ._lib import _ERR, available, device_name
from .ops import (
    TrainableInt8Linear,
    dequant,
    dequant_act_quantize,
    dequant_slice,
    dequant_weight,
    dequant_weight_torch,
    ffn,
    int8_linear,
    int_mm,
    linear,
    linear_acc,
    linear_dw,
    linear_dw_int8,
    linear_dx,
    linear_dx_int8,
    prepare_weight,
    prepare_weight_fused,
    quantize,
    quantize_act,
    quantize_row,
    quantize_row_torch,
)


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


def selftest(verbose: bool = True) -> bool:
    """Quick end-to-end check on this machine.  Returns True when it passes."""
    if not available():
        if verbose:
            from . import _lib as L
            print(f"libxpuint8 unavailable: {L._ERR or _ERR}")
        return False
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(0)
    M, K, N = 512, 1024, 512
    x = (torch.randn(M, K, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.05).to(torch.bfloat16)
    bias = torch.randn(N, generator=g, device=dev) * 0.1

    w8, ws = prepare_weight(w)
    y = linear(x, w8, ws, bias)
    ref = (x.float() @ w.float().t() + bias).to(torch.bfloat16)
    rel = _rel(y, ref)

    acc, xs = linear_acc(x, w8, ws)
    same = dequant(acc, xs, ws, bias).view(torch.int16).equal(y.view(torch.int16))

    xq, _ = quantize(x)
    acc_ref = (xq.double() @ w8.double().t()).to(torch.int32)
    gemm_exact = bool(acc.equal(acc_ref))

    acc_w, xs_w = linear_acc(x, torch.cat([w8, w8], 0), torch.cat([ws, ws]))
    half = acc_w[:, :N]
    sl = dequant_slice(half, xs_w, ws, bias)
    slice_same = sl.view(torch.int16).equal(dequant(half.contiguous(), xs_w, ws, bias).view(torch.int16))

    kff = 1024
    wup = (torch.randn(2 * kff, K, generator=g, device=dev) * 0.05).to(torch.bfloat16)
    wup8, wup_s = prepare_weight(wup)
    xup = (torch.randn(M, K, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    acc2, xs2 = linear_acc(xup, wup8, wup_s)
    q2, s2 = dequant_act_quantize(acc2, xs2, wup_s)
    d = dequant(acc2, xs2, wup_s)
    q2_ref, s2_ref = quantize_act(d, "situ")
    code_diff = int((q2.to(torch.int16) - q2_ref.to(torch.int16)).abs().max())
    scale_rel = float(((s2 - s2_ref).abs() / s2_ref.clamp_min(1e-20)).max())

    wdown = (torch.randn(K, kff, generator=g, device=dev) * 0.05).to(torch.bfloat16)
    wdown8, wdown_s = prepare_weight(wdown)
    ffn_fused = ffn(xup, wup8, wup_s, wdown8, wdown_s, act="geglu_erf")
    hidden, gate = d.chunk(2, dim=-1)
    q2_g, xs2_g = quantize(hidden * torch.nn.functional.gelu(gate))
    ffn_ref = dequant(int_mm(q2_g, wdown8), xs2_g, wdown_s)
    geglu_diff = int((ffn_fused.view(torch.int16) != ffn_ref.view(torch.int16)).sum())

    dy = (torch.randn(M, N, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    xr = x.detach().clone().requires_grad_(True)
    torch.nn.functional.linear(xr, w).backward(dy)
    grad = xr.grad
    dx_rel = _rel(linear_dx(dy, w), grad)
    w_deq = dequant_weight(w8, ws)
    dequant_same = bool(w_deq.view(torch.int16).eq(dequant_weight_torch(w8, ws).view(torch.int16)).all())
    w_rel = _rel(w_deq, w)
    dx_int8_rel = _rel(linear_dx(dy, w_deq), grad)
    dx_q_rel = _rel(linear_dx_int8(dy, w8, ws), grad)

    q_fused, s_fused = quantize_row(dy)
    q_chain, s_chain = quantize_row_torch(dy)
    quant_diff = int((q_fused.view(torch.int8) != q_chain.view(torch.int8)).sum())
    quant_rel = _rel(q_fused, q_chain)
    scale_same = bool(s_fused.view(torch.int32).equal(s_chain.view(torch.int32)))

    xi = x.detach().clone().requires_grad_(True)
    int8_linear(xi, w8, ws, None, mode="dense").backward(dy)
    dx_gemm_rel = _rel(xi.grad, dy @ w_deq)
    dw = linear_dw(dy, x)
    xr2 = x.detach().clone().requires_grad_(True)
    wr2 = w_deq.detach().clone().requires_grad_(True)
    torch.nn.functional.linear(xr2, wr2).backward(dy)
    dw_rel = _rel(dw, wr2.grad)
    dw_int8_rel = _rel(linear_dw_int8(dy, xq, xs), wr2.grad)

    tr = TrainableInt8Linear(w, bias)
    y_tr = tr(x)
    w8_f, ws_f = prepare_weight_fused(w)
    y_tr_ref = linear(x, w8_f, ws_f, tr.bias.detach())
    tr_same = bool(y_tr.view(torch.int16).eq(y_tr_ref.view(torch.int16)).all())
    y_tr.backward(dy)
    dw_same = bool(tr.weight.grad.view(torch.int16).eq(dw.view(torch.int16)).all())
    torch.cuda.synchronize()

    ok = (same and slice_same and gemm_exact and rel < 0.02 and code_diff <= 1
          and scale_rel < 0.05 and dx_rel < 1e-6 and w_rel < 0.02 and dx_int8_rel < 0.03
          and dx_q_rel < 0.04 and quant_diff == 0 and scale_same and dequant_same
          and dx_gemm_rel < 1e-6 and dw_rel < 1e-6 and geglu_diff == 0 and tr_same
          and dw_same and dw_int8_rel < 0.04)
    if verbose:
        print(f"device            : {device_name()}")
        print(f"INT8 vs bf16      : relative error {rel:.4f} (expect < 0.02)")
        print(f"acc path == linear: {same}")
        print(f"int8 GEMM exact   : {gemm_exact}")
        print(f"strided slice     : {slice_same}")
        print(f"fused situ vs chain: max code diff {code_diff}, max scale rel {scale_rel:.4f}")
        print(f"fused GEGLU FFN vs the unfused chain: {geglu_diff} bf16 values differ (expect 0)")
        print(f"trainable INT8 linear: forward is the INT8 model's {tr_same}, "
              f"dW is the bf16 model's {dw_same}")
        print(f"backward dx vs autograd: rel {dx_rel:.2e} (expect 0)")
        print(f"dequant_weight    : rel {w_rel:.4f} (the INT8 weight itself)")
        print(f"backward dx, INT8 : rel {dx_int8_rel:.4f}")
        print(f"backward dx, int8 GEMM (weight stays quantized): rel {dx_q_rel:.4f}")
        print(f"backward dW, int8 GEMM: rel {dw_int8_rel:.4f}")
        print(f"fused quantizer vs chain: {quant_diff} of {q_fused.numel()} values "
              f"differ, rel {quant_rel:.2e}, scales exact: {scale_same}")
        print(f"fused dequant vs the chain: bit-identical {dequant_same}")
        print(f"autograd op: dx vs the same GEMM rel {dx_gemm_rel:.2e}, "
              f"dW vs autograd rel {dw_rel:.2e}")
        print("PASS" if ok else "FAIL")
    return ok
