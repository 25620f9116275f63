"""The INT8 API: weight preparation, the linear, the FFN, the accumulator paths
and the backward -- the B200 build of python/xpu_kernels/int8/ops.py.

Every function takes and returns torch tensors on a CUDA device; the kernels
are enqueued on torch's current stream, so nothing here synchronises.  The
names, arguments, return values and error messages are the reference's; what
changed is underneath:

* every ``torch._int_mm`` of the reference (ops.py:371, :587, :634, :714,
  :716) is the library's tcgen05 int8 GEMM (``xpuint8_int_mm*_stream``);
* ``linear`` is two launches (rotate+quantize, then the GEMM with the dequant
  epilogue fused into its accumulator drain) instead of three;
* ``ffn`` with ``geglu_erf`` fuses the dequant + GEGLU into the up-projection
  GEMM's epilogue; the other activations keep the reference's
  ``dequant_act_quantize`` step;
* ``quantize_row`` is the library's row quantizer (no Triton);
* new: ``linear_dw_int8``, the weight gradient with both GEMM operands int8.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from .._capture import is_capturing
from ._lib import (
    ACTIVATIONS,
    PAIRED_ACTIVATIONS,
    _err,
    _flat2d,
    _lib,
    _ptr,
    _stream,
    load,
)

_P = ctypes.c_void_p


def rotate(x):
    """ConvRot rotation only: bf16 [.., K] in, bf16 [.., K] out, no quantization."""
    lib = _lib()
    x2, shape = _flat2d(x)
    out = torch.empty_like(x2)
    m, k = x2.shape
    rc = lib.xpuint8_convrot_rotate_bf16_stream(_stream(x.device), _ptr(x2), _ptr(out), m, k)
    if rc != 0:
        _err(lib, "rotate")
    return out.reshape(shape)


def quantize(x):
    """Rotate and quantize an activation: bf16 [.., K] -> (int8 [.., K], fp32 [..])."""
    lib = _lib()
    x2, shape = _flat2d(x)
    m, k = x2.shape
    q = torch.empty((m, k), device=x.device, dtype=torch.int8)
    scale = torch.empty((m,), device=x.device, dtype=torch.float32)
    rc = lib.xpuint8_convrot_quantize_stream(_stream(x.device), _ptr(x2), _ptr(q), _ptr(scale),
                                             m, k)
    if rc != 0:
        _err(lib, "quantize")
    return q.reshape(*shape[:-1], k), scale.reshape(shape[:-1])


def quantize_act(x, activation: str):
    """Rotate+quantize with an activation fused into the load.

    ``gelu_tanh`` and ``gelu_erf`` consume [.., K]; ``swiglu``, ``situ`` and
    ``geglu_erf`` consume [.., 2K] (``[gate, up]`` for swiglu, ``[hidden, gate]``
    for the others); the result is [.., K].  ``K`` is the *output* width in all
    cases -- the C API takes it that way, because for the pair activations it
    doubles as the stride between the two halves.
    """
    lib = _lib()
    x2, shape = _flat2d(x)
    m, k2 = x2.shape
    act = ACTIVATIONS[activation]
    k = k2 // 2 if activation in PAIRED_ACTIVATIONS else k2
    q = torch.empty((m, k), device=x.device, dtype=torch.int8)
    scale = torch.empty((m,), device=x.device, dtype=torch.float32)
    rc = lib.xpuint8_convrot_quantize_act_stream(_stream(x.device), _ptr(x2), _ptr(q),
                                                 _ptr(scale), m, k, act)
    if rc != 0:
        _err(lib, "quantize_act")
    return q.reshape(*shape[:-1], k), scale.reshape(shape[:-1])


def _div(a, b):
    # A true (IEEE) division.  On CUDA, ``tensor / python_scalar`` is computed
    # as a multiplication by the reciprocal, which is not what the reference
    # chains compute (CPU and XPU divide); a 0-dim device tensor divides.
    if not isinstance(b, torch.Tensor):
        b = torch.tensor(float(b), dtype=a.dtype, device=a.device)
    return torch.div(a, b)


def prepare_weight(w, group: int = 256):
    """Prepare an INT8 weight for :func:`linear`.

    ``w`` is bf16 or fp32 [N, K] in the *unrotated* orientation, i.e. the
    matrix a plain ``x @ w.T`` would use.  Returns ``(int8 [N, K], fp32 [N])``:
    the row-rotated weights and the per-output-channel scale the dequant
    epilogue expects.  Round to nearest, symmetric, clipped to +-127.
    Same arithmetic as the reference (ops.py:83-100), divisions IEEE.
    """
    if w.shape[1] % group:
        raise ValueError(f"K={w.shape[1]} is not a multiple of the group size {group}")
    wr = rotate(w.detach().to(device=w.device, dtype=torch.bfloat16).contiguous())
    amax = wr.abs().amax(dim=1).clamp_min(1e-30)
    scale = _div(amax.float(), 127.0)
    q = torch.round(_div(wr.float(), scale[:, None])).clamp_(-127, 127).to(torch.int8)
    return q, scale.contiguous()


def prepare_weight_fused(w, group: int = 256):
    """Prepare an INT8 weight for :func:`linear`, in one kernel.

    The same result as :func:`prepare_weight` up to the last bit: the kernel
    rotates and quantizes in one pass and keeps the rotated values in fp32
    where the chain rounds them to bf16 first, so the row's scale can differ by
    one ULP and a few percent of the values by one unit (the reference measures
    5.7 %, ops.py:106-113).  It is a separate function so that stored weights
    never change.
    """
    if w.shape[1] % group:
        raise ValueError(f"K={w.shape[1]} is not a multiple of the group size {group}")
    return quantize(w.detach().to(device=w.device, dtype=torch.bfloat16).contiguous())


def dequant_weight(w8, w_scale):
    """The unrotated bf16 weight behind an INT8 ConvRot weight, ``rotate(bf16(w8 * s))``.

    One fused kernel: int8 in, bf16 out (3 bytes per parameter), bit-identical
    to :func:`dequant_weight_torch`.
    """
    if w8.dtype != torch.int8:
        raise TypeError(f"w8 must be int8, got {w8.dtype}")
    if w8.dim() != 2 or w8.shape[1] % 256 or w_scale.numel() not in (1, w8.shape[0]):
        return dequant_weight_torch(w8, w_scale)
    lib = _lib()
    scale = expand_scale(w_scale.detach(), w8.shape[0], w8.device)
    w8c = w8.contiguous()
    out = torch.empty(w8.shape, dtype=torch.bfloat16, device=w8.device)
    rc = lib.xpuint8_dequant_weight_stream(_stream(w8.device), _ptr(w8c), _ptr(scale), _ptr(out),
                                           w8.shape[0], w8.shape[1])
    if rc != 0:
        _err(lib, "dequant_weight")
    return out


def dequant_weight_torch(w8, w_scale):
    """The weight dequantization as a torch chain -- the definition
    (ops.py:169-191): the fp32 multiply by the row's scale, the bf16 rounding,
    and then the rotation undone."""
    if w8.dtype != torch.int8:
        raise TypeError(f"w8 must be int8, got {w8.dtype}")
    if is_capturing():
        raise RuntimeError(
            "dequant_weight() materializes a full-precision copy of the "
            "weight; inside a device-graph capture it would be captured and "
            "re-computed on every replay. Call it before capturing, or use "
            "the int8 backward (xpu_kernels.int8_linear(..., mode='int8')), "
            "which needs no copy at all.")
    w = w8.to(torch.float32) * w_scale.to(torch.float32).reshape(-1, 1)
    return rotate(w.to(torch.bfloat16))


def linear_dx(dy, w):
    """``dL/dx`` for a linear with weight ``w``: ``dy [.., N] @ w [N, K] -> [.., K]``.

    ``w`` is the *unrotated* ``[N, K]`` weight -- ``dequant_weight(...)`` of an
    INT8 weight, or the bf16 weight itself.
    """
    if dy.shape[-1] != w.shape[0]:
        raise ValueError(f"dy has {dy.shape[-1]} columns but w has {w.shape[0]} rows")
    return dy @ w


def linear_dw(dy, x):
    """``dL/dW`` for a linear: ``dy [.., N]^T @ x [.., K] -> [N, K]`` (bf16).

    The batch dimension is the contraction, so the batch dims must agree.
    ``x`` is the unrotated activation.  See :func:`linear_dw_int8` for the
    variant whose GEMM operands are both int8.
    """
    if dy.shape[-2] != x.shape[-2]:
        raise ValueError(
            f"dy has {dy.shape[-2]} rows but x has {x.shape[-2]}: the batch "
            f"dims must match for dy^T @ x")
    return dy.reshape(-1, dy.shape[-1]).transpose(0, 1) @ x.reshape(-1, x.shape[-1])


def linear_dw_int8(dy, xq, x_scale):
    """``dL/dW`` with both GEMM operands int8 (no counterpart in the reference).

    ``xq`` and ``x_scale`` are the forward's rotated int8 activation and its
    row scales (``quantize(x)``).  The forward computed, in the rotated basis,
    ``y = (xs[m] xq[m,:]) . (ws[n] w8[n,:])``; with the straight-through
    convention the gradient of the rotated weight is ``dy^T (xs xq)`` and,
    because the rotation H is symmetric and its own inverse,
    ``dW = rotate_K(dy^T (xs xq))``.  ``g = dy * xs`` is quantized per column
    (the scale must not depend on the contraction index m), the int8 GEMM
    ``gq^T xq`` is exact in int32, and the epilogue applies the column scale
    before the rotation: ``dW = rotate(bf16(acc[n,k] * tg[n]))``.
    Returns bf16 [N, K].
    """
    lib = _lib()
    if dy.dtype != torch.bfloat16:
        dy = dy.to(torch.bfloat16)
    dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
    xq2 = xq.reshape(-1, xq.shape[-1]).contiguous()
    m, n = dy2.shape
    k = xq2.shape[1]
    if xq2.shape[0] != m:
        raise ValueError(f"dy has {m} rows but xq has {xq2.shape[0]}: the batch "
                         f"dims must match for dy^T @ x")
    if xq2.dtype != torch.int8:
        raise TypeError("xq must be the int8 activation of the forward")
    xs = expand_scale(x_scale.reshape(-1), m, dy.device)
    # one C call: column quantizer -> int8 GEMM (both operands MN-major) -> rotation
    ws_bytes = lib.xpuint8_linear_dw_int8_workspace_bytes(m, n, k)
    if ws_bytes < 0:
        raise ValueError(f"linear_dw_int8: bad sizes M={m}, N={n}, K={k}")
    work = torch.empty((ws_bytes,), dtype=torch.uint8, device=dy.device)
    dw = torch.empty((n, k), dtype=torch.bfloat16, device=dy.device)
    rc = lib.xpuint8_linear_dw_int8_stream(_stream(dy.device), _ptr(dy2), _ptr(xq2), _ptr(xs),
                                           _ptr(dw), _ptr(work), m, n, k)
    if rc != 0:
        _err(lib, "linear_dw_int8")
    return dw


class _Int8LinearFn(torch.autograd.Function):
    """The INT8 linear as an autograd op (ops.py:241-289).

    The backward is :func:`linear_dx` against the dequantized weight
    (``mode="dense"``) or :func:`linear_dx_int8`, which keeps the weight in
    int8 and quantizes ``dy`` instead.  No weight gradient: the INT8 weight is
    a frozen int8 buffer.
    """

    @staticmethod
    def forward(ctx, x, w8, w_scale, bias, mode):
        ctx.save_for_backward(w8, w_scale)
        ctx.mode = mode
        ctx.input_dtype = x.dtype
        return linear(x, w8, w_scale, bias)

    @staticmethod
    def backward(ctx, dy):
        w8, w_scale = ctx.saved_tensors
        dbias = dy.reshape(-1, dy.shape[-1]).sum(dim=0) if ctx.needs_input_grad[3] else None
        dy = dy.to(torch.bfloat16)
        if ctx.mode == "int8":
            dx = linear_dx_int8(dy, w8, w_scale)
        elif ctx.mode == "dense":
            dx = linear_dx(dy, dequant_weight(w8, w_scale))
        else:
            raise ValueError(f"unknown backward mode {ctx.mode!r}; "
                             f"use 'dense' or 'int8'")
        return dx.to(ctx.input_dtype), None, None, dbias, None


def int8_linear(x, w8, w_scale, bias=None, *, mode="dense"):
    """The INT8 linear, differentiable (ops.py:292-317).

    ``mode="dense"`` dequantizes the weight for the backward; ``mode="int8"``
    keeps it in int8 and quantizes ``dy`` (:func:`linear_dx_int8`).
    """
    if mode not in ("dense", "int8"):
        raise ValueError(f"unknown backward mode {mode!r}; use 'dense' or 'int8'")
    return _Int8LinearFn.apply(x, w8, w_scale, bias, mode)


def quantize_row_torch(x):
    """The per-row quantizer as a torch chain -- the definition (ops.py:320-330).

    ``scale = (amax / 127).clamp_min(1e-30)``, ``round(x / scale)`` clamped to
    +-127, both true divisions (see ``_div``: on CUDA a division by a python
    scalar would be a reciprocal multiply).
    """
    xf = x.to(torch.float32)
    scale = _div(xf.abs().amax(dim=-1, keepdim=True), 127.0).clamp_min(1e-30)
    q = torch.round(_div(xf, scale)).clamp_(-127, 127).to(torch.int8)
    return q.contiguous(), scale.squeeze(-1).contiguous()


def quantize_row(x, col_scale=None):
    """Per-row symmetric int8 quantization, no rotation: bf16 [.., K] -> (int8, fp32).

    The library's fused quantizer (one read pass for the maximum, one for the
    values; true divisions, so it is bit-identical to
    :func:`quantize_row_torch`).  With ``col_scale`` ([K]) the quantized
    tensor is ``bf16(x * bf16(col_scale))`` -- the column-scaled gradient of
    :func:`linear_dx_int8`, computed inside the same pass.
    """
    lib = _lib()
    x2, shape = _flat2d(x)
    m, k = x2.shape
    cs = None
    if col_scale is not None:
        cs = expand_scale(col_scale, k, x.device)
    q = torch.empty((m, k), device=x.device, dtype=torch.int8)
    scale = torch.empty((m,), device=x.device, dtype=torch.float32)
    rc = lib.xpuint8_quantize_row_stream(_stream(x.device), _ptr(x2), _ptr(cs), _ptr(q),
                                         _ptr(scale), m, k)
    if rc != 0:
        _err(lib, "quantize_row")
    return q.reshape(*shape[:-1], k), scale.reshape(shape[:-1])


def linear_dx_int8(dy, w8, w_scale):
    """``dL/dx`` against the weight *still in int8* (ops.py:353-377).

    ``dx = (dy * s) @ W8``, then the ConvRot rotation undone.  Here the column
    scale and the row quantizer are one kernel, and the int8 GEMM reads ``w8``
    as stored ([N, K], N the contraction: an MN-major B operand) and applies
    the row scales in its epilogue.
    """
    lib = _lib()
    d2 = dy.to(torch.bfloat16).reshape(-1, dy.shape[-1])
    if not d2.is_contiguous():
        d2 = d2.contiguous()
    n, k = w8.shape
    if d2.shape[1] != n:
        raise ValueError(f"dy has {d2.shape[1]} columns but w8 has {n} rows")
    m = d2.shape[0]
    ws = expand_scale(w_scale, n, dy.device)
    # one C call: column-scaled row quantizer -> int8 GEMM -> rotation
    ws_bytes = lib.xpuint8_linear_dx_int8_workspace_bytes(m, n, k)
    if ws_bytes < 0:
        raise ValueError(f"linear_dx_int8: bad sizes M={m}, N={n}, K={k}")
    work = torch.empty((ws_bytes,), dtype=torch.uint8, device=dy.device)
    dx = torch.empty((m, k), dtype=torch.bfloat16, device=dy.device)
    rc = lib.xpuint8_linear_dx_int8_stream(_stream(dy.device), _ptr(d2), _ptr(w8.contiguous()),
                                           _ptr(ws), _ptr(dx), _ptr(work), m, n, k)
    if rc != 0:
        _err(lib, "linear_dx_int8")
    return dx.reshape(*dy.shape[:-1], k)


def expand_scale(scale, n, device=None):
    """A flat fp32 ``[n]`` scale, broadcasting a per-tensor scalar (ops.py:380-408).

    The kernels index ``scale[i]`` for every ``i < n``, so a scalar *must* be
    materialised.  A flat fp32 ``[n]`` tensor on the right device is returned
    unchanged (no copy on the hot path).
    """
    if not isinstance(scale, torch.Tensor):
        if not isinstance(scale, (float, int)):
            raise TypeError(f"scale must be a tensor or a python float, "
                            f"got {type(scale).__name__}")
        if device is None:
            raise TypeError("a python-scalar scale needs an explicit device")
        return torch.full((n,), float(scale), device=device, dtype=torch.float32)
    if (scale.dtype == torch.float32 and scale.dim() == 1 and scale.numel() == n
            and scale.is_contiguous() and (device is None or scale.device == device)):
        return scale
    s = scale.reshape(-1).to(device=device or scale.device, dtype=torch.float32)
    if s.numel() == 1 and n != 1:
        s = s.expand(n)
    return s.contiguous()


def _dims(x, w8, act):
    m = 1
    for d in x.shape[:-1]:
        m *= int(d)
    return m, int(w8.shape[0]), int(w8.shape[1])


def unsupported_reason(x, w8, w_scale, act=None):
    """Why this call cannot use the fused kernels, or ``None`` if it can
    (ops.py:418-476; the messages are the reference's, with CUDA for XPU)."""
    if not isinstance(x, torch.Tensor) or not isinstance(w8, torch.Tensor):
        return "activation and weight must be torch tensors"
    if x.dtype not in (torch.bfloat16, torch.float32):
        return (f"activation dtype {x.dtype} is not bfloat16 or float32 "
                f"(the kernels consume bf16)")
    if w8.dtype != torch.int8 or w8.dim() != 2:
        return f"weight must be an int8 [N, K] tensor, got {w8.dtype} {tuple(w8.shape)}"
    if act is not None and act not in ACTIVATIONS:
        return (f"unknown activation {act!r}; expected None or one of "
                f"{', '.join(sorted(ACTIVATIONS))}")
    k = int(w8.shape[1])
    want = k * 2 if act in PAIRED_ACTIVATIONS else k
    if x.shape[-1] != want:
        return (f"activation has {x.shape[-1]} columns but this weight wants "
                f"{want} (K={k}{' with two halves' if want != k else ''})")
    # 256 is a multiple of 16, so this covers the vector width too
    if k % 256:
        return f"K={k} is not a multiple of the ConvRot group size (256)"
    if w8.shape[0] % 16:
        return (f"N={w8.shape[0]} is not a multiple of 16; the dequant epilogue "
                f"reads the output 16 columns at a time and would drop the tail")
    if isinstance(w_scale, torch.Tensor):
        if not w_scale.is_floating_point():
            return (f"weight scale dtype {w_scale.dtype} is not floating point; "
                    f"a per-channel scale is amax/127")
        if w_scale.dim() > 2:
            return (f"weight scale has {w_scale.dim()} dims; expected a scalar, "
                    f"[N] or [N, 1]")
        if w_scale.numel() not in (1, w8.shape[0]):
            return (f"weight scale has {w_scale.numel()} values; expected 1 or "
                    f"N={w8.shape[0]}")
    elif not isinstance(w_scale, (float, int)):
        return "weight scale must be a tensor or a python float"
    if load() is None:
        return "libxpuint8.so is not available (see xpu_kernels.int8._lib)"
    if x.device.type != "cuda":
        return (f"activation is on {x.device}; the kernels need a CUDA tensor "
                f"(this build of libxpuint8 has no XPU or CPU path)")
    if w8.device != x.device:
        return (f"weight is on {w8.device} but the activation is on {x.device}; "
                f"the kernels take raw pointers into one stream")
    return None


def dequant(acc, x_scale, w_scale, bias=None):
    """bf16 dequant of an int32 [M, N] accumulator with per-row and per-column scales."""
    lib = _lib()
    if acc.dim() != 2 or acc.dtype != torch.int32:
        raise TypeError("acc must be an int32 [M, N] tensor")
    acc = acc.contiguous()
    m, n = acc.shape
    out = torch.empty((m, n), device=acc.device, dtype=torch.bfloat16)
    xs, ws = expand_scale(x_scale, m, acc.device), expand_scale(w_scale, n, acc.device)
    b = None if bias is None else expand_scale(bias, n, acc.device)
    rc = lib.xpuint8_dequant_epilogue_stream(_stream(acc.device), _ptr(acc), _ptr(out), _ptr(xs),
                                             _ptr(ws), _ptr(b), m, n)
    if rc != 0:
        _err(lib, "dequant")
    return out


def dequant_slice(acc, x_scale, w_scale, bias=None):
    """As :func:`dequant`, for a [M, N] column slice of a wider [M, S] accumulator
    read in place with its row stride (ops.py:500-525)."""
    lib = _lib()
    if acc.dim() != 2 or acc.dtype != torch.int32:
        raise TypeError("acc must be an int32 [M, N] tensor")
    if acc.stride(1) != 1:
        raise TypeError("acc must have unit column stride")
    m, n = acc.shape
    out = torch.empty((m, n), device=acc.device, dtype=torch.bfloat16)
    xs, ws = expand_scale(x_scale, m, acc.device), expand_scale(w_scale, n, acc.device)
    b = None if bias is None else expand_scale(bias, n, acc.device)
    rc = lib.xpuint8_dequant_epilogue_slice_stream(_stream(acc.device), _ptr(acc), _ptr(out),
                                                   _ptr(xs), _ptr(ws), _ptr(b), m, n,
                                                   acc.stride(0))
    if rc != 0:
        _err(lib, "dequant_slice")
    return out


def dequant_act_quantize(acc, x_scale, w_scale, activation="situ"):
    """Dequant, activate, rotate and quantize an up-projection accumulator in one
    pass (ops.py:528-568): int32 [M, 2K] ([hidden | gate]) for ``situ`` and
    ``geglu_erf``, [M, K] for ``gelu_erf`` -> ``(int8 [M, K], fp32 [M])``."""
    lib = _lib()
    act_id = ACTIVATIONS[activation]
    paired = activation in PAIRED_ACTIVATIONS
    if acc.dim() != 2 or acc.dtype != torch.int32:
        raise TypeError("acc must be an int32 [M, N] tensor")
    acc = acc.contiguous()
    m, n = acc.shape
    if paired:
        if n % 2:
            raise TypeError(f"acc must be an int32 [M, 2K] tensor for {activation}, got {n} columns")
        k = n // 2
    else:
        k = n
    q = torch.empty((m, k), device=acc.device, dtype=torch.int8)
    scale = torch.empty((m,), device=acc.device, dtype=torch.float32)
    xs = expand_scale(x_scale, m, acc.device)
    ws = expand_scale(w_scale, n, acc.device)
    rc = lib.xpuint8_dequant_act_quantize_stream(_stream(acc.device), _ptr(acc), _ptr(q),
                                                 _ptr(scale), _ptr(xs), _ptr(ws), m, k, act_id)
    if rc != 0:
        _err(lib, "dequant_act_quantize")
    return q, scale


def int_mm(a, b, layout: int = 0):
    """The library's exact int8 GEMM: ``layout=0`` is ``a @ b.T`` (``a`` [M,K],
    ``b`` [N,K], what ``torch._int_mm(a, b.t())`` computes), ``1`` is
    ``a @ b`` (``b`` [K,N]), ``2`` is ``a.T @ b`` (``a`` [K,M])."""
    lib = _lib()
    if a.dtype != torch.int8 or b.dtype != torch.int8 or a.dim() != 2 or b.dim() != 2:
        raise TypeError("int_mm takes two int8 matrices")
    a, b = a.contiguous(), b.contiguous()
    if layout == 0:
        m, k = a.shape
        n = b.shape[0]
        kb = b.shape[1]
    elif layout == 1:
        m, k = a.shape
        kb, n = b.shape
    elif layout == 2:
        k, m = a.shape
        kb, n = b.shape
    else:
        raise ValueError("layout must be 0, 1 or 2")
    if kb != k:
        raise ValueError(f"K mismatch: {k} vs {kb}")
    c = torch.empty((m, n), dtype=torch.int32, device=a.device)
    rc = lib.xpuint8_int_mm_stream(_stream(a.device), _ptr(a), _ptr(b), _ptr(c), m, n, k, layout, n)
    if rc != 0:
        _err(lib, "int_mm")
    return c


def _linear_from_quantized(xq, xs, w8, w_scale, bias=None):
    """The GEMM with the fused dequant epilogue on an already quantized
    activation: bf16 [M, N]."""
    lib = _lib()
    m, k = xq.shape
    n = w8.shape[0]
    dev = xq.device
    ws = expand_scale(w_scale, n, dev)
    b = None if bias is None else expand_scale(bias, n, dev)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    rc = lib.xpuint8_int_mm_dequant_stream(_stream(dev), _ptr(xq), _ptr(w8.contiguous()),
                                           _ptr(out), _ptr(xs), _ptr(ws), _ptr(b), m, n, k, 0, n)
    if rc != 0:
        _err(lib, "linear")
    return out


def linear_acc(x, w8, w_scale, act: Optional[str] = None):
    """The GEMM without the output dequant: ``(int32 [M, N], fp32 [M])`` (ops.py:571-588)."""
    if act is None:
        xq, xs = quantize(x)
    else:
        xq, xs = quantize_act(x, act)
    if w8.dtype != torch.int8 or w8.dim() != 2:
        raise TypeError("w8 must be an int8 [N, K] tensor")
    if xq.shape[-1] != w8.shape[1]:
        raise ValueError(f"K mismatch: activation {xq.shape[-1]} vs weight {w8.shape[1]}")
    acc = int_mm(xq.reshape(-1, xq.shape[-1]), w8)
    return acc, xs.reshape(-1)


def linear(x, w8, w_scale, bias=None, act: Optional[str] = None, residual=None,
           residual_scale=None, return_acc: bool = False):
    """INT8 ConvRot linear: bf16/fp32 [.., K] -> bf16/fp32 [.., N] (ops.py:591-646).

    ``act`` folds an activation into the input quantizer; ``residual`` /
    ``residual_scale`` apply ``residual + residual_scale * out`` after the
    dequant; ``return_acc`` returns ``(int32 [M, N], fp32 [M], fp32 [N])``
    instead of the output.  Raises ``TypeError`` with the message of
    :func:`unsupported_reason`.
    """
    reason = unsupported_reason(x, w8, w_scale, act)
    if reason is not None:
        raise TypeError(reason)
    if return_acc and (bias is not None or residual is not None):
        raise ValueError("return_acc skips the epilogue, so bias and residual "
                         "cannot be applied")
    m, n, k = _dims(x, w8, act)
    input_dtype = x.dtype
    x2 = x.reshape(m, -1)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(dtype=torch.bfloat16)
    if not x2.is_contiguous():
        x2 = x2.contiguous()

    if return_acc:
        acc, xs = linear_acc(x2, w8, w_scale, act)
        return acc, xs, expand_scale(w_scale, n, acc.device)

    lib = _lib()
    dev = x.device
    ws = expand_scale(w_scale, n, dev)
    b = None if bias is None else expand_scale(bias, n, dev)
    xq = torch.empty((m, k), dtype=torch.int8, device=dev)
    xs = torch.empty((m,), dtype=torch.float32, device=dev)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    w8c = w8 if w8.is_contiguous() else w8.contiguous()
    rc = lib.xpuint8_linear_stream(_stream(dev), _ptr(x2), _ptr(w8c), _ptr(ws), _ptr(b),
                                   _ptr(out), _ptr(xq), _ptr(xs), m, n, k,
                                   0 if act is None else ACTIVATIONS[act])
    if rc != 0:
        _err(lib, "linear")
    if residual is not None:
        residual = residual.reshape(m, n).to(
            out.dtype if input_dtype == torch.bfloat16 else input_dtype)
        if input_dtype != torch.bfloat16:
            out = out.to(dtype=input_dtype)
        out = torch.addcmul(residual, out, residual_scale)
    out = out.reshape(*x.shape[:-1], n)
    return out if input_dtype == torch.bfloat16 else out.to(dtype=input_dtype)


def linear_split(x, w8, w_scale, bias=None, parts: int = 3, act: Optional[str] = None):
    """The INT8 linear against ``parts`` concatenated projections, one output
    per projection: ``(y_0, .., y_{parts-1})``, each bf16 [.., N] with
    ``N = w8.shape[0] // parts``.

    The fused qkv projection: ``w8 = cat([Wq8, Wk8, Wv8])`` (prepared as one
    weight, or the parts' prepared weights concatenated with their scales),
    ``bias`` the concatenated biases or None.  One quantizer launch and one
    GEMM whose drain dequantizes each part straight into its own output --
    bit-identical to ``linear_acc`` followed by :func:`dequant_slice` per part
    (the reference's pattern, ops.py:500-525 with selftest.py:67-72), without
    the int32 [M, parts*N] accumulator round trip through HBM.
    """
    reason = unsupported_reason(x, w8, w_scale, act)
    if reason is not None:
        raise TypeError(reason)
    m, n_all, k = _dims(x, w8, act)
    if parts < 1 or parts > 8 or n_all % parts:
        raise ValueError(f"{n_all} output channels do not split into {parts} equal parts "
                         f"(1 <= parts <= 8)")
    n = n_all // parts
    if n % 32:
        raise ValueError(f"each part's width must be a multiple of 32 (got {n})")
    x2 = x.reshape(m, -1)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(dtype=torch.bfloat16)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    lib = _lib()
    dev = x.device
    ws = expand_scale(w_scale, n_all, dev)
    b = None if bias is None else expand_scale(bias, n_all, dev)
    xq = torch.empty((m, k), dtype=torch.int8, device=dev)
    xs = torch.empty((m,), dtype=torch.float32, device=dev)
    outs = [torch.empty((m, n), dtype=torch.bfloat16, device=dev) for _ in range(parts)]
    table = (ctypes.c_void_p * parts)(*[o.data_ptr() for o in outs])
    w8c = w8 if w8.is_contiguous() else w8.contiguous()
    rc = lib.xpuint8_linear_split_stream(_stream(dev), _ptr(x2), _ptr(w8c), _ptr(ws), _ptr(b),
                                         table, parts, _ptr(xq), _ptr(xs), m, n, k,
                                         0 if act is None else ACTIVATIONS[act])
    if rc != 0:
        _err(lib, "linear_split")
    return tuple(o.reshape(*x.shape[:-1], n) for o in outs)


def _rope_rows(x, what):
    """(row stride, B, S, H, D) of a [B, S, H, D] view whose heads are
    contiguous within a row and whose rows are uniformly strided (a slice of a
    fused qkv tensor qualifies)."""
    if x.dim() != 4:
        raise ValueError(f"{what} must be [B, S, H, D], got {tuple(x.shape)}")
    B, S, H, D = x.shape
    st = x.stride()
    if st[3] != 1 or st[2] != D or (B > 1 and st[0] != S * st[1]):
        raise ValueError(f"{what}: the heads of a row must be contiguous and the rows "
                         f"uniformly strided (strides {st})")
    return st[1], B, S, H, D


def _rope_freqs(freqs_cis, B, S, D, dev):
    f = freqs_cis
    if f.dim() == 6:              # [B or 1, S or 1, 1, D/2, 2, 2]
        f = f.squeeze(2)
    if f.dim() != 5 or f.shape[2:] != (D // 2, 2, 2) or f.shape[0] not in (1, B) or \
            f.shape[1] not in (1, S):
        raise ValueError(f"freqs_cis must be [1|B, 1|S, 1, D/2, 2, 2], got {tuple(freqs_cis.shape)}")
    return f.to(device=dev, dtype=torch.float32).contiguous()


def _aligned16(t):
    return t.clone() if t.data_ptr() % 16 else t


def _rms_rope(x, freqs_cis, scale, epsilon, split_half, x_scale=None, w_scale=None):
    lib = _lib()
    is_acc = x_scale is not None
    if is_acc and x.dtype != torch.int32:
        raise TypeError("the accumulator must be int32")
    if not is_acc and x.dtype != torch.bfloat16:
        raise TypeError("x must be bfloat16")
    ld, B, S, H, D = _rope_rows(x, "x")
    # the kernel reads runs of four elements: 16-byte (int32) / 8-byte (bf16)
    # aligned rows; an odd view is copied first
    if x.data_ptr() % (16 if is_acc else 8) or ld % 4:
        x = x.contiguous() if not x.is_contiguous() else x.clone()
        ld = H * D
    dev = x.device
    f = _aligned16(_rope_freqs(freqs_cis, B, S, D, dev))
    w = _aligned16(scale.reshape(-1).to(device=dev, dtype=torch.float32).contiguous())
    if w.numel() != D:
        raise ValueError(f"scale must have {D} elements")
    xs = ws = None
    if is_acc:
        xs = x_scale.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
        ws = _aligned16(w_scale.reshape(-1).to(device=dev, dtype=torch.float32).contiguous())
        if xs.numel() != B * S or ws.numel() != H * D:
            raise ValueError("x_scale must have B*S elements and w_scale H*D")
    out = torch.empty((B, S, H, D), dtype=torch.bfloat16, device=dev)
    if out.numel() == 0:
        return out
    rc = lib.xpuint8_rms_rope_stream(_stream(dev), ctypes.c_void_p(x.data_ptr()), 1 if is_acc else 0,
                                     ld, _ptr(xs), _ptr(ws), _ptr(w), _ptr(f), f.shape[0], f.shape[1],
                                     _ptr(out), H * D, B, S, H, D, float(epsilon),
                                     1 if split_half else 0)
    if rc != 0:
        _err(lib, "rms_rope")
    return out


def rms_rope(x, freqs_cis, scale, epsilon=1e-6, split_half=True):
    """RMS norm (with the per-dim ``scale``) then rotary embedding of attention
    heads, bf16 ``[B, S, H, D]`` -> bf16 (triton/rope.py:360-376 ``_rows``; the
    chain ``rope_split_half(rms_norm(x, scale, eps), freqs_cis)`` of
    triton/reference.py:63-98).  ``freqs_cis`` is ``[1|B, 1|S, 1, D/2, 2, 2]``
    holding ``[[cos, -sin], [sin, cos]]`` per pair; ``split_half`` rotates
    ``(d, d + D/2)``, otherwise ``(2i, 2i + 1)``.  D is 64, 128 or 256."""
    return _rms_rope(x, freqs_cis, scale, epsilon, split_half)


def rms_rope_dequant(acc, freqs_cis, scale, x_scale, w_scale, epsilon=1e-6, split_half=True):
    """:func:`rms_rope` reading the INT8 GEMM's int32 accumulator (a
    ``[B, S, H, D]`` view, e.g. a slice of the fused qkv accumulator) with the
    dequant folded into the load: ``bf16(float(acc) * (w_scale * x_scale))``
    (triton/rope.py:378-408 ``_rows_dq``).  ``x_scale`` is ``[B, S]`` or
    ``[B*S]``, ``w_scale`` the slice's ``[H*D]`` column scales."""
    return _rms_rope(acc, freqs_cis, scale, epsilon, split_half, x_scale, w_scale)


def rms_rope_split_half(q, k, freqs_cis, q_scale, k_scale=None, epsilon=1e-6):
    """``(rms_rope(q), rms_rope(k))`` with split-half rotation
    (triton/rope.py:694)."""
    if k_scale is None:
        k_scale = q_scale
    return (rms_rope(q, freqs_cis, q_scale, epsilon), rms_rope(k, freqs_cis, k_scale, epsilon))


def rms_rope_split_half_dequant(q_acc, k_acc, freqs_cis, q_w, k_w, x_scale, q_scale,
                                k_scale=None, epsilon=1e-6, split_half=True):
    """The q and k slices of a fused qkv accumulator through
    :func:`rms_rope_dequant` (triton/rope.py:643-652: ``q_w`` / ``k_w`` are
    the slices' column scales, ``q_scale`` / ``k_scale`` the norms')."""
    if k_scale is None:
        k_scale = q_scale
    if k_w is None:
        k_w = q_w
    return (rms_rope_dequant(q_acc, freqs_cis, q_scale, x_scale, q_w, epsilon, split_half),
            rms_rope_dequant(k_acc, freqs_cis, k_scale, x_scale, k_w, epsilon, split_half))


def ffn(x, up_w8, up_scale, down_w8, down_scale, down_bias=None, act="situ"):
    """``act(up(x)) @ down.T`` with the bf16 [M, 2*ffn] intermediate never
    written (ops.py:649-719).

    ``up_w8`` is [2*ffn, K] holding ``[hidden | gate]`` for a paired activation
    (``situ``, ``geglu_erf``) and [ffn, K] for ``gelu_erf``; ``down_w8`` is
    [K, ffn].  For ``geglu_erf`` the dequant and the GEGLU run in the
    up-projection GEMM's epilogue, which writes ``y`` (bf16 [M, ffn]); the
    rotate+quantize of ``y`` is then exactly the reference chain's
    ``quantize(hidden * gelu(gate))``.
    """
    if act not in ACTIVATIONS:
        raise TypeError(f"unknown activation {act!r}; "
                        f"known: {', '.join(sorted(ACTIVATIONS))}")
    if act not in ("situ", "geglu_erf", "gelu_erf"):
        raise TypeError(f"the fused FFN supports situ, geglu_erf and gelu_erf, "
                        f"not {act!r}")
    paired = act in PAIRED_ACTIVATIONS
    reason = unsupported_reason(x, up_w8, up_scale, None)
    if reason is not None:
        raise TypeError(reason)
    m, n, k = _dims(x, up_w8, None)
    if paired and n % 2:
        raise TypeError(f"up-projection N={n} must be 2*ffn for the {act} "
                        f"activation")
    inner = n // 2 if paired else n
    if inner % 256 or inner % 16:
        raise TypeError(f"the FFN's inner width {inner} must be a multiple of "
                        f"256 (and of 16) for the fused {act} epilogue")
    if down_w8.dtype != torch.int8 or down_w8.dim() != 2:
        raise TypeError(f"down weight must be an int8 [K, ffn] tensor, got "
                        f"{down_w8.dtype} {tuple(down_w8.shape)}")
    if tuple(down_w8.shape) != (k, inner):
        raise TypeError(f"down weight is {tuple(down_w8.shape)}, expected "
                        f"{(k, inner)}")
    if down_w8.device != x.device:
        raise TypeError(f"down weight is on {down_w8.device} but the activation "
                        f"is on {x.device}")
    if isinstance(down_scale, torch.Tensor):
        if down_scale.dtype != torch.float32 or down_scale.dim() > 2:
            raise TypeError("down weight scale must be a float32 scalar or [K]")
        if down_scale.numel() not in (1, k):
            raise TypeError(f"down weight scale has {down_scale.numel()} values; "
                            f"expected 1 or K={k}")
    elif not isinstance(down_scale, (float, int)):
        raise TypeError("down weight scale must be a tensor or a python float")

    lib = _lib()
    device = x.device
    input_dtype = x.dtype
    x2 = x.reshape(m, k)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(dtype=torch.bfloat16)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    act_id = ACTIVATIONS[act]
    nbytes = lib.xpuint8_ffn_workspace_bytes(m, k, inner, act_id)
    ws = torch.empty((nbytes,), dtype=torch.uint8, device=device)
    out = torch.empty((m, k), dtype=torch.bfloat16, device=device)
    us = expand_scale(up_scale, n, device)
    dsc = expand_scale(down_scale, k, device)
    db = None if down_bias is None else expand_scale(down_bias, k, device)
    rc = lib.xpuint8_ffn_stream(_stream(device), _ptr(x2), _ptr(up_w8.contiguous()), _ptr(us),
                                _ptr(down_w8.contiguous()), _ptr(dsc), _ptr(db), _ptr(out),
                                _ptr(ws), m, k, inner, act_id)
    if rc != 0:
        _err(lib, "ffn")
    out = out.reshape(*x.shape[:-1], k)
    return out if input_dtype == torch.bfloat16 else out.to(dtype=input_dtype)


def ffn_situ(x, up_w8, up_scale, down_w8, down_scale, down_bias=None):
    """``situ(up(x)) @ down.T`` -- :func:`ffn` with MossImage's activation."""
    return ffn(x, up_w8, up_scale, down_w8, down_scale, down_bias, act="situ")


class TrainableInt8Linear(torch.nn.Module):
    """A linear whose parameter stays bf16 and is quantized on every forward
    (ops.py:730-789): the straight-through estimator.

    ``backward="ste"`` computes ``dx = dy @ W`` with the bf16 parameter;
    ``backward="dense"`` uses the dequantized weight.  ``dw="bf16"`` (the
    reference's) computes ``dW = dy^T @ x`` in bf16; ``dw="int8"`` uses
    :func:`linear_dw_int8` on the forward's int8 activation.
    """

    def __init__(self, weight, bias=None, *, backward="ste", dw="bf16"):
        super().__init__()
        if weight.dtype not in (torch.bfloat16, torch.float32):
            raise TypeError(f"the weight must be bfloat16 or float32, got {weight.dtype}")
        if backward not in ("ste", "dense"):
            raise ValueError(f"unknown backward mode {backward!r}; "
                             f"use 'ste' or 'dense'")
        if dw not in ("bf16", "int8"):
            raise ValueError(f"unknown weight-gradient mode {dw!r}; use 'bf16' or 'int8'")
        self.weight = torch.nn.Parameter(weight.detach())
        self.bias = None if bias is None else torch.nn.Parameter(
            bias.detach().to(self.weight.dtype))
        self.backward = backward
        self.dw = dw

    @classmethod
    def from_linear(cls, mod, *, backward="ste", dw="bf16"):
        return cls(mod.weight.detach(), getattr(mod, "bias", None), backward=backward, dw=dw)

    def forward(self, x):
        return _TrainableInt8LinearFn.apply(x, self.weight, self.bias, self.backward, self.dw)

    def extra_repr(self):
        return (f"{tuple(self.weight.shape)}, backward={self.backward}, dw={self.dw}, "
                f"bias={self.bias is not None}")


class _TrainableInt8LinearFn(torch.autograd.Function):
    """The autograd op behind :class:`TrainableInt8Linear` (ops.py:792-824)."""

    @staticmethod
    def forward(ctx, x, weight, bias, mode, dw_mode):
        w8, ws = prepare_weight_fused(weight)
        if dw_mode == "int8":
            reason = unsupported_reason(x, w8, ws)
            if reason is not None:
                raise TypeError(reason)
            x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
            xq, xs = quantize(x2)
            y = _linear_from_quantized(xq, xs, w8, ws, bias).reshape(*x.shape[:-1], w8.shape[0])
            y = y if x.dtype == torch.bfloat16 else y.to(x.dtype)
            ctx.save_for_backward(x, weight, w8, ws, xq, xs)
        else:
            y = linear(x, w8, ws, bias)
            ctx.save_for_backward(x, weight, w8, ws)
        ctx.mode = mode
        ctx.dw_mode = dw_mode
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        saved = ctx.saved_tensors
        x, weight, w8, ws = saved[:4]
        dy = dy.reshape(-1, dy.shape[-1])
        x2 = x.reshape(-1, x.shape[-1])
        w = dequant_weight(w8, ws) if ctx.mode == "dense" else weight
        dx = dy @ w.to(dy.dtype)
        if ctx.dw_mode == "int8":
            dw = linear_dw_int8(dy, saved[4], saved[5])
        else:
            dw = linear_dw(dy, x2)
        db = dy.sum(dim=0) if ctx.has_bias else None
        if dw.dtype != weight.dtype:
            dw = dw.to(weight.dtype)
        return (dx.reshape(x.shape[:-1] + (dx.shape[-1],)), dw, db, None, None)


class Int8Linear(torch.nn.Module):
    """Drop-in ``nn.Linear`` replacement for inference with prepared weights
    (ops.py:831-902)."""

    def __init__(self, w8, w_scale, bias=None, *, backward="dense"):
        super().__init__()
        self.register_buffer("w8", w8.detach())
        self.register_buffer("w_scale", w_scale.detach().to(torch.float32))
        self.bias = None if bias is None else torch.nn.Parameter(
            bias.detach().to(torch.float32), requires_grad=False)
        if backward not in ("dense", "int8"):
            raise ValueError(f"unknown backward mode {backward!r}; "
                             f"use 'dense' or 'int8'")
        self.backward = backward

    @classmethod
    def from_linear(cls, mod, *, backward="dense"):
        q, scale = prepare_weight(mod.weight.detach())
        return cls(q, scale, getattr(mod, "bias", None), backward=backward)

    def forward(self, x):
        return int8_linear(x, self.w8, self.w_scale, self.bias, mode=self.backward)

    def dense_weight(self, refresh=False):
        """The unrotated bf16 weight, dequantized once and cached (not inside a
        device-graph capture)."""
        cached = getattr(self, "_dense", None)
        if cached is None or refresh:
            if is_capturing():
                raise RuntimeError(
                    "Int8Linear.dense_weight() materializes a second, "
                    "full-precision copy of the weight; inside a device-graph "
                    "capture it would be captured and re-computed on every "
                    "replay. Call it before capturing -- "
                    "xpu_kernels.prepare_for_capture(model) does it for a whole "
                    "model.")
            cached = dequant_weight(self.w8, self.w_scale)
            self._dense = cached
        return cached

    def dx(self, dy):
        """``dL/dx`` given ``dL/dy`` -- the backward's activation gradient."""
        return linear_dx(dy, self.dense_weight())

    def extra_repr(self):
        n, k = self.w8.shape
        return f"in_features={k}, out_features={n}, bias={self.bias is not None}"
