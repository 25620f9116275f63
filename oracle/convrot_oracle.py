"""CPU oracle for the ConvRot INT8 linear path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the arithmetic of the reference library's
ConvRot INT8 path (okolenmi/oko-xpu-kernels v0.4.0).  It is the checker the
CUDA kernels are compared against.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import it; the product path
(``xpu_kernels``) never does, and fails loudly when its CUDA library is absent.

Every function names the reference file:line it follows (paths are relative to
the reference project root).  The reference's device code is SYCL for an Intel
Xe2 GPU (``src/xpuint8.cpp``) and cannot be compiled or run here, so this
restatement follows its source; the parts of the reference that are plain torch
(``quantize_row_torch``, ``linear_dw``, ``expand_scale``,
``reference/convrot_linear.py``, the chains of ``prepare_weight`` and
``dequant_weight_torch``) were run on CPU to produce the golden fixtures under
``tests/golden/`` that pin this file (see ``tests/golden/make_golden.py``).

Floating point follows the reference kernel's source order:

* bf16 <-> fp32 conversions are exact widenings / round-to-nearest-even;
* the group-256 rotation applies the four radix-4 ``H4/2`` butterflies in the
  reference's order and association (``rotate_groups``), every step in fp32;
* row scales are ``max(amax / 127, 1e-30)`` with an IEEE division, and the
  activation quantizer multiplies by the IEEE reciprocal ``1/s``;
* integer GEMMs are exact (int8 x int8 accumulated in int32).

``order="kernel"`` selects the association the CUDA kernels use where it
differs from the reference's (it does not today: the kernels follow the
reference order, so both names give identical bits); the tests compare the two
orders with the +-1 code tolerance to show the order does not matter beyond
the stated rate.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "GROUP", "H4", "hadamard_matrix",
    "f32_to_bf16_bits", "bf16_bits_to_f32", "round_bf16", "as_bf16_bits",
    "rotate_groups", "rotate_groups_dense_f64", "rotate_bf16",
    "activation", "ACT_IDS", "PAIRED_ACT_IDS",
    "convrot_quantize", "dequant_epilogue", "dequant_act_quantize",
    "dequant_weight", "prepare_weight", "prepare_weight_fused", "quantize_row",
    "int_mm", "linear", "linear_acc", "ffn", "linear_dx_int8", "linear_dw",
    "linear_dw_int8", "colquant_scaled", "convrot_linear_reference", "rms_rope",
]

GROUP = 256

# H4 of the reference (src/xpuint8.cpp:75); H = kron(H4,H4,H4,H4)/16
# (docs/architecture.md:29-35).
H4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]],
              dtype=np.float64)

#: activation ids of the C API (include/xpu_kernels/convrot.h:49-57,
#: src/xpuint8.cpp:179-188)
ACT_IDS = {"none": 0, "gelu_tanh": 1, "swiglu": 2, "situ": 3, "geglu_erf": 4,
           "gelu_erf": 5}
PAIRED_ACT_IDS = (2, 3, 4)


def hadamard_matrix() -> np.ndarray:
    """The dense 256x256 rotation ``kron(H4,H4,H4,H4)/16`` in float64
    (docs/architecture.md:29-35).  Symmetric and orthogonal: ``H @ H = I``."""
    h = H4
    for _ in range(3):
        h = np.kron(h, H4)
    return h / 16.0


# ---------------------------------------------------------------------------
# bf16 helpers
# ---------------------------------------------------------------------------

def f32_to_bf16_bits(a) -> np.ndarray:
    """Round fp32 to bf16 (round to nearest, ties to even), returned as uint16
    bit patterns.  NaN maps to the canonical quiet NaN 0x7FC0."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    """Exact widening of bf16 bit patterns (uint16) to fp32
    (``load_reg``, src/xpuint8.cpp:109-117)."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def round_bf16(a) -> np.ndarray:
    """fp32 -> bf16 -> fp32: the ``convert<BF>().convert<float>()`` rounding
    point the reference applies after each activation step
    (src/xpuint8.cpp:190-261)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


def as_bf16_bits(x) -> np.ndarray:
    """Accept bf16 bit patterns (uint16) or a float array (rounded to bf16)."""
    x = np.asarray(x)
    if x.dtype == np.uint16:
        return x
    return f32_to_bf16_bits(x.astype(np.float32))


# ---------------------------------------------------------------------------
# the group-256 rotation
# ---------------------------------------------------------------------------

_HALF = np.float32(0.5)


def _axis_seq(v: np.ndarray, axis: int) -> np.ndarray:
    """One radix-4 ``H4/2`` butterfly written as the reference's in-register
    accumulation chain (``inreg``, src/xpuint8.cpp:290-301):
    ``t = c0*a0; t += c1*a1; t += c2*a2; t += c3*a3`` with ``c_j = 0.5*H4[r][j]``.
    Every product is exact (a signed half), so each ``+=`` rounds once."""
    a = [np.take(v, j, axis=axis) for j in range(4)]
    outs = []
    for r in range(4):
        t = (np.float32(0.5 * H4[r][0]) * a[0]).astype(np.float32)
        for j in range(1, 4):
            t = (t + np.float32(0.5 * H4[r][j]) * a[j]).astype(np.float32)
        outs.append(t)
    return np.stack(outs, axis=axis)


def _axis_bfly(v: np.ndarray, axis: int) -> np.ndarray:
    """One radix-4 ``H4/2`` butterfly in the reference's cross-register form
    (``bfly4``, src/xpuint8.cpp:279-285; the cross-lane ``bfly_xor`` of
    :441-448 produces the same bits): ``p=a0+a1, m=a0-a1, q=a2+a3, n=a2-a3``,
    ``out = ((p+n), (p-n), (m+q), (q-m)) * 0.5``."""
    a0, a1, a2, a3 = (np.take(v, j, axis=axis) for j in range(4))
    p = (a0 + a1).astype(np.float32)
    m = (a0 - a1).astype(np.float32)
    q = (a2 + a3).astype(np.float32)
    n = (a2 - a3).astype(np.float32)
    return np.stack([((p + n) * _HALF).astype(np.float32),
                     ((p - n) * _HALF).astype(np.float32),
                     ((m + q) * _HALF).astype(np.float32),
                     ((q - m) * _HALF).astype(np.float32)], axis=axis)


def rotate_groups(v, order: str = "reference") -> np.ndarray:
    """ConvRot rotation of fp32 values along the last axis, per 256-group.

    The element ``i = 16w + q`` of a group has base-4 digits ``i0 = q&3,
    i1 = q>>2, i2 = w&3, i3 = w>>2`` (src/xpuint8.cpp:55-67).  Axes 0 and 1
    are applied in the in-register accumulation form, axes 2 and 3 in the
    butterfly form, in that order -- exactly the sequence of
    ``launch_convrot_quant_warp`` (src/xpuint8.cpp:473-476) and of
    ``launch_rotate_bf16`` (:602-614).  All arithmetic is fp32.
    """
    if order not in ("reference", "kernel"):
        raise ValueError(f"unknown order {order!r}")
    v = np.ascontiguousarray(v, dtype=np.float32)
    k = v.shape[-1]
    if k % GROUP:
        raise ValueError(f"K={k} is not a multiple of {GROUP}")
    lead = v.shape[:-1]
    # [..., G, i3, i2, i1, i0]
    t = v.reshape(*lead, k // GROUP, 4, 4, 4, 4)
    t = _axis_seq(t, -1)    # axis 0 (i0)
    t = _axis_seq(t, -2)    # axis 1 (i1)
    t = _axis_bfly(t, -3)   # axis 2 (i2)
    t = _axis_bfly(t, -4)   # axis 3 (i3)
    return np.ascontiguousarray(t.reshape(*lead, k))


def rotate_groups_dense_f64(v) -> np.ndarray:
    """The rotation as a dense float64 product ``x_group @ H`` -- the ground
    truth the reference's pipeline benchmark uses (benchmarks/bench_pipeline.py:128-142)."""
    v = np.asarray(v, dtype=np.float64)
    k = v.shape[-1]
    g = v.reshape(*v.shape[:-1], k // GROUP, GROUP)
    return (g @ hadamard_matrix()).reshape(v.shape)


def rotate_bf16(x, order: str = "reference") -> np.ndarray:
    """bf16 [.., K] -> bf16 [.., K] (uint16 bits): rotate in fp32 and round once
    at the store (``launch_rotate_bf16``, src/xpuint8.cpp:588-635)."""
    xf = bf16_bits_to_f32(as_bf16_bits(x))
    return f32_to_bf16_bits(rotate_groups(xf, order))


# ---------------------------------------------------------------------------
# activations (src/xpuint8.cpp:128-261)
# ---------------------------------------------------------------------------

def _erf_f32(x: np.ndarray) -> np.ndarray:
    from scipy.special import erf
    return np.asarray(erf(x.astype(np.float64)), dtype=np.float64).astype(np.float32)


def _gelu_erf(x: np.ndarray) -> np.ndarray:
    """``0.5 * x * (1 + erf(x * 0.7071067811865476))`` in fp32
    (``gelu_erf_reg``, src/xpuint8.cpp:175-177); erf is evaluated in float64
    and rounded, i.e. correctly rounded, where the device's erf is within its
    documented ulp bound."""
    t = (x * np.float32(0.7071067811865476)).astype(np.float32)
    e = _erf_f32(t)
    return ((np.float32(0.5) * x).astype(np.float32)
            * (np.float32(1.0) + e).astype(np.float32)).astype(np.float32)


def _tanh_f32(z: np.ndarray) -> np.ndarray:
    return np.tanh(z.astype(np.float64)).astype(np.float32)


def _situ(h: np.ndarray, g: np.ndarray) -> np.ndarray:
    """MossImage's situ ``tanh(g/4)*sigmoid(g)*tanh(h/25)`` with the reference's
    bf16 rounding points (``situ_reg``, src/xpuint8.cpp:142-160)."""
    tg = round_bf16(_tanh_f32(round_bf16((g / np.float32(4.0)).astype(np.float32))))
    sg = round_bf16((np.float32(1.0) / (np.float32(1.0) + np.exp(-g.astype(np.float64)).astype(np.float32))).astype(np.float32))
    th = round_bf16(_tanh_f32(round_bf16((h / np.float32(25.0)).astype(np.float32))))
    p = round_bf16((tg * sg).astype(np.float32))
    return round_bf16((p * th).astype(np.float32))


def activation(act: int, a: np.ndarray, b: np.ndarray | None = None) -> np.ndarray:
    """The fused input activation on fp32 values that are exact bf16
    (``load_activated_reg<ACT>``, src/xpuint8.cpp:190-220).  For the paired ids
    ``a`` is the first half and ``b`` the second: swiglu is ``[gate, up]``,
    situ and geglu are ``[hidden, gate]`` (include/xpu_kernels/convrot.h:49-57).
    Returns fp32 values that are exact bf16 (every id rounds at the end)."""
    a = a.astype(np.float32)
    if act == 0:
        return a
    if act == 1:
        x = a
        x2 = (x * x).astype(np.float32)
        inner = (np.float32(0.7978845608028654) * x).astype(np.float32)
        inner = (inner * (np.float32(1.0) + (np.float32(0.044715) * x2).astype(np.float32)).astype(np.float32)).astype(np.float32)
        y = ((np.float32(0.5) * x).astype(np.float32)
             * (np.float32(1.0) + _tanh_f32(inner)).astype(np.float32)).astype(np.float32)
        return round_bf16(y)
    if act == 2:
        g, u = a, b.astype(np.float32)
        den = (np.float32(1.0) + np.exp(-g.astype(np.float64)).astype(np.float32)).astype(np.float32)
        silu = round_bf16((g / den).astype(np.float32))
        return round_bf16((silu * u).astype(np.float32))
    if act == 3:
        return _situ(a, b.astype(np.float32))
    if act == 4:
        h, g = a, b.astype(np.float32)
        y = round_bf16(_gelu_erf(g))
        return round_bf16((h * y).astype(np.float32))
    if act == 5:
        return round_bf16(_gelu_erf(a))
    raise ValueError(f"unknown activation id {act}")


# ---------------------------------------------------------------------------
# quantizers
# ---------------------------------------------------------------------------

def _row_scale(amax: np.ndarray) -> np.ndarray:
    # s = fmax(amax / 127.0f, 1e-30f)   (src/xpuint8.cpp:366, :496)
    return np.maximum((amax.astype(np.float32) / np.float32(127.0)).astype(np.float32),
                      np.float32(1e-30)).astype(np.float32)


def _quantize_rotated(v: np.ndarray):
    """Row abs-max -> scale -> ``clamp(rint(v * (1/s)), +-127)``: the
    reciprocal multiply of ``store_reg`` / ``quantize_vec``
    (src/xpuint8.cpp:264-277, :366-370, :496-498)."""
    amax = np.abs(v).max(axis=-1)
    s = _row_scale(amax)
    inv = (np.float32(1.0) / s).astype(np.float32)
    r = (v * inv[..., None]).astype(np.float32)
    q = np.clip(np.rint(r), -127, 127).astype(np.int8)
    return q, s


def convrot_quantize(x, act: int = 0, order: str = "reference"):
    """Rotate + per-row int8 quantize (``xpuint8_convrot_quantize`` /
    ``_quantize_act``, src/xpuint8.cpp:450-502, :793-838).

    ``x`` is bf16 bits [M, K] (or [M, 2K] for a paired activation).  Returns
    ``(int8 [M, K], fp32 [M])``.
    """
    xb = as_bf16_bits(x)
    xf = bf16_bits_to_f32(xb)
    if act in PAIRED_ACT_IDS:
        k = xf.shape[-1] // 2
        v = activation(act, xf[..., :k], xf[..., k:])
    else:
        v = activation(act, xf)
    return _quantize_rotated(rotate_groups(v, order))


def prepare_weight_fused(w, order: str = "reference"):
    """``prepare_weight_fused`` = ``quantize(bf16(w))`` (python/xpu_kernels/int8/ops.py:103-124)."""
    return convrot_quantize(w, 0, order)


def prepare_weight(w, order: str = "reference"):
    """The offline weight preparation (python/xpu_kernels/int8/ops.py:83-100):
    ``wr = rotate(bf16(w))`` (bf16 output), ``amax = |wr|.amax(1).clamp_min(1e-30)``
    (bf16), ``scale = float(amax) / 127`` (IEEE division), then
    ``round(wr / scale)`` with a true fp32 division, clamped to +-127."""
    wr = bf16_bits_to_f32(rotate_bf16(w, order))
    amax = np.maximum(np.abs(wr).max(axis=-1), np.float32(1e-30))
    # the clamp happens on a bf16 tensor: 1e-30 rounds to bf16 first
    amax = np.where(np.abs(wr).max(axis=-1) < np.float32(1e-30),
                    round_bf16(np.float32(1e-30)), amax).astype(np.float32)
    scale = (amax / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.rint((wr / scale[:, None]).astype(np.float32)), -127, 127).astype(np.int8)
    return q, scale


def quantize_row(x):
    """Per-row symmetric int8, no rotation: the torch chain
    ``quantize_row_torch`` (python/xpu_kernels/int8/ops.py:320-330):
    ``scale = (amax / 127).clamp_min(1e-30)``, ``round(x / scale)`` -- both
    true fp32 divisions -- clamped to +-127."""
    xf = bf16_bits_to_f32(as_bf16_bits(x)) if np.asarray(x).dtype == np.uint16 \
        else np.asarray(x, dtype=np.float32)
    amax = np.abs(xf).max(axis=-1, keepdims=True)
    scale = np.maximum((amax / np.float32(127.0)).astype(np.float32), np.float32(1e-30))
    q = np.clip(np.rint((xf / scale).astype(np.float32)), -127, 127).astype(np.int8)
    return q, scale[..., 0].astype(np.float32)


# ---------------------------------------------------------------------------
# GEMM and epilogues
# ---------------------------------------------------------------------------

def int_mm(a, b_t):
    """Exact int8 x int8 -> int32: ``a [M,K] @ b_t [N,K]^T`` -- what
    ``torch._int_mm(xq, w8.t())`` computes at python/xpu_kernels/int8/ops.py:634.
    Evaluated in float64 BLAS, which is exact while |acc| < 2^53 (always, for
    K < 2^39)."""
    a = np.asarray(a, dtype=np.int8).astype(np.float64)
    b = np.asarray(b_t, dtype=np.int8).astype(np.float64)
    return (a @ b.T).astype(np.int32)


def dequant_epilogue(acc, x_scale, w_scale, bias=None):
    """``bf16(float(acc) * (w_scale[n] * x_scale[m]) + bias[n])`` with an fp32
    bias and one rounding to bf16 (``launch_dequant_epilogue``,
    src/xpuint8.cpp:692-710).  The product and the add round separately.
    Returns bf16 bits [M, N]."""
    acc = np.asarray(acc, dtype=np.int32)
    xs = np.asarray(x_scale, dtype=np.float32).reshape(-1)
    ws = np.asarray(w_scale, dtype=np.float32).reshape(-1)
    sc = (ws[None, :] * xs[:, None]).astype(np.float32)
    v = (acc.astype(np.float32) * sc).astype(np.float32)
    if bias is not None:
        v = (v + np.asarray(bias, dtype=np.float32).reshape(1, -1)).astype(np.float32)
    return f32_to_bf16_bits(v)


def dequant_act_quantize(acc, x_scale, w_scale, act: int, order: str = "reference"):
    """Dequant -> activation -> rotate -> quantize of an up-projection
    accumulator (``launch_dequant_act_quant_warp``, src/xpuint8.cpp:517-573;
    ``load_dequant_act_reg`` :238-261).  ``acc`` is int32 [M, 2K] for the
    paired ids (3 situ, 4 geglu_erf; hidden first) and [M, K] for 5 gelu_erf.
    Returns ``(int8 [M, K], fp32 [M])``."""
    if act not in (3, 4, 5):
        raise ValueError("dequant_act_quantize supports activation 3, 4 or 5")
    acc = np.asarray(acc, dtype=np.int32)
    xs = np.asarray(x_scale, dtype=np.float32).reshape(-1, 1)
    ws = np.asarray(w_scale, dtype=np.float32).reshape(1, -1)
    d = round_bf16((acc.astype(np.float32) * (ws * xs).astype(np.float32)).astype(np.float32))
    if act == 5:
        v = round_bf16(_gelu_erf(d))
    else:
        k = d.shape[-1] // 2
        v = activation(act, d[:, :k], d[:, k:])
    return _quantize_rotated(rotate_groups(v, order))


def dequant_weight(w8, w_scale, order: str = "reference"):
    """The unrotated bf16 weight: ``rotate(bf16(float(w8) * s[n]))``
    (``dequant_weight_torch``, python/xpu_kernels/int8/ops.py:169-191; the bf16
    round happens before the rotation, src/xpuint8.cpp:98-107).  bf16 bits."""
    w = (np.asarray(w8, dtype=np.int8).astype(np.float32)
         * np.asarray(w_scale, dtype=np.float32).reshape(-1, 1)).astype(np.float32)
    return rotate_bf16(f32_to_bf16_bits(w), order)


# ---------------------------------------------------------------------------
# compositions (python/xpu_kernels/int8/ops.py)
# ---------------------------------------------------------------------------

def _expand(scale, n):
    s = np.asarray(scale, dtype=np.float32).reshape(-1)
    return np.full(n, s[0], np.float32) if s.size == 1 and n != 1 else s


def linear_acc(x, w8, act: int = 0, order: str = "reference"):
    """``linear_acc`` (python/xpu_kernels/int8/ops.py:571-588): the int32
    accumulator and the activation row scales."""
    xq, xs = convrot_quantize(x, act, order)
    return int_mm(xq, w8), xs


def linear(x, w8, w_scale, bias=None, act: int = 0, order: str = "reference"):
    """The INT8 ConvRot linear (python/xpu_kernels/int8/ops.py:591-646):
    rotate+quantize -> int8 GEMM -> dequant(+bias).  bf16 bits [M, N]."""
    acc, xs = linear_acc(x, w8, act, order)
    n = np.asarray(w8).shape[0]
    b = None if bias is None else _expand(bias, n)
    return dequant_epilogue(acc, xs, _expand(w_scale, n), b)


def ffn(x, up8, up_s, down8, down_s, down_bias=None, act: int = 4,
        order: str = "reference"):
    """The fused FFN (python/xpu_kernels/int8/ops.py:649-719): quantize ->
    GEMM -> dequant+act+rotate+quantize -> GEMM -> dequant.  bf16 bits."""
    xq, xs = convrot_quantize(x, 0, order)
    acc = int_mm(xq, up8)
    q2, xs2 = dequant_act_quantize(acc, xs, _expand(up_s, acc.shape[1]), act, order)
    acc2 = int_mm(q2, down8)
    n = np.asarray(down8).shape[0]
    b = None if down_bias is None else _expand(down_bias, n)
    return dequant_epilogue(acc2, xs2, _expand(down_s, n), b)


def linear_dx_int8(dy, w8, w_scale, order: str = "reference"):
    """dL/dx with the weight kept in int8 (python/xpu_kernels/int8/ops.py:353-377):
    ``d = bf16(bf16(dy) * bf16(w_scale))``, row-quantize d, ``acc = q @ w8``
    (w8 as stored, [N, K]), dequant with unit column scales, rotate back.
    bf16 bits [M, K]."""
    dyf = bf16_bits_to_f32(as_bf16_bits(dy))
    wsb = round_bf16(np.asarray(w_scale, dtype=np.float32).reshape(1, -1))
    d = round_bf16((dyf * wsb).astype(np.float32))
    q, a = quantize_row(d)
    w8 = np.asarray(w8, dtype=np.int8)
    acc = (q.astype(np.float64) @ w8.astype(np.float64)).astype(np.int32)
    dx = dequant_epilogue(acc, a, np.ones(acc.shape[1], np.float32))
    return rotate_bf16(dx, order)


def linear_dw(dy, x):
    """``dy^T @ x`` (python/xpu_kernels/int8/ops.py:207-238) in fp32 with a bf16
    result, for bf16 operands (what a bf16 matmul computes up to the
    accumulation order).  bf16 bits [N, K]."""
    dyf = bf16_bits_to_f32(as_bf16_bits(dy)).reshape(-1, np.asarray(dy).shape[-1])
    xf = bf16_bits_to_f32(as_bf16_bits(x)).reshape(-1, np.asarray(x).shape[-1])
    return f32_to_bf16_bits((dyf.astype(np.float64).T @ xf.astype(np.float64)).astype(np.float32))


def colquant_scaled(dy, x_scale):
    """Column quantization of ``g[m, n] = dy[m, n] * x_scale[m]`` over m: the
    operand of the int8 weight gradient (no reference counterpart; the
    formulation is this build's, see ``linear_dw_int8``).
    ``tg[n] = max(amax_m |g| / 127, 1e-30)``, ``gq = clamp(rint(g / tg), +-127)``,
    true fp32 divisions.  Returns ``(int8 [M, N], fp32 [N])``."""
    dyf = bf16_bits_to_f32(as_bf16_bits(dy))
    xs = np.asarray(x_scale, dtype=np.float32).reshape(-1, 1)
    g = (dyf * xs).astype(np.float32)
    amax = np.abs(g).max(axis=0)
    tg = np.maximum((amax / np.float32(127.0)).astype(np.float32), np.float32(1e-30))
    gq = np.clip(np.rint((g / tg[None, :]).astype(np.float32)), -127, 127).astype(np.int8)
    return gq, tg.astype(np.float32)


def linear_dw_int8(dy, xq, x_scale, order: str = "reference"):
    """The int8 weight gradient (new in this build; the reference's only dW is
    the bf16 ``dy^T @ x`` of python/xpu_kernels/int8/ops.py:207-238).

    The forward computed ``y = (xs[m] xq[m,:]) . (ws[n] w8[n,:])`` in the
    rotated basis, ``xs xq ~ x H``; with the straight-through convention the
    gradient of the rotated weight is ``dy^T (xs xq)`` and, H being symmetric
    and an involution, ``dW = rotate_K(dy^T (xs xq))``.  Both GEMM operands
    are int8: ``g = dy * xs`` is column-quantized (scale per n, constant over
    the contraction index m), ``acc[n,k] = sum_m gq[m,n] xq[m,k]`` exactly,
    ``dW = rotate(bf16(acc * tg[n]))``.  bf16 bits [N, K].
    """
    gq, tg = colquant_scaled(dy, x_scale)
    acc = (gq.astype(np.float64).T @ np.asarray(xq, dtype=np.int8).astype(np.float64)).astype(np.int32)
    dwr = dequant_epilogue(acc, tg, np.ones(acc.shape[1], np.float32))
    return rotate_bf16(dwr, order)


def convrot_linear_reference(x, w8, w_scale, bias=None, rotation: str = "hadamard"):
    """``reference/convrot_linear.py:5-23`` restated.  ``rotation="identity"`` is
    the file exactly as shipped (it multiplies by ``torch.eye``, :10-12);
    ``"hadamard"`` puts the normalized Hadamard in, as its own comment asks.
    The rotation is a bf16 matmul (fp32 accumulate, bf16 result); the quantizer
    divides (``x_rot.float() / x_scale``); the dequant is
    ``bf16((acc * xs) * ws)`` followed by a bf16 ``+ bias``.  bf16 bits."""
    xf = bf16_bits_to_f32(as_bf16_bits(x))
    m, k = xf.shape
    if rotation == "identity":
        xr = xf
    elif rotation == "hadamard":
        h = hadamard_matrix().astype(np.float32)  # entries +-1/16: exact in bf16
        xr = round_bf16((xf.reshape(m, k // GROUP, GROUP).astype(np.float64) @ h.astype(np.float64))
                        .astype(np.float32).reshape(m, k))
    else:
        raise ValueError(rotation)
    amax = np.abs(xr).max(axis=-1, keepdims=True)
    xs = np.maximum((amax / np.float32(127.0)).astype(np.float32), np.float32(1e-30))
    xq = np.clip(np.rint((xr / xs).astype(np.float32)), -127, 127).astype(np.int8)
    acc = int_mm(xq, w8)
    ws = np.asarray(w_scale, dtype=np.float32).reshape(1, -1)
    r = ((acc.astype(np.float32) * xs).astype(np.float32) * ws).astype(np.float32)
    out = round_bf16(r)
    if bias is not None:
        out = round_bf16((out + round_bf16(np.asarray(bias, dtype=np.float32).reshape(1, -1))).astype(np.float32))
    return f32_to_bf16_bits(out)


# ---------------------------------------------------------------------------
# the int32-accumulator consumer of the fused qkv projection
# ---------------------------------------------------------------------------

def rms_rope(x, freqs, weight, eps: float = 1e-6, split_half: bool = True,
             x_scale=None, w_scale=None):
    """RMS norm + rotary embedding per head (python/xpu_kernels/triton/rope.py
    :378-408 ``_rows_dq`` and :360-376 ``_rows``; the torch chain they restate,
    triton/reference.py:63-98).

    ``x``: bf16 bits ``[B, S, H, D]``, or int32 ``[B, S, H, D]`` with
    ``x_scale [B*S]`` and ``w_scale [H*D]`` (then first
    ``bf16(float(acc) * (w_scale * x_scale))``, rope.py:398-401).  Per head:
    ``inv = rsqrt(mean(x^2) + eps)``, ``y = bf16((x * inv) * weight)``, then the
    pairs ``(d, d + D/2)`` (split half) or ``(2i, 2i + 1)`` rotated by
    ``freqs [fb, fs, D/2, 2, 2]`` (fp32; size-1 leading dims broadcast):
    ``out = bf16(f00 y_a + f01 y_b)``, ``bf16(f10 y_a + f11 y_b)``, every
    product and sum rounded in fp32.  The mean of squares is summed in float64
    and rounded (the kernels' own summation orders differ from each other in
    the last bit; the tests' tolerance covers it).  Returns bf16 bits."""
    if x_scale is not None:
        acc = np.asarray(x, dtype=np.int32)
        B, S, H, D = acc.shape
        xs = np.asarray(x_scale, dtype=np.float32).reshape(B, S, 1, 1)
        ws = np.asarray(w_scale, dtype=np.float32).reshape(1, 1, H, D)
        xf = round_bf16((acc.astype(np.float32) * (ws * xs).astype(np.float32)).astype(np.float32))
    else:
        xf = bf16_bits_to_f32(as_bf16_bits(x))
        B, S, H, D = xf.shape
    ss = (xf.astype(np.float64) ** 2).sum(axis=-1, keepdims=True).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(((ss / np.float32(D)).astype(np.float32)
                                      + np.float32(eps)).astype(np.float64))).astype(np.float32)
    wt = np.asarray(weight, dtype=np.float32).reshape(1, 1, 1, D)
    y = round_bf16(((xf * inv).astype(np.float32) * wt).astype(np.float32))
    f = np.asarray(freqs, dtype=np.float32)
    f = np.broadcast_to(f.reshape(f.shape[0], f.shape[1], 1, D // 2, 2, 2), (B, S, 1, D // 2, 2, 2))
    if split_half:
        ya, yb = y[..., :D // 2], y[..., D // 2:]
    else:
        ya, yb = y[..., 0::2], y[..., 1::2]
    f00, f01, f10, f11 = f[..., 0, 0], f[..., 0, 1], f[..., 1, 0], f[..., 1, 1]
    oa = ((f00 * ya).astype(np.float32) + (f01 * yb).astype(np.float32)).astype(np.float32)
    ob = ((f10 * ya).astype(np.float32) + (f11 * yb).astype(np.float32)).astype(np.float32)
    out = np.empty_like(y)
    if split_half:
        out[..., :D // 2], out[..., D // 2:] = oa, ob
    else:
        out[..., 0::2], out[..., 1::2] = oa, ob
    return f32_to_bf16_bits(out)
