"""Fused ConvRot INT8 primitives for NVIDIA B200 (sm_100a), on torch CUDA tensors.

A thin, torch-only binding over ``libxpuint8.so`` -- the B200 build of the
reference package's ``xpu_kernels.int8`` with the same API:

    bf16 [M,K] --rotate+quantize------------------------------> int8 [M,K] + fp32 [M]
    int8 [M,K] x int8 [N,K].T --tcgen05 GEMM + fused dequant--> bf16 [M,N]
                               --raw---------------------------> int32 [M,N]
    int32 [M,N] --dequant(+bias)-------------------------------> bf16 [M,N]
                --or dequant+activation+rotate+quantize--------> int8 [M,K2] + fp32 [M]

    import xpu_kernels, torch
    w8, ws = xpu_kernels.prepare_weight(w)              # once, offline
    y = xpu_kernels.linear(x, w8, ws)                   # bf16 [M,K] -> bf16 [M,N]
    y = xpu_kernels.ffn(x, up8, up_s, down8, down_s, act="geglu_erf")

Bit-exactness contract (as the reference's): ``dequant(linear_acc(x, w8,
ws)[0], ...)`` is bit-identical to ``linear(x, ...)``; the dequant arithmetic is
``float(acc) * (w_scale[n] * x_scale[m])`` (+ fp32 bias) rounded once to bf16.
``K`` must be a multiple of 256 and ``N`` of 16.  There is no CPU or XPU path
and no fallback: without the library every op raises ``RuntimeError``.
"""

from __future__ import annotations

from ._lib import ACTIVATIONS, PAIRED_ACTIVATIONS, available, device_name, load
from .ops import (
    Int8Linear,
    TrainableInt8Linear,
    dequant,
    dequant_act_quantize,
    dequant_slice,
    dequant_weight,
    dequant_weight_torch,
    expand_scale,
    ffn,
    ffn_situ,
    int8_linear,
    int_mm,
    linear,
    linear_acc,
    linear_split,
    rms_rope,
    rms_rope_dequant,
    rms_rope_split_half,
    rms_rope_split_half_dequant,
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
    rotate,
    unsupported_reason,
)
from .selftest import selftest

__all__ = [
    "ACTIVATIONS", "Int8Linear", "PAIRED_ACTIVATIONS", "TrainableInt8Linear", "available",
    "dequant", "dequant_act_quantize", "dequant_slice", "dequant_weight",
    "dequant_weight_torch", "device_name", "expand_scale", "ffn", "ffn_situ", "int8_linear",
    "int_mm", "linear", "linear_acc", "linear_split", "rms_rope", "rms_rope_dequant", "rms_rope_split_half",
    "rms_rope_split_half_dequant", "linear_dw", "linear_dw_int8", "linear_dx",
    "linear_dx_int8", "load", "prepare_weight", "prepare_weight_fused", "quantize",
    "quantize_act", "quantize_row", "quantize_row_torch", "rotate", "selftest",
    "unsupported_reason",
]
