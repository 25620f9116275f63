"""xpu-kernels for NVIDIA B200: the ConvRot INT8 linear path.

The B200-native build of the reference package's INT8 half
(``xpu_kernels.int8``): a C-ABI library ``libxpuint8.so`` with hand-written
sm_100a CUDA kernels (rotate+quantize, a tcgen05 int8 GEMM with fused dequant
and GEGLU epilogues, the row quantizers and the backward) and this torch-only
binding.  The flat namespace below is the INT8 API (the same names are
available as ``xpu_kernels.int8.<name>``).  The reference's Triton half (norm,
rope, attention, NF4) is not part of this build.

Run ``python -m xpu_kernels`` to self-test the library on this machine.
"""

from __future__ import annotations

from .int8 import (
    ACTIVATIONS,
    Int8Linear,
    PAIRED_ACTIVATIONS,
    TrainableInt8Linear,
    available,
    dequant,
    dequant_act_quantize,
    dequant_slice,
    dequant_weight,
    dequant_weight_torch,
    device_name,
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
    load,
    prepare_weight,
    prepare_weight_fused,
    quantize,
    quantize_act,
    quantize_row,
    quantize_row_torch,
    rotate,
    selftest,
    unsupported_reason,
)
from .capture import (
    capture_status,
    is_capturing,
    prepare_for_capture,
    require_capture_ready,
)
from . import int8

__version__ = "0.4.0+b200"

__all__ = [
    "ACTIVATIONS", "Int8Linear", "PAIRED_ACTIVATIONS", "TrainableInt8Linear", "available",
    "capture_status", "dequant", "dequant_act_quantize", "dequant_slice", "dequant_weight",
    "dequant_weight_torch", "device_name", "expand_scale", "ffn", "ffn_situ", "int8_linear",
    "int_mm", "is_capturing", "linear", "linear_acc", "linear_split", "rms_rope", "rms_rope_dequant", "rms_rope_split_half",
    "rms_rope_split_half_dequant", "linear_dw", "linear_dw_int8",
    "linear_dx", "linear_dx_int8", "load", "prepare_for_capture", "prepare_weight",
    "prepare_weight_fused", "quantize", "quantize_act", "quantize_row", "quantize_row_torch",
    "require_capture_ready", "rotate", "selftest", "unsupported_reason", "int8",
]
