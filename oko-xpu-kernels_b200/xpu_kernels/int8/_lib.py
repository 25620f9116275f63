"""Loading and calling ``libxpuint8.so``: the ctypes surface, nothing else.

The B200 build of the reference's loader (python/xpu_kernels/int8/_lib.py):
the same search order and environment variables (``$XPU_KERNELS_LIB``, then the
legacy ``$XPU_INT8_LIB``, then beside this file, ...), the same
``available()`` / ``device_name()`` / ``_lib()`` / ``_err()`` contract, with the
SYCL queue replaced by the CUDA stream handle of torch's current stream.

There is no fallback: when the library cannot be loaded every op raises
``RuntimeError`` naming the reason (``_lib()``), and ``unsupported_reason``
reports it without raising.
"""

from __future__ import annotations

import ctypes
import os
import sys
from typing import Optional

import torch

_LIB = None
_TRIED = False
_PATH = None
_ERR = None


def _candidate_paths():
    for var in ("XPU_KERNELS_LIB", "XPU_INT8_LIB"):   # the old name still works
        env = os.environ.get(var)
        if env:
            yield env
    here = os.path.dirname(os.path.abspath(__file__))       # .../xpu_kernels/int8
    pkg = os.path.dirname(here)                             # .../xpu_kernels
    for base in (here, pkg):
        yield os.path.join(base, "libxpuint8.so")           # built beside the code
    root = os.path.dirname(os.path.dirname(pkg))            # the repo, when run in place
    yield os.path.join(root, "build", "libxpuint8.so")
    yield os.path.join(root, "lib", "libxpuint8.so")
    yield os.path.join(sys.prefix, "lib", "libxpuint8.so")
    yield "/usr/local/lib/libxpuint8.so"


def library_path() -> Optional[str]:
    """The first candidate path that exists (loaded or not), for diagnostics."""
    for p in _candidate_paths():
        if p and os.path.exists(p):
            return p
    return None


#: every entry point of include/xpu_kernels/convrot.h with its ctypes argtypes
def _signatures():
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
    return {
        "xpuint8_convrot_quantize": [vp, vp, vp, i64, i64],
        "xpuint8_convrot_quantize_stream": [vp] * 4 + [i64] * 2,
        "xpuint8_convrot_quantize_act": [vp, vp, vp, i64, i64, i32],
        "xpuint8_convrot_quantize_act_stream": [vp] * 4 + [i64] * 2 + [i32],
        "xpuint8_dequant_weight": [vp, vp, vp, i64, i64],
        "xpuint8_dequant_weight_stream": [vp] * 4 + [i64] * 2,
        "xpuint8_convrot_rotate_bf16": [vp, vp, i64, i64],
        "xpuint8_convrot_rotate_bf16_stream": [vp] * 3 + [i64] * 2,
        "xpuint8_dequant_epilogue": [vp] * 5 + [i64] * 2,
        "xpuint8_dequant_epilogue_stream": [vp] * 6 + [i64] * 2,
        "xpuint8_dequant_epilogue_slice": [vp] * 5 + [i64] * 3,
        "xpuint8_dequant_epilogue_slice_stream": [vp] * 6 + [i64] * 3,
        "xpuint8_dequant_act_quantize": [vp] * 5 + [i64] * 2 + [i32],
        "xpuint8_dequant_act_quantize_stream": [vp] * 6 + [i64] * 2 + [i32],
        "xpuint8_int_mm_stream": [vp] * 4 + [i64] * 3 + [i32, i64],
        "xpuint8_int_mm_dequant_stream": [vp] * 7 + [i64] * 3 + [i32, i64],
        "xpuint8_int_mm_geglu_stream": [vp] * 6 + [i64] * 3,
        "xpuint8_linear_stream": [vp] * 8 + [i64] * 3 + [i32],
        "xpuint8_linear_split_stream": [vp] * 6 + [i32, vp, vp] + [i64] * 3 + [i32],
        "xpuint8_ffn_workspace_bytes": [i64, i64, i64, i32],
        "xpuint8_ffn_stream": [vp] * 9 + [i64] * 3 + [i32],
        "xpuint8_quantize_row_stream": [vp] * 5 + [i64] * 2,
        "xpuint8_colquant_stream": [vp] * 5 + [i64] * 2,
        "xpuint8_linear_dx_int8_workspace_bytes": [i64] * 3,
        "xpuint8_linear_dx_int8_stream": [vp] * 6 + [i64] * 3,
        "xpuint8_linear_dw_int8_workspace_bytes": [i64] * 3,
        "xpuint8_linear_dw_int8_stream": [vp] * 6 + [i64] * 3,
        "xpuint8_rms_rope_stream": [vp, vp, i32, i64] + [vp] * 4 + [i64, i64, vp] + [i64] * 5
                                   + [ctypes.c_float, i32],
        "xpuint8_fault_status": [i32],
        "xpuint8_wait_probe": [i64, i32, vp],
        "xpuint8_check_scale_math": [vp, vp],
        "xpuint8_linear_allgather_stream": [vp] * 6 + [i32, i32, vp, vp] + [i64] * 3 + [i32],
        "xpuint8_linear_allgather_cols_stream": [vp] * 6 + [i32, i64, i64, vp, vp] + [i64] * 3
                                                + [i32],
        "xpuint8_ipc_alloc": [i64, vp, vp],
        "xpuint8_ipc_open": [vp, vp],
        "xpuint8_ipc_close": [vp],
        "xpuint8_ipc_free": [vp],
        "xpuint8_linear_noalloc_stream": [vp] * 6 + [i64] * 3 + [i32],
    }


def _bind(lib):
    """Declare every argtype: an undeclared pointer argument is truncated to 32
    bits by ctypes, which is a device fault, not an error code."""
    for name, args in _signatures().items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int64 if name.endswith("_workspace_bytes") else ctypes.c_int


def load():
    """Load, bind and initialise the library.  Returns the ctypes handle or None."""
    global _LIB, _TRIED, _PATH, _ERR
    if _LIB is not None or _TRIED:
        return _LIB
    _TRIED = True
    for path in _candidate_paths():
        if not path or not os.path.exists(path):
            continue
        try:
            lib = ctypes.CDLL(path)
        except OSError as exc:
            _ERR = f"{path}: {exc}"
            continue
        try:
            lib.xpuint8_init.restype = ctypes.c_int
            lib.xpuint8_device_name.restype = ctypes.c_char_p
            lib.xpuint8_last_error.restype = ctypes.c_char_p
            lib.xpuint8_convrot_groupsize.restype = ctypes.c_int
            _bind(lib)
        except AttributeError as exc:
            _ERR = f"{path}: {exc}"
            continue
        if lib.xpuint8_init() != 0:
            _ERR = f"{path}: {lib.xpuint8_last_error()!r}"
            continue
        _LIB, _PATH = lib, path
        return lib
    if _ERR is None:
        tried = ", ".join(p for p in _candidate_paths() if p)
        _ERR = (f"no libxpuint8.so found (tried: {tried}); build it with "
                f"`make -C oko-xpu-kernels_b200/csrc` or __graft_entry__.build()")
    return None


def available() -> bool:
    """True when the library loaded and found a B200 (sm_100) on this machine."""
    return load() is not None


def device_name() -> Optional[str]:
    lib = load()
    if lib is None:
        return None
    name = lib.xpuint8_device_name()
    return name.decode() if name else None


def _lib():
    lib = load()
    if lib is None:
        raise RuntimeError(f"libxpuint8 unavailable: {_ERR or 'not found'}")
    return lib


def _err(lib, what):
    raise RuntimeError(f"{what}: {lib.xpuint8_last_error()!r}")


def _stream(device):
    """torch's current CUDA stream on ``device`` as the library's stream handle."""
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _fp32(t):
    return t.reshape(-1).to(dtype=torch.float32).contiguous()


def _flat2d(x):
    if x.dtype != torch.bfloat16:
        raise TypeError(f"expected bfloat16, got {x.dtype}")
    if x.device.type != "cuda":
        raise TypeError(f"expected a CUDA tensor, got {x.device}")
    x = x if x.is_contiguous() else x.contiguous()
    return x.reshape(-1, x.shape[-1]), x.shape


ACTIVATIONS = {"gelu_tanh": 1, "swiglu": 2, "situ": 3, "geglu_erf": 4, "gelu_erf": 5}

#: The activations that read a *pair* of halves (``[hidden, gate]`` or
#: ``[gate, up]``) rather than a single tensor.
PAIRED_ACTIVATIONS = ("swiglu", "situ", "geglu_erf")
