"""The C-ABI library: it loads, and it exports every symbol the header declares.

No compute calls here -- this runs without a GPU.  The header is parsed for its
function declarations, and the built libxpuint8.so must export each one.
"""

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "xpu_kernels", "convrot.h")
LIB = os.path.join(ROOT, "oko-xpu-kernels_b200", "xpu_kernels", "int8", "libxpuint8.so")

# the reference's 18 entry points (its include/xpu_kernels/convrot.h:30-114)
REFERENCE_SYMBOLS = {
    "xpuint8_init", "xpuint8_device_name", "xpuint8_convrot_groupsize",
    "xpuint8_convrot_quantize", "xpuint8_convrot_quantize_stream",
    "xpuint8_convrot_quantize_act", "xpuint8_convrot_quantize_act_stream",
    "xpuint8_dequant_weight", "xpuint8_dequant_weight_stream",
    "xpuint8_convrot_rotate_bf16", "xpuint8_convrot_rotate_bf16_stream",
    "xpuint8_dequant_epilogue", "xpuint8_dequant_epilogue_stream",
    "xpuint8_dequant_epilogue_slice", "xpuint8_dequant_epilogue_slice_stream",
    "xpuint8_dequant_act_quantize", "xpuint8_dequant_act_quantize_stream",
    "xpuint8_last_error",
}


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(xpuint8_\w+)\s*\(", text))


def test_the_header_keeps_the_reference_abi():
    assert REFERENCE_SYMBOLS <= declared_symbols()


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is not built; run __graft_entry__.build()")
    import torch  # noqa: F401  (loads the CUDA runtime the library links)
    return ctypes.CDLL(LIB)


def test_the_library_exports_every_declared_symbol(lib):
    missing = [s for s in sorted(declared_symbols()) if not hasattr(lib, s)]
    assert not missing, missing


def test_the_python_binding_declares_every_entry_point():
    from xpu_kernels.int8 import _lib as L
    bound = set(L._signatures()) | {"xpuint8_init", "xpuint8_device_name",
                                    "xpuint8_last_error", "xpuint8_convrot_groupsize"}
    assert declared_symbols() <= bound


def test_group_size_needs_no_device(lib):
    lib.xpuint8_convrot_groupsize.restype = ctypes.c_int
    assert lib.xpuint8_convrot_groupsize() == 256
