"""The INT8 linear entry point that allocates nothing.

xpuint8_linear_noalloc_stream serves callers that cannot allocate device
memory (a plugin whose host application owns the GPU's memory pool, a C caller
without a device allocator, a path where cudaMalloc would synchronise): it
keeps the int8 activation and its row scales in a fixed array inside the
library instead of taking scratch buffers.  Its results must be those of
xpuint8_linear_stream with caller-provided scratch -- bit for bit, the
tolerance every linear parity test here uses -- on two calls in a row (the
second call finds the array holding the first call's contents), and it must
refuse shapes beyond the array with an error instead of launching.

This file is collected last so that a run stopping at its first failure has
already run every other test; it passes alone in a fresh process too.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import xpu_kernels
    from xpu_kernels.int8 import _lib as L
    if not torch.cuda.is_available() or not xpu_kernels.available():
        pytest.fail(f"libxpuint8 did not load: {L._ERR}")
    return L, L.load()


def _case(m, k, n, seed):
    from xpu_kernels import int8
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(m, k, generator=g, device="cuda")).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    w8, ws = int8.prepare_weight(w)
    bias = torch.randn(n, generator=g, device="cuda") * 0.01
    return x, w8, ws, bias


def _with_scratch(L, lib, x, w8, ws, bias):
    m, k = x.shape
    n = w8.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    xq = torch.empty(m, k, dtype=torch.int8, device="cuda")
    xs = torch.empty(m, dtype=torch.float32, device="cuda")
    rc = lib.xpuint8_linear_stream(L._stream(x.device), L._ptr(x), L._ptr(w8), L._ptr(ws),
                                   L._ptr(bias), L._ptr(out), L._ptr(xq), L._ptr(xs), m, n, k, 0)
    assert rc == 0, lib.xpuint8_last_error()
    return out


def _no_alloc(L, lib, x, w8, ws, bias):
    m, k = x.shape
    n = w8.shape[0]
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    rc = lib.xpuint8_linear_noalloc_stream(L._stream(x.device), L._ptr(x), L._ptr(w8),
                                           L._ptr(ws), L._ptr(bias), L._ptr(out), m, n, k, 0)
    assert rc == 0, lib.xpuint8_last_error()
    return out


def test_no_alloc_linear_matches_the_scratch_entry_point_twice():
    L, lib = _lib()
    # the second call uses another shape and other data: the array still
    # holds the first call's values when it starts
    for m, k, n, seed in ((2048, 1280, 1280, 1), (300, 1024, 272, 2)):
        x, w8, ws, bias = _case(m, k, n, seed)
        ref = _with_scratch(L, lib, x, w8, ws, bias)
        got = _no_alloc(L, lib, x, w8, ws, bias)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    assert lib.xpuint8_fault_status(1) == 0


def test_no_alloc_linear_refuses_shapes_beyond_its_array():
    L, lib = _lib()
    lib.xpuint8_last_error.restype = ctypes.c_char_p
    x = torch.empty(1, 256, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(1, 16, dtype=torch.bfloat16, device="cuda")
    w8 = torch.empty(16, 256, dtype=torch.int8, device="cuda")
    ws = torch.ones(16, dtype=torch.float32, device="cuda")
    # more rows than the row-scale array holds: refused before any launch
    rc = lib.xpuint8_linear_noalloc_stream(L._stream(x.device), L._ptr(x), L._ptr(w8), L._ptr(ws),
                                           None, L._ptr(out), 16385, 16, 256, 0)
    assert rc == 2 and b"scratch" in lib.xpuint8_last_error()
    # more activation bytes than the array holds
    rc = lib.xpuint8_linear_noalloc_stream(L._stream(x.device), L._ptr(x), L._ptr(w8), L._ptr(ws),
                                           None, L._ptr(out), 4096, 16, 4096, 0)
    assert rc == 2 and b"scratch" in lib.xpuint8_last_error()
