"""Device-side failure detection: a bounded wait that runs out returns an error
status instead of hanging the GPU.

The GEMM's mbarrier waits give up after a time limit, record a site number in a
device fault word and let the kernel return.  ``xpuint8_wait_probe`` runs that
same wait on an mbarrier that nothing ever arrives on (no TMA, no tensor core,
no trap), with a short limit; the test checks that the kernel returned after
about that limit, that ``xpuint8_fault_status`` reports the site, that a reset
clears it, and that the GPU still computes correctly afterwards.  The
reference's own failure model is the return code plus ``last_error``
(src/xpuint8.cpp:47-50); this is the device-side half of it.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    import xpu_kernels
    from xpu_kernels.int8 import _lib as L
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device")
    if not xpu_kernels.available():
        pytest.fail(f"libxpuint8 did not load: {L._ERR}")
    lib = L.load()
    assert lib.xpuint8_fault_status(1) == 0, "a fault was left over before the probe"
    yield lib
    lib.xpuint8_fault_status(1)


@pytest.mark.parametrize("limit_ms", [1, 5])
def test_a_wait_that_runs_out_returns_and_reports_its_site(lib, limit_ms):
    elapsed = ctypes.c_int64(-1)
    site = 40 + limit_ms
    rc = lib.xpuint8_wait_probe(limit_ms * 1_000_000, site, ctypes.addressof(elapsed))
    assert rc == 0, lib.xpuint8_last_error()
    # it waited at least its limit, and returned well inside the library's 2 s bound
    assert limit_ms * 1_000_000 <= elapsed.value < 500_000_000, elapsed.value
    print(f"\nwait probe: limit {limit_ms} ms, gave up after {elapsed.value / 1e6:.3f} ms")
    assert lib.xpuint8_fault_status(0) == site      # read without clearing
    assert lib.xpuint8_fault_status(1) == site      # read and clear
    assert lib.xpuint8_fault_status(0) == 0


def test_the_first_site_wins_until_reset(lib):
    for site in (7, 8):
        assert lib.xpuint8_wait_probe(100_000, site, None) == 0, lib.xpuint8_last_error()
    assert lib.xpuint8_fault_status(1) == 7
    assert lib.xpuint8_fault_status(0) == 0


def test_the_probe_rejects_site_zero(lib):
    assert lib.xpuint8_wait_probe(100_000, 0, None) == 2
    assert b"site" in lib.xpuint8_last_error()


def test_the_gpu_still_computes_after_a_probe(lib):
    """A probe fault neither poisons the context nor stops the GEMM's own waits."""
    from xpu_kernels import int8
    assert lib.xpuint8_wait_probe(200_000, 9, None) == 0
    a = torch.randint(-127, 128, (256, 512), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (384, 512), dtype=torch.int8, device="cuda")
    got = int8.int_mm(a, b)
    ref = (a.double() @ b.double().t()).to(torch.int32)
    assert torch.equal(got, ref)
    assert lib.xpuint8_fault_status(1) == 9   # only the probe's site: no GEMM wait gave up
    assert lib.xpuint8_fault_status(0) == 0
