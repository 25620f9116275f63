"""Capture readiness and CUDA-graph replay of the INT8 path.

A captured step replays whatever was enqueued inside it, on every replay.  Two
things can make an INT8 step wrong or wasteful inside a capture, and neither
is an error by itself:

* work enqueued on another stream than torch's current one is not part of the
  graph: the replay then returns the first input's answer (a stale result,
  not an exception);
* the "dense" backward's dequantized weight, a full-precision copy of the
  weight, would be re-computed on every replay.

The CPU tests pin the readiness contract of ``xpu_kernels.capture`` (what is
reported, what raises), mirroring the reference's tests/test_capture.py for
its INT8 half.  The GPU tests capture the forward, the fused FFN and the int8
backward in a CUDA graph, replay them on new data and compare the result bit
for bit with the eager call on the same data (the reference's
debug/verify_int8_capture.py, as tests).
"""

from unittest import mock

import pytest
import torch

import xpu_kernels
from xpu_kernels import capture, int8


def _model(backward="dense"):
    """A model with one INT8 linear, built by hand (``prepare_weight`` needs the
    device library; the readiness contract does not)."""
    w8 = torch.randint(-127, 128, (32, 512), dtype=torch.int8,
                       generator=torch.Generator().manual_seed(0))
    scale = torch.full((32,), 0.01, dtype=torch.float32)
    mod = torch.nn.Module()
    mod.proj = int8.Int8Linear(w8, scale, backward=backward)
    return mod


# -------------------------------------------------------------------- CPU: the contract

def test_is_capturing_is_false_and_never_raises():
    assert xpu_kernels.is_capturing() is False


def test_is_capturing_survives_a_backend_that_cannot_answer():
    def broken():
        raise RuntimeError("no device")
    with mock.patch.object(torch.cuda, "is_current_stream_capturing", broken):
        assert xpu_kernels.is_capturing() is False


def test_status_is_empty_without_a_model():
    assert capture.capture_status() == []
    assert capture.capture_status(need=()) == []


def test_status_rejects_an_unknown_kernel_name():
    # this build has no self-tested fused kernels to name: any name is a typo,
    # and a typo must not read as "everything is fine"
    with pytest.raises(ValueError) as exc:
        capture.capture_status(need=("rms_rope",))
    assert "rms_rope" in str(exc.value)


def test_status_reports_a_missing_dense_weight():
    problems = capture.capture_status(model=_model())
    assert len(problems) == 1
    assert "dense weight" in problems[0] and "proj" in problems[0]


def test_require_ready_raises_with_the_problems():
    with pytest.raises(RuntimeError) as exc:
        capture.require_capture_ready(model=_model())
    assert "dense weight" in str(exc.value)
    capture.require_capture_ready(model=_model(backward="int8"))  # nothing to do


def test_prepare_materializes_the_dense_weight():
    model = _model()
    calls = []

    def fake_dequant(w8, w_scale):
        calls.append(tuple(w8.shape))
        return torch.zeros(w8.shape, dtype=torch.bfloat16)

    with mock.patch("xpu_kernels.int8.ops.dequant_weight", fake_dequant):
        summary = capture.prepare_for_capture(model)
        assert summary["dense_weights"] == 1
        assert summary["problems"] == []
        # cached: a second prepare does not dequantize again
        capture.prepare_for_capture(model)
    assert calls == [(32, 512)]
    assert capture.capture_status(model=model) == []


def test_the_dense_weight_is_only_demanded_where_it_is_needed():
    # "int8" backward keeps the weight in int8: it never needs a dense copy,
    # and materializing one would spend the memory the mode exists to save
    model = torch.nn.Module()
    model.dense = int8.Int8Linear(torch.zeros(16, 256, dtype=torch.int8),
                                  torch.ones(16, dtype=torch.float32), backward="dense")
    model.cheap = int8.Int8Linear(torch.zeros(16, 256, dtype=torch.int8),
                                  torch.ones(16, dtype=torch.float32), backward="int8")
    problems = capture.capture_status(model=model)
    assert any("dense" in p for p in problems)
    assert not any("cheap" in p for p in problems)
    with mock.patch("xpu_kernels.int8.ops.dequant_weight",
                    lambda w8, s: torch.zeros(w8.shape, dtype=torch.bfloat16)):
        assert capture.prepare_for_capture(model)["dense_weights"] == 1
    assert getattr(model.cheap, "_dense", None) is None


def test_dense_weight_refuses_to_allocate_inside_a_capture():
    model = _model()
    with mock.patch("xpu_kernels.int8.ops.is_capturing", return_value=True):
        with pytest.raises(RuntimeError) as exc:
            model.proj.dense_weight()
    assert "capture" in str(exc.value)
    assert getattr(model.proj, "_dense", None) is None


def test_a_cached_dense_weight_is_served_inside_a_capture():
    model = _model()
    with mock.patch("xpu_kernels.int8.ops.dequant_weight",
                    lambda w8, s: torch.ones(w8.shape, dtype=torch.bfloat16)):
        capture.prepare_for_capture(model)
    with mock.patch("xpu_kernels.int8.ops.is_capturing", return_value=True):
        w = model.proj.dense_weight()
    assert w.shape == (32, 512)


# -------------------------------------------------------------------- GPU: replay

DEV = "cuda"


def _weights(n, k, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn((n, k), generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    return int8.prepare_weight(w)


def _x(shape, seed, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(torch.bfloat16).to(DEV)


def _same(a, b):
    return a.dtype == b.dtype and a.shape == b.shape and torch.equal(
        a.contiguous().view(torch.int16), b.contiguous().view(torch.int16))


def _capture(fn, warmup=2):
    """Warm ``fn`` up on a side stream, then capture it; returns (graph, outputs)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(warmup):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = fn()
    torch.cuda.synchronize()
    return g, out


@pytest.mark.gpu
def test_is_capturing_is_true_inside_a_capture():
    seen = []
    x = torch.zeros(16, device=DEV)

    def fn():
        seen.append(xpu_kernels.is_capturing())
        return x + 1

    _capture(fn, warmup=1)
    assert seen == [False, True]


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(512, 1024, 3072), (77, 160, 1280)])
def test_linear_replays_bit_for_bit(m, n, k):
    w8, ws = _weights(n, k, 1)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(2)) * 0.01).to(DEV)
    x_static = _x((m, k), 3)
    g, y_static = _capture(lambda: int8.linear(x_static, w8, ws, bias))

    x_new = _x((m, k), 4)
    want = int8.linear(x_new, w8, ws, bias)
    x_static.copy_(x_new)
    g.replay()
    torch.cuda.synchronize()
    assert _same(y_static, want), "the replay does not recompute the linear"

    # back to a first input: a stale graph would still hold x_new's answer
    x_first = _x((m, k), 5)
    x_static.copy_(x_first)
    g.replay()
    torch.cuda.synchronize()
    assert _same(y_static, int8.linear(x_first, w8, ws, bias))
    del g


@pytest.mark.gpu
@pytest.mark.parametrize("act", ["situ", "geglu_erf"])
def test_ffn_replays_bit_for_bit(act):
    m, k, inner = 256, 1280, 1024
    up8, up_s = _weights(2 * inner, k, 11)
    dn8, dn_s = _weights(k, inner, 12)
    x_static = _x((m, k), 13)
    g, f_static = _capture(lambda: int8.ffn(x_static, up8, up_s, dn8, dn_s, act=act))
    x_new = _x((m, k), 14)
    want = int8.ffn(x_new, up8, up_s, dn8, dn_s, act=act)
    x_static.copy_(x_new)
    g.replay()
    torch.cuda.synchronize()
    assert _same(f_static, want)
    del g


@pytest.mark.gpu
def test_int8_backward_replays_bit_for_bit():
    """Forward and backward of the int8-mode linear in one graph: the output,
    dx (row quantizer with column scales, MN-major int8 GEMM, rotation) and
    dbias all replay."""
    m, n, k = 384, 1024, 1280
    w8, ws = _weights(n, k, 21)
    bias = torch.zeros(n, device=DEV, requires_grad=True)
    x_static = _x((m, k), 22).requires_grad_(True)
    dy_static = _x((m, n), 23, scale=1e-3)

    def step():
        x_static.grad = None
        bias.grad = None
        y = int8.int8_linear(x_static, w8, ws, bias, mode="int8")
        y.backward(dy_static)
        return y

    g, y_static = _capture(step)
    dx_static, db_static = x_static.grad, bias.grad

    x_new, dy_new = _x((m, k), 24), _x((m, n), 25, scale=1e-3)
    xe = x_new.clone().requires_grad_(True)
    be = torch.zeros(n, device=DEV, requires_grad=True)
    ye = int8.int8_linear(xe, w8, ws, be, mode="int8")
    ye.backward(dy_new)
    with torch.no_grad():
        x_static.copy_(x_new)
        dy_static.copy_(dy_new)
    g.replay()
    torch.cuda.synchronize()
    assert _same(y_static.detach(), ye.detach())
    assert _same(dx_static, xe.grad)
    assert torch.equal(db_static, be.grad)
    del g


@pytest.mark.gpu
def test_prepared_dense_dx_replays_bit_for_bit():
    """``Int8Linear.dx`` after ``prepare_for_capture``: the cached dense weight
    is served inside the capture and the bf16 GEMM replays."""
    n, k, m = 512, 1280, 256
    w8, ws = _weights(n, k, 31)
    mod = torch.nn.Module()
    mod.proj = int8.Int8Linear(w8, ws)
    summary = xpu_kernels.prepare_for_capture(mod)
    assert summary["dense_weights"] == 1 and summary["problems"] == []
    xpu_kernels.require_capture_ready(model=mod)
    dy_static = _x((m, n), 32, scale=1e-3)
    g, dx_static = _capture(lambda: mod.proj.dx(dy_static))
    dy_new = _x((m, n), 33, scale=1e-3)
    want = mod.proj.dx(dy_new)
    dy_static.copy_(dy_new)
    g.replay()
    torch.cuda.synchronize()
    assert _same(dx_static, want)
    del g


@pytest.mark.gpu
def test_int8_dw_replays_bit_for_bit():
    """The int8 weight gradient (column quantizer, MN-major int8 GEMM,
    rotation) in a graph."""
    m, n, k = 512, 640, 1280
    x_static = _x((m, k), 41)
    dy_static = _x((m, n), 42, scale=1e-3)

    def dw():
        xq, xs = int8.quantize(x_static)
        return int8.linear_dw_int8(dy_static, xq, xs)

    g, dw_static = _capture(dw)
    x_new, dy_new = _x((m, k), 43), _x((m, n), 44, scale=1e-3)
    xq, xs = int8.quantize(x_new)
    want = int8.linear_dw_int8(dy_new, xq, xs)
    x_static.copy_(x_new)
    dy_static.copy_(dy_new)
    g.replay()
    torch.cuda.synchronize()
    assert _same(dw_static, want)
    del g
