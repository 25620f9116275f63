"""The INT8 API contract that can be checked without a device.

The same checks as the reference's tests/test_int8_api.py: ``unsupported_reason``
returns the specific reason and ``linear`` raises with that same string, so the
messages are part of the API.  Without a B200 (or without the library) only the
argument checks that run before the device is touched are testable; the
"library or device" part of each answer must name libxpuint8 or the device.
"""

import pytest
import torch

from xpu_kernels import int8


def _w(n=32, k=512):
    return torch.zeros((n, k), dtype=torch.int8)


def _x(m=4, k=512):
    return torch.zeros((m, k), dtype=torch.bfloat16)


def _scale(n=32):
    return torch.full((n,), 0.01, dtype=torch.float32)


def _device_or_lib(reason):
    return reason is None or "libxpuint8" in reason or "CUDA" in reason


def test_valid_call_passes_the_argument_checks():
    assert _device_or_lib(int8.unsupported_reason(_x(), _w(), _scale()))


def test_activation_dtype_is_reported():
    assert "float16" in int8.unsupported_reason(_x().to(torch.float16), _w(), _scale())


def test_weight_must_be_int8_2d():
    assert "int8" in int8.unsupported_reason(_x(), _w().float(), _scale())
    assert "int8" in int8.unsupported_reason(_x(), _w()[0], _scale())


def test_column_count_must_match_the_weight():
    reason = int8.unsupported_reason(_x(k=512), _w(k=1024), _scale())
    assert "512" in reason and "1024" in reason


def test_pair_activation_wants_two_halves():
    reason = int8.unsupported_reason(_x(k=512), _w(k=512), _scale(), act="situ")
    assert "1024" in reason
    assert int8.unsupported_reason(_x(k=1024), _w(k=512), _scale(), act="situ") is not None \
        or torch.cuda.is_available()
    assert "situ" in int8.unsupported_reason(_x(), _w(), _scale(), act="silu")


def test_the_activation_set():
    assert set(int8.ACTIVATIONS) >= {"gelu_tanh", "swiglu", "situ", "geglu_erf", "gelu_erf"}
    assert "situ" in int8.PAIRED_ACTIVATIONS
    assert "geglu_erf" in int8.PAIRED_ACTIVATIONS
    assert "gelu_erf" not in int8.PAIRED_ACTIVATIONS
    # the C ids of include/xpu_kernels/convrot.h
    assert int8.ACTIVATIONS == {"gelu_tanh": 1, "swiglu": 2, "situ": 3, "geglu_erf": 4,
                                "gelu_erf": 5}


def test_the_new_activations_in_the_argument_checks():
    assert "1024" in int8.unsupported_reason(_x(k=512), _w(k=512), _scale(), act="geglu_erf")
    assert _device_or_lib(int8.unsupported_reason(_x(k=512), _w(k=512), _scale(),
                                                  act="gelu_erf"))


def test_ffn_rejects_an_unknown_activation_before_anything_else():
    with pytest.raises(TypeError) as exc:
        int8.ffn(_x(), _w(), _scale(), _w(), _scale(), act="silu")
    assert "silu" in str(exc.value)
    with pytest.raises(TypeError) as exc:
        int8.ffn(_x(), _w(), _scale(), _w(), _scale(), act="swiglu")
    assert "swiglu" in str(exc.value)


def test_group_size_multiple():
    assert "256" in int8.unsupported_reason(_x(k=384), _w(k=384), _scale())


def test_output_width_multiple_of_16():
    reason = int8.unsupported_reason(_x(), _w(n=24), _scale(24))
    assert "24" in reason and "16" in reason


def test_scale_shapes():
    assert "floating point" in int8.unsupported_reason(
        _x(), _w(), torch.zeros(32, dtype=torch.int32))
    assert "dims" in int8.unsupported_reason(_x(), _w(), torch.zeros((2, 2, 8), dtype=torch.float32))
    assert "values" in int8.unsupported_reason(_x(), _w(), torch.zeros(7))
    assert "tensor or a python float" in int8.unsupported_reason(_x(), _w(), "0.01")
    for scale in (torch.zeros(1), torch.zeros(32), torch.zeros(32, 1), 0.01):
        assert _device_or_lib(int8.unsupported_reason(_x(), _w(), scale))


def test_cpu_tensors_are_refused_with_a_reason():
    # no fallback: a CPU activation is never computed, whatever the machine
    reason = int8.unsupported_reason(_x(), _w(), _scale())
    assert reason is not None
    assert "libxpuint8" in reason or "CUDA" in reason


def test_linear_raises_the_same_message():
    reason = int8.unsupported_reason(_x(), _w(k=384), _scale())
    with pytest.raises(TypeError) as exc:
        int8.linear(_x(), _w(k=384), _scale())
    assert str(exc.value) == reason


def test_linear_on_cpu_raises_instead_of_falling_back():
    with pytest.raises(TypeError) as exc:
        int8.linear(_x(), _w(), _scale())
    assert "libxpuint8" in str(exc.value) or "CUDA" in str(exc.value)


def test_prepare_weight_fused_checks_the_group_size():
    with pytest.raises(ValueError) as exc:
        int8.prepare_weight_fused(torch.zeros((32, 384), dtype=torch.bfloat16))
    assert "384" in str(exc.value) and "256" in str(exc.value)


def test_the_trainable_linear_checks_its_arguments():
    w = torch.zeros((32, 512), dtype=torch.bfloat16)
    with pytest.raises(ValueError) as exc:
        int8.TrainableInt8Linear(w, backward="exact")
    assert "exact" in str(exc.value)
    with pytest.raises(TypeError) as exc:
        int8.TrainableInt8Linear(torch.zeros((32, 512), dtype=torch.float16))
    assert "bfloat16" in str(exc.value)
    with pytest.raises(ValueError) as exc:
        int8.TrainableInt8Linear(w, dw="fp8")
    assert "fp8" in str(exc.value)


def test_expand_scale():
    flat = _scale(32)
    assert int8.expand_scale(flat, 32, flat.device) is flat
    one = torch.tensor(0.25)
    got = int8.expand_scale(one, 5, one.device)
    assert got.shape == (5,) and got.dtype == torch.float32
    assert torch.equal(got, torch.full((5,), 0.25))
    col = torch.arange(4, dtype=torch.float32).reshape(4, 1)
    assert torch.equal(int8.expand_scale(col, 4, col.device), col.reshape(-1))
    assert int8.expand_scale(0.5, 3, torch.device("cpu")).shape == (3,)
    with pytest.raises(TypeError):
        int8.expand_scale(0.5, 3)
    with pytest.raises(TypeError):
        int8.expand_scale("0.5", 3, torch.device("cpu"))


def test_ops_raise_when_the_library_is_missing(monkeypatch):
    # the product path fails loudly: no silent CPU computation
    from xpu_kernels.int8 import _lib as L
    monkeypatch.setattr(L, "_LIB", None)
    monkeypatch.setattr(L, "_TRIED", True)
    monkeypatch.setattr(L, "_ERR", "simulated: not found")
    with pytest.raises(RuntimeError) as exc:
        int8.quantize(_x())
    assert "libxpuint8 unavailable" in str(exc.value)
    assert "libxpuint8" in int8.unsupported_reason(_x(), _w(), _scale())
