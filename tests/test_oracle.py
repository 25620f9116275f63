"""The CPU oracle, pinned before it is trusted.

Everything here runs without a GPU.  The oracle (oracle/convrot_oracle.py) is
checked against
* the golden fixtures made by running the reference's own torch code on CPU
  (tests/golden/make_golden.py -> reference_cpu.npz): quantize_row_torch,
  reference/convrot_linear.py, linear_dw, the prepare_weight and
  dequant_weight_torch chains, linear_dx_int8, torch's GELU on every bf16;
* the reference's known-answer tests: the ties row of tests/test_quantize.py,
  the float64 formula of the row quantizer;
* properties of the rotation: H @ H = I, rotate(rotate(x)) = x, the butterfly
  form against the dense float64 matrix.
"""

import os

import numpy as np
import pytest

from oracle import convrot_oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "reference_cpu.npz")


@pytest.fixture(scope="module")
def G():
    return np.load(GOLDEN)


def _bits_equal(a, b):
    return np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8))


# ------------------------------------------------------------------ golden fixtures

def test_quantize_row_matches_the_reference_chain(G):
    q, s = O.quantize_row(G["qrow_x"])
    assert np.array_equal(q, G["qrow_q"])
    assert _bits_equal(s, G["qrow_s"])


def test_convrot_linear_as_shipped(G):
    bias = O.bf16_bits_to_f32(G["cl_bias"])
    y = O.convrot_linear_reference(G["cl_x"], G["cl_w8"], G["cl_ws"], bias, rotation="identity")
    assert np.array_equal(y, G["cl_out"])
    y0 = O.convrot_linear_reference(G["cl_x"], G["cl_w8"], G["cl_ws"], None, rotation="identity")
    assert np.array_equal(y0, G["cl_out_nobias"])


def test_linear_dw_within_accumulation_order(G):
    d = O.linear_dw(G["dw_dy"], G["dw_x"])
    ref = O.bf16_bits_to_f32(G["dw_out"])
    got = O.bf16_bits_to_f32(d)
    # the bf16 matmul's accumulation order is torch's; the values agree to a bf16 ulp
    assert np.abs(got - ref).max() <= np.abs(ref).max() * 2 ** -7
    assert (d != G["dw_out"]).mean() < 1e-3


def test_prepare_weight_chain(G):
    q, s = O.prepare_weight(O.bf16_bits_to_f32(G["pw_w"]))
    assert np.array_equal(q, G["pw_q"])
    assert _bits_equal(s, G["pw_s"])


def test_dequant_weight_chain(G):
    assert np.array_equal(O.dequant_weight(G["pw_q"], G["pw_s"]), G["dq_w"])


def test_linear_dx_int8_chain(G):
    assert np.array_equal(O.linear_dx_int8(G["dx_dy"], G["pw_q"], G["pw_s"]), G["dx_out"])


def test_gelu_erf_equals_torch_on_every_bf16_of_the_core_range(G):
    x = O.bf16_bits_to_f32(G["gelu_in"])
    with np.errstate(all="ignore"):
        got = O.f32_to_bf16_bits(O._gelu_erf(x))
    # for 1e-30 <= |x| <= 3 the oracle and torch agree bit for bit; outside
    # it 1 + erf cancels, the product overflows, or the result is subnormal
    # (torch's CPU kernel flushes those to zero), and erf implementations
    # round differently there
    core = np.isfinite(x) & (np.abs(x) <= 3.0) & ((np.abs(x) >= 1e-30) | (x == 0))
    assert np.array_equal(got[core], G["gelu_out"][core])
    assert (got != G["gelu_out"])[np.isfinite(x)].mean() < 0.02


def test_gelu_tanh_and_geglu_within_a_few_values(G):
    x = O.bf16_bits_to_f32(G["gelu_in"])
    fin = np.isfinite(x) & (np.abs(x) < 1e30)
    with np.errstate(all="ignore"):
        gt = O.f32_to_bf16_bits(O.activation(1, x))
    assert (gt != G["gelu_tanh_out"])[fin].sum() <= 16
    y = O.f32_to_bf16_bits(O.activation(4, O.bf16_bits_to_f32(G["geglu_h"]),
                                        O.bf16_bits_to_f32(G["geglu_g"])))
    assert (y != G["geglu_y"]).mean() < 1e-3


# ------------------------------------------------------------------ known answers

def test_geglu_reads_hidden_then_gate():
    """The reference's half-order probe (debug/verify_ffn_geglu.py:116-127):
    hidden = 1, gate = -2 must give bf16(1 * bf16(gelu(-2))), not
    bf16(-2 * bf16(gelu(1))); the activated row is constant, and the rotation
    (each radix-4 stage's rows sum to 2, scaled by 1/2) keeps a constant row
    constant: every code is -127."""
    m, k = 8, 256
    x = np.zeros((m, 2 * k), np.float32)
    x[:, :k], x[:, k:] = 1.0, -2.0
    q, s = O.convrot_quantize(O.f32_to_bf16_bits(x), O.ACT_IDS["geglu_erf"])
    y = O.bf16_bits_to_f32(O.f32_to_bf16_bits(O.activation(4, np.float32(1.0), np.float32(-2.0))))
    assert -0.05 < float(y) < -0.04  # gelu(-2) = -0.0455; the swapped halves give -1.68
    qr, sr = O.convrot_quantize(O.f32_to_bf16_bits(np.full((m, k), y, np.float32)))
    assert np.array_equal(q, qr) and np.array_equal(s.view(np.uint32), sr.view(np.uint32))
    assert (q == -127).all()


def test_ties_round_to_even():
    # tests/test_quantize.py:84-91 of the reference
    q, s = O.quantize_row(np.array([[127.0, 254.0, -254.0, 63.0]], np.float32))
    assert q[0].tolist() == [64, 127, -127, 32]
    assert s[0] == np.float32(2.0)


def test_the_row_quantizer_is_the_float64_formula():
    # tests/test_quantize.py:42-52 of the reference
    rng = np.random.default_rng(0)
    x = O.round_bf16((rng.standard_normal((8, 64)) * 0.4).astype(np.float32))
    q, _ = O.quantize_row(x)
    xf = x.astype(np.float64)
    scale = np.maximum(np.abs(xf).max(axis=-1, keepdims=True) / 127.0, 1e-30)
    want = np.clip(np.rint(xf / scale), -127, 127)
    assert np.array_equal(q.astype(np.int16), want.astype(np.int16))


def test_hadamard_is_orthogonal_and_symmetric():
    H = O.hadamard_matrix()
    assert np.allclose(H @ H, np.eye(256), atol=1e-12)
    assert np.array_equal(H, H.T)
    assert set(np.unique(np.abs(H))) == {1.0 / 16}


def test_rotation_of_a_basis_vector_is_a_column_of_H():
    e = np.zeros((1, 256), np.float32)
    e[0, 37] = 1.0
    assert np.array_equal(O.rotate_groups(e)[0].astype(np.float64), O.hadamard_matrix()[37])


def test_butterflies_match_the_dense_matrix():
    rng = np.random.default_rng(1)
    x = O.round_bf16(rng.standard_normal((16, 1024)).astype(np.float32))
    got = O.rotate_groups(x).astype(np.float64)
    ref = O.rotate_groups_dense_f64(x)
    assert np.abs(got - ref).max() <= 1e-6 * np.abs(ref).max()


def test_rotation_is_its_own_inverse():
    rng = np.random.default_rng(2)
    x = O.round_bf16(rng.standard_normal((8, 512)).astype(np.float32))
    back = O.rotate_groups(O.rotate_groups(x))
    assert np.abs(back - x).max() <= 1e-6 * np.abs(x).max()


def test_quantize_round_trip_recovers_the_rotation():
    rng = np.random.default_rng(3)
    x = O.round_bf16(rng.standard_normal((32, 1280)).astype(np.float32))
    q, s = O.convrot_quantize(x)
    rot = O.rotate_groups(x)
    err = np.abs(q.astype(np.float32) * s[:, None] - rot).max(axis=1)
    assert np.all(err <= s * 0.5 * (1 + 1e-5))


def test_the_two_forward_definitions_agree_within_the_gate():
    # the kernel semantics and convrot_linear.py with the Hadamard in
    rng = np.random.default_rng(4)
    x = O.round_bf16(rng.standard_normal((64, 512)).astype(np.float32))
    w = O.round_bf16((rng.standard_normal((128, 512)) * 0.02).astype(np.float32))
    w8, ws = O.prepare_weight(w)
    a = O.bf16_bits_to_f32(O.linear(x, w8, ws)).astype(np.float64)
    b = O.bf16_bits_to_f32(O.convrot_linear_reference(x, w8, ws)).astype(np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-2


def test_int8_dw_is_close_to_the_bf16_gradient():
    rng = np.random.default_rng(5)
    m, n, k = 256, 64, 512
    x = O.round_bf16(rng.standard_normal((m, k)).astype(np.float32))
    dy = O.round_bf16((rng.standard_normal((m, n)) * 1e-3).astype(np.float32))
    xq, xs = O.convrot_quantize(x)
    dw = O.bf16_bits_to_f32(O.linear_dw_int8(dy, xq, xs)).astype(np.float64)
    ref = dy.astype(np.float64).T @ x.astype(np.float64)
    assert np.linalg.norm(dw - ref) / np.linalg.norm(ref) < 0.03


def test_int_mm_is_exact():
    rng = np.random.default_rng(6)
    a = rng.integers(-127, 128, (33, 160), dtype=np.int8)
    b = rng.integers(-127, 128, (48, 160), dtype=np.int8)
    ref = a.astype(np.int64) @ b.astype(np.int64).T
    assert np.array_equal(O.int_mm(a, b), ref.astype(np.int32))


def test_torch_cpu_restatement_of_convrot_linear_as_shipped(G):
    """oracle/convrot_torch_cpu.py (the benchmark's reference arm) gives the
    shipped reference/convrot_linear.py's bits, and with the Hadamard the numpy
    restatement's."""
    import torch
    from oracle import convrot_torch_cpu as T

    def t16(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)

    x, w8 = t16(G["cl_x"]), torch.from_numpy(G["cl_w8"])
    ws, b = torch.from_numpy(G["cl_ws"]), t16(G["cl_bias"])
    y = T.convrot_int8_linear_cpu(x, w8, ws, b, rotation="identity")
    assert np.array_equal(y.view(torch.int16).numpy().view(np.uint16), G["cl_out"])
    y0 = T.convrot_int8_linear_cpu(x, w8, ws, None, rotation="identity")
    assert np.array_equal(y0.view(torch.int16).numpy().view(np.uint16), G["cl_out_nobias"])
    yh = T.convrot_int8_linear_cpu(x, w8, ws, b, rotation="hadamard")
    ref = O.convrot_linear_reference(G["cl_x"], G["cl_w8"], G["cl_ws"],
                                     O.bf16_bits_to_f32(G["cl_bias"]), rotation="hadamard")
    got = yh.view(torch.int16).numpy().view(np.uint16)
    # the bf16 matmul's accumulation order may differ from float64-then-round in
    # rare last bits of x_rot; the outputs agree to a bf16 ulp at most there
    d = np.abs(O.bf16_bits_to_f32(got).astype(np.float64) - O.bf16_bits_to_f32(ref))
    assert (got != ref).mean() < 0.02 and d.max() <= 0.02 * np.abs(O.bf16_bits_to_f32(ref)).max()
    assert np.array_equal(T.hadamard_bf16().float().numpy(), O.hadamard_matrix().astype(np.float32))


def test_rms_rope_restatement_matches_the_reference_chain():
    """The oracle's RMS norm + rotary embedding (the consumer of the fused qkv
    accumulator) against the reference's torch chain
    (python/xpu_kernels/triton/reference.py:63-98) on the bf16 dequant of an
    int32 accumulator slice, exactly as the reference's own probe builds its
    expected value (tests/golden/reference_rope.npz); the int32 form with the
    dequant folded in gives the same bits."""
    import os
    R = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_rope.npz"))
    B, S, H, D = 1, 48, 3, 128
    pe = R["pe"].reshape(B, S, D // 2, 2, 2)
    for name, lo in (("q", 0), ("k", H * D)):
        got = O.rms_rope(R[f"{name}_x"], pe, R["scale"], 1e-6, True)
        assert np.array_equal(got, R[f"{name}_out"].reshape(got.shape))
        acc = R["acc"][:, lo:lo + H * D].reshape(B, S, H, D)
        got_acc = O.rms_rope(acc, pe, R["scale"], 1e-6, True, R["xs"], R["ws"][lo:lo + H * D])
        assert np.array_equal(got_acc, got)
