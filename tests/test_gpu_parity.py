"""GPU parity: every CUDA kernel against the CPU oracle on the same seeded inputs.

Integer and byte results must be bit-exact (int32 accumulators, int8 codes of
the pure rotation paths, bf16 outputs of the rotation / dequant paths whose
fp32 arithmetic the oracle restates operation for operation).  Where a device
transcendental (erf, tanh, exp) enters, the north-star tolerance applies:
int8 codes may differ by 1 at a rate below 1e-4 (counted over every code a
test produces, and printed), bf16 outputs by a relative L2 of 1e-2; and every
row whose codes match the oracle's exactly must give bit-identical outputs.

Large shapes are checked through size-independent properties: rows are
independent in every kernel of the forward, so a sample of rows of a full-size
call is compared exactly with the oracle run on those rows alone.
"""

import numpy as np
import pytest
import torch

from oracle import convrot_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    import xpu_kernels
    from xpu_kernels.int8 import _lib as L
    if not torch.cuda.is_available():
        pytest.fail("no CUDA device")
    if not xpu_kernels.available():
        pytest.fail(f"libxpuint8 did not load: {L._ERR}")
    yield
    torch.cuda.synchronize()
    assert L.load().xpuint8_fault_status(1) == 0


def bits(t):
    """torch tensor -> numpy (bf16 as uint16 bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def dev_bf16(a):
    """numpy uint16 bits -> CUDA bf16 tensor."""
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(DEV)


def rand_bf16(shape, seed, scale=1.0, outliers=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=g) * scale
    if outliers:
        cols = torch.randperm(shape[-1], generator=g)[:outliers]
        x[..., cols] *= 20
    return x.to(torch.bfloat16)


def rand_i8(shape, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(-127, 128, shape, generator=g, dtype=torch.int8)


#: the north-star bound on int8 codes that differ (by 1) where a device
#: transcendental enters the activation
CODE_RATE = 1e-4


def code_mismatches(got, ref):
    """(number of codes that differ, number of codes); every difference must be +-1."""
    d = np.abs(got.astype(np.int16) - ref.astype(np.int16))
    assert d.max(initial=0) <= 1, f"max code difference {d.max()}"
    return int((d > 0).sum()), int(d.size)


def codes_close(got, ref, rate=CODE_RATE, what="codes"):
    bad, n = code_mismatches(got, ref)
    print(f"\n{what}: {bad} of {n} codes differ by 1 (rate {bad / max(n, 1):.2e})")
    assert bad / max(n, 1) < rate, f"mismatch rate {bad / n:.2e}"


def scales_close(got, ref, ulps=1):
    gi = got.view(np.int32).astype(np.int64)
    ri = ref.view(np.int32).astype(np.int64)
    assert np.abs(gi - ri).max() <= ulps


def rel_l2(a, b):
    a = O.bf16_bits_to_f32(a).astype(np.float64) if a.dtype == np.uint16 else a.astype(np.float64)
    b = O.bf16_bits_to_f32(b).astype(np.float64) if b.dtype == np.uint16 else b.astype(np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


SHAPES = [(1, 256), (3, 1024), (127, 1280), (300, 4096), (37, 5120), (9, 10240), (5, 32768)]


# ------------------------------------------------------------------------ rotation family

@pytest.mark.parametrize("m,k", SHAPES)
def test_rotate_bf16_is_bit_exact(m, k):
    from xpu_kernels import int8
    x = rand_bf16((m, k), 10 + k, outliers=4)
    got = bits(int8.rotate(x.to(DEV)))
    assert np.array_equal(got, O.rotate_bf16(bits(x)))


@pytest.mark.parametrize("m,k", SHAPES)
def test_quantize_is_bit_exact(m, k):
    from xpu_kernels import int8
    x = rand_bf16((m, k), 20 + k, outliers=8)
    q, s = int8.quantize(x.to(DEV))
    qr, sr = O.convrot_quantize(bits(x))
    assert np.array_equal(bits(s).view(np.uint32), sr.view(np.uint32))
    assert np.array_equal(bits(q), qr)


@pytest.mark.parametrize("k", [1024, 2048, 3072, 4096, 5120, 6144, 7168, 8192])
@pytest.mark.parametrize("m", [1, 3, 333])
def test_quantize_four_group_teams_are_bit_exact(m, k):
    """Row widths that are multiples of 1024 run the four-groups-per-slot
    quantizer (teams of 4 to 14 slots, 1 to 4 rows per batch); ragged row
    counts leave partial last batches.  Codes and scales equal the oracle's."""
    from xpu_kernels import int8
    x = rand_bf16((m, k), 90 + k + m, outliers=6)
    q, s = int8.quantize(x.to(DEV))
    qr, sr = O.convrot_quantize(bits(x))
    assert np.array_equal(bits(s).view(np.uint32), sr.view(np.uint32))
    assert np.array_equal(bits(q), qr)


def test_quantize_edge_rows():
    from xpu_kernels import int8
    x = torch.zeros(6, 512, dtype=torch.bfloat16)
    x[1, 7] = 1.0                       # one-hot row
    x[2] = -3.0                         # constant row
    x[3, ::2] = 1e-20                   # tiny values
    x[4] = rand_bf16((512,), 5) * 1e4   # large values
    x[5, :4] = torch.tensor([127.0, 254.0, -254.0, 63.0])
    q, s = int8.quantize(x.to(DEV))
    qr, sr = O.convrot_quantize(bits(x))
    assert np.array_equal(bits(q), qr)
    assert np.array_equal(bits(s).view(np.uint32), sr.view(np.uint32))
    assert bits(s)[0] == np.float32(1e-30) and not bits(q)[0].any()


def test_scale_math_matches_the_ieee_definition():
    """The quantizers' row scale (s = max(amax/127, 1e-30), 1/s) without the
    library divide equals the IEEE form on every non-negative float, the packed
    code arithmetic rounds the product and the sum separately, and the row
    quantizer's division gives the IEEE division's code on every pair of bf16
    value and bf16 row maximum."""
    import ctypes
    from xpu_kernels.int8 import _lib as L
    bad_scale, bad_quant = ctypes.c_int64(-1), ctypes.c_int64(-1)
    rc = L.load().xpuint8_check_scale_math(ctypes.addressof(bad_scale), ctypes.addressof(bad_quant))
    assert rc == 0, L.load().xpuint8_last_error()
    assert (bad_scale.value, bad_quant.value) == (0, 0), L.load().xpuint8_last_error()


def test_quantize_full_c5_every_code():
    """Config C5's activation (x [65536, 4096], 0.5 % outlier channels x20):
    every code and every row scale of the GPU rotate+quantize equals the
    oracle's."""
    from xpu_kernels import int8
    m, k = 65536, 4096
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(m, k, generator=g, device=DEV)
    x[:, torch.randperm(k, device=DEV, generator=g)[:20]] *= 20
    x = x.to(torch.bfloat16)
    q, s = int8.quantize(x)
    for r in range(0, m, 8192):
        qr, sr = O.convrot_quantize(bits(x[r:r + 8192]))
        assert np.array_equal(bits(s[r:r + 8192]).view(np.uint32), sr.view(np.uint32)), r
        assert np.array_equal(bits(q[r:r + 8192]), qr), r


def test_geglu_halves_are_not_swapped():
    """The reference's half-order probe (debug/verify_ffn_geglu.py:116-127):
    hidden = 1, gate = -2 through the fused quantizer equals the torch chain
    quantize(hidden * gelu(gate)) bit for bit (the swapped halves would give
    -2 * gelu(1)); the same for the dequant + activation path, whose int32
    accumulators dequantize to those values."""
    from xpu_kernels import int8
    m, k = 8, 256
    x = torch.zeros(m, 2 * k, dtype=torch.bfloat16, device=DEV)
    x[:, :k], x[:, k:] = 1.0, -2.0
    hidden, gate = x.chunk(2, dim=-1)
    q_ref, s_ref = int8.quantize((hidden * torch.nn.functional.gelu(gate)).contiguous())
    q, s = int8.quantize_act(x, "geglu_erf")
    assert torch.equal(q, q_ref) and torch.equal(s.view(torch.int32), s_ref.view(torch.int32))
    acc = torch.zeros(m, 2 * k, dtype=torch.int32, device=DEV)
    acc[:, :k], acc[:, k:] = 1, -2
    ones = torch.ones(m, dtype=torch.float32, device=DEV)
    q2, s2 = int8.dequant_act_quantize(acc, ones, torch.ones(2 * k, dtype=torch.float32, device=DEV), "geglu_erf")
    assert torch.equal(q2, q_ref) and torch.equal(s2.view(torch.int32), s_ref.view(torch.int32))


@pytest.mark.parametrize("act", ["gelu_tanh", "swiglu", "situ", "geglu_erf", "gelu_erf"])
def test_quantize_act(act):
    """Each fused input activation over three shapes (edge, C2-like, C5-like
    rows): codes within +-1 of the oracle's at a rate below 1e-4 of all the
    codes, and every row whose scale is the oracle's has the oracle's codes
    wherever its activations round to the same bf16."""
    from xpu_kernels import int8
    bad = total = 0
    for m, k in [(5, 256), (512, 1280), (65, 4096)]:
        kin = 2 * k if act in int8.PAIRED_ACTIVATIONS else k
        x = rand_bf16((m, kin), 30 + k, scale=2.0)
        q, s = int8.quantize_act(x.to(DEV), act)
        qr, sr = O.convrot_quantize(bits(x), int8.ACTIVATIONS[act])
        b, n = code_mismatches(bits(q), qr)
        bad, total = bad + b, total + n
        scales_close(bits(s), sr, ulps=2 ** 16)  # a 1-ulp bf16 activation can move the row max
        assert np.abs(bits(s) / sr - 1).max() < 1e-2
    print(f"\nquantize_act {act}: {bad} of {total} codes differ by 1 (rate {bad / total:.2e})")
    assert bad / total < CODE_RATE


@pytest.mark.parametrize("n,k", [(16, 256), (300, 1280), (64, 5120)])
def test_dequant_weight_is_bit_exact(n, k):
    from xpu_kernels import int8
    w8 = rand_i8((n, k), 40 + k)
    g = torch.Generator().manual_seed(41)
    ws = torch.rand(n, generator=g) * 0.01 + 1e-4
    got = bits(int8.dequant_weight(w8.to(DEV), ws.to(DEV)))
    assert np.array_equal(got, O.dequant_weight(bits(w8), bits(ws)))
    # and it is the torch chain of the reference
    chain = bits(int8.dequant_weight_torch(w8.to(DEV), ws.to(DEV)))
    assert np.array_equal(got, chain)


@pytest.mark.parametrize("act", ["situ", "geglu_erf", "gelu_erf"])
def test_dequant_act_quantize(act):
    """Dequant + activation + rotate + quantize of an up-projection accumulator
    over three shapes: codes within +-1 at a rate below 1e-4 of all codes."""
    from xpu_kernels import int8
    bad = total = 0
    for m, k in [(7, 256), (512, 1280), (19, 5120)]:
        n = 2 * k if act in int8.PAIRED_ACTIVATIONS else k
        g = torch.Generator().manual_seed(50 + k)
        acc = torch.randint(-200000, 200000, (m, n), generator=g, dtype=torch.int32)
        xs = torch.rand(m, generator=g) * 1e-3 + 1e-5
        ws = torch.rand(n, generator=g) * 1e-3 + 1e-5
        q, s = int8.dequant_act_quantize(acc.to(DEV), xs.to(DEV), ws.to(DEV), act)
        qr, sr = O.dequant_act_quantize(bits(acc), bits(xs), bits(ws), int8.ACTIVATIONS[act])
        b, nn = code_mismatches(bits(q), qr)
        bad, total = bad + b, total + nn
        assert np.abs(bits(s) / sr - 1).max() < 1e-2
    print(f"\ndequant_act_quantize {act}: {bad} of {total} codes differ by 1 "
          f"(rate {bad / total:.2e})")
    assert bad / total < CODE_RATE


# ------------------------------------------------------------------------ dequant epilogue

@pytest.mark.parametrize("m,n", [(1, 16), (129, 272), (300, 1280)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_dequant_epilogue_is_bit_exact(m, n, with_bias):
    from xpu_kernels import int8
    g = torch.Generator().manual_seed(60 + n)
    acc = torch.randint(-(2 ** 24), 2 ** 24, (m, n), generator=g, dtype=torch.int32)
    xs = torch.rand(m, generator=g) * 1e-3
    ws = torch.rand(n, generator=g) * 1e-2
    b = torch.randn(n, generator=g) * 0.1 if with_bias else None
    got = bits(int8.dequant(acc.to(DEV), xs.to(DEV), ws.to(DEV), None if b is None else b.to(DEV)))
    ref = O.dequant_epilogue(bits(acc), bits(xs), bits(ws), None if b is None else bits(b))
    assert np.array_equal(got, ref)


def test_dequant_slice_reads_in_place():
    from xpu_kernels import int8
    g = torch.Generator().manual_seed(70)
    big = torch.randint(-(2 ** 20), 2 ** 20, (77, 3 * 320), generator=g, dtype=torch.int32).to(DEV)
    xs = (torch.rand(77, generator=g) * 1e-3).to(DEV)
    ws = (torch.rand(320, generator=g) * 1e-2).to(DEV)
    for j in range(3):
        sl = big[:, j * 320:(j + 1) * 320]
        got = int8.dequant_slice(sl, xs, ws)
        ref = int8.dequant(sl.contiguous(), xs, ws)
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16))
    # an odd offset (not 16-byte aligned) takes the scalar path
    sl = big[:, 3:3 + 320]
    assert torch.equal(int8.dequant_slice(sl, xs, ws).view(torch.int16),
                       int8.dequant(sl.contiguous(), xs, ws).view(torch.int16))


# ------------------------------------------------------------------------ the int8 GEMM

GEMM_SHAPES = [(1, 16, 256), (129, 272, 1280), (300, 1024, 4096), (128, 256, 128),
               (257, 528, 48), (2048, 1280, 1280)]


def _exact(a, b):
    return (a.astype(np.float64) @ b.astype(np.float64)).astype(np.int32)


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_int_mm_nt_is_bit_exact(m, n, k):
    from xpu_kernels import int8
    a, b = rand_i8((m, k), 80 + m), rand_i8((n, k), 81 + n)
    got = bits(int8.int_mm(a.to(DEV), b.to(DEV), 0))
    assert np.array_equal(got, _exact(bits(a), bits(b).T))


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_int_mm_nn_is_bit_exact(m, n, k):
    from xpu_kernels import int8
    a, b = rand_i8((m, k), 90 + m), rand_i8((k, n), 91 + n)
    got = bits(int8.int_mm(a.to(DEV), b.to(DEV), 1))
    assert np.array_equal(got, _exact(bits(a), bits(b)))


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_int_mm_tn_is_bit_exact(m, n, k):
    from xpu_kernels import int8
    if m % 16:
        pytest.skip("an MN-major A needs M % 16 == 0 (its row length)")
    a, b = rand_i8((k, m), 100 + m), rand_i8((k, n), 101 + n)
    got = bits(int8.int_mm(a.to(DEV), b.to(DEV), 2))
    assert np.array_equal(got, _exact(bits(a).T, bits(b)))


@pytest.mark.parametrize("bn", [128, 160, 192, 224, 256])
@pytest.mark.parametrize("m,n,k", [(300, 1040, 1280), (2048, 2080, 1280)])
def test_every_tile_width_is_bit_exact(monkeypatch, bn, m, n, k):
    """The GEMM picks its output-tile width (128..256 columns) from the shape;
    XPUINT8_GEMM_BN pins it.  Every width gives the exact int32 product and the
    same dequant bits, with ragged last tiles and several tiles per CTA."""
    from xpu_kernels import int8
    from xpu_kernels.int8 import _lib as L
    monkeypatch.setenv("XPUINT8_GEMM_BN", str(bn))
    lib = L.load()
    a, b = rand_i8((m, k), 120 + bn), rand_i8((n, k), 121 + bn)
    exact = _exact(bits(a), bits(b).T)
    ad, bd = a.to(DEV), b.to(DEV)
    assert np.array_equal(bits(int8.int_mm(ad, bd, 0)), exact)
    g = torch.Generator().manual_seed(122)
    xs, ws, bias = torch.rand(m, generator=g) * 1e-3, torch.rand(n, generator=g) * 1e-2, \
        torch.randn(n, generator=g) * 0.1
    out = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    xsd, wsd, bdd = (t.to(DEV) for t in (xs, ws, bias))
    rc = lib.xpuint8_int_mm_dequant_stream(L._stream(out.device), L._ptr(ad), L._ptr(bd),
                                           L._ptr(out), L._ptr(xsd), L._ptr(wsd), L._ptr(bdd),
                                           m, n, k, 0, n)
    assert rc == 0, lib.xpuint8_last_error()
    assert np.array_equal(bits(out), O.dequant_epilogue(exact, bits(xs), bits(ws), bits(bias)))


def test_int_mm_extreme_values_do_not_overflow():
    from xpu_kernels import int8
    k = 4096
    a = torch.full((128, k), -127, dtype=torch.int8)
    b = torch.full((256, k), -127, dtype=torch.int8)
    got = int8.int_mm(a.to(DEV), b.to(DEV))
    assert int(got.min()) == int(got.max()) == 127 * 127 * k


@pytest.mark.parametrize("m,n,k", [(129, 272, 1280), (2048, 1280, 1280)])
def test_gemm_dequant_epilogue_is_bit_exact(m, n, k):
    from xpu_kernels import int8
    from xpu_kernels.int8 import _lib as L
    lib = L.load()
    a, b = rand_i8((m, k), 110), rand_i8((n, k), 111)
    g = torch.Generator().manual_seed(112)
    xs, ws, bias = torch.rand(m, generator=g) * 1e-3, torch.rand(n, generator=g) * 1e-2, \
        torch.randn(n, generator=g) * 0.1
    out = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    ad, bd, xsd, wsd, bdd = (t.to(DEV) for t in (a, b, xs, ws, bias))
    rc = lib.xpuint8_int_mm_dequant_stream(L._stream(out.device), L._ptr(ad), L._ptr(bd),
                                           L._ptr(out), L._ptr(xsd), L._ptr(wsd), L._ptr(bdd),
                                           m, n, k, 0, n)
    assert rc == 0, lib.xpuint8_last_error()
    ref = O.dequant_epilogue(_exact(bits(a), bits(b).T), bits(xs), bits(ws), bits(bias))
    assert np.array_equal(bits(out), ref)
    # and equal to the standalone epilogue on the raw accumulator
    acc = int8.int_mm(ad, bd)
    assert torch.equal(int8.dequant(acc, xsd, wsd, bdd).view(torch.int16), out.view(torch.int16))


@pytest.mark.parametrize("m,inner,k", [(64, 256, 256), (300, 1280, 1280)])
def test_gemm_geglu_epilogue(m, inner, k):
    from xpu_kernels.int8 import _lib as L
    lib = L.load()
    a, b = rand_i8((m, k), 120), rand_i8((2 * inner, k), 121)
    g = torch.Generator().manual_seed(122)
    xs, ws = torch.rand(m, generator=g) * 1e-3, torch.rand(2 * inner, generator=g) * 1e-2
    y = torch.empty((m, inner), dtype=torch.bfloat16, device=DEV)
    ad, bd, xsd, wsd = (t.to(DEV) for t in (a, b, xs, ws))
    rc = lib.xpuint8_int_mm_geglu_stream(L._stream(y.device), L._ptr(ad), L._ptr(bd), L._ptr(y),
                                         L._ptr(xsd), L._ptr(wsd), m, inner, k)
    assert rc == 0, lib.xpuint8_last_error()
    acc = _exact(bits(a), bits(b).T)
    d = O.round_bf16((acc.astype(np.float32) * (bits(ws)[None, :] * bits(xs)[:, None]).astype(np.float32)).astype(np.float32))
    ref = O.f32_to_bf16_bits(O.activation(4, d[:, :inner], d[:, inner:]))
    got = bits(y)
    # The device erf differs from the correctly rounded one in rare last bits,
    # which can move the bf16 rounding of gelu(g) and so of y by one bf16 ulp
    # (measured on B200: 42 of 384000 values, 1.1e-4); where 1 + erf(g/sqrt 2)
    # cancels (g < -3) gelu(g) is tiny and its few significant bits may differ
    # more, by a negligible absolute amount.  The gate: every difference is one
    # ulp or below 1e-3 of the largest |y|, at most 5e-4 of the values differ,
    # rel-L2 below 1e-3.
    diff = got != ref
    ulps = np.abs(got.view(np.int16).astype(np.int32) - ref.view(np.int16).astype(np.int32))
    gf, rf = O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(ref)
    tiny = np.abs(gf - rf) <= 1e-3 * np.abs(rf).max()
    print(f"\nGEGLU epilogue {m}x{inner}x{k}: {int(diff.sum())} of {got.size} bf16 values "
          f"differ (rate {diff.mean():.2e}; {int((diff & (ulps > 1)).sum())} by more than one "
          f"ulp, all below 1e-3 of max|y|), rel-L2 {rel_l2(got, ref):.2e}")
    assert np.all((ulps <= 1) | tiny)
    assert diff.mean() < 5e-4
    assert rel_l2(got, ref) < 1e-3


# ------------------------------------------------------------------------ compositions

def _prep(n, k, seed):
    w = rand_bf16((n, k), seed, scale=0.02)
    w8, ws = O.prepare_weight(bits(w))
    return w, w8, ws


@pytest.mark.parametrize("m,n,k", [(256, 1024, 1024), (77, 272, 512)])
def test_linear_matches_the_oracle(m, n, k):
    from xpu_kernels import int8
    x = rand_bf16((m, k), 130, outliers=8)
    _, w8, ws = _prep(n, k, 131)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(132)) * 0.01)
    got = bits(int8.linear(x.to(DEV), torch.from_numpy(w8).to(DEV), torch.from_numpy(ws).to(DEV),
                           bias.to(DEV)))
    ref = O.linear(bits(x), w8, ws, bits(bias))
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("m,n_local,k", [(1000, 1040, 1280), (256, 64, 256), (77, 1792, 4096)])
def test_allgather_epilogue_on_one_gpu(m, n_local, k):
    """The all-gather linear's multi-destination, wide-store epilogue on one GPU:
    two 'ranks' (two calls with rank 0 and 1 and their own weight blocks) store
    their column blocks into two local buffers; both buffers must equal the
    linear of the whole weight, bit for bit."""
    import ctypes
    from xpu_kernels import int8
    from xpu_kernels.int8 import _lib as L
    lib = L.load()
    n = 2 * n_local
    _, w8n, wsn = _prep(n, k, 180 + k)
    w8, ws = torch.from_numpy(w8n).to(DEV), torch.from_numpy(wsn).to(DEV)
    x = rand_bf16((m, k), 181 + m, outliers=4).to(DEV)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(n)) * 0.01).to(DEV)
    full = int8.linear(x, w8, ws, bias)
    outs = [torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(2)]
    table = (ctypes.c_void_p * 2)(*[o.data_ptr() for o in outs])
    xq = torch.empty(m, k, dtype=torch.int8, device=DEV)
    xs = torch.empty(m, dtype=torch.float32, device=DEV)
    for r in range(2):
        sl = slice(r * n_local, (r + 1) * n_local)
        w8r, wsr, br = w8[sl].contiguous(), ws[sl].contiguous(), bias[sl].contiguous()
        rc = lib.xpuint8_linear_allgather_stream(L._stream(torch.device(DEV)), L._ptr(x), L._ptr(w8r),
                                                 L._ptr(wsr), L._ptr(br), table, 2, r, L._ptr(xq),
                                                 L._ptr(xs), m, n_local, k, 0)
        assert rc == 0, lib.xpuint8_last_error()
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o.view(torch.int16), full.view(torch.int16))


def test_prepare_weight_matches_the_reference_fixture():
    from xpu_kernels import int8
    import os
    G = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_cpu.npz"))
    q, s = int8.prepare_weight(dev_bf16(G["pw_w"]))
    assert np.array_equal(bits(q), G["pw_q"])
    assert np.array_equal(bits(s).view(np.uint32), G["pw_s"].view(np.uint32))
    dq = int8.dequant_weight(q, s)
    assert np.array_equal(bits(dq), G["dq_w"])
    dx = int8.linear_dx_int8(dev_bf16(G["dx_dy"]), q, s)
    assert np.array_equal(bits(dx), G["dx_out"])


def test_quantize_row_matches_the_reference_fixture():
    from xpu_kernels import int8
    import os
    G = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_cpu.npz"))
    q, s = int8.quantize_row(dev_bf16(G["qrow_x"]))
    assert np.array_equal(bits(q), G["qrow_q"])
    assert np.array_equal(bits(s).view(np.uint32), G["qrow_s"].view(np.uint32))
    tie = torch.tensor([[127.0, 254.0, -254.0, 63.0] + [0.0] * 4], dtype=torch.bfloat16)
    q, _ = int8.quantize_row(tie.to(DEV))
    assert bits(q)[0, :4].tolist() == [64, 127, -127, 32]


def test_quantize_row_reference_probe_rows():
    """The rows of the reference's own probe of its Triton row quantizer
    (triton/quantize.py:234-255): 64 x 3072 and 64 x 8192 of N(0, 0.4), and
    the tie rows arange(-8, 8) / 2, bit-exact against the oracle."""
    from xpu_kernels import int8
    g = torch.Generator().manual_seed(0)
    tie = (torch.arange(-8, 8, dtype=torch.float32) * 0.5).repeat(64, 1).to(torch.bfloat16)
    for x in [(torch.randn(64, 3072, generator=g) * 0.4).to(torch.bfloat16),
              (torch.randn(64, 8192, generator=g) * 0.4).to(torch.bfloat16), tie]:
        q, s = int8.quantize_row(x.to(DEV))
        qr, sr = O.quantize_row(bits(x))
        assert np.array_equal(bits(q), qr)
        assert np.array_equal(bits(s).view(np.uint32), sr.view(np.uint32))


@pytest.mark.parametrize("m,k", [(64, 5120), (3, 24), (100, 1000), (40, 8192), (7, 8200)])
def test_quantize_row_is_bit_exact(m, k):
    from xpu_kernels import int8
    x = rand_bf16((m, k), 140 + k, scale=1e-3)
    q, s = int8.quantize_row(x.to(DEV))
    qr, sr = O.quantize_row(bits(x))
    assert np.array_equal(bits(q), qr)
    assert np.array_equal(bits(s).view(np.uint32), sr.view(np.uint32))
    qt, st = int8.quantize_row_torch(x.to(DEV))
    assert torch.equal(qt.cpu(), torch.from_numpy(qr))


@pytest.mark.parametrize("m,k", [(33, 5120), (5, 1032), (9, 8200)])
def test_quantize_row_column_scaled_is_bit_exact(m, k):
    """bf16(x * bf16(col_scale)) then the row quantizer (linear_dx_int8's operand)."""
    from xpu_kernels import int8
    x = rand_bf16((m, k), 160 + k, scale=1e-3)
    cs = torch.rand(k, generator=torch.Generator().manual_seed(k)) * 0.04 + 1e-4
    q, s = int8.quantize_row(x.to(DEV), cs.to(DEV))
    d = O.f32_to_bf16_bits(O.bf16_bits_to_f32(bits(x)) * O.round_bf16(cs.numpy().astype(np.float32)))
    qr, sr = O.quantize_row(d)
    assert np.array_equal(bits(q), qr)
    assert np.array_equal(bits(s).view(np.uint32), sr.view(np.uint32))


@pytest.mark.parametrize("m,n", [(1000, 5136), (3, 16), (129, 272)])
def test_colquant_is_bit_exact(m, n):
    """The int8 weight gradient's column quantizer on ragged tiles."""
    import ctypes
    from xpu_kernels.int8 import _lib as L
    dy = rand_bf16((m, n), 170 + n, scale=1e-3)
    xs = (torch.rand(m, generator=torch.Generator().manual_seed(m)) * 0.05 + 1e-3).float()
    gq = torch.empty(m, n, dtype=torch.int8, device=DEV)
    tg = torch.empty(n, dtype=torch.float32, device=DEV)
    dyd, xsd = dy.to(DEV), xs.to(DEV)
    rc = L.load().xpuint8_colquant_stream(L._stream(torch.device(DEV)), L._ptr(dyd), L._ptr(xsd),
                                          L._ptr(gq), L._ptr(tg), m, n)
    assert rc == 0, L.load().xpuint8_last_error()
    qr, tr = O.colquant_scaled(bits(dy), xs.numpy())
    assert np.array_equal(bits(tg).view(np.uint32), tr.view(np.uint32))
    assert np.array_equal(bits(gq), qr)


@pytest.mark.parametrize("m,n,k", [(256, 512, 1280), (100, 208, 768), (333, 1040, 256), (4000, 640, 1280)])
def test_linear_dx_int8_matches_the_oracle(m, n, k):
    """The one-call entry (row quantizer, GEMM with MN-major B, rotate), with
    ragged M and N."""
    from xpu_kernels import int8
    _, w8, ws = _prep(n, k, 150)
    dy = rand_bf16((m, n), 151, scale=1e-3)
    got = bits(int8.linear_dx_int8(dy.to(DEV), torch.from_numpy(w8).to(DEV),
                                   torch.from_numpy(ws).to(DEV)))
    assert np.array_equal(got, O.linear_dx_int8(bits(dy), w8, ws))


@pytest.mark.parametrize("m,n,k", [(512, 256, 1280), (272, 208, 512), (100, 256, 768), (384, 3872, 1280)])
def test_linear_dw_int8_matches_the_oracle(m, n, k):
    """The one-call entry (column quantizer, GEMM with both operands MN-major,
    rotate), with ragged M and N."""
    from xpu_kernels import int8
    x = rand_bf16((m, k), 160)
    dy = rand_bf16((m, n), 161, scale=1e-3)
    xq, xs = int8.quantize(x.to(DEV))
    got = bits(int8.linear_dw_int8(dy.to(DEV), xq, xs))
    ref = O.linear_dw_int8(bits(dy), bits(xq), bits(xs))
    assert np.array_equal(got, ref)


def _ffn_codes(x, up8, up_s, act):
    """The FFN's intermediate int8 codes on the GPU, step by step through the
    library (the same kernels the fused entry runs)."""
    import ctypes  # noqa: F401
    from xpu_kernels import int8
    from xpu_kernels.int8 import _lib as L
    lib = L.load()
    xq, xs = int8.quantize(x)
    if act == "geglu_erf":
        inner = up8.shape[0] // 2
        y = torch.empty((x.shape[0], inner), dtype=torch.bfloat16, device=DEV)
        rc = lib.xpuint8_int_mm_geglu_stream(L._stream(y.device), L._ptr(xq), L._ptr(up8), L._ptr(y),
                                             L._ptr(xs), L._ptr(up_s), x.shape[0], inner, x.shape[1])
        assert rc == 0, lib.xpuint8_last_error()
        return int8.quantize(y)
    acc = int8.int_mm(xq, up8)
    return int8.dequant_act_quantize(acc, xs, up_s, act)


def _check_ffn_rows(x, up8, up_s, dn8, dn_s, dn_b, act, got, rows, ref):
    """The FFN on `rows` (got: the fused entry's output on those rows; ref: the
    oracle's): the intermediate codes differ from the oracle's by +-1 at a rate
    below 1e-4, the bf16 output is within rel-L2 1e-2, and every row whose
    intermediate codes equal the oracle's gives bit-identical outputs."""
    from xpu_kernels import int8
    q2, _ = _ffn_codes(x, up8, up_s, act)
    q2 = bits(q2)[rows]
    xq_r, xs_r = O.convrot_quantize(bits(x)[rows])
    acc_r = O.int_mm(xq_r, bits(up8))
    q2r, _ = O.dequant_act_quantize(acc_r, xs_r, O._expand(bits(up_s), acc_r.shape[1]),
                                    int8.ACTIVATIONS[act])
    codes_close(q2, q2r, what=f"FFN {act} intermediate")
    same = np.all(q2 == q2r, axis=1)
    assert rel_l2(got, ref) < 1e-2, rel_l2(got, ref)
    assert np.array_equal(got[same], ref[same]), "a row with the oracle's codes differs"
    print(f"FFN {act}: {int(same.sum())} of {len(rows)} rows bit-exact, "
          f"rel-L2 {rel_l2(got, ref):.2e}")


@pytest.mark.parametrize("act", ["geglu_erf", "situ", "gelu_erf"])
def test_ffn_matches_the_oracle(act):
    from xpu_kernels import int8
    m, k, inner = 96, 512, 768
    n_up = 2 * inner if act in int8.PAIRED_ACTIVATIONS else inner
    x = rand_bf16((m, k), 170)
    _, up8, up_s = _prep(n_up, k, 171)
    _, dn8, dn_s = _prep(k, inner, 172)
    got = bits(int8.ffn(x.to(DEV), torch.from_numpy(up8).to(DEV), torch.from_numpy(up_s).to(DEV),
                        torch.from_numpy(dn8).to(DEV), torch.from_numpy(dn_s).to(DEV), act=act))
    ref = O.ffn(bits(x), up8, up_s, dn8, dn_s, None, int8.ACTIVATIONS[act])
    assert rel_l2(got, ref) < 1e-2
    _check_ffn_rows(x.to(DEV), torch.from_numpy(up8).to(DEV), torch.from_numpy(up_s).to(DEV),
                    torch.from_numpy(dn8).to(DEV), torch.from_numpy(dn_s).to(DEV), None, act,
                    got, np.arange(m), ref)


def test_geglu_ffn_equals_the_unfused_chain():
    # the reference's self-test: fused GEGLU FFN == dequant -> hidden*gelu(gate) -> quantize
    from xpu_kernels import int8
    m, k, inner = 128, 1280, 1280
    x = rand_bf16((m, k), 180).to(DEV)
    w1 = rand_bf16((2 * inner, k), 181, scale=0.02).to(DEV)
    w2 = rand_bf16((k, inner), 182, scale=0.02).to(DEV)
    up8, up_s = int8.prepare_weight(w1)
    dn8, dn_s = int8.prepare_weight(w2)
    fused = int8.ffn(x, up8, up_s, dn8, dn_s, act="geglu_erf")
    acc, xs = int8.linear_acc(x, up8, up_s)
    d = int8.dequant(acc, xs, up_s)
    h, gt = d.chunk(2, dim=-1)
    q2, xs2 = int8.quantize(h * torch.nn.functional.gelu(gt))
    chain = int8.dequant(int8.int_mm(q2, dn8), xs2, dn_s)
    diff = int((fused.view(torch.int16) != chain.view(torch.int16)).sum().item())
    print(f"\nfused GEGLU FFN vs the unfused chain: {diff} of {fused.numel()} values differ")
    assert diff / fused.numel() < CODE_RATE


@pytest.mark.parametrize("act", ["situ", "gelu_erf"])
def test_ffn_equals_the_accumulator_chain(act):
    """The fused FFN (the activation in the up-projection's epilogue, y stored
    as bf16 and rotated + quantized) equals the reference's own structure run
    on the GPU -- the int32 accumulator, dequant_act_quantize, the down GEMM
    (ops.py:713-718) -- bit for bit, on a ragged row count."""
    from xpu_kernels import int8
    m, k, inner = 300, 1280, 1280
    n_up = 2 * inner if act in int8.PAIRED_ACTIVATIONS else inner
    x = rand_bf16((m, k), 185).to(DEV)
    up8, up_s = int8.prepare_weight(rand_bf16((n_up, k), 186, scale=0.02).to(DEV))
    dn8, dn_s = int8.prepare_weight(rand_bf16((k, inner), 187, scale=0.02).to(DEV))
    fused = int8.ffn(x, up8, up_s, dn8, dn_s, act=act)
    xq, xs = int8.quantize(x)
    q2, xs2 = int8.dequant_act_quantize(int8.int_mm(xq, up8), xs, up_s, act)
    chain = int8.dequant(int8.int_mm(q2, dn8), xs2, dn_s)
    assert torch.equal(fused.view(torch.int16), chain.view(torch.int16))


def test_selftest_passes():
    from xpu_kernels import int8
    from xpu_kernels.int8.selftest import run_checks
    failed = [r for r in run_checks() if not r["ok"]]
    assert not failed, failed
    assert int8.selftest(verbose=True)


# ------------------------------------------------------------------------ full-size properties

@pytest.mark.parametrize("cfg", ["C2", "C3", "C4", "C5"])
def test_full_size_linear_on_sampled_rows(cfg):
    """The BASELINE configs at full size: every row of the output is independent,
    so sampled rows are checked bit for bit against the oracle."""
    from xpu_kernels import int8
    m, k, n, seed = {"C2": (2048, 1280, 1280, 1), "C3": (2048, 1280, 10240, 2),
                     "C4": (4096, 1280, 5120, 3), "C5": (65536, 4096, 14336, 4)}[cfg]
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[:, torch.randperm(k, generator=g)[:max(1, k // 100)]] *= 10
    x = x.to(torch.bfloat16).to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    w8, ws = int8.prepare_weight(w)
    y = int8.linear(x, w8, ws)
    rows = torch.randperm(m, generator=g)[:24].sort().values
    ref = O.linear(bits(x[rows.to(DEV)]), bits(w8), bits(ws))
    assert np.array_equal(bits(y[rows.to(DEV)]), ref)
    # and the accumulators of those rows are exact
    acc, xs = int8.linear_acc(x, w8, ws)
    xq_rows, _ = O.convrot_quantize(bits(x[rows.to(DEV)]))
    assert np.array_equal(bits(acc[rows.to(DEV)]), _exact(xq_rows, bits(w8).T))
    rel = torch.linalg.norm((y.float() - (x.float() @ w.float().t()))) / \
        torch.linalg.norm(x.float() @ w.float().t())
    assert rel.item() < 2e-2


def test_full_size_ffn_c3_on_sampled_rows():
    """Config C3 at full size: x [2048, 1280] through the GEGLU FFN, W1 [10240,
    1280] (hidden | gate halves of 5120) and W2 [1280, 5120], prepared with
    prepare_weight.  Rows are independent, so 24 sampled rows are checked
    against the oracle: intermediate codes at a +-1 rate below 1e-4, output
    rel-L2 below 1e-2, rows with the oracle's codes bit-exact."""
    from xpu_kernels import int8
    m, k, inner = 2048, 1280, 5120
    g = torch.Generator().manual_seed(2)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    w1 = (torch.randn(2 * inner, k, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    w2 = (torch.randn(k, inner, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    up8, up_s = int8.prepare_weight(w1)
    dn8, dn_s = int8.prepare_weight(w2)
    y = int8.ffn(x, up8, up_s, dn8, dn_s, act="geglu_erf")
    rows = torch.randperm(m, generator=g)[:24].sort().values.numpy()
    ref = O.ffn(bits(x)[rows], bits(up8), bits(up_s), bits(dn8), bits(dn_s), None, 4)
    _check_ffn_rows(x, up8, up_s, dn8, dn_s, None, "geglu_erf", bits(y)[rows], rows, ref)
    # against the unquantized bf16 FFN (reported: the quantization error of the path)
    h, gt = (x.float() @ w1.float().t()).chunk(2, dim=-1)
    dense = (h * torch.nn.functional.gelu(gt)) @ w2.float().t()
    rel = (torch.linalg.norm(y.float() - dense) / torch.linalg.norm(dense)).item()
    print(f"C3 FFN vs the unquantized fp32 FFN: rel-L2 {rel:.3e}")
    assert rel < 5e-2


def test_full_size_backward_c4():
    """Config C4 at full size (x [4096, 1280], W [5120, 1280], dy [4096, 5120]
    ~ N(0, 1e-3)): linear_dx_int8 bit-exact on 24 sampled rows (rows are
    independent) and linear_dw_int8 bit-exact on 24 sampled output channels (the
    column quantizer scales each column of dy on its own, so a subset of dy's
    columns gives exactly those rows of dW).  The relative L2 error of both
    against the unquantized fp32 autograd of the linear is printed."""
    from xpu_kernels import int8
    m, k, n = 4096, 1280, 5120
    g = torch.Generator().manual_seed(3)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    dy = (torch.randn(m, n, generator=g) * 1e-3).to(torch.bfloat16).to(DEV)
    w8, ws = int8.prepare_weight(w)
    dx = int8.linear_dx_int8(dy, w8, ws)
    rows = torch.randperm(m, generator=g)[:24].sort().values.numpy()
    assert np.array_equal(bits(dx)[rows], O.linear_dx_int8(bits(dy)[rows], bits(w8), bits(ws)))
    xq, xs = int8.quantize(x)
    dw = int8.linear_dw_int8(dy, xq, xs)
    cols = torch.randperm(n, generator=g)[:24].sort().values.numpy()
    ref_dw = O.linear_dw_int8(bits(dy)[:, cols], bits(xq), bits(xs))
    assert np.array_equal(bits(dw)[cols], ref_dw)
    # the torch autograd of the unquantized linear y = x W^T
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    (xf @ wf.t()).backward(dy.float())
    rdx = (torch.linalg.norm(dx.float() - xf.grad) / torch.linalg.norm(xf.grad)).item()
    rdw = (torch.linalg.norm(dw.float() - wf.grad) / torch.linalg.norm(wf.grad)).item()
    print(f"\nC4 backward vs the unquantized fp32 autograd: dx rel-L2 {rdx:.3e}, "
          f"dW rel-L2 {rdw:.3e}")
    assert rdx < 5e-2 and rdw < 5e-2


@pytest.mark.parametrize("m,widths,k", [(1000, (1040, 1024), 1280), (77, (48, 32, 64), 512)])
def test_allgather_ragged_blocks_on_one_gpu(m, widths, k):
    """The all-gather linear with column blocks of unequal widths (the
    explicit-offset entry): each 'rank' stores its block at its own offset of
    every buffer; every buffer equals the linear of the whole weight."""
    import ctypes
    from xpu_kernels import int8
    from xpu_kernels.int8 import _lib as L
    lib = L.load()
    n = sum(widths)
    _, w8n, wsn = _prep(n, k, 190 + k)
    w8, ws = torch.from_numpy(w8n).to(DEV), torch.from_numpy(wsn).to(DEV)
    x = rand_bf16((m, k), 191 + m, outliers=4).to(DEV)
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(n)) * 0.01).to(DEV)
    full = int8.linear(x, w8, ws, bias)
    nr = len(widths)
    outs = [torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=DEV) for _ in range(nr)]
    table = (ctypes.c_void_p * nr)(*[o.data_ptr() for o in outs])
    xq = torch.empty(m, k, dtype=torch.int8, device=DEV)
    xs = torch.empty(m, dtype=torch.float32, device=DEV)
    c0 = 0
    for wdt in widths:
        sl = slice(c0, c0 + wdt)
        w8r, wsr, br = w8[sl].contiguous(), ws[sl].contiguous(), bias[sl].contiguous()
        rc = lib.xpuint8_linear_allgather_cols_stream(
            L._stream(torch.device(DEV)), L._ptr(x), L._ptr(w8r), L._ptr(wsr), L._ptr(br), table,
            nr, c0, n, L._ptr(xq), L._ptr(xs), m, wdt, k, 0)
        assert rc == 0, lib.xpuint8_last_error()
        c0 += wdt
    torch.cuda.synchronize()
    for o in outs:
        assert torch.equal(o.view(torch.int16), full.view(torch.int16))


@pytest.mark.parametrize("m,n,k,with_bias", [(2048, 1280, 1280, True), (333, 96, 512, False),
                                             (1, 64, 256, True)])
def test_split_projection_equals_acc_and_slices(m, n, k, with_bias):
    """The fused qkv projection (one GEMM over cat(Wq, Wk, Wv), each third
    dequantized straight into its own output) is bit-identical to the
    reference's pattern: linear_acc, then dequant_slice of each third
    (python/xpu_kernels/int8/selftest.py:67-72), and to a linear per part."""
    from xpu_kernels import int8
    x = rand_bf16((m, k), 200 + m, outliers=6).to(DEV)
    ws_parts, w8_parts = [], []
    for i in range(3):
        _, w8i, wsi = _prep(n, k, 201 + i)
        w8_parts.append(torch.from_numpy(w8i).to(DEV))
        ws_parts.append(torch.from_numpy(wsi).to(DEV))
    w8, ws = torch.cat(w8_parts), torch.cat(ws_parts)
    g = torch.Generator().manual_seed(n)
    bias = (torch.randn(3 * n, generator=g) * 0.01).to(DEV) if with_bias else None
    q, kk, v = int8.linear_split(x, w8, ws, bias, parts=3)
    acc, xs = int8.linear_acc(x, w8, ws)
    for i, got in enumerate((q, kk, v)):
        sl = slice(i * n, (i + 1) * n)
        ref = int8.dequant_slice(acc[:, sl], xs, ws[sl], None if bias is None else bias[sl])
        assert torch.equal(got.view(torch.int16), ref.view(torch.int16)), i
        one = int8.linear(x, w8_parts[i], ws_parts[i], None if bias is None else bias[sl])
        assert torch.equal(got.view(torch.int16), one.view(torch.int16)), i
    # and the oracle on a few rows
    rows = np.arange(0, m, max(1, m // 7))
    ref_all = O.linear(bits(x)[rows], bits(w8), bits(ws), None if bias is None else bits(bias))
    got_all = np.concatenate([bits(t)[rows] for t in (q, kk, v)], axis=1)
    assert np.array_equal(got_all, ref_all)


def test_split_projection_rejects_bad_parts():
    from xpu_kernels import int8
    x = rand_bf16((4, 256), 1).to(DEV)
    w8 = torch.zeros((3 * 48, 256), dtype=torch.int8, device=DEV)
    ws = torch.ones(3 * 48, device=DEV)
    with pytest.raises(ValueError):
        int8.linear_split(x, w8, ws, parts=3)      # 48 columns: not a multiple of 32
    with pytest.raises(ValueError):
        int8.linear_split(x, w8, ws, parts=5)      # 144 rows do not split in 5


# ------------------------------------------------------------------------ qkv consumer: RMS norm + rope

def _pe(B, S, D, seed, fb=None):
    g = torch.Generator().manual_seed(seed)
    ang = torch.rand(B if fb is None else fb, S, 1, D // 2, generator=g) * 3.0
    return torch.stack([torch.stack([ang.cos(), -ang.sin()], -1),
                        torch.stack([ang.sin(), ang.cos()], -1)], -2)


def _rope_close(got, ref, what):
    """Same arithmetic, summed in a different order: a few outputs may move by a
    bf16 ulp (the reference's own budget for that, triton/reference.py:45-53,
    is 1e-3 relative)."""
    ulps = np.abs(got.view(np.int16).astype(np.int32) - ref.view(np.int16).astype(np.int32))
    rel = rel_l2(got, ref)
    print(f"\n{what}: {int((ulps > 0).sum())} of {got.size} differ, max {ulps.max()} ulp, "
          f"rel-L2 {rel:.2e}")
    assert (ulps > 0).mean() < 1e-2 and rel < 1e-3


def test_rms_rope_dequant_matches_the_reference_fixture():
    """The int32-accumulator consumer on the q and k slices of a fused qkv
    accumulator (strided views, row stride 3*H*D) against the reference's torch
    chain run on CPU (tests/golden/reference_rope.npz); the bf16 form on the
    dequantized slices gives the same bits as the int32 form."""
    from xpu_kernels import int8
    import os
    R = np.load(os.path.join(os.path.dirname(__file__), "golden", "reference_rope.npz"))
    B, S, H, D = 1, 48, 3, 128
    acc = torch.from_numpy(R["acc"]).to(DEV)
    xs, ws = torch.from_numpy(R["xs"]).to(DEV), torch.from_numpy(R["ws"]).to(DEV)
    scale, pe = torch.from_numpy(R["scale"]).to(DEV), torch.from_numpy(R["pe"]).to(DEV)
    view = acc.view(B, S, 3 * H * D)
    q_acc = view[:, :, :H * D].unflatten(-1, (H, D))
    k_acc = view[:, :, H * D:2 * H * D].unflatten(-1, (H, D))
    q, k = int8.rms_rope_split_half_dequant(q_acc, k_acc, pe, ws[:H * D], ws[H * D:2 * H * D],
                                            xs.view(B, S), scale)
    for name, got in (("q", q), ("k", k)):
        _rope_close(bits(got), R[f"{name}_out"].reshape(B, S, H, D), f"rms_rope {name} vs reference")
        xb = dev_bf16(R[f"{name}_x"].reshape(B, S, H, D))
        assert torch.equal(int8.rms_rope(xb, pe, scale).view(torch.int16), got.view(torch.int16))


@pytest.mark.parametrize("B,S,H,D,split,fb", [(2, 33, 5, 64, True, None), (1, 100, 2, 256, True, 1),
                                             (3, 17, 4, 128, False, None), (2, 8, 1, 64, False, 1),
                                             (4, 512, 40, 128, True, None)])
def test_rms_rope_matches_the_oracle(B, S, H, D, split, fb):
    """Both rotations (split half, interleaved), D = 64 / 128 / 256, freqs per
    batch or broadcast, several batches: the int32 form against the oracle,
    and the bf16 form on the dequantized values equal to it."""
    from xpu_kernels import int8
    g = torch.Generator().manual_seed(B * 1000 + S + D)
    acc = torch.randint(-(2 ** 22), 2 ** 22, (B, S, H, D), generator=g, dtype=torch.int32)
    xs = torch.rand(B * S, generator=g) * 0.02 + 0.001
    ws = torch.rand(H * D, generator=g) * 0.02 + 0.001
    scale = torch.rand(D, generator=g) * 0.2 + 0.9
    pe = _pe(B, S, D, D + S, fb)
    got = int8.rms_rope_dequant(acc.to(DEV), pe.to(DEV), scale.to(DEV), xs.to(DEV), ws.to(DEV),
                                1e-6, split)
    ref = O.rms_rope(acc.numpy(), pe.numpy().reshape(pe.shape[0], S, D // 2, 2, 2), scale.numpy(),
                     1e-6, split, xs.numpy(), ws.numpy())
    _rope_close(bits(got), ref, f"rms_rope {B}x{S}x{H}x{D} split={split}")
    x = torch.from_numpy(O.f32_to_bf16_bits(O.round_bf16(
        (acc.numpy().astype(np.float32) * (ws.numpy().reshape(1, 1, H, D)
                                           * xs.numpy().reshape(B, S, 1, 1)).astype(np.float32))
        .astype(np.float32))).view(np.int16)).view(torch.bfloat16)
    same = int8.rms_rope(x.to(DEV), pe.to(DEV), scale.to(DEV), 1e-6, split)
    assert torch.equal(same.view(torch.int16), got.view(torch.int16))


def test_rms_rope_empty_rows():
    """No rows: an empty [B, 0, H, D] result and no launch (the reference's
    wrappers launch a (S, B) grid, empty here: triton/rope.py:360-376)."""
    from xpu_kernels import int8
    pe = _pe(1, 1, 128, 0).to(DEV)
    out = int8.rms_rope(torch.empty(1, 0, 4, 128, dtype=torch.bfloat16, device=DEV), pe[:, :0],
                        torch.ones(128, device=DEV))
    assert out.shape == (1, 0, 4, 128)


def test_split_projection_then_rms_rope_equals_the_accumulator_path():
    """The fused pipeline (linear_split writes bf16 q, k, v; rms_rope reads them)
    equals the reference's (linear_acc over cat(Wq, Wk, Wv), then the dequant
    consumer on the int32 q and k slices), bit for bit."""
    from xpu_kernels import int8
    B, S, H, D, K = 2, 64, 4, 128, 1024
    n = H * D
    x = rand_bf16((B * S, K), 330, outliers=4).to(DEV)
    w8s, wss = [], []
    for i in range(3):
        _, w8i, wsi = _prep(n, K, 331 + i)
        w8s.append(torch.from_numpy(w8i).to(DEV))
        wss.append(torch.from_numpy(wsi).to(DEV))
    w8, ws = torch.cat(w8s), torch.cat(wss)
    scale = (torch.rand(D, generator=torch.Generator().manual_seed(5)) * 0.2 + 0.9).to(DEV)
    pe = _pe(B, S, D, 6).to(DEV)
    q, k, v = int8.linear_split(x, w8, ws, None, parts=3)
    fused = int8.rms_rope_split_half(q.view(B, S, H, D), k.view(B, S, H, D), pe, scale)
    acc, xs = int8.linear_acc(x, w8, ws)
    a3 = acc.view(B, S, 3 * n)
    ref = int8.rms_rope_split_half_dequant(a3[:, :, :n].unflatten(-1, (H, D)),
                                           a3[:, :, n:2 * n].unflatten(-1, (H, D)), pe,
                                           ws[:n], ws[n:2 * n], xs.view(B, S), scale)
    for a, b in zip(fused, ref):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
