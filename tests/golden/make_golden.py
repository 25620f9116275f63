"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run from the repository root in a container where the reference project is
mounted (``--reference`` points at its root; nothing else reads it)::

    python tests/golden/make_golden.py --reference <path-to-oko-xpu-kernels>

It imports the reference's own Python code (``python/xpu_kernels`` and
``reference/convrot_linear.py``), runs every part of the ConvRot INT8 path that
is plain torch on CPU, and stores inputs and outputs in ``reference_cpu.npz``.
The reference's device kernels (SYCL, ``src/xpuint8.cpp``) cannot run here;
where a reference chain calls one of them (``rotate``, ``dequant``) the oracle's
restatement is patched in, so the fixture pins the reference's *torch* part of
that chain (its bf16 rounding points, divisions and clamps) around it.

Arrays are stored as raw bit patterns: bf16 as uint16, fp32 as float32, int8 as
int8.  Seeds are fixed; re-running reproduces the file bit for bit on the same
torch version.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.contiguous().numpy().copy()


def _from_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of the reference project (read only)")
    ap.add_argument("--out", default=os.path.join(HERE, "reference_cpu.npz"))
    args = ap.parse_args()

    sys.path.insert(0, os.path.join(args.reference, "python"))
    sys.path.insert(0, os.path.join(args.reference, "reference"))
    sys.path.insert(0, ROOT)
    from xpu_kernels import int8 as ref            # the reference package
    from xpu_kernels.int8 import ops as ref_ops
    import convrot_linear                           # reference/convrot_linear.py
    from oracle import convrot_oracle as O

    torch.manual_seed(0)
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(1234)

    # 1. quantize_row_torch (ops.py:320-330) on seeded rows, a zero row, a
    #    ties row (tests/test_quantize.py:84-91) and a row with outliers.
    x = (torch.randn(32, 768, generator=g) * 0.4).to(torch.bfloat16)
    x[3] = 0
    x[5, :4] = torch.tensor([127.0, 254.0, -254.0, 63.0])
    x[5, 4:] = 0
    x[7, ::97] *= 50
    q, s = ref.quantize_row_torch(x)
    out["qrow_x"], out["qrow_q"], out["qrow_s"] = _bits(x), _bits(q), _bits(s)

    # 2. reference/convrot_linear.py:5-23 exactly as shipped (identity rotation)
    m, k, n = 64, 512, 256
    xl = torch.randn(m, k, generator=g)
    xl[:, torch.randperm(k, generator=g)[:8]] *= 20
    xl = xl.to(torch.bfloat16)
    wq = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    ws = (torch.rand(n, generator=g) * 0.01 + 1e-3).float()
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
    y = convrot_linear.convrot_int8_linear(xl, wq, ws, bias)
    out["cl_x"], out["cl_w8"], out["cl_ws"] = _bits(xl), _bits(wq), _bits(ws)
    out["cl_bias"], out["cl_out"] = _bits(bias), _bits(y)
    y0 = convrot_linear.convrot_int8_linear(xl, wq, ws, None)
    out["cl_out_nobias"] = _bits(y0)

    # 3. linear_dw (ops.py:207-238): a bf16 matmul dy^T @ x
    dy = (torch.randn(48, 64, generator=g) * 0.1).to(torch.bfloat16)
    xa = torch.randn(48, 256, generator=g).to(torch.bfloat16)
    out["dw_dy"], out["dw_x"], out["dw_out"] = _bits(dy), _bits(xa), _bits(ref.linear_dw(dy, xa))

    # The reference chains below call the device library for the rotation and
    # the dequant; the oracle's restatements stand in for those two calls.
    def rot(t):
        return _from_bits(O.rotate_bf16(_bits(t.to(torch.bfloat16)))).reshape(t.shape)

    def deq(acc, x_scale, w_scale, bias=None):
        a = acc.numpy()
        xs_ = ref.expand_scale(x_scale, a.shape[0], torch.device("cpu")).numpy()
        ws_ = ref.expand_scale(w_scale, a.shape[1], torch.device("cpu")).numpy()
        b = None if bias is None else ref.expand_scale(bias, a.shape[1], torch.device("cpu")).numpy()
        return _from_bits(O.dequant_epilogue(a, xs_, ws_, b))

    ref_ops.rotate = rot
    ref_ops.dequant = deq

    # 4. prepare_weight (ops.py:83-100): the torch chain around rotate()
    w = (torch.randn(64, 512, generator=g) * 0.02).to(torch.bfloat16)
    w[2] = 0
    q, sc = ref.prepare_weight(w)
    out["pw_w"], out["pw_q"], out["pw_s"] = _bits(w), _bits(q), _bits(sc)

    # 5. dequant_weight_torch (ops.py:169-191): bf16(w8 * s) then rotate()
    dwq = ref.dequant_weight_torch(q, sc)
    out["dq_w"] = _bits(dwq)

    # 6. linear_dx_int8 (ops.py:353-377): column scale in bf16, quantize_row
    #    (its torch chain on CPU), torch._int_mm, dequant, rotate()
    dyx = (torch.randn(40, 64, generator=g) * 1e-3).to(torch.bfloat16)
    dx = ref.linear_dx_int8(dyx, q, sc)
    out["dx_dy"], out["dx_out"] = _bits(dyx), _bits(dx)

    # 7. the erf GELU the fused activations are defined by: torch's F.gelu on
    #    every bf16 value (docs/performance.md:830-837 claims bit-identity of
    #    the SYCL erf-GELU with it); and the GEGLU product chain
    allb = torch.arange(0, 1 << 16, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    out["gelu_in"] = _bits(allb)
    out["gelu_out"] = _bits(torch.nn.functional.gelu(allb))
    out["gelu_tanh_out"] = _bits(torch.nn.functional.gelu(allb, approximate="tanh"))
    out["silu_out"] = _bits(torch.nn.functional.silu(allb))
    hid = torch.randn(16, 512, generator=g).to(torch.bfloat16)
    gat = torch.randn(16, 512, generator=g).to(torch.bfloat16)
    out["geglu_h"], out["geglu_g"] = _bits(hid), _bits(gat)
    out["geglu_y"] = _bits(hid * torch.nn.functional.gelu(gat))

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, torch {torch.__version__}")
    _rope_fixture(args.reference, os.path.join(os.path.dirname(args.out), "reference_rope.npz"))


def _rope_fixture(reference: str, path: str) -> None:
    """The consumer of the fused qkv accumulator: the reference's torch chain
    (python/xpu_kernels/triton/reference.py:63-98, ``rms_rope_split_half``)
    run on the bf16 dequant of an int32 accumulator slice, exactly as its
    probe builds the expected value (triton/rope.py:484-521)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "ref_triton_reference", os.path.join(reference, "python", "xpu_kernels", "triton", "reference.py"))
    tref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tref)
    g = torch.Generator().manual_seed(77)
    B, S, H, D = 1, 48, 3, 128
    M, C = B * S, 3 * H * D
    acc = torch.randint(-(2 ** 23), 2 ** 23, (M, C), generator=g, dtype=torch.int32)
    xs = torch.rand(M, generator=g) * 0.02 + 0.001
    ws = torch.rand(C, generator=g) * 0.02 + 0.001
    scale = torch.rand(D, generator=g) * 0.2 + 0.9
    ang = torch.rand(B, S, 1, D // 2, generator=g) * 3.0
    pe = torch.stack([torch.stack([ang.cos(), -ang.sin()], -1),
                      torch.stack([ang.sin(), ang.cos()], -1)], -2)
    out = {"acc": _bits(acc), "xs": _bits(xs), "ws": _bits(ws), "scale": _bits(scale),
           "pe": _bits(pe.contiguous())}
    for name, lo in (("q", 0), ("k", H * D)):
        x = (acc[:, lo:lo + H * D].to(torch.float32) * (ws[lo:lo + H * D] * xs[:, None])
             ).to(torch.bfloat16).view(B, S, H, D)
        out[f"{name}_x"] = _bits(x)
        out[f"{name}_out"] = _bits(tref.rms_rope_split_half(x, pe, scale, 1e-6))
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays")


if __name__ == "__main__":
    main()
