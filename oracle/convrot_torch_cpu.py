"""The reference's own CPU path of the ConvRot INT8 linear, as torch CPU ops --
TEST AND BENCHMARK INFRASTRUCTURE ONLY.

``reference/convrot_linear.py:5-23`` (okolenmi/oko-xpu-kernels v0.4.0) is the
reference's plain-PyTorch ConvRot INT8 linear: a bf16 matmul of each 256-group
with the rotation matrix, a per-row abs-max scale ``max(amax/127, 1e-30)``,
``round(x_rot / scale)`` clamped to +-127, ``torch._int_mm`` against the
transposed int8 weight, ``bf16((acc * x_scale) * w_scale)`` and a bf16 bias
add.  As shipped it multiplies by ``torch.eye`` (its :10-12, with a comment
that a real implementation would use the normalized Hadamard);
``rotation="hadamard"`` puts that matrix in, which is the ConvRot path this
library implements.

This module restates that op sequence in torch (the same library calls, so the
same CPU kernels: oneDNN's bf16 matmul and int8 GEMM) for the benchmark's
reference arm and CPU baseline, where the reference tree itself is not
available.  ``tests/test_oracle.py`` pins it bit for bit to the fixture that
``tests/golden/make_golden.py`` produced by running the shipped file.  Only
``tests/`` and ``bench.py``'s CPU legs use it; the product path never does.
"""

from __future__ import annotations

import torch

GROUP = 256


def hadamard_bf16(group: int = GROUP) -> torch.Tensor:
    """The normalized rotation ``kron(H4, H4, H4, H4) / 16`` (entries +-1/16,
    exact in bf16), H4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]]
    (src/xpuint8.cpp:75)."""
    h4 = torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]],
                      dtype=torch.float64)
    h = h4
    while h.shape[0] < group:
        h = torch.kron(h, h4)
    return (h / torch.sqrt(torch.tensor(float(group)))).to(torch.bfloat16)


def convrot_int8_linear_cpu(x, w8, w_scale, bias=None, rotation: str = "hadamard",
                            h: torch.Tensor | None = None):
    """``reference/convrot_linear.py:5-23`` in torch on CPU.

    x bf16 [M, K] (K % 256 == 0); w8 int8 [N, K] (the prepared weight);
    w_scale fp32 [N]; bias bf16 [N] or None.  Returns bf16 [M, N].  ``h`` may
    pass a cached rotation matrix (bf16 [256, 256])."""
    m, k = x.shape
    if rotation == "identity":
        rot = torch.eye(GROUP, dtype=x.dtype)
    elif rotation == "hadamard":
        rot = hadamard_bf16() if h is None else h
    else:
        raise ValueError(rotation)
    # one bf16 matmul per 256-group (fp32 accumulation, bf16 result)
    xr = torch.matmul(x.reshape(m, k // GROUP, GROUP), rot).reshape(m, k)
    amax = xr.abs().amax(dim=-1, keepdim=True)
    xs = (amax.float() / 127.0).clamp(min=1e-30)
    xq = torch.round(xr.float() / xs).clamp(-127, 127).to(torch.int8)
    # the int8 GEMM against the transposed weight (the reference copies the
    # transpose on every call)
    acc = torch._int_mm(xq, w8.t().contiguous())
    y = ((acc.float() * xs) * w_scale.reshape(1, -1)).to(x.dtype)
    if bias is not None:
        y = y + bias
    return y
