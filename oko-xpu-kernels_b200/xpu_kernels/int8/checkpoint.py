"""Prepared INT8 weights on disk: the ConvRot storage format, validated.

A layer prepared by :func:`xpu_kernels.prepare_weight` is an int8 ``[N, K]``
weight rotated along K by the group-256 Hadamard and quantized per output
channel, plus its fp32 scale (``[N]``, ``[N, 1]`` or a scalar, as the
reference's ``expand_scale`` accepts, python/xpu_kernels/int8/ops.py:380-408).
That pair is the format the reference documents as interchangeable with
ComfyUI's ``TensorWiseINT8Layout`` with ``convrot`` (python/xpu_kernels/int8/
__init__.py, "Weights must be prepared with prepare_weight (or an equivalent
... TensorWiseINT8Layout with convrot)"), so a checkpoint written by either
loads here unchanged.

A checkpoint is a ``torch.save`` dictionary: ``"<layer>.weight"`` (int8),
``"<layer>.weight_scale"`` (fp32), optionally ``"<layer>.bias"`` (any float
dtype, kept as fp32), and a ``"__xpu_int8__"`` entry ``{"format":
"convrot-int8", "group": 256, "version": 1}``.  Loading validates every layer
(:func:`validate_weight`) before anything reaches the GPU, so a malformed file
fails with the layer and the rule it breaks instead of a wrong result: a plain
``w / amax * 127`` quantization is indistinguishable by shape, which is why the
metadata entry is required unless ``require_meta=False``.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

FORMAT = {"format": "convrot-int8", "group": 256, "version": 1}
META_KEY = "__xpu_int8__"

__all__ = ["FORMAT", "META_KEY", "validate_weight", "save_int8_linear", "load_int8_linear",
           "prepare_state_dict"]

Layer = Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]


def validate_weight(w8: torch.Tensor, w_scale, name: str = "weight") -> None:
    """Raise ``ValueError`` naming ``name`` unless ``(w8, w_scale)`` is a prepared
    ConvRot INT8 weight the linear kernels accept: int8 ``[N, K]`` with
    ``K % 256 == 0`` and ``N % 16 == 0``, codes in ``[-127, 127]`` (the
    symmetric quantizers never produce -128), and an fp32 scale of ``N``
    elements (``[N]`` or ``[N, 1]``) or one element, finite and positive."""
    if not isinstance(w8, torch.Tensor) or w8.dtype != torch.int8:
        raise ValueError(f"{name}: the weight must be an int8 tensor, got "
                         f"{getattr(w8, 'dtype', type(w8).__name__)}")
    if w8.dim() != 2:
        raise ValueError(f"{name}: the weight must be [N, K], got shape {tuple(w8.shape)}")
    n, k = w8.shape
    if k % FORMAT["group"]:
        raise ValueError(f"{name}: K={k} is not a multiple of the ConvRot group size "
                         f"{FORMAT['group']}")
    if n % 16:
        raise ValueError(f"{name}: N={n} is not a multiple of 16")
    if w8.numel() and int(w8.min()) == -128:
        raise ValueError(f"{name}: the weight holds -128, which no ConvRot quantizer produces")
    s = torch.as_tensor(w_scale)
    if s.dtype != torch.float32:
        raise ValueError(f"{name}: the scale must be fp32, got {s.dtype}")
    if not (s.numel() == 1 or (s.numel() == n and (s.dim() == 1 or tuple(s.shape) == (n, 1)))):
        raise ValueError(f"{name}: the scale must be [N], [N, 1] or a scalar for N={n}, got "
                         f"shape {tuple(s.shape)}")
    if not bool(torch.isfinite(s).all()) or not bool((s > 0).all()):
        raise ValueError(f"{name}: the scale must be finite and positive")


def save_int8_linear(path, layers: Dict[str, Layer]) -> None:
    """Write prepared layers ``{name: (w8, w_scale, bias or None)}`` to ``path``
    (each validated first; tensors are saved from the CPU)."""
    sd = {META_KEY: dict(FORMAT)}
    for name, (w8, ws, bias) in layers.items():
        validate_weight(w8, ws, name)
        sd[f"{name}.weight"] = w8.detach().cpu().contiguous()
        sd[f"{name}.weight_scale"] = torch.as_tensor(ws).detach().float().cpu().contiguous()
        if bias is not None:
            sd[f"{name}.bias"] = bias.detach().float().cpu().contiguous()
    torch.save(sd, path)


def load_int8_linear(path, device=None, require_meta: bool = True) -> Dict[str, Layer]:
    """Read a checkpoint written by :func:`save_int8_linear` (or any state dict
    with the same keys) and return ``{name: (w8, w_scale, bias or None)}`` on
    ``device``, every layer validated.  ``require_meta=False`` accepts a file
    without the format entry (the caller vouches for the rotation)."""
    sd = torch.load(path, map_location="cpu", weights_only=True)
    meta = sd.get(META_KEY)
    if meta is None:
        if require_meta:
            raise ValueError(f"{path}: no {META_KEY!r} entry; not a ConvRot INT8 checkpoint "
                             "(pass require_meta=False to load it anyway)")
    elif meta.get("format") != FORMAT["format"] or meta.get("group") != FORMAT["group"]:
        raise ValueError(f"{path}: format {meta!r} is not {FORMAT!r}")
    layers: Dict[str, Layer] = {}
    for key in sd:
        if not key.endswith(".weight"):
            continue
        name = key[: -len(".weight")]
        if f"{name}.weight_scale" not in sd:
            raise ValueError(f"{path}: layer {name!r} has no weight_scale")
        w8, ws = sd[key], sd[f"{name}.weight_scale"]
        validate_weight(w8, ws, name)
        bias = sd.get(f"{name}.bias")
        layers[name] = (w8.to(device), ws.to(device),
                        None if bias is None else bias.float().to(device))
    return layers


def prepare_state_dict(state_dict: Dict[str, torch.Tensor], names=None,
                       device=None) -> Dict[str, Layer]:
    """Prepare the bf16/fp32 linear weights ``"<name>.weight"`` (``[N, K]``) of a
    state dict with :func:`xpu_kernels.prepare_weight` on ``device`` (a CUDA
    device); ``names`` restricts the layers.  Layers whose shape breaks the
    K % 256 / N % 16 rules are skipped, as a caller that falls back per layer
    would (``unsupported_reason``)."""
    from .ops import prepare_weight
    out: Dict[str, Layer] = {}
    for key, w in state_dict.items():
        if not key.endswith(".weight") or w.dim() != 2 or not w.is_floating_point():
            continue
        name = key[: -len(".weight")]
        if names is not None and name not in names:
            continue
        n, k = w.shape
        if k % FORMAT["group"] or n % 16:
            continue
        w8, ws = prepare_weight(w.to(device=device, dtype=torch.bfloat16))
        bias = state_dict.get(f"{name}.bias")
        out[name] = (w8, ws, None if bias is None else bias.float().to(device))
    return out
