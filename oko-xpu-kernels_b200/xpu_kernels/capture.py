"""Capture readiness: what must be true before a step is captured in a CUDA graph
(the reference's python/xpu_kernels/capture.py, for the INT8 half).

Every INT8 kernel enqueues on torch's current stream with no host
synchronisation and allocates nothing, so a captured forward or backward
replays bit for bit.  The one thing that must not happen inside a capture is
the "dense" backward's weight dequantization: a full-precision copy of the
weight that would be re-computed on every replay.  ``prepare_for_capture``
materializes it beforehand; ``require_capture_ready`` checks; ``capture_status``
lists the problems without raising.  This build has no Triton kernels, so
``need`` names nothing: any name is refused as unknown.

All three must be called outside a capture.
"""

from __future__ import annotations

from typing import Iterable

from ._capture import is_capturing

__all__ = ["capture_status", "is_capturing", "prepare_for_capture", "require_capture_ready"]

_KERNELS: tuple = ()  # self-tested fused kernels a step may name (none in this build)


def _check_need(need):
    if need is None:
        return list(_KERNELS)
    wanted = list(need)
    unknown = [n for n in wanted if n not in _KERNELS]
    if unknown:
        raise ValueError(f"unknown kernel(s) {unknown!r}; this package has {sorted(_KERNELS)}")
    return wanted


def _int8_modules(model):
    from .int8 import Int8Linear
    if model is None:
        return []
    if isinstance(model, Int8Linear):
        return [(getattr(model, "_name", "int8_linear"), model)]
    return [(name, m) for name, m in model.named_modules() if isinstance(m, Int8Linear)]


def capture_status(need: Iterable[str] | None = None, model=None) -> list[str]:
    """Everything that would make a captured step wrong or wasteful; empty when ready."""
    _check_need(need)
    problems: list[str] = []
    for name, module in _int8_modules(model):
        if getattr(module, "backward", "dense") != "dense":
            continue
        if getattr(module, "_dense", None) is None:
            problems.append(
                f"{name}: the dense weight is not materialized -- the dequant "
                f"would be captured and re-run on every replay; call "
                f"prepare_for_capture(model) first")
    return problems


def require_capture_ready(need: Iterable[str] | None = None, model=None) -> None:
    """Raise ``RuntimeError`` unless the step is ready to be captured."""
    problems = capture_status(need=need, model=model)
    if problems:
        raise RuntimeError("not ready to capture a step:\n  " + "\n  ".join(problems))


def prepare_for_capture(model=None, need: Iterable[str] | None = None) -> dict:
    """Materialize the dense weight of every ``Int8Linear`` in "dense" backward
    mode, and report what was done.  Call it outside a capture."""
    wanted = _check_need(need)
    materialized = 0
    for _name, module in _int8_modules(model):
        if getattr(module, "backward", "dense") != "dense":
            continue
        module.dense_weight()
        materialized += 1
    return {"verified": wanted, "dense_weights": materialized,
            "problems": capture_status(need=wanted, model=model)}
