"""Is a device-graph capture in progress?  (python/xpu_kernels/_capture.py)

Kept in its own module so it can be imported from anywhere without a cycle.
"""

from __future__ import annotations

import torch

__all__ = ["is_capturing"]


def is_capturing() -> bool:
    """True while a CUDA graph is being captured on the current stream.
    Never raises: no CUDA, or a backend that cannot answer, is "not capturing"."""
    probe = getattr(getattr(torch, "cuda", None), "is_current_stream_capturing", None)
    if probe is None:
        return False
    try:
        return bool(probe())
    except Exception:  # noqa: BLE001 - a backend that cannot answer is not capturing
        return False
