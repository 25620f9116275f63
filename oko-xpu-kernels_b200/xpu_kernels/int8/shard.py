"""Multi-GPU drivers for the INT8 linear (one process per GPU, torch.distributed).

The reference has no distributed code; rows of the INT8 linear are independent
(per-row activation scales, per-channel static weights), so the path shards in
two ways:

* **M-sharding** (the default; BASELINE config C5 "M-sharded with replicated
  weights"): rank r owns rows ``row_range(M, P, r)`` of the activation and a full
  copy of the weight, and runs :func:`xpu_kernels.linear` on its rows.  No data
  moves between GPUs; every row's result is bit-identical to a one-GPU run.
* **N-sharding** (config C5's variant for the large weight): rank r owns the
  weight rows ``col_range(N, P, r)`` (output columns) and the whole activation,
  computes ``y_r = linear(x, w8_r, ws_r)`` ([M, N/P]) and the ranks all-gather
  the column blocks into the full ``[M, N]`` (:func:`gather_columns`).  The
  gather is NCCL over NVLink; each rank's GEMM writes its block contiguously
  and the assembly into row-major ``[M, N]`` is one strided copy.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch

__all__ = ["row_range", "col_range", "split_rows", "shard_weight", "linear_mshard",
           "gather_columns", "linear_nshard"]


def _balanced(n: int, parts: int, index: int, align: int = 1) -> Tuple[int, int]:
    if parts <= 0 or not 0 <= index < parts:
        raise ValueError(f"index {index} is not in [0, {parts})")
    if n % align:
        raise ValueError(f"{n} is not a multiple of {align}")
    units = n // align
    base, extra = divmod(units, parts)
    start = index * base + min(index, extra)
    stop = start + base + (1 if index < extra else 0)
    return start * align, stop * align


def row_range(m: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows ``[start, stop)`` of an ``m``-row activation owned by ``rank`` (balanced)."""
    return _balanced(m, world, rank)


def col_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Output columns (weight rows) ``[start, stop)`` owned by ``rank``.  Blocks are
    multiples of 16 columns, the dequant epilogue's granularity, so ``n`` must be
    a multiple of 16 (the INT8 linear's N rule)."""
    return _balanced(n, world, rank, align=16)


def split_rows(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """This rank's rows of ``x`` (a view, no copy)."""
    a, b = row_range(x.shape[0], world, rank)
    return x[a:b]


def shard_weight(w8: torch.Tensor, w_scale: torch.Tensor, world: int, rank: int,
                 bias: Optional[torch.Tensor] = None):
    """This rank's block of output channels of a prepared weight: ``(w8[a:b], ws[a:b],
    bias[a:b] or None)``."""
    a, b = col_range(w8.shape[0], world, rank)
    ws = w_scale.reshape(-1)
    ws = ws[a:b] if ws.numel() == w8.shape[0] else ws
    return w8[a:b], ws, (None if bias is None else bias.reshape(-1)[a:b])


def linear_mshard(x_local, w8, w_scale, bias=None, linear: Optional[Callable] = None):
    """The M-sharded INT8 linear: this rank's rows against the replicated weight.
    No collective; the caller keeps its rows."""
    if linear is None:
        from .ops import linear as linear
    return linear(x_local, w8, w_scale, bias)


def gather_columns(y_local: torch.Tensor, n_total: int, group=None) -> torch.Tensor:
    """All-gather the column blocks ``y_r`` ([M, n_r], rank-ordered, balanced by
    :func:`col_range`) of every rank into the full ``[M, n_total]``.

    One ``all_gather_into_tensor`` into the rank-major ``[P, M, n]`` buffer
    (ragged blocks are padded to the widest and trimmed), then one strided copy
    into row-major ``[M, N]``.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    m = y_local.shape[0]
    widths = [b - a for a, b in (col_range(n_total, world, r) for r in range(world))]
    wmax = max(widths)
    y_local = y_local.contiguous()
    if y_local.shape[1] != wmax:
        pad = torch.zeros((m, wmax), dtype=y_local.dtype, device=y_local.device)
        pad[:, :y_local.shape[1]] = y_local
        y_local = pad
    # 2-byte elements travel as int32 pairs (blocks are multiples of 16
    # columns): a bit view that every backend can gather
    wire = y_local.view(torch.int32) if y_local.element_size() == 2 else y_local
    buf = torch.empty((world * m, wire.shape[1]), dtype=wire.dtype, device=wire.device)
    dist.all_gather_into_tensor(buf, wire, group=group)
    buf = buf.view(y_local.dtype).view(world, m, wmax)
    if len(set(widths)) == 1:
        return buf.permute(1, 0, 2).reshape(m, n_total)
    return torch.cat([buf[r, :, :w] for r, w in enumerate(widths)], dim=1)


def linear_nshard(x, w8_local, w_scale_local, bias_local=None, n_total: Optional[int] = None,
                  group=None, linear: Optional[Callable] = None):
    """The N-sharded INT8 linear: every rank multiplies the whole activation by its
    block of output channels and the blocks are all-gathered into ``[M, N]``."""
    import torch.distributed as dist
    if linear is None:
        from .ops import linear as linear
    if n_total is None:
        n_total = w8_local.shape[0] * dist.get_world_size(group)
    y = linear(x, w8_local, w_scale_local, bias_local)
    return gather_columns(y.reshape(-1, y.shape[-1]), n_total, group).reshape(
        *x.shape[:-1], n_total)
