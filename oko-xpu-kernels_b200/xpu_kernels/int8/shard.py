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
  the column blocks into the full ``[M, N]``.  Two forms:

  - :func:`linear_nshard_fused`: the GEMM's epilogue stores every output tile
    of this rank's block straight into every rank's ``[M, N]`` buffer
    (:class:`PeerOutput`, mapped across the processes with CUDA IPC) over
    NVLink, so the exchange overlaps the GEMM tile by tile and lands in
    row-major order; two one-element all-reduces on the stream order the
    ranks around it;
  - :func:`linear_nshard`: the GEMM, then an NCCL all-gather of the blocks
    (:func:`gather_columns`) and a strided copy into row-major ``[M, N]`` (the
    form that runs on any backend, e.g. gloo on CPU).
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch

__all__ = ["row_range", "col_range", "split_rows", "shard_weight", "linear_mshard",
           "gather_columns", "linear_nshard", "PeerOutput", "linear_nshard_fused"]


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


class _CudaBuffer:
    """A raw device allocation seen through ``__cuda_array_interface__`` (int16
    elements; viewed as bf16 by the caller)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape),
                                         "typestr": "<i2", "version": 3, "strides": None}


class PeerOutput:
    """The all-gathered output of :func:`linear_nshard_fused`: a bf16 buffer
    ``[m, n_total]`` on every rank of ``group``, mapped into every other rank's
    process (CUDA IPC), so that each rank's GEMM can store its column block into
    all of them.  Collective: every rank constructs it with the same shape, on
    its current CUDA device, and calls :meth:`close` when done.  ``tensor`` is
    this rank's buffer (valid until the next call that writes it)."""

    def __init__(self, m: int, n_total: int, group=None):
        import ctypes
        import torch.distributed as dist
        from ._lib import _lib

        self._lib = _lib()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the fused all-gather supports at most 8 ranks")
        self.m, self.n_total = int(m), int(n_total)
        self.device = torch.device("cuda", torch.cuda.current_device())
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        if self._lib.xpuint8_ipc_alloc(self.m * self.n_total * 2, ctypes.byref(ptr), handle) != 0:
            raise RuntimeError(f"PeerOutput: {self._lib.xpuint8_last_error()!r}")
        self._own = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            hb = (ctypes.c_char * 64).from_buffer_copy(h)
            if self._lib.xpuint8_ipc_open(hb, ctypes.byref(p)) != 0:
                raise RuntimeError(f"PeerOutput (rank {r}): {self._lib.xpuint8_last_error()!r}")
            self._opened.append(p.value)
            ptrs.append(p.value)
        self.table = (ctypes.c_void_p * self.world)(*ptrs)
        self.tensor = torch.as_tensor(_CudaBuffer(self._own, (self.m, self.n_total)),
                                      device=self.device).view(torch.bfloat16)

    def close(self):
        """Unmap the peers' buffers, wait for every rank to do the same, free this
        rank's buffer (collective)."""
        import ctypes
        import torch.distributed as dist
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self._lib.xpuint8_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        dist.barrier(group=self.group)
        self.tensor = None
        self._lib.xpuint8_ipc_free(ctypes.c_void_p(self._own))
        self._own = None


def _device_barrier(group, device):
    """Orders every rank's earlier work on its stream before every rank's later
    work (a one-element all-reduce on the current stream; no host wait)."""
    import torch.distributed as dist
    dist.all_reduce(torch.zeros(1, device=device), group=group)


def linear_nshard_fused(x, w8_local, w_scale_local, bias_local, out: PeerOutput):
    """The N-sharded INT8 linear with the all-gather fused into the GEMM: this
    rank quantizes the whole activation, multiplies it by its block of output
    channels and stores every output tile into all ranks' ``out`` buffers (the
    TMA unit over NVLink), at this rank's columns.  Returns ``out.tensor[:M]``,
    the full ``[M, N]`` output (rows of x beyond ``out.m`` are an error).

    Collective over ``out.group``: every rank calls it with its own weight block,
    the output channels ``col_range(N, P, rank)`` of :func:`shard_weight` (blocks
    of multiples of 16 columns, equal or not).  Before the GEMM the ranks wait
    for each other's readers of the previous output; after it, for each other's
    stores.
    """
    from . import ops
    from ._lib import _err, _lib, _ptr, _stream

    k = x.shape[-1]
    x2 = x.reshape(-1, k)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    m, n = x2.shape[0], w8_local.shape[0]
    reason = ops.unsupported_reason(x2, w8_local, w_scale_local)
    if reason is not None:
        raise TypeError(reason)
    c0, c1 = col_range(out.n_total, out.world, out.rank)
    if n != c1 - c0:
        raise ValueError(f"rank {out.rank} holds {n} output channels; its block of the "
                         f"output's {out.n_total} columns is [{c0}, {c1})")
    if m > out.m:
        raise ValueError(f"{m} rows do not fit the output's {out.m}")
    dev = x2.device
    lib = _lib()
    ws = ops.expand_scale(w_scale_local, n, dev)
    b = None if bias_local is None else ops.expand_scale(bias_local, n, dev)
    w8c = w8_local if w8_local.is_contiguous() else w8_local.contiguous()
    xq = torch.empty((m, k), dtype=torch.int8, device=dev)
    xs = torch.empty((m,), dtype=torch.float32, device=dev)
    _device_barrier(out.group, dev)
    rc = lib.xpuint8_linear_allgather_cols_stream(_stream(dev), _ptr(x2), _ptr(w8c), _ptr(ws),
                                                  _ptr(b), out.table, out.world, c0, out.n_total,
                                                  _ptr(xq), _ptr(xs), m, n, k, 0)
    if rc != 0:
        _err(lib, "linear_nshard_fused")
    _device_barrier(out.group, dev)
    return out.tensor[:m].reshape(*x.shape[:-1], out.n_total)
