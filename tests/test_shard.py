"""The multi-GPU drivers' host logic, on CPU with two gloo ranks.

The per-rank compute is the CPU oracle (the CUDA kernels need a GPU); what is
tested is the sharding arithmetic and the collective plumbing of
``xpu_kernels.int8.shard``: M-sharded results concatenate to the single-process
result bit for bit, N-sharded column blocks all-gather into it bit for bit
(equal and ragged blocks), and a rank that dies before the collective makes the
others fail with an error instead of waiting forever.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import convrot_oracle as O
from xpu_kernels.int8 import shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _problem(m=96, k=512, n=272, seed=7):
    rng = np.random.default_rng(seed)
    x = O.f32_to_bf16_bits(rng.standard_normal((m, k)).astype(np.float32))
    w = O.round_bf16((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
    w8, ws = O.prepare_weight(w)
    bias = (rng.standard_normal(n) * 0.01).astype(np.float32)
    return x, w8, ws, bias


def _oracle_linear(x, w8, ws, bias):
    """CPU stand-in for xpu_kernels.linear: torch tensors in, bf16 bits out."""
    xb = x.numpy() if x.dtype == torch.int16 else x.numpy()
    y = O.linear(xb.view(np.uint16), w8.numpy(), ws.numpy(), None if bias is None else bias.numpy())
    return torch.from_numpy(y.view(np.int16).copy())


def _run(fn, world, *args):
    port = _free_port()
    ctx = mp.start_processes(fn, args=(world, port) + args, nprocs=world, join=False,
                             start_method="spawn")
    ok = ctx.join(timeout=120)
    while not ok:
        ok = ctx.join(timeout=120)


def _mshard_worker(rank, world, port, outdir):
    _init(rank, world, port)
    x, w8, ws, bias = _problem()
    xl = shard.split_rows(torch.from_numpy(x.view(np.int16)), world, rank)
    y = shard.linear_mshard(xl, torch.from_numpy(w8), torch.from_numpy(ws), torch.from_numpy(bias),
                            linear=_oracle_linear)
    np.save(os.path.join(outdir, f"m{rank}.npy"), y.numpy())
    dist.barrier()
    dist.destroy_process_group()


def _nshard_worker(rank, world, port, outdir, n):
    _init(rank, world, port)
    x, w8, ws, bias = _problem(n=n)
    w8l, wsl, bl = shard.shard_weight(torch.from_numpy(w8), torch.from_numpy(ws), world, rank,
                                      torch.from_numpy(bias))
    y = shard.linear_nshard(torch.from_numpy(x.view(np.int16)), w8l, wsl, bl, n_total=n,
                            linear=_oracle_linear)
    np.save(os.path.join(outdir, f"n{rank}.npy"), y.numpy())
    dist.destroy_process_group()


def _dying_worker(rank, world, port, outdir):
    _init(rank, world, port, timeout_s=10)
    if rank == 1:
        os._exit(3)  # leaves between steps, with nothing in flight
    y = torch.zeros(4, 16, dtype=torch.int16)
    try:
        shard.gather_columns(y, 32)
        result = "returned"
    except Exception as exc:  # noqa: BLE001 - any error is the expected outcome
        result = f"error: {type(exc).__name__}"
    with open(os.path.join(outdir, "dying.txt"), "w") as f:
        f.write(result)
    os._exit(0)


def test_ranges_cover_and_balance():
    for m, world in ((96, 2), (97, 4), (65536, 8), (3, 8)):
        spans = [shard.row_range(m, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == m
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        sizes = [b - a for a, b in spans]
        assert max(sizes) - min(sizes) <= 1
    spans = [shard.col_range(14336, 8, r) for r in range(8)]
    assert [b - a for a, b in spans] == [1792] * 8
    spans = [shard.col_range(272, 2, r) for r in range(2)]
    assert spans == [(0, 144), (144, 272)]
    with pytest.raises(ValueError):
        shard.col_range(40, 2, 0)


def test_mshard_concatenates_to_the_single_process_result(tmp_path):
    world = 2
    _run(_mshard_worker, world, str(tmp_path))
    got = np.concatenate([np.load(tmp_path / f"m{r}.npy") for r in range(world)])
    x, w8, ws, bias = _problem()
    assert np.array_equal(got.view(np.uint16), O.linear(x, w8, ws, bias))


@pytest.mark.parametrize("n", [256, 272])  # equal blocks (128+128), ragged (144+128)
def test_nshard_gathers_to_the_single_process_result(tmp_path, n):
    world = 2
    _run(_nshard_worker, world, str(tmp_path), n)
    x, w8, ws, bias = _problem(n=n)
    ref = O.linear(x, w8, ws, bias)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"n{r}.npy").view(np.uint16), ref)


def test_a_dead_rank_makes_the_collective_fail_not_hang(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_dying_worker, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=90)
    assert all(not p.is_alive() for p in ctx.processes)
    assert (tmp_path / "dying.txt").read_text().startswith("error")
