"""The sharded INT8 linear on every visible GPU (2 to 8), bit for bit against one GPU.

Rows are independent, so the M-sharded result of each rank must equal the
single-GPU result on those rows exactly; the N-sharded all-gather (NCCL, and
the GEMM whose epilogue stores into the peers' buffers over NVLink) must
rebuild the single-GPU output exactly.  The tests use every visible GPU, up
to 8 ranks, and are skipped when fewer than two are visible.  NVLS is off (NCCL_NVLS_ENABLE=0) and the fused path uses plain peer
stores, no multicast.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(dev):
    import xpu_kernels
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(512, 1024, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(1024, 1024, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    w8, ws = xpu_kernels.prepare_weight(w)
    bias = torch.randn(1024, generator=g, device=dev) * 0.01
    return x, w8, ws, bias


def _worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    import xpu_kernels
    from xpu_kernels.int8 import shard
    x, w8, ws, bias = _problem(dev)
    full = xpu_kernels.linear(x, w8, ws, bias)
    a, b = shard.row_range(x.shape[0], world, rank)
    ym = shard.linear_mshard(shard.split_rows(x, world, rank), w8, ws, bias)
    w8l, wsl, bl = shard.shard_weight(w8, ws, world, rank, bias)
    yn = shard.linear_nshard(x, w8l, wsl, bl, n_total=w8.shape[0])
    torch.cuda.synchronize()
    ok_m = torch.equal(ym.view(torch.int16), full[a:b].view(torch.int16))
    ok_n = torch.equal(yn.view(torch.int16), full.view(torch.int16))
    with open(os.path.join(outdir, f"r{rank}.txt"), "w") as f:
        f.write(f"{int(ok_m)} {int(ok_n)}")
    dist.barrier()
    dist.destroy_process_group()


def _world():
    n = min(torch.cuda.device_count(), 8)
    if n < 2:
        pytest.skip("needs two GPUs")
    return n


def test_sharded_linear_on_all_gpus(tmp_path):
    world = _world()
    ctx = mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                             join=False, start_method="spawn")
    while not ctx.join(timeout=300):
        pass
    for r in range(world):
        assert (tmp_path / f"r{r}.txt").read_text() == "1 1"


def _fused_worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    import xpu_kernels
    from xpu_kernels.int8 import shard
    g = torch.Generator(device=dev).manual_seed(21)
    k = 1280
    oks = []
    # n = 2048 splits into equal blocks at 2, 4 and 8 ranks and into ragged ones
    # (e.g. 688/688/672) at 3, 5, 6 and 7; n = 2064 (129 blocks of 16) is ragged
    # at every rank count
    for n in (2048, 2064):
        w = (torch.randn(n, k, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        w8, ws = xpu_kernels.prepare_weight(w)
        bias = torch.randn(n, generator=g, device=dev) * 0.01
        w8l, wsl, bl = shard.shard_weight(w8, ws, world, rank, bias)
        out = shard.PeerOutput(1000, n)
        # two calls in a row (the second overwrites the first's output in every
        # rank's buffer), a ragged row count, then fewer rows than the buffer holds
        for m, seed in ((1000, 1), (1000, 2), (333, 3)):
            gx = torch.Generator(device=dev).manual_seed(seed)
            x = torch.randn(m, k, generator=gx, device=dev).to(torch.bfloat16)
            full = xpu_kernels.linear(x, w8, ws, bias)
            y = shard.linear_nshard_fused(x, w8l, wsl, bl, out)
            torch.cuda.synchronize()
            oks.append(int(torch.equal(y.view(torch.int16), full.view(torch.int16))))
        out.close()
    from xpu_kernels.int8 import _lib as L
    oks.append(int(L.load().xpuint8_fault_status(1) == 0))
    with open(os.path.join(outdir, f"f{rank}.txt"), "w") as f:
        f.write(" ".join(map(str, oks)))
    dist.barrier()
    dist.destroy_process_group()


def test_fused_allgather_linear_on_all_gpus(tmp_path):
    world = _world()
    ctx = mp.start_processes(_fused_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                             join=False, start_method="spawn")
    while not ctx.join(timeout=300):
        pass
    for r in range(world):
        assert (tmp_path / f"f{r}.txt").read_text() == "1 1 1 1 1 1 1"
