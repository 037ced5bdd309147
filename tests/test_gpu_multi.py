"""Mode T on two GPUs over NCCL: the column-parallel gated MLP equals the same MLP on one
GPU bit for bit.  Skipped unless two GPUs are visible."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(m_total=512, d=1024, inter=2048, seed=5):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m_total, d, generator=g)
    x = torch.where(torch.rand(m_total, d, generator=g) < 0.01, x * 20.0, x).half()
    H = torch.rand(m_total, generator=g) * 2.5
    wg = (torch.randn(inter, d, generator=g) * 0.03).half()
    wu = (torch.randn(inter, d, generator=g) * 0.03).half()
    wd = (torch.randn(d, inter, generator=g) * 0.03).half()
    return x, H, wg, wu, wd


def _pkg():
    import sys

    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import __graft_entry__ as g

    return g.load_package()


def _worker(rank, world, port, out_path):
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    pkg = _pkg()
    from importlib import import_module

    sh = import_module(pkg.__name__ + ".sharding")
    x, H, wg, wu, wd = _inputs()
    m = x.shape[0] // world
    mlp = sh.ColumnParallelGatedMLP(wg.to(dev), wu.to(dev), wd.to(dev), world, rank)
    rows = slice(rank * m, (rank + 1) * m)
    y = mlp.forward(x[rows].to(dev), H[rows].to(dev))
    y_all = torch.empty(world * m, y.shape[1], dtype=y.dtype, device=dev)
    dist.all_gather_into_tensor(y_all, y.contiguous())
    torch.cuda.synchronize()
    if rank == 0:
        torch.save(y_all.cpu(), out_path)
    dist.barrier(device_ids=[rank])
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_mode_t_two_gpus_equals_one(pkg, cuda, tmp_path):
    out = str(tmp_path / "y.pt")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    got = torch.load(out)
    from importlib import import_module

    sh = import_module(pkg.__name__ + ".sharding")
    x, H, wg, wu, wd = _inputs()
    single = sh.ColumnParallelGatedMLP(wg.to(cuda), wu.to(cuda), wd.to(cuda), 1, 0)
    want = single.forward(x.to(cuda), H.to(cuda)).cpu()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
