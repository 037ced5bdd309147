"""Multi-rank host logic on CPU (gloo, world size 2): row partitioning of the gated
path, gathering of the ranks' results, and host-side failure detection of a rank
that never reaches a step.  No GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ee_oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _sharding():
    import sys

    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import __graft_entry__ as g

    g.load_package()
    from importlib import import_module

    return import_module("tko_b200.sharding")


def test_row_shard_covers_rows_exactly():
    sh = _sharding()
    for total in (0, 1, 7, 4096, 4097):
        for world in (1, 2, 3, 8):
            spans = [sh.row_shard(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sh.row_shard(10, 2, 2)


def _worker_gated(rank, world, port, inp, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sh = _sharding()
    M = inp["A"].shape[0]
    a, b = sh.row_shard(M, world, rank)
    w_kn, w_s = orc.quantize_weights_int8(inp["W"])
    res = orc.gated_linear(inp["logits"][a:b], inp["A"][a:b], w_kn, w_s, 0.41, 1.68)
    y = torch.from_numpy(res["Y"].view(np.int16).astype(np.int32))  # gloo has no int16
    r = torch.from_numpy(res["route"].astype(np.int64))
    y_all = sh.gather_rows(y, world)
    r_all = sh.gather_rows(r, world)
    if rank == 0:
        np.savez(out_path, Y=y_all.numpy(), route=r_all.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_row_sharded_gated_linear_equals_single_rank(tmp_path):
    inp = orc.make_gating_inputs(M=37, n=256, K=128, N=64, seed=7)
    out = str(tmp_path / "gathered.npz")
    mp.start_processes(_worker_gated, args=(2, _free_port(), inp, out), nprocs=2, start_method="spawn")
    got = np.load(out)
    w_kn, w_s = orc.quantize_weights_int8(inp["W"])
    ref = orc.gated_linear(inp["logits"], inp["A"], w_kn, w_s, 0.41, 1.68)
    assert np.array_equal(got["route"], ref["route"].astype(np.int64))
    assert np.array_equal(got["Y"], ref["Y"].view(np.int16).astype(np.int32))


def _worker_liveness(rank, world, port, result_path):
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    sh = _sharding()
    store = dist.distributed_c10d._get_default_store()
    sh.check_peers(store, world, rank, "step0", timeout_s=5.0)  # everyone is alive
    if rank == 1:
        return  # this rank "dies" between steps: it never reaches step1
    try:
        sh.check_peers(store, world, rank, "step1", timeout_s=1.0)
        msg = "no error"
    except sh.PeerTimeout as exc:
        msg = str(exc)
    with open(result_path, "w") as f:
        f.write(msg)


def test_missing_rank_is_detected_on_the_host(tmp_path):
    out = str(tmp_path / "liveness.txt")
    mp.start_processes(_worker_liveness, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    msg = open(out).read()
    assert "ranks [1] did not reach 'step1'" in msg


class _OracleOps:
    """Mode T's device operations restated with the CPU oracle (per-row tiers)."""

    def __init__(self, tau_low, tau_high):
        self.tl, self.th = tau_low, tau_high

    @staticmethod
    def pack(weight):
        return orc.quantize_weights_int8(weight.numpy())

    def _lin(self, x, H, w):
        tiers = orc.route(H.numpy(), self.tl, self.th)
        xn = x.numpy()
        out = np.zeros((xn.shape[0], w[0].shape[1]), dtype=np.float16)
        for t in (0, 1, 2):
            idx = np.nonzero(tiers == t)[0]
            if idx.size:
                out[idx] = orc.linear_by_tier(xn[idx], w[0], w[1], t)
        return torch.from_numpy(out)

    @staticmethod
    def pack_swiglu(w_gate, w_up):
        return _OracleOps.pack(w_gate), _OracleOps.pack(w_up)

    def swiglu(self, x, H, gate_up):
        g, u = self._lin(x, H, gate_up[0]), self._lin(x, H, gate_up[1])
        return torch.nn.functional.silu(g.float()).half() * u

    def down(self, h, H, down):
        return self._lin(h, H, down)


def _mlp_inputs(m_total=24, d=64, inter=256, seed=11):
    rng = np.random.default_rng(seed)
    return {"x": orc.activations(m_total, d, rng, outliers=True),
            "H": rng.uniform(0.0, 2.5, size=m_total).astype(np.float32),
            "wg": (rng.standard_normal((inter, d)) * 0.05).astype(np.float16),
            "wu": (rng.standard_normal((inter, d)) * 0.05).astype(np.float16),
            "wd": (rng.standard_normal((d, inter)) * 0.05).astype(np.float16)}


def _worker_mode_t(rank, world, port, inp, out_path, chunks):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sh = _sharding()
    m = inp["x"].shape[0] // world
    mlp = sh.ColumnParallelGatedMLP(torch.from_numpy(inp["wg"]), torch.from_numpy(inp["wu"]),
                                    torch.from_numpy(inp["wd"]), world, rank, ops=_OracleOps(0.41, 1.68),
                                    chunks=chunks)
    assert mlp.cols[rank][1] - mlp.cols[rank][0] == inp["wg"].shape[0] // world
    rows = slice(rank * m, (rank + 1) * m)
    y = mlp.forward(torch.from_numpy(inp["x"][rows]), torch.from_numpy(inp["H"][rows]))
    y_all = sh.gather_rows(y.view(torch.int16).to(torch.int32), world)  # gloo has no int16
    if rank == 0:
        np.save(out_path, y_all.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("chunks", [1, 2])
def test_column_parallel_mlp_equals_single_rank(tmp_path, chunks):
    """Mode T (gate / up split by column, rows exchanged with an all-gather and an
    all-to-all, in one or two pipelined row chunks) gives the single-rank MLP bit for bit."""
    inp = _mlp_inputs()
    out = str(tmp_path / "mode_t.npy")
    mp.start_processes(_worker_mode_t, args=(2, _free_port(), inp, out, chunks), nprocs=2, start_method="spawn")
    sh = _sharding()
    single = sh.ColumnParallelGatedMLP(torch.from_numpy(inp["wg"]), torch.from_numpy(inp["wu"]),
                                       torch.from_numpy(inp["wd"]), 1, 0, ops=_OracleOps(0.41, 1.68))
    want = single.forward(torch.from_numpy(inp["x"]), torch.from_numpy(inp["H"]))
    got = np.load(out)
    assert np.array_equal(got, want.view(torch.int16).to(torch.int32).numpy())
    tiers = orc.route(inp["H"], 0.41, 1.68)
    assert set(np.unique(tiers).tolist()) == {0, 1, 2}


def test_column_shard_groups():
    sh = _sharding()
    spans = [sh.column_shard(14336, 8, r) for r in range(8)]
    assert spans[0] == (0, 1792) and spans[-1] == (12544, 14336)
    assert all(a % 128 == 0 and b % 128 == 0 for a, b in spans)
    with pytest.raises(ValueError):
        sh.column_shard(100, 2, 0)

