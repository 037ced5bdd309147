"""Mode T on two GPUs over NCCL: the column-parallel gated MLP (in two pipelined row
chunks) equals the same MLP on one GPU bit for bit, and that one-GPU MLP agrees with the
CPU oracle's linears per tier; the mode-T decoder stack equals the decoder engine (mode
R) on each rank's sequences bit for bit.  Skipped unless two GPUs are visible."""
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
    mlp = sh.ColumnParallelGatedMLP(wg.to(dev), wu.to(dev), wd.to(dev), world, rank, chunks=2)
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
    # the one-GPU MLP against the oracle's linears: silu(gate) * up in fp16, then down,
    # every row in the tier of its entropy
    import numpy as np
    from oracle import ee_oracle as orc

    tiers = orc.route(H.numpy(), 0.41, 1.68)
    qg, qu, qd = (orc.quantize_weights_int8(w.numpy()) for w in (wg, wu, wd))
    for t in (0, 1, 2):
        idx = np.nonzero(tiers == t)[0]
        assert idx.size > 0
        xt = x.numpy()[idx]
        g = torch.from_numpy(orc.linear_by_tier(xt, *qg, t))
        u = torch.from_numpy(orc.linear_by_tier(xt, *qu, t))
        h = (torch.nn.functional.silu(g.float()).half() * u).numpy()
        ref = orc.linear_by_tier(h, *qd, t).astype(np.float64)
        diff = want.numpy()[idx].astype(np.float64) - ref
        assert np.linalg.norm(diff) / np.linalg.norm(ref) < 1e-2, t


def _worker_decoder(rank, world, port, out_path):
    import torch.distributed as dist
    import torch.nn as nn
    from datetime import timedelta
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaModel

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    pkg = _pkg()
    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=512, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
                      intermediate_size=1024, vocab_size=512, rms_norm_eps=1e-5, rope_theta=10000.0,
                      max_position_embeddings=4096, attn_implementation="eager", initializer_range=0.02)
    with torch.device(dev):
        model = LlamaModel(cfg)
    model = model.half().eval().requires_grad_(False)
    B, S = 2, 256  # per rank
    ids = torch.randint(0, 512, (world * B, S), generator=torch.Generator().manual_seed(3))[rank * B:(rank + 1) * B]
    eng = pkg.DecoderEngine.from_model(model, B, S, 2.0, 4.0, routing="token")
    h0 = model.embed_tokens(ids.to(dev)).half()
    eng.forward(h0)
    pos = torch.arange(S, device=dev).unsqueeze(0).expand(B, S)
    pe = model.rotary_emb(h0, pos)
    mt = pkg.sharding.ColumnParallelDecoder(eng.blocks, model.norm.weight, pe, world, rank, tau_low=2.0,
                                            tau_high=4.0, chunks=2)
    y, h_last = mt.forward(h0)
    torch.cuda.synchronize()
    ok = torch.equal(h_last.reshape(eng.residual.shape), eng.residual) and torch.equal(
        y.reshape(eng.output.shape), eng.output)
    mix = eng.layer_counts.sum(dim=0).cpu().tolist()
    flags = [None] * world
    dist.all_gather_object(flags, (ok, mix))
    if rank == 0:
        torch.save(flags, out_path)
    dist.barrier(device_ids=[rank])
    eng.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_mode_t_decoder_equals_engine_two_gpus(pkg, cuda, tmp_path):
    out = str(tmp_path / "flags.pt")
    mp.start_processes(_worker_decoder, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    flags = torch.load(out)
    assert all(ok for ok, _ in flags), flags
    assert all(sum(1 for c in mix if c > 0) >= 2 for _, mix in flags), flags  # rows in several tiers
