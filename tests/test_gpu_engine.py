"""The native launchers on the GPU: the CUDA-Graph gated layer loop reproduces the
per-call API bit for bit (same kernels, same routing), eagerly and replayed, and the
reference-compatible CubinEngine matches the INT8 GEMM (EE/csrc/engine.cpp:106-166)."""
import json
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layer_inputs(rows, n, dims, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    s = torch.exp(torch.rand(rows, 1, generator=g, device=dev) * (math.log(9.5) - math.log(7.0)) + math.log(7.0))
    logits = (torch.randn(rows, n, generator=g, device=dev) * s).half()
    acts = [torch.randn(rows, K, generator=g, device=dev).half() for K, _ in dims]
    return logits, acts


def test_graph_engine_matches_per_call_api(pkg, cuda):
    rows, n = 512, 1024
    dims = [(512, 768), (768, 512)]
    g = torch.Generator(device=cuda).manual_seed(3)
    packs = [pkg.WeightPack(*pkg.quantize_weights_int8((torch.randn(N, K, generator=g, device=cuda) * 0.02).half()))
             for K, N in dims]
    layers, want = [], []
    for li in range(3):
        logits, acts = _layer_inputs(rows, n, dims, 10 + li, cuda)
        ys = [torch.zeros(rows, N, dtype=torch.float16, device=cuda) for _, N in dims]
        layers.append((logits, [(a, p, y) for a, p, y in zip(acts, packs, ys)]))
        router = pkg.EntropyRouter(0.41, 1.68)
        router.reserve(rows, max(K for K, _ in dims), cuda)
        router.route(logits)
        want.append([router.gated_linear(a, p).clone() for a, p in zip(acts, packs)])
    eng = pkg.GatedLayerEngine(layers, 0.41, 1.68)
    eng.run()
    torch.cuda.synchronize()
    for (_, projs), w in zip(layers, want):
        for (_, _, y), yw in zip(projs, w):
            assert torch.equal(y.view(torch.int16), yw.view(torch.int16))
    for _, projs in layers:
        for _, _, y in projs:
            y.zero_()
    eng.capture()
    eng.launch()
    eng.launch()
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    for (_, projs), w in zip(layers, want):
        for (_, _, y), yw in zip(projs, w):
            assert torch.equal(y.view(torch.int16), yw.view(torch.int16))
    eng.close()


def test_cubin_engine_contract(pkg, cuda, tmp_path):
    meta = tmp_path / "gemm_int8_meta.json"
    meta.write_text(json.dumps({"shared": 36864, "num_warps": 8, "name": "gemm_int8_kernel", "BLOCK_M": 64,
                                "BLOCK_N": 128, "BLOCK_K": 64}))
    eng = pkg.CubinEngine.from_metadata(None, str(meta), "gemm_int8_kernel")
    g = torch.Generator().manual_seed(4)
    M, K, N = 256, 512, 384
    a = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    b = torch.randint(-127, 128, (K, N), generator=g, dtype=torch.int32).to(torch.int8).to(cuda)
    sa = (torch.rand(M, generator=g) * 0.01 + 1e-3).to(cuda)
    sb = (torch.rand(N, generator=g) * 0.01 + 1e-3).to(cuda)
    y = eng.forward(a, b, sa, sb)
    acc = (a.double() @ b.double()).round()
    ref = ((acc.float() * sa[:, None]) * sb[None, :]).half()
    torch.cuda.synchronize()
    assert y.dtype == torch.float16 and y.shape == (M, N)
    assert torch.equal(y.view(torch.int16), ref.view(torch.int16))
    with pytest.raises(RuntimeError, match="b must be int8"):
        eng.forward(a, b.float(), sa, sb)
    with pytest.raises(RuntimeError, match="K mismatch"):
        eng.forward(a, b[:-16], sa, sb)
    with pytest.raises(RuntimeError):
        pkg.CubinEngine(None, "gemm_fp8_kernel")
