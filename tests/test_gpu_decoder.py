"""The decoder-stack engine (ee_decoder_*, DecoderEngine) against the Python layer loop
of EntropyDispatchedLlamaBlock(attention="flash") through the same kernels: the last
block's output bit for bit, eagerly and as a replayed CUDA graph, for per-token and
batch-max routing, MLP-only and every-linear routing, online and exact entropies.  A small random-init Llama
(transformers) with thresholds that put rows in all three tiers."""
import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu

TAU = (2.0, 4.0)  # causal rows of 256 keys: early positions INT8, middle FP8, late FP16


def _model(layers=2, hidden=256, heads=4, kv=2, inter=512, vocab=512, seed=0):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaModel

    torch.manual_seed(seed)
    cfg = LlamaConfig(hidden_size=hidden, num_hidden_layers=layers, num_attention_heads=heads, num_key_value_heads=kv,
                      intermediate_size=inter, vocab_size=vocab, rms_norm_eps=1e-5, rope_theta=10000.0,
                      max_position_embeddings=4096, attn_implementation="eager", initializer_range=0.02)
    model = LlamaModel(cfg).cuda().half().eval()
    wrap = nn.Module()
    wrap.model = model
    return wrap


@pytest.mark.parametrize("routing,route_all,exact", [("token", False, False), ("token", True, False),
                                                     ("batch", False, False), ("batch", True, False),
                                                     ("token", False, True), ("batch", True, True)])
@torch.no_grad()
def test_decoder_engine_equals_block_loop(pkg, cuda, routing, route_all, exact):
    wrap = _model()
    model = wrap.model
    blocks, disp = pkg.build_dispatched_llama(wrap, *TAU, routing=routing, attention="flash", route_all=route_all,
                                              exact_entropy=exact)
    B, S = 2, 256
    ids = torch.randint(0, 512, (B, S), generator=torch.Generator().manual_seed(3)).to(cuda)
    h0 = model.embed_tokens(ids).half()
    pos = torch.arange(S, device=cuda).unsqueeze(0).expand(B, S)
    pe = model.rotary_emb(h0, pos)
    h = h0
    for blk in blocks:
        h = blk(h, dispatcher=disp, position_ids=pos, position_embeddings=pe)[0]
    want_out = pkg.add_rmsnorm(h, model.norm.weight, model.norm.variance_epsilon)

    eng = pkg.DecoderEngine(blocks, model.norm.weight, pe, B, S, *TAU, routing=routing, route_all=route_all)
    eng.run(h0.reshape(B * S, -1).contiguous())  # eager
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert torch.equal(eng.residual.view(B, S, -1), h)
    assert torch.equal(eng.output.view(B, S, -1), want_out)
    counts = eng.layer_counts.cpu()
    assert (counts.sum(dim=1) == B * S).all()
    if routing == "token":
        assert (counts > 0).sum() >= 4, counts  # the thresholds split the rows
    else:
        assert ((counts > 0).sum(dim=1) == 1).all(), counts  # one tier per layer

    out = eng.forward(h0)  # one graph replay
    torch.cuda.synchronize()
    assert torch.equal(eng.residual.view(B, S, -1), h)
    assert torch.equal(out, want_out)
    x2 = (h0 * 0.5).contiguous()  # new input, same graph
    out2 = eng.forward(x2).clone()
    h2 = x2
    for blk in blocks:
        h2 = blk(h2, dispatcher=disp, position_ids=pos, position_embeddings=pe)[0]
    torch.cuda.synchronize()
    assert torch.equal(eng.residual.view(B, S, -1), h2)
    assert torch.equal(out2, pkg.add_rmsnorm(h2, model.norm.weight, model.norm.variance_epsilon))
    eng.close()


@torch.no_grad()
def test_head_mean_entropy_matches_torch(pkg, cuda):
    g = torch.Generator(device=cuda).manual_seed(5)
    rows = torch.rand(3, 32, 1000, generator=g, device=cuda) * 7.0
    token, batch = pkg.head_mean_entropy(rows)
    torch.testing.assert_close(token, rows.mean(dim=1), rtol=2e-6, atol=0)
    torch.testing.assert_close(batch, rows.mean(dim=(1, 2)), rtol=2e-6, atol=0)
    token2, _ = pkg.head_mean_entropy(rows)
    assert torch.equal(token, token2)  # one fixed summation order
    assert (token.double() - rows.double().sum(dim=1) / 32).abs().max().item() < 1e-5


@torch.no_grad()
def test_linear_f16_matches_torch(pkg, cuda):
    g = torch.Generator(device=cuda).manual_seed(6)
    x = torch.randn(300, 512, generator=g, device=cuda).half()
    w = (torch.randn(776, 512, generator=g, device=cuda) * 0.05).half()
    y = pkg.linear_f16(x, w)
    ref = (x.double() @ w.double().t())
    rel = ((y.double() - ref).norm() / ref.norm()).item()
    assert rel < 1e-3


@torch.no_grad()
def test_blocks_from_pack_file_equal_quantised_blocks(pkg, cuda, tmp_path):
    """A model whose routed linears come from a weight-pack file (no quantisation at load)
    computes the same forward as the one quantised from its weights, bit for bit."""
    wrap = _model()
    model = wrap.model
    blocks, disp = pkg.build_dispatched_llama(wrap, *TAU, routing="token", attention="flash", route_all=True)
    path = str(tmp_path / "model.eepack")
    pkg.packfile.save_dispatched_llama(blocks, path)
    packs = pkg.packfile.load_packs(path, device=cuda)
    assert len(packs) == 5 * len(blocks)
    blocks2, disp2 = pkg.build_dispatched_llama(wrap, *TAU, routing="token", attention="flash", route_all=True,
                                                packs=packs)
    B, S = 2, 256
    ids = torch.randint(0, 512, (B, S), generator=torch.Generator().manual_seed(4)).to(cuda)
    h0 = model.embed_tokens(ids).half()
    pos = torch.arange(S, device=cuda).unsqueeze(0).expand(B, S)
    pe = model.rotary_emb(h0, pos)
    h, h2 = h0, h0
    for b1, b2 in zip(blocks, blocks2):
        assert b2.gate_proj._pack().w_i8.data_ptr() == packs[f"layers.{b1.layer_idx}.gate_proj"].w_i8.data_ptr()
        h = b1(h, dispatcher=disp, position_ids=pos, position_embeddings=pe)[0]
        h2 = b2(h2, dispatcher=disp2, position_ids=pos, position_embeddings=pe)[0]
    torch.cuda.synchronize()
    assert torch.equal(h, h2)
