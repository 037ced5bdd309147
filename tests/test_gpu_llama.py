"""The Llama block surface (EE/python/dispatch.py:150-259) on the GPU, checked against
the CPU oracle: the attention module is the block's own (transformers, eager), so
everything after it is compared with the oracle's linears on the same inputs."""
import numpy as np
import pytest
import torch

from oracle import ee_oracle as orc

pytestmark = pytest.mark.gpu


def _relf(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


@pytest.fixture(scope="module")
def layer(cuda):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaDecoderLayer, LlamaRotaryEmbedding

    torch.manual_seed(7)
    cfg = LlamaConfig(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, intermediate_size=512,
                      num_hidden_layers=1, vocab_size=64, attn_implementation="eager")
    lay = LlamaDecoderLayer(cfg, layer_idx=0).to(cuda).half().eval()
    rope = LlamaRotaryEmbedding(cfg).to(cuda)
    B, S = 2, 64
    x = (torch.randn(B, S, 256, device=cuda) * 0.5).half()
    pos = torch.arange(S, device=cuda)[None].expand(B, S)
    pe = rope(x, pos)
    mask = torch.full((S, S), float("-inf"), device=cuda).triu(1)[None, None].half()
    return lay, x, pos, pe, mask


def _mlp_inputs(lay, x, pe, mask):
    """residual + attention, the post-norm rows and the attention probabilities, via
    the layer's own modules (what the block computes before its MLP)."""
    with torch.no_grad():
        h = lay.input_layernorm(x)
        attn_out, p = lay.self_attn(h, position_embeddings=pe, attention_mask=mask, output_attentions=True)[:2]
        mid = x + attn_out
        post = lay.post_attention_layernorm(mid)
    return mid, post, p


def _oracle_mlp(post, block, tiers, cuda):
    """gate / up / down through the oracle's per-tier linears; tiers: one per row."""
    x = post.reshape(-1, post.shape[-1]).cpu().numpy()

    def lin(a, proj):
        w_kn = proj.weight_int8.cpu().numpy()
        s_w = proj.weight_scale.cpu().numpy()
        out = np.zeros((a.shape[0], proj.out_features), dtype=np.float16)
        for t in (0, 1, 2):
            idx = np.nonzero(tiers == t)[0]
            if idx.size:
                out[idx] = orc.linear_by_tier(a[idx], w_kn, s_w, t)
        return out

    gate = torch.from_numpy(lin(x, block.gate_proj)).to(cuda)
    up = torch.from_numpy(lin(x, block.up_proj)).to(cuda)
    h = (torch.nn.functional.silu(gate) * up).cpu().numpy()  # the same torch ops the block runs
    return lin(h, block.down_proj)


def _capture(obj, name):
    """Wraps obj.name so the value it returns is recorded in the returned dict."""
    rec = {}
    real = getattr(obj, name)

    def wrapped(*a, **k):
        rec["out"] = real(*a, **k)
        return rec["out"]

    setattr(obj, name, wrapped)
    return rec


@pytest.mark.parametrize("taus,tier", [((100.0, 200.0), 0), ((-1.0, 100.0), 1), ((-2.0, -1.0), 2)])
def test_batch_routing_matches_oracle(pkg, cuda, layer, taus, tier):
    lay, x, pos, pe, mask = layer
    block = pkg.EntropyDispatchedLlamaBlock(lay).to(cuda)
    disp = pkg.PipelinedEntropyDispatcher(*taus)
    rec = _capture(block.down_proj, "forward")
    with torch.no_grad():
        out = block(x, dispatcher=disp, attention_mask=mask, position_ids=pos, position_embeddings=pe)[0]
    torch.cuda.synchronize()
    mid, post, p = _mlp_inputs(lay, x, pe, mask)
    want_batch, _ = orc.attention_entropy(p.cpu().numpy())
    np.testing.assert_allclose(block.layer_entropy.cpu().numpy(), want_batch, rtol=1e-4)
    assert orc.batch_max_tier(want_batch, *taus) == tier
    assert disp.get_stats()[["INT8", "FP8", "FP16"][tier]]["count"] == 1
    rows = x.shape[0] * x.shape[1]
    mlp = rec["out"].reshape(rows, -1)
    want = _oracle_mlp(post, block, np.full(rows, tier), cuda)
    if tier == 0:  # INT8: every linear bit-exact, so the MLP branch is too
        assert np.array_equal(mlp.cpu().numpy().view(np.uint16), want.view(np.uint16))
    else:
        assert _relf(mlp.cpu().numpy(), want) < 1e-2
    assert torch.equal(out, mid + rec["out"])  # the residual add of the reference block


def test_token_routing_matches_oracle(pkg, cuda, layer):
    lay, x, pos, pe, mask = layer
    mid, post, p = _mlp_inputs(lay, x, pe, mask)
    _, rows_h = orc.attention_entropy(p.cpu().numpy())
    tok = rows_h.mean(axis=1).reshape(-1)  # [B*S]: per query position, mean over heads
    lo, hi = (float(v) for v in np.quantile(tok, [0.3, 0.7]))  # a mix of all three tiers
    block = pkg.EntropyDispatchedLlamaBlock(lay, routing="token").to(cuda)
    disp = pkg.PipelinedEntropyDispatcher(lo, hi)
    rec = _capture(block, "_mlp_per_token")
    with torch.no_grad():
        out = block(x, dispatcher=disp, attention_mask=mask, position_ids=pos, position_embeddings=pe)[0]
    torch.cuda.synchronize()
    np.testing.assert_allclose(block.token_entropy.reshape(-1).cpu().numpy(), tok, rtol=1e-4, atol=1e-6)
    far = (np.abs(tok - lo) > 1e-5) & (np.abs(tok - hi) > 1e-5)
    tiers = orc.route(tok, lo, hi)
    assert set(np.unique(tiers[far]).tolist()) == {0, 1, 2}
    rows = tok.shape[0]
    got = rec["out"].reshape(rows, -1).cpu().numpy()
    want = _oracle_mlp(post, block, tiers, cuda)
    i8 = np.nonzero(far & (tiers == 0))[0]
    assert np.array_equal(got[i8].view(np.uint16), want[i8].view(np.uint16))
    for t in (1, 2):
        sel = np.nonzero(far & (tiers == t))[0]
        assert _relf(got[sel], want[sel]) < 1e-2
    assert torch.equal(out, mid + rec["out"])


def test_build_dispatched_llama(pkg, cuda):
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(3)
    cfg = LlamaConfig(hidden_size=128, num_attention_heads=4, num_key_value_heads=4, intermediate_size=256,
                      num_hidden_layers=2, vocab_size=64, attn_implementation="eager")
    model = LlamaForCausalLM(cfg).to(cuda).half().eval()
    blocks, disp = pkg.build_dispatched_llama(model, 0.41, 1.68)
    assert len(blocks) == 2 and isinstance(disp, pkg.PipelinedEntropyDispatcher)
    assert blocks[1].layer_idx == 1 and blocks[0].gate_proj.weight_int8.dtype == torch.int8


def test_dispatched_forward_tracks_the_model(pkg, cuda):
    """The whole model through the dispatched blocks (the reference's evaluation
    forward): with every layer in the FP16 tier the logits stay within the W8A16 weight
    quantisation error of the transformers model; the gated run gives finite perplexity
    and a small KL divergence from the all-FP16-tier run."""
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(5)
    cfg = LlamaConfig(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, intermediate_size=512,
                      num_hidden_layers=2, vocab_size=128, attn_implementation="eager")
    model = LlamaForCausalLM(cfg).to(cuda).half().eval()
    ids = torch.randint(0, 128, (2, 64), generator=torch.Generator().manual_seed(1)).to(cuda)
    with torch.no_grad():
        ref = model(ids).logits.float()
    blocks, disp = pkg.build_dispatched_llama(model, -1.0, -1.0)  # every layer in the FP16 tier
    fp16 = pkg.dispatched_forward(model, blocks, disp, ids).float()
    assert torch.isfinite(fp16).all()
    assert _relf(fp16.cpu().numpy(), ref.cpu().numpy()) < 5e-2
    assert disp.get_stats()["FP16"]["count"] == 2
    for routing in ("batch", "token"):
        blocks, disp = pkg.build_dispatched_llama(model, 0.41, 1.68, routing=routing)
        gated = pkg.dispatched_forward(model, blocks, disp, ids).float()
        lp, lq = torch.log_softmax(gated, -1), torch.log_softmax(fp16, -1)
        kl = float((lp.exp() * (lp - lq)).sum(-1).mean())
        assert 0.0 <= kl < 0.05
        ppl, stats = pkg.eval_dispatched(model, blocks, disp, [list(range(65)), list(range(3, 68))], cuda)
        assert np.isfinite(ppl) and ppl > 1.0
        # batch routing reads one tier per layer per chunk on the host; token routing none
        assert sum(v["count"] for v in stats.values()) == (4 if routing == "batch" else 0)


@pytest.mark.parametrize("routing", ["batch", "token"])
def test_flash_attention_block_tracks_eager(pkg, cuda, layer, routing):
    """attention="flash": the same block with the attention computed by the flash kernel
    (no probabilities in HBM) -- entropies and outputs track the eager block."""
    lay, x, pos, pe, mask = layer
    eager = pkg.EntropyDispatchedLlamaBlock(lay, routing=routing).to(cuda)
    flash = pkg.EntropyDispatchedLlamaBlock(lay, routing=routing, attention="flash").to(cuda)
    d1 = pkg.PipelinedEntropyDispatcher(-1.0, -1.0)  # every token in FP16: compares the attention paths
    d2 = pkg.PipelinedEntropyDispatcher(-1.0, -1.0)
    with torch.no_grad():
        out_e = eager(x, dispatcher=d1, attention_mask=mask, position_ids=pos, position_embeddings=pe)[0]
        out_f = flash(x, dispatcher=d2, attention_mask=mask, position_ids=pos, position_embeddings=pe)[0]
    torch.cuda.synchronize()
    np.testing.assert_allclose(flash.layer_entropy.cpu().numpy(), eager.layer_entropy.cpu().numpy(), rtol=2e-3)
    np.testing.assert_allclose(flash.token_entropy.cpu().numpy(), eager.token_entropy.cpu().numpy(), rtol=5e-3,
                               atol=5e-3)
    assert _relf(out_f.float().cpu().numpy(), out_e.float().cpu().numpy()) < 1e-2


@pytest.mark.parametrize("routing", ["batch", "token"])
def test_every_linear_routed(pkg, cuda, routing):
    """route_all: q / k / v / o dispatched too.  With every tier forced to FP16 the
    model tracks the transformers model within the W8A16 quantisation error; with the
    real thresholds the routed model's KL from the all-FP16 run stays small."""
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(11)
    cfg = LlamaConfig(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, intermediate_size=512,
                      num_hidden_layers=3, vocab_size=128, attn_implementation="eager")
    model = LlamaForCausalLM(cfg).to(cuda).half().eval()
    ids = torch.randint(0, 128, (2, 128), generator=torch.Generator().manual_seed(2)).to(cuda)
    with torch.no_grad():
        ref = model(ids).logits.float()
    blocks, disp = pkg.build_dispatched_llama(model, -1.0, -1.0, routing=routing, attention="flash", route_all=True)
    fp16 = pkg.dispatched_forward(model, blocks, disp, ids).float()
    assert torch.isfinite(fp16).all()
    assert _relf(fp16.cpu().numpy(), ref.cpu().numpy()) < 5e-2
    lo, hi = (0.41, 1.68) if routing == "batch" else tuple(
        float(v) for v in np.quantile(torch.cat([b.token_entropy.reshape(-1) for b in blocks]).cpu().numpy(),
                                      [0.3, 0.7]))
    blocks, disp = pkg.build_dispatched_llama(model, lo, hi, routing=routing, attention="flash", route_all=True)
    gated = pkg.dispatched_forward(model, blocks, disp, ids).float()
    lp, lq = torch.log_softmax(gated, -1), torch.log_softmax(fp16, -1)
    kl = float((lp.exp() * (lp - lq)).sum(-1).mean())
    assert 0.0 <= kl < 0.1

