"""The reference's entropy-dispatched Llama block (EE/python/dispatch.py:150-259) on the
B200 kernels.

``EntropyDispatchedLlamaBlock`` keeps the reference's constructor, ``forward``
signature and outputs: the block's own attention module (transformers, eager, so it
returns the [B, H, S, S] probabilities) -> attention entropy (``attention_entropy``,
one HBM pass on the device instead of torch's log / mul / sum / mean chain) -> the
dispatcher -> gate / up / down as ``EntropyDispatchedLinear``.

``routing="batch"`` is the reference's granularity: one tier per block from the
batch max of the per-batch entropies (dispatch.py:64), read on the host.
``routing="token"`` routes every token by its own attention entropy (the mean over
heads of its query row) on the device: the MLP runs as gated GEMMs over per-token
buckets, with no host round trip; gate and up share one packing of their input and
one GEMM whose epilogue applies SiLU and the product (``SwiGLUPack``).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from .dispatch import EntropyDispatchedLinear, EntropyRouter, PipelinedEntropyDispatcher, PrecisionTier
from .kernels import (SwiGLUPack, _require, add_rmsnorm, attention_entropy, flash_attention_entropy,
                      flash_attention_rope_entropy, head_mean_entropy, linear_f16)


class EntropyDispatchedLlamaBlock(nn.Module):
    """EE/python/dispatch.py:150-247 with the sm_100a kernels."""

    def __init__(self, llama_block, layer_idx: int = 0, routing: str = "batch", attention: str = "eager",
                 route_all: bool = False, exact_entropy: bool = False, packs: Optional[dict] = None):
        super().__init__()
        _require(routing in ("batch", "token"), "routing must be 'batch' or 'token'")
        _require(attention in ("eager", "flash"), "attention must be 'eager' or 'flash'")
        _require(not route_all or attention == "flash", "route_all needs attention='flash'")
        self.layer_idx = layer_idx
        self.routing = routing
        self.attention = attention
        self.route_all = route_all
        # flash attention: route by the entropy of the fp16-rounded probabilities, as the
        # reference's eager block computes it (a second pass over the keys), or online
        self.exact_entropy = bool(exact_entropy)
        self.self_attn = llama_block.self_attn
        self.input_layernorm = llama_block.input_layernorm
        self.post_attention_layernorm = llama_block.post_attention_layernorm
        def routed(name, make_linear):
            # from a weight-pack file when it holds this linear (no quantisation at load)
            if packs is not None and name in packs:
                p = packs[name]
                p = p.to_weight_pack() if hasattr(p, "to_weight_pack") else p
                return EntropyDispatchedLinear.from_pack(p, scale_dtype=torch.float16)
            return EntropyDispatchedLinear.from_linear(make_linear())

        mlp = llama_block.mlp
        self.gate_proj = routed("gate_proj", lambda: mlp.gate_proj)
        self.up_proj = routed("up_proj", lambda: mlp.up_proj)
        self.down_proj = routed("down_proj", lambda: mlp.down_proj)
        self.act_fn = nn.SiLU()
        if route_all:
            # every linear of the block entropy-dispatched: q / k / v as one concatenated
            # projection (per-output-channel scales: concatenation changes nothing), o
            a = llama_block.self_attn
            self.qkv_proj = routed("qkv_proj", lambda: _concat_linears(a.q_proj, a.k_proj, a.v_proj))
            self.o_proj = routed("o_proj", lambda: a.o_proj)
        a = llama_block.self_attn
        self._qkv_split = (a.q_proj.out_features, a.k_proj.out_features, a.v_proj.out_features)
        self.layer_entropy: Optional[torch.Tensor] = None
        self.token_entropy: Optional[torch.Tensor] = None
        self._router: Optional[EntropyRouter] = None

    def forward(self, hidden_states: torch.Tensor, dispatcher: Optional[PipelinedEntropyDispatcher] = None,
                attention_mask: Optional[torch.Tensor] = None, position_ids: Optional[torch.Tensor] = None,
                past_key_value=None, use_cache: bool = False, **kwargs) -> Tuple[torch.Tensor, ...]:
        residual = hidden_states
        fused = self.attention == "flash" and hidden_states.dtype == torch.float16
        if fused:  # one pass instead of transformers' chain of fp32 ops
            hidden_states = add_rmsnorm(hidden_states, self.input_layernorm.weight,
                                        self.input_layernorm.variance_epsilon)
        else:
            hidden_states = self.input_layernorm(hidden_states)
        if self.route_all:
            kwargs["_dispatcher"] = dispatcher
        attn_output, entropy_batch, present_kv = self._attention_with_fused_entropy(
            hidden_states, attention_mask=attention_mask, position_ids=position_ids, past_key_value=past_key_value,
            use_cache=use_cache, **kwargs)
        self.layer_entropy = entropy_batch
        if dispatcher is not None and not (self.route_all and self.routing == "batch"):
            dispatcher.submit_entropy(entropy_batch)  # (route_all / batch submitted it before o)
        if dispatcher is not None and self.routing == "token":
            dispatcher._prev_token_entropy = self.token_entropy.reshape(-1)  # the next layer's q / k / v
        if fused:  # residual + attention output and the second norm in one pass
            hidden_states, residual = add_rmsnorm(attn_output, self.post_attention_layernorm.weight,
                                                  self.post_attention_layernorm.variance_epsilon, residual=residual)
        else:
            hidden_states = residual + attn_output
            residual = hidden_states
            hidden_states = self.post_attention_layernorm(hidden_states)
        if self.routing == "token" and dispatcher is not None:
            hidden_states = self._mlp_per_token(hidden_states, dispatcher)
        else:
            tier = dispatcher.get_tier() if dispatcher is not None else PrecisionTier.FP16
            gate = self.gate_proj(hidden_states, tier=tier)
            up = self.up_proj(hidden_states, tier=tier)
            hidden_states = self.down_proj(self.act_fn(gate) * up, tier=tier)
        hidden_states = residual + hidden_states

        outputs = (hidden_states,)
        if use_cache:
            outputs += (present_kv,)
        return outputs

    def swiglu_pack(self) -> Optional[SwiGLUPack]:
        """Gate and up packs interleaved for the fused SwiGLU GEMM (None when the
        intermediate size is not a multiple of 128)."""
        gp, up = self.gate_proj._pack(), self.up_proj._pack()
        if gp.N % 128 != 0:
            return None
        key = (id(gp), id(up))
        if getattr(self, "_gu_key", None) != key:
            self._gu, self._gu_key = SwiGLUPack(gp, up), key
        return self._gu

    def qkv_weight(self) -> torch.Tensor:
        """The attention's q / k / v weights concatenated by rows (fp16 [(Hq + 2 Hkv) d,
        hidden]): one GEMM for the three projections."""
        a = self.self_attn
        ws = (a.q_proj.weight, a.k_proj.weight, a.v_proj.weight)
        key = tuple((w.data_ptr(), w._version) for w in ws)
        if getattr(self, "_qkv_key", None) != key:
            self._qkv_w = torch.cat([w.detach().to(torch.float16) for w in ws], dim=0).contiguous()
            self._qkv_key = key
        return self._qkv_w

    def _mlp_per_token(self, x: torch.Tensor, dispatcher: PipelinedEntropyDispatcher) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.float16).contiguous()
        M = x2.shape[0]
        r = self._router_for(dispatcher, M, max(self.gate_proj.in_features, self.down_proj.in_features), x2.device)
        r.route_entropy(self.token_entropy.reshape(-1))
        r.pack_rows(x2)  # one packing of the post-norm rows serves gate and up
        gu = self.swiglu_pack()
        if gu is not None:
            h = r.swiglu_packed(gu)  # gate, up, SiLU and the product in one GEMM
        else:
            h = self.act_fn(r.gemm_packed(self.gate_proj._pack())) * r.gemm_packed(self.up_proj._pack())
        out = r.gated_linear(h, self.down_proj._pack())
        return out.reshape(shape[:-1] + (self.down_proj.out_features,))

    def _flash_attention(self, hidden_states: torch.Tensor, position_embeddings, dispatcher=None):
        """The attention module's projections and rotary embedding, then causal flash
        attention with the row entropies in one kernel (no [B, H, S, S] probabilities).
        With ``route_all`` the q / k / v projection runs in the precision of the previous
        layer's entropy (per token, or its batch tier) and o in this layer's."""
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

        attn = self.self_attn
        B, S, _ = hidden_states.shape
        d = attn.head_dim
        # the unrouted projections run on the library's fp16 GEMM (bias-free Llama linears)
        own_gemm = hidden_states.dtype == torch.float16 and all(
            getattr(attn, n).bias is None for n in ("q_proj", "k_proj", "v_proj", "o_proj"))
        if self.route_all:
            qkv = self._routed(hidden_states, self.qkv_proj, dispatcher, prev=True)
            q, k, v = qkv.split(self._qkv_split, dim=-1)
        elif own_gemm:  # q / k / v as one GEMM of the concatenated weights
            qkv = linear_f16(hidden_states.reshape(B * S, -1), self.qkv_weight()).reshape(B, S, -1)
            q, k, v = qkv.split(self._qkv_split, dim=-1)
        else:
            q, k, v = attn.q_proj(hidden_states), attn.k_proj(hidden_states), attn.v_proj(hidden_states)
        cos, sin = position_embeddings
        if q.dtype == torch.float16 and cos.dtype == torch.float16:
            # rotary embedding, head layout and V transpose in the attention's own launches
            Hkv = k.shape[-1] // d
            out, batch, rows, token = flash_attention_rope_entropy(q, k, v, cos, sin, q.shape[-1] // d, Hkv,
                                                                   causal=True, scale=attn.scaling, return_token=True,
                                                                   exact_entropy=self.exact_entropy)
        else:
            q = q.reshape(B, S, -1, d).transpose(1, 2)
            k = k.reshape(B, S, -1, d).transpose(1, 2)
            v = v.reshape(B, S, -1, d).transpose(1, 2)
            q, k = apply_rotary_pos_emb(q, k, cos, sin)
            out, batch, rows, token = flash_attention_entropy(q.half(), k.half(), v.half(), causal=True,
                                                              scale=attn.scaling, return_token=True)
        out = out.reshape(B, S, -1).to(hidden_states.dtype)
        self.token_entropy = token  # [B, S]: per query position, mean over heads
        if self.route_all:
            if self.routing == "batch" and dispatcher is not None:
                dispatcher.submit_entropy(batch)
            return self._routed(out, self.o_proj, dispatcher, prev=False), batch, rows
        if own_gemm:
            return linear_f16(out.reshape(B * S, -1), attn.o_proj.weight).reshape(B, S, -1), batch, rows
        return attn.o_proj(out), batch, rows

    def _routed(self, x: torch.Tensor, proj: "EntropyDispatchedLinear", dispatcher, prev: bool) -> torch.Tensor:
        """One linear of the attention in the precision the dispatcher chose: per token
        (``routing="token"``) from the previous layer's token entropies (prev) or this
        layer's; per batch from the dispatcher's current tier.  No entropy yet: FP16."""
        if self.routing == "batch" or dispatcher is None:
            first = prev and self.layer_idx == 0  # no earlier layer's entropy yet: FP16
            tier = dispatcher.get_tier() if dispatcher is not None and not first else PrecisionTier.FP16
            return proj(x, tier=tier)
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).to(torch.float16).contiguous()
        H = getattr(dispatcher, "_prev_token_entropy", None) if prev else self.token_entropy.reshape(-1)
        if H is None or H.numel() != x2.shape[0] or (prev and self.layer_idx == 0):  # the first layer: FP16
            H = torch.full((x2.shape[0],), float("inf"), device=x2.device)
        r = self._router_for(dispatcher, x2.shape[0], max(proj.in_features, self.down_proj.in_features), x2.device)
        r.route_entropy(H)
        return r.gated_linear(x2, proj._pack()).reshape(shape[:-1] + (proj.out_features,))

    def _router_for(self, dispatcher, M: int, K: int, device) -> EntropyRouter:
        r = self._router
        if r is None or r.tau_low != dispatcher.tau_low or r.tau_high != dispatcher.tau_high:
            r = self._router = EntropyRouter(dispatcher.tau_low, dispatcher.tau_high)
        r.reserve(M, K, device)
        return r

    def _attention_with_fused_entropy(self, hidden_states: torch.Tensor, attention_mask=None, position_ids=None,
                                      past_key_value=None, use_cache: bool = False, **kwargs):
        """EE/python/dispatch.py:212-247: the attention module with its probabilities
        returned, then their entropy (per batch, and per token for token routing).  With
        ``attention="flash"`` the probabilities never reach HBM: causal flash attention
        computes the output and every row's entropy in one pass (the explicit
        ``attention_mask`` is then taken to be the causal mask; no KV cache)."""
        if self.attention == "flash":
            _require(not use_cache and past_key_value is None, "flash attention here has no KV cache")
            pe = kwargs.get("position_embeddings")
            if pe is None:
                pe = self.self_attn.rotary_emb(hidden_states, position_ids)
            attn_output, entropy_batch, rows = self._flash_attention(hidden_states, pe, kwargs.get("_dispatcher"))
            return attn_output, entropy_batch, None
        attn_kwargs = dict(attention_mask=attention_mask, position_ids=position_ids, past_key_value=past_key_value,
                           output_attentions=True, use_cache=use_cache)
        attn_kwargs.update(kwargs)
        if "position_embeddings" not in attn_kwargs and hasattr(self.self_attn, "rotary_emb"):
            attn_kwargs["position_embeddings"] = self.self_attn.rotary_emb(hidden_states, position_ids)
        attn_outputs = self.self_attn(hidden_states, **attn_kwargs)
        attn_output = attn_outputs[0]
        attn_weights = attn_outputs[1]  # [B, H, S, S] post-softmax
        _require(attn_weights is not None, "the attention module returned no probabilities (use eager attention)")
        present_kv = attn_outputs[2] if use_cache and len(attn_outputs) > 2 else None
        entropy_batch, rows = attention_entropy(attn_weights, return_rows=True)
        if rows.dim() == 3:  # [B, S]: per query position, mean over heads
            self.token_entropy, _ = head_mean_entropy(rows)
        else:
            self.token_entropy = rows.mean(dim=1)
        return attn_output, entropy_batch, present_kv


def _concat_linears(*linears: nn.Linear) -> nn.Linear:
    out = nn.Linear(linears[0].in_features, sum(l.out_features for l in linears), bias=False)
    out = out.to(device=linears[0].weight.device, dtype=linears[0].weight.dtype)
    with torch.no_grad():
        out.weight.copy_(torch.cat([l.weight for l in linears], dim=0))
    return out


def build_dispatched_llama(model, tau_low: float, tau_high: float, routing: str = "batch",
                           attention: str = "eager", route_all: bool = False, exact_entropy: bool = False,
                           packs: Optional[dict] = None):
    """EE/python/dispatch.py:250-259: wraps every decoder layer of a transformers Llama
    model; returns (blocks, dispatcher).  ``route_all`` also dispatches q / k / v / o
    (with ``attention="flash"``).  ``packs`` (``packfile.load_packs`` of a file written by
    ``packfile.save_dispatched_llama``) supplies the routed linears' packs instead of
    quantising the model's weights."""
    device = next(model.parameters()).device
    blocks = []
    for i, layer in enumerate(model.model.layers):
        mine = None
        if packs is not None:
            pre = f"layers.{i}."
            mine = {k[len(pre):]: v for k, v in packs.items() if k.startswith(pre)}
        block = EntropyDispatchedLlamaBlock(layer, layer_idx=i, routing=routing, attention=attention,
                                            route_all=route_all, exact_entropy=exact_entropy, packs=mine)
        block = block.to(device).half()
        block.eval()
        blocks.append(block)
    dispatcher = PipelinedEntropyDispatcher(tau_low=tau_low, tau_high=tau_high)
    return blocks, dispatcher


@torch.no_grad()
def dispatched_forward(model, blocks, dispatcher, input_ids: torch.Tensor) -> torch.Tensor:
    """Logits of a transformers Llama model with its decoder layers replaced by
    ``blocks``: embedding -> fp16 -> rotary -> causal mask -> blocks -> norm -> lm_head,
    the forward of the reference's evaluation loop (EE/python/quality_eval.py:111-141)."""
    B, S = input_ids.shape
    device = input_ids.device
    hidden = model.model.embed_tokens(input_ids).to(torch.float16)
    position_ids = torch.arange(S, device=device).unsqueeze(0).expand(B, S)
    position_embeddings = model.model.rotary_emb(hidden, position_ids)
    causal_mask = torch.full((1, 1, S, S), torch.finfo(torch.float16).min, device=device, dtype=torch.float16)
    causal_mask = torch.triu(causal_mask, diagonal=1)
    for block in blocks:
        hidden = block(hidden, dispatcher=dispatcher, position_ids=position_ids,
                       position_embeddings=position_embeddings, attention_mask=causal_mask)[0]
    hidden = model.model.norm(hidden)
    return model.lm_head(hidden)


@torch.no_grad()
def eval_dispatched(model, blocks, dispatcher, chunks, device):
    """EE/python/quality_eval.py:111-152: perplexity of token chunks (each a list of ids,
    the last one the final target) through the dispatched blocks; returns (ppl, stats)."""
    import math

    total_loss, total_tokens = 0.0, 0
    dispatcher.reset_stats()
    for chunk in chunks:
        ids = torch.tensor([chunk[:-1]], device=device, dtype=torch.long)
        target = torch.tensor([chunk[1:]], device=device, dtype=torch.long)
        logits = dispatched_forward(model, blocks, dispatcher, ids)
        total_loss += torch.nn.functional.cross_entropy(logits.float().view(-1, logits.size(-1)), target.view(-1),
                                                        reduction="sum").item()
        total_tokens += target.numel()
    return math.exp(total_loss / total_tokens), dispatcher.get_stats()

