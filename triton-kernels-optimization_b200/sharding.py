"""Row partitioning of the gated path across the GPUs of one node (mode R), and the
column-parallel gated MLP (mode T).

Every quantity on the path is row-local -- per-row entropy, route and activation
scales (EE/python/kernels.py:272, :336, :361) -- and the weight scales are per output
column (EE/python/dispatch.py:45-46), so splitting the rows across ranks with a full
weight replica on each changes no result: the concatenation of the ranks' outputs is
the single-GPU output, bit for bit.  No collective runs inside a step; the helpers
below are for placing rows and for collecting results afterwards.
"""
from __future__ import annotations

import time
from datetime import timedelta

import torch
import torch.distributed as dist


def row_shard(total_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced [start, stop) of ``total_rows`` for ``rank`` of ``world``
    (the first ``total_rows % world`` ranks take one extra row)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(int(total_rows), world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_rows(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather row blocks of possibly different lengths, concatenated in rank order."""
    if world == 1:
        return local
    n = torch.tensor([local.shape[0]], dtype=torch.int64, device=local.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    pad = max(sizes)
    buf = local.new_zeros((pad,) + tuple(local.shape[1:]))
    buf[: local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], dim=0)


def column_shard(total_cols: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """Contiguous [start, stop) of ``total_cols`` output columns for ``rank``, in whole
    ``align``-column groups (the GEMM's N granularity); the first ranks take the extra
    groups."""
    if total_cols % align:
        raise ValueError(f"{total_cols} columns are not a multiple of {align}")
    a, b = row_shard(total_cols // align, world, rank)
    return a * align, b * align


def exchange_blocks(send: list, recv: list, rank: int, group=None, async_op: bool = False):
    """All-to-all of one block per rank pair: ``send[s]`` goes to rank s and
    ``recv[s]`` receives rank s's block for this rank.  Grouped point-to-point
    transfers (one NCCL group on GPUs; gloo, which has no all-to-all, runs the same
    code on CPU).  With ``async_op`` the requests are returned instead of waited for
    (on NCCL, waiting makes the current stream wait, not the host)."""
    ops = []
    for peer in range(len(send)):
        if peer == rank:
            recv[peer].copy_(send[peer])
            continue
        gpeer = dist.get_global_rank(group, peer) if group is not None else peer
        ops.append(dist.P2POp(dist.isend, send[peer], gpeer, group))
        ops.append(dist.P2POp(dist.irecv, recv[peer], gpeer, group))
    reqs = dist.batch_isend_irecv(ops) if ops else []
    if async_op:
        return reqs
    for req in reqs:
        req.wait()
    return []


class GatedMLPOps:
    """The device operations mode T needs, on the sm_100a kernels: routing from given
    entropies, the fused SwiGLU GEMM over the gate / up column block and the bucketed
    down GEMM.  The routers keep every tile whole (no K split), so a row's result does
    not depend on how many rows share its call: mode T equals one GPU bit for bit."""

    def __init__(self, tau_low: float, tau_high: float):
        from .dispatch import EntropyRouter

        self._all = EntropyRouter(tau_low, tau_high, k_split=False)
        self._local = EntropyRouter(tau_low, tau_high, k_split=False)

    @staticmethod
    def pack(weight: torch.Tensor):
        from .kernels import WeightPack

        return WeightPack.from_weight(weight)

    @staticmethod
    def pack_swiglu(w_gate: torch.Tensor, w_up: torch.Tensor):
        from .kernels import SwiGLUPack, WeightPack

        return SwiGLUPack(WeightPack.from_weight(w_gate), WeightPack.from_weight(w_up))

    def swiglu(self, x: torch.Tensor, H: torch.Tensor, gate_up):
        """fp16(fp16(silu(x gate^T)) * (x up^T)) for this rank's columns, one GEMM."""
        r = self._all
        r.reserve(x.shape[0], x.shape[1], x.device)
        r.route_entropy(H)
        r.pack_rows(x)
        return r.swiglu_packed(gate_up)

    def down(self, h: torch.Tensor, H: torch.Tensor, down):
        r = self._local
        r.reserve(h.shape[0], h.shape[1], h.device)
        r.route_entropy(H)
        return r.gated_linear(h, down)


class ColumnParallelGatedMLP:
    """Mode T of the gated SwiGLU MLP: ``down(silu(gate(x)) * up(x))`` with gate and up
    split by output column across the ranks and the rows of x split by row.

    Per call, for the ``m`` rows a rank owns (equal on every rank), in ``chunks`` row
    chunks pipelined against each other:
      1. all-gather the chunk's rows x [m / chunks, d] from every rank and their
         entropies H (all chunks' gathers are issued up front and run on the
         collective stream while earlier chunks compute);
      2. route the gathered rows (every rank derives the same routes from the same H)
         and run this rank's gate / up columns over them in one fused SwiGLU GEMM
         -> h [world * m / chunks, I / world];
      3. all-to-all (NCCL's, or grouped point-to-point transfers on gloo): the row block
         of every other rank goes to it and this rank's rows come back from every rank ->
         [m / chunks, I] (columns in rank order), issued as soon as the chunk's h exists,
         so it overlaps the next chunk's GEMM;
      4. the down projection (full weight) on the rank's own rows of the chunk.
    Per-row activation scales span the whole row (steps 2 and 4 see full rows), weight
    scales are per output column and no tile's K loop is split, so the result equals
    the single-GPU MLP bit for bit.  The collectives are the layer-boundary exchange of
    this mode (NCCL over NVLink on GPUs).
    """

    def __init__(self, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, world: int, rank: int,
                 ops=None, group=None, tau_low: float = 0.41, tau_high: float = 1.68, chunks: int = 1):
        inter = w_gate.shape[0]
        if w_up.shape[0] != inter or w_down.shape[1] != inter:
            raise ValueError("gate / up must be [I, d] and down [d, I]")
        self.world, self.rank, self.group = world, rank, group
        self.chunks = max(1, int(chunks))
        self.ops = ops if ops is not None else GatedMLPOps(tau_low, tau_high)
        self.cols = [column_shard(inter, world, r) for r in range(world)]
        c0, c1 = self.cols[rank]
        self.gate_up = self.ops.pack_swiglu(w_gate[c0:c1], w_up[c0:c1])
        self.down_w = self.ops.pack(w_down)
        self._set_exchange()

    def _set_exchange(self) -> None:
        # NCCL has a native all-to-all (equal column blocks); gloo exchanges by grouped
        # point-to-point transfers
        self._nccl = self.world > 1 and dist.is_initialized() and dist.get_backend(self.group) == "nccl"
        self._equal_cols = len({c1 - c0 for c0, c1 in self.cols}) == 1

    @classmethod
    def from_blocks_mlp(cls, block, world: int, rank: int, group=None, tau_low: float = 0.41,
                        tau_high: float = 1.68, chunks: int = 1) -> "ColumnParallelGatedMLP":
        """Mode T over the already quantised MLP of an EntropyDispatchedLlamaBlock: this
        rank's gate / up columns are slices of the block's int8 [K, N] weights and their
        scales (per output column), so the packs equal those of the whole block."""
        from .kernels import SwiGLUPack, WeightPack

        self = cls.__new__(cls)
        self.world, self.rank, self.group = world, rank, group
        self.chunks = max(1, int(chunks))
        self.ops = GatedMLPOps(tau_low, tau_high)
        inter = block.gate_proj.out_features
        self.cols = [column_shard(inter, world, r) for r in range(world)]
        c0, c1 = self.cols[rank]

        def sliced(lin):
            return WeightPack(lin.weight_int8[:, c0:c1].contiguous(), lin.weight_scale[c0:c1].float())

        self.gate_up = SwiGLUPack(sliced(block.gate_proj), sliced(block.up_proj))
        self.down_w = block.down_proj._pack()
        self._set_exchange()
        return self

    def forward(self, x: torch.Tensor, H: torch.Tensor) -> torch.Tensor:
        m, d = x.shape
        world, C = self.world, self.chunks
        if m % C:
            raise ValueError(f"{m} rows do not split into {C} chunks")
        mc = m // C
        x, H = x.contiguous(), H.contiguous()
        xs, Hs, gathers = [], [], []
        for c in range(C):  # every chunk's gather up front: they run while earlier chunks compute
            x_all = x.new_empty((world * mc, d))
            H_all = H.new_empty((world * mc,))
            xc, Hc = x[c * mc:(c + 1) * mc], H[c * mc:(c + 1) * mc]
            if world > 1:
                gathers.append((dist.all_gather_into_tensor(x_all, xc, group=self.group, async_op=True),
                                dist.all_gather_into_tensor(H_all, Hc, group=self.group, async_op=True)))
            else:
                x_all.copy_(xc)
                H_all.copy_(Hc)
                gathers.append(None)
            xs.append(x_all)
            Hs.append(H_all)
        exchanged = []
        for c in range(C):
            if gathers[c] is not None:
                for w in gathers[c]:
                    w.wait()
            h_cols = self.ops.swiglu(xs[c], Hs[c], self.gate_up)  # [world * mc, I_r]
            if world > 1 and self._nccl and self._equal_cols:
                # one NCCL all-to-all: row block r of h_cols goes to rank r
                recv = torch.empty_like(h_cols)
                work = dist.all_to_all_single(recv, h_cols, group=self.group, async_op=True)
                exchanged.append(("a2a", recv, [work]))
            elif world > 1:
                recv = [h_cols.new_empty((mc, c1 - c0)) for c0, c1 in self.cols]
                reqs = exchange_blocks([b.contiguous() for b in h_cols.split(mc, dim=0)], recv, self.rank,
                                       self.group, async_op=True)
                exchanged.append(("p2p", recv, reqs))
            else:
                exchanged.append(("p2p", [h_cols], []))
        outs = []
        for c, (kind, recv, reqs) in enumerate(exchanged):
            for req in reqs:
                req.wait()
            if kind == "a2a":  # [world, mc, I_r] -> [mc, world * I_r], columns in rank order
                h = recv.view(world, mc, -1).permute(1, 0, 2).reshape(mc, -1)
            else:
                h = torch.cat(recv, dim=1) if len(recv) > 1 else recv[0]
            outs.append(self.ops.down(h.contiguous(), H[c * mc:(c + 1) * mc], self.down_w))
        return outs[0] if C == 1 else torch.cat(outs, dim=0)


class ColumnParallelDecoder:
    """Mode T of the decoder stack (BASELINE config 5's "MLP up/gate column-sharded, NCCL
    all-gather over NVLink"): every rank runs norms, projections and attention for its
    own sequences, and each layer's MLP as ``ColumnParallelGatedMLP`` (gate / up split
    by column across the ranks, rows all-gathered at the layer boundary, the SwiGLU
    output exchanged back by row blocks).  Built over the same EntropyDispatchedLlamaBlock
    layers as ``DecoderEngine`` with per-token routing and the reference's MLP-only mode,
    it computes the same values as the engine on the rank's rows, bit for bit.
    ``position_embeddings`` are the rotary (cos, sin) tables of this rank's [batch, seq]."""

    def __init__(self, blocks, final_norm: torch.Tensor, position_embeddings, world: int, rank: int, group=None,
                 tau_low: float = 0.41, tau_high: float = 1.68, chunks: int = 2):
        self.blocks = blocks
        self.world, self.rank = world, rank
        self.mlps = [ColumnParallelGatedMLP.from_blocks_mlp(b, world, rank, group, tau_low, tau_high, chunks)
                     for b in blocks]
        self.final_norm = final_norm
        self.pe = position_embeddings

    @torch.no_grad()
    def forward(self, hidden: torch.Tensor):
        """hidden fp16 [batch, seq, d] of this rank's sequences -> (final-norm output, the
        last block's output), both [batch, seq, d]."""
        from .kernels import add_rmsnorm, flash_attention_rope_entropy, linear_f16

        B, S, d = hidden.shape
        h, s_prev, m_prev = hidden, None, None
        for blk, mlp in zip(self.blocks, self.mlps):
            attn = blk.self_attn
            eps = blk.input_layernorm.variance_epsilon
            if s_prev is None:
                x = add_rmsnorm(h, blk.input_layernorm.weight, eps)
            else:
                x, h = add_rmsnorm(m_prev, blk.input_layernorm.weight, eps, residual=s_prev)
            qkv = linear_f16(x.reshape(B * S, d), blk.qkv_weight()).reshape(B, S, -1)
            q, k, v = qkv.split(blk._qkv_split, dim=-1)
            hd = attn.head_dim
            cos, sin = self.pe
            out, _, _, token = flash_attention_rope_entropy(q, k, v, cos, sin, q.shape[-1] // hd, k.shape[-1] // hd,
                                                            causal=True, scale=attn.scaling, return_token=True)
            o = linear_f16(out.reshape(B * S, -1), attn.o_proj.weight).reshape(B, S, d)
            x2, s_prev = add_rmsnorm(o, blk.post_attention_layernorm.weight,
                                     blk.post_attention_layernorm.variance_epsilon, residual=h)
            m_prev = mlp.forward(x2.reshape(B * S, d), token.reshape(-1)).reshape(B, S, d)
        y, h_last = add_rmsnorm(m_prev, self.final_norm, self.blocks[-1].input_layernorm.variance_epsilon,
                                residual=s_prev)
        return y, h_last


class PeerTimeout(RuntimeError):
    """A rank did not report in time (it died, hung or never joined)."""


def check_peers(store, world: int, rank: int, tag: str, timeout_s: float = 10.0) -> None:
    """Host-side liveness check before a step: every rank publishes ``tag`` in the
    store, then waits (bounded) for all others.  Raises PeerTimeout naming the missing
    ranks instead of letting the next collective hang."""
    store.set(f"{tag}/{rank}", "1")
    deadline = time.monotonic() + timeout_s
    missing = list(range(world))
    while missing:
        missing = [r for r in missing if not _has_key(store, f"{tag}/{r}")]
        if not missing:
            return
        if time.monotonic() > deadline:
            raise PeerTimeout(f"ranks {missing} did not reach '{tag}' within {timeout_s:.1f} s")
        time.sleep(0.01)


def _has_key(store, key: str) -> bool:
    try:
        store.wait([key], timedelta(milliseconds=1))
        return True
    except Exception:  # the store reports a timeout as an exception
        return False
