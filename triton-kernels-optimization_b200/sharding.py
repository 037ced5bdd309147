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


def exchange_blocks(send: list, recv: list, rank: int, group=None) -> None:
    """All-to-all of one block per rank pair: ``send[s]`` goes to rank s and
    ``recv[s]`` receives rank s's block for this rank.  Grouped point-to-point
    transfers (one NCCL group on GPUs; gloo, which has no all-to-all, runs the same
    code on CPU)."""
    ops = []
    for peer in range(len(send)):
        if peer == rank:
            recv[peer].copy_(send[peer])
            continue
        gpeer = dist.get_global_rank(group, peer) if group is not None else peer
        ops.append(dist.P2POp(dist.isend, send[peer], gpeer, group))
        ops.append(dist.P2POp(dist.irecv, recv[peer], gpeer, group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()


class GatedMLPOps:
    """The device operations mode T needs, on the sm_100a kernels: routing from given
    entropies and the bucketed GEMMs (gate and up share one packing of their input)."""

    def __init__(self, tau_low: float, tau_high: float):
        from .dispatch import EntropyRouter

        self._all = EntropyRouter(tau_low, tau_high)
        self._local = EntropyRouter(tau_low, tau_high)

    @staticmethod
    def pack(weight: torch.Tensor):
        from .kernels import WeightPack

        return WeightPack.from_weight(weight)

    def gate_up(self, x: torch.Tensor, H: torch.Tensor, gate, up):
        r = self._all
        r.reserve(x.shape[0], x.shape[1], x.device)
        r.route_entropy(H)
        r.pack_rows(x)
        return r.gemm_packed(gate), r.gemm_packed(up)

    def down(self, h: torch.Tensor, H: torch.Tensor, down):
        r = self._local
        r.reserve(h.shape[0], h.shape[1], h.device)
        r.route_entropy(H)
        return r.gated_linear(h, down)


class ColumnParallelGatedMLP:
    """Mode T of the gated SwiGLU MLP: ``down(silu(gate(x)) * up(x))`` with gate and up
    split by output column across the ranks and the rows of x split by row.

    Per step, for the ``m`` rows a rank owns (equal on every rank):
      1. all-gather the rows x [m, d] -> [world*m, d] and their entropies H [m];
      2. route all rows (every rank derives the same routes from the same H) and run
         this rank's gate / up columns over all of them -> [world*m, I/world] each;
      3. h = silu(gate) * up on that column block;
      4. all-to-all: the row block of every other rank goes to it, and this rank's
         rows come back from every rank -> h [m, I] (columns in rank order);
      5. the down projection (full weight) on the rank's own rows.
    Per-row activation scales span the whole row (steps 2 and 5 see full rows) and
    weight scales are per output column, so the result equals the single-GPU MLP bit
    for bit.  The two collectives are the layer-boundary exchange of this mode.
    """

    def __init__(self, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, world: int, rank: int,
                 ops=None, group=None, tau_low: float = 0.41, tau_high: float = 1.68):
        inter = w_gate.shape[0]
        if w_up.shape[0] != inter or w_down.shape[1] != inter:
            raise ValueError("gate / up must be [I, d] and down [d, I]")
        self.world, self.rank, self.group = world, rank, group
        self.ops = ops if ops is not None else GatedMLPOps(tau_low, tau_high)
        self.cols = [column_shard(inter, world, r) for r in range(world)]
        c0, c1 = self.cols[rank]
        self.gate = self.ops.pack(w_gate[c0:c1])
        self.up = self.ops.pack(w_up[c0:c1])
        self.down_w = self.ops.pack(w_down)

    def forward(self, x: torch.Tensor, H: torch.Tensor) -> torch.Tensor:
        m, d = x.shape
        world = self.world
        x_all = x.new_empty((world * m, d))
        H_all = H.new_empty((world * m,))
        if world > 1:
            dist.all_gather_into_tensor(x_all, x.contiguous(), group=self.group)
            dist.all_gather_into_tensor(H_all, H.contiguous(), group=self.group)
        else:
            x_all.copy_(x)
            H_all.copy_(H)
        g, u = self.ops.gate_up(x_all, H_all, self.gate, self.up)
        h_cols = torch.nn.functional.silu(g) * u  # [world*m, I_r]
        if world > 1:
            recv = [h_cols.new_empty((m, c1 - c0)) for c0, c1 in self.cols]
            exchange_blocks([b.contiguous() for b in h_cols.split(m, dim=0)], recv, self.rank, self.group)
            h = torch.cat(recv, dim=1)
        else:
            h = h_cols
        return self.ops.down(h.contiguous(), H, self.down_w)


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
