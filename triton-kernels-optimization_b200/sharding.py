"""Row partitioning of the gated path across the GPUs of one node.

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
