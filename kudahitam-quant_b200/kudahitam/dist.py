"""Multi-GPU plumbing (one process per GPU, torch.distributed).

* Compression is row-independent: ``shard_range`` gives each rank a
  contiguous slice of the flattened batch x head axis and ranks compress their
  slices with no communication.
* Decode attention over a sequence-sharded cache: every rank runs the split-K
  partial kernel over its own slice of S and writes (m, l, acc[D]) records into
  its slot of a zero-initialised [G, world * n_splits, D+2] buffer; one
  all-reduce(SUM) turns that buffer into the gathered records of all ranks
  (slots of other ranks are zero and records with l == 0 are ignored by the
  merge), and every rank merges them locally with ``kh_decode_combine``.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from . import ops


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced slice [start, stop) of n items for ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _world(group) -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


def gather_partials(local: torch.Tensor, group=None) -> torch.Tensor:
    """[G, P, R] records of this rank -> [G, world * P, R] records of all ranks
    (rank r at slots [r*P, (r+1)*P)), by one all-reduce over a zero buffer."""
    world, rank = _world(group)
    G, P, R = local.shape
    if world == 1:
        return local
    buf = torch.zeros((G, world * P, R), dtype=local.dtype, device=local.device)
    buf[:, rank * P:(rank + 1) * P] = local
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    return buf


def decode_attention_seq_sharded(q: torch.Tensor, k_local: ops.PackedKV,
                                 v_local: ops.PackedKV, dk, dv, centroids,
                                 sm_scale: Optional[float] = None,
                                 n_splits: Optional[int] = None, group=None,
                                 partials: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode attention where each rank holds S_local cached rows per group
    (k_local / v_local: G * S_local rows).  q is [G, D] or [G, n_q, D]
    (grouped-query heads).  Returns float32 with q's shape on every rank."""
    world, rank = _world(group)
    G, D = q.shape[0], q.shape[-1]
    R = q.numel() // D  # query rows: G * n_q
    S_loc = k_local.n_rows // max(G, 1)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if n_splits is None:
        n_splits = ops.default_splits(R, S_loc, q.device)
    parts = world * n_splits
    if partials is None or partials.numel() < R * parts * (D + 2):
        partials = torch.empty(R * parts * (D + 2), dtype=torch.float32, device=q.device)
    buf = partials[: R * parts * (D + 2)].view(R, parts, D + 2)
    buf.zero_()
    ops.decode_partial(q, k_local, v_local, dk, dv, centroids, sm_scale, n_splits, buf,
                       part_stride=parts, part_offset=rank * n_splits, seq_len=S_loc)
    if world > 1:
        dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    return ops.decode_combine(buf, parts, dv, out)


def max_over_ranks(value: float, group=None, device=None) -> float:
    """Maximum of a per-rank scalar (e.g. a CUDA-event time) over all ranks."""
    world, _ = _world(group)
    if world == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
