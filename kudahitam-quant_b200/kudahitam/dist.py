"""Multi-GPU plumbing (one process per GPU, torch.distributed).

* Compression is row-independent: ``shard_range`` gives each rank a
  contiguous slice of the flattened batch x head axis and ranks compress their
  slices with no communication.
* Decode attention over a sequence-sharded cache: every rank runs the split-K
  partial kernel over its own slice of S, merges its splits into one
  (m, l, acc[D]) record per query row (``kh_decode_merge``), and one
  all-gather gives every rank the [world, R, D+2] records of all ranks, which
  ``kh_decode_combine_strided`` merges into the output (records with l == 0,
  from ranks or splits that own no rows, are ignored).  Each rank sends
  R * (D+2) floats: 266 KB for 512 query rows at D = 128.
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


def gather_records(local: torch.Tensor, group=None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """This rank's [R, D+2] merged records -> [world, R, D+2], the records of
    every rank (rank r at [r]), by one all-gather."""
    world, _ = _world(group)
    R, W = local.shape
    if out is None:
        out = torch.empty((world, R, W), dtype=local.dtype, device=local.device)
    if world == 1:
        out[0].copy_(local)
        return out
    dist.all_gather_into_tensor(out.view(world * R, W), local.contiguous(), group=group)
    return out


def seq_sharded_workspace_numel(n_rows: int, n_splits: int, world: int, head_dim: int) -> int:
    """Floats of workspace ``decode_attention_seq_sharded`` uses: the local
    split records, and with world > 1 the merged record and the gathered
    records of every rank."""
    extra = 1 + world if world > 1 else 0
    return n_rows * (head_dim + 2) * (n_splits + extra)


def next_epoch(epoch: int) -> int:
    """Epoch of the peer exchange's next call: 1, 2, ..., 0xFFFFFFFF, then 2.
    0 is reserved (flags start at 0, "never written").  Wrapping to 2 rather
    than 1 keeps the parity (which buffer/flag set a call uses) alternating
    across the wrap, so two consecutive calls never share a set."""
    return epoch + 1 if epoch < 0xFFFFFFFF else 2


class PeerRecordExchange:
    """Buffers for the record exchange of a sequence-sharded decode over peer
    memory: one symmetric-memory allocation per rank, addressable by every
    rank over NVLink, holding two sets (alternating between calls) of a
    record buffer [world, n_rows, n_parts, D+2] and a flag array [world],
    plus a local counter.  Two ways to use it:

    * ``decode``: the partial kernel itself stores its split records into
      every rank's buffer (``kh_decode_partial_to_peers``, up to n_parts
      records per query row) and one combine kernel merges them
      (``kh_decode_combine_peer_records``): two kernels per step, no
      collective call;
    * ``combine``: after a local partial kernel, ``kh_decode_merge_to_peers``
      merges each rank's splits and stores one record per row, then
      ``kh_decode_combine_from_peers`` merges the world records.

    Collective to create: every rank of the group builds one with the same
    arguments, and every rank must make the same sequence of calls.  Release
    it (``del``) after a device synchronisation and before
    ``destroy_process_group``.  world <= 8."""

    def __init__(self, n_rows: int, head_dim: int, group=None, device=None, n_parts: int = 1):
        import torch.distributed._symmetric_memory as symm
        world, rank = _world(group)
        if world > 8:
            raise ValueError("the peer record exchange supports at most 8 ranks")
        if n_parts < 1:
            raise ValueError("n_parts must be at least 1")
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.world, self.rank, self.n_rows, self.head_dim = world, rank, n_rows, head_dim
        self.n_parts = n_parts
        self.rec_bytes = world * n_rows * n_parts * (head_dim + 2) * 4
        self.flag_off = 2 * self.rec_bytes
        total = self.flag_off + 2 * world * 4
        total = (total + 255) // 256 * 256
        self.buf = symm.empty(total, dtype=torch.uint8, device=dev)
        self.buf.zero_()
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        grp = group if group is not None else dist.group.WORLD
        self.handle = symm.rendezvous(self.buf, grp)
        self.handle.barrier()  # every rank's buffer is zero before any peer store
        self.ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.epoch = 0

    def combine(self, local: torch.Tensor, dv, out: torch.Tensor,
                checked: bool = False) -> torch.Tensor:
        """local: this rank's [R, P, D+2] split records; out: [R, D] (any
        shape of R * D floats).  Merges, exchanges and combines.

        If a peer's records do not arrive within about a second, the combine
        kernel stops waiting, writes ZEROS to ``out`` and sets bit 2 of the
        library's sticky device error word (``_lib.device_error()``); the
        call itself returns normally, because the wait runs on the GPU after
        this function has returned.  With ``checked=True`` the call
        synchronises the stream, reads that word and raises
        ``PeerTimeoutError`` (clearing the word) when bit 2 is set."""
        R, P, gs, ps = ops._record_view(local, self.head_dim)
        if R != self.n_rows:
            raise ValueError(f"exchange built for {self.n_rows} rows, got {R}")
        self.epoch = next_epoch(self.epoch)
        par = self.epoch & 1
        w = self.world
        K = ops.ext()
        K.decode_merge_to_peers(local, R, P, gs, ps, self.head_dim,
                                [p + par * self.rec_bytes for p in self.ptrs],
                                [p + self.flag_off + par * w * 4 for p in self.ptrs],
                                self.rank, self.epoch, self.counter)
        K.decode_combine_from_peers(self.buf, par * self.rec_bytes, self.flag_off + par * w * 4,
                                    self.epoch, R, w, ops._host_f32(dv), out)
        dev = local.device
        if checked:
            check_peer_timeout(dev)
        return out

    def decode(self, q: torch.Tensor, k_local: ops.PackedKV, v_local: ops.PackedKV, dk, dv,
               centroids, sm_scale: float, n_splits: int, out: torch.Tensor,
               checked: bool = False) -> torch.Tensor:
        """The whole sequence-sharded decode step in one kernel: this rank's
        split-K partial kernel stores its records straight into every rank's
        buffer, and once every rank's flag has arrived its CTAs merge the
        world x n_splits records of each query row into ``out`` (a second
        kernel does the merge if the launch does not fit on the GPU at once).
        q: [G, D] or [G, n_q, D] (float32 on this rank's GPU); the caches hold
        G * S_local rows.  Timeouts behave as in ``combine``."""
        if n_splits > self.n_parts:
            raise ValueError(f"exchange built for {self.n_parts} records per row, "
                             f"got n_splits={n_splits}")
        G, D = q.shape[0], q.shape[-1]
        R = q.numel() // D
        if R != self.n_rows or D != self.head_dim:
            raise ValueError(f"exchange built for {self.n_rows} rows of {self.head_dim}")
        S_loc = k_local.n_rows // max(G, 1)
        qf = q if (q.dtype == torch.float32 and q.is_contiguous()) else \
            q.to(torch.float32).contiguous()
        self.epoch = next_epoch(self.epoch)
        par = self.epoch & 1
        w = self.world
        K = ops.ext()
        K.decode_partial_to_peers(qf, k_local.code, k_local.res, k_local.norms, k_local.rnorms,
                                  v_local.code, v_local.res, v_local.norms, v_local.rnorms,
                                  S_loc, 0, S_loc, ops._host_f32(dk), ops._host_f32(centroids),
                                  float(sm_scale), n_splits,
                                  [p + par * self.rec_bytes for p in self.ptrs],
                                  [p + self.flag_off + par * w * 4 for p in self.ptrs],
                                  self.rank, self.epoch, self.counter, ops._host_f32(dv), out)
        if checked:
            check_peer_timeout(q.device)
        return out


class PeerTimeoutError(RuntimeError):
    """A peer-memory record exchange stopped waiting for a peer's records
    (its output holds zeros)."""


def check_peer_timeout(device=None) -> None:
    """Synchronise ``device`` and raise PeerTimeoutError if a peer-memory
    combine gave up waiting since the device error word was last cleared
    (bit 2 of ``kh_device_error``); the word is cleared before raising."""
    from . import _lib
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    with ops._on(dev):
        torch.cuda.synchronize(dev)
        if _lib.device_error() & 4:
            _lib.call("kh_clear_device_error")
            raise PeerTimeoutError(
                "a peer's decode records did not arrive within about a second; the "
                "combined output was set to zeros")


def decode_attention_seq_sharded(q: torch.Tensor, k_local: ops.PackedKV,
                                 v_local: ops.PackedKV, dk, dv, centroids,
                                 sm_scale: Optional[float] = None,
                                 n_splits: Optional[int] = None, group=None,
                                 partials: Optional[torch.Tensor] = None,
                                 exchange: Optional[PeerRecordExchange] = None,
                                 checked: bool = False) -> torch.Tensor:
    """Decode attention where each rank holds S_local cached rows per group
    (k_local / v_local: G * S_local rows).  q is [G, D] or [G, n_q, D]
    (grouped-query heads).  Returns float32 with q's shape on every rank.
    With ``exchange`` (a PeerRecordExchange of this group and shape) the
    records cross NVLink by plain stores instead of one NCCL all-gather: from
    the partial kernel itself when the exchange holds n_splits records per
    row (and the codebook has a table kernel), else from the merge kernel.
    If a peer never arrives these paths return zeros and flag bit 2 of the
    device error word, and ``checked=True`` turns that into a
    PeerTimeoutError (at the cost of a stream synchronisation)."""
    world, _ = _world(group)
    G, D = q.shape[0], q.shape[-1]
    R = q.numel() // D  # query rows: G * n_q
    S_loc = k_local.n_rows // max(G, 1)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if n_splits is None:
        n_splits = ops.default_splits(R, S_loc, q.device, 1 if q.dim() == 2 else q.shape[1])
    rec = D + 2
    need = seq_sharded_workspace_numel(R, n_splits, world, D)
    if partials is None or partials.numel() < need:
        partials = torch.empty(need, dtype=torch.float32, device=q.device)
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    if (world > 1 and exchange is not None and n_splits <= exchange.n_parts
            and (ops._check_codebook(centroids)[0] == 2 or D == 128)):
        # the partial kernel stores its records into every rank's buffer
        return exchange.decode(q, k_local, v_local, dk, dv, centroids, sm_scale, n_splits, out,
                               checked=checked)
    local = partials[: R * n_splits * rec].view(R, n_splits, rec)
    ops.decode_partial(q, k_local, v_local, dk, dv, centroids, sm_scale, n_splits, local,
                       part_stride=n_splits, part_offset=0, seq_len=S_loc)
    if world == 1:
        return ops.decode_combine(local, n_splits, dv, out)
    if exchange is not None:
        return exchange.combine(local, dv, out, checked=checked)
    off = R * n_splits * rec
    merged = partials[off: off + R * rec].view(R, rec)
    ops.decode_merge(local, merged)
    gathered = partials[off + R * rec: need].view(world, R, rec)
    gather_records(merged, group, out=gathered)
    return ops.decode_combine_records(gathered.transpose(0, 1), dv, out)


def max_over_ranks(value: float, group=None, device=None) -> float:
    """Maximum of a per-rank scalar (e.g. a CUDA-event time) over all ranks."""
    world, _ = _world(group)
    if world == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
