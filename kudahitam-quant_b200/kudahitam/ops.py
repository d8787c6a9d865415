"""Torch-facing operators: Python wrappers of ``torch.ops.kudahitam.*``.

The operators are registered by the engine's torch extension
(``_lib/libkh_torch.so``, built from ``csrc/kh_torch.cpp``), a thin layer over
the C ABI: each takes CUDA tensors, allocates its outputs with PyTorch's
caching allocator and launches on the tensors' device and its current
stream.  There is no CPU path: CPU inputs raise ``ValueError`` and a missing
engine raises ``NativeLibraryError``.  (``_lib`` binds the same C ABI with
ctypes for the pure-C tests.)
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import torch

from . import _lib

_DTYPE_CODE = {torch.float32: _lib.KH_F32, torch.float16: _lib.KH_F16,
               torch.bfloat16: _lib.KH_BF16}

HEAD_DIMS = (128, 256)


_EXT = None


def ext():
    """``torch.ops.kudahitam`` (loads the engine's torch extension once)."""
    global _EXT
    if _EXT is None:
        path = _lib.library_path().parent / "libkh_torch.so"
        if not path.exists():
            raise _lib.NativeLibraryError(
                f"{path} not found: build it with `python kudahitam-quant_b200/build.py`")
        try:
            torch.ops.load_library(str(path))
        except OSError as e:  # pragma: no cover
            raise _lib.NativeLibraryError(f"cannot load {path}: {e}") from e
        _EXT = torch.ops.kudahitam
    return _EXT


def _host_f32(t) -> torch.Tensor:
    """Contiguous float32 CPU copy (d vectors and centroids travel by value)."""
    if (isinstance(t, torch.Tensor) and t.dtype == torch.float32 and not t.is_cuda
            and not t.requires_grad and t.is_contiguous()):
        return t  # already in the form the library reads
    t = torch.as_tensor(t)
    return t.detach().to(device="cpu", dtype=torch.float32).contiguous()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class _Nothing:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NOTHING = _Nothing()


def _on(dev: torch.device):
    """``torch.cuda.device(dev)`` when dev is not the current device (the
    switch costs microseconds per call on the common single-device path)."""
    return _NOTHING if dev.index == torch.cuda.current_device() else torch.cuda.device(dev)


def _require_cuda(*ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("kudahitam ops run on CUDA tensors only (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


@dataclass
class PackedKV:
    """The packed cache of one tensor of N = prod(shape[:-1]) rows.

    code   int32 [N, D/32] (bits=1) or [N, D/16] (bits=2), bit patterns of the
           uint32 words described in include/kudahitam.h
    res    int32 [N, D/32] residual sign plane, or None (1-bit mode)
    norms  float32 [N]
    rnorms float32 [N] or None
    """
    shape: tuple
    bits: int
    code: torch.Tensor
    norms: torch.Tensor
    res: Optional[torch.Tensor] = None
    rnorms: Optional[torch.Tensor] = None

    @property
    def head_dim(self) -> int:
        return int(self.shape[-1])

    @property
    def n_rows(self) -> int:
        return int(self.norms.numel())

    @property
    def residual(self) -> bool:
        return self.res is not None

    @property
    def device(self) -> torch.device:
        return self.norms.device

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in
                   (self.code, self.norms, self.res, self.rnorms) if t is not None)

    def rows(self, start: int, stop: int) -> "PackedKV":
        """Rows [start, stop) as a flat PackedKV (views, no copy)."""
        sl = slice(start, stop)
        return PackedKV((stop - start, self.head_dim), self.bits, self.code[sl],
                        self.norms[sl], None if self.res is None else self.res[sl],
                        None if self.rnorms is None else self.rnorms[sl])


def empty_packed(shape, bits: int, residual: bool, device) -> PackedKV:
    D = int(shape[-1])
    n = math.prod(int(s) for s in shape[:-1])
    words = D // 32 if bits == 1 else D // 16
    return PackedKV(tuple(int(s) for s in shape), bits,
                    torch.empty((n, words), dtype=torch.int32, device=device),
                    torch.empty(n, dtype=torch.float32, device=device),
                    torch.empty((n, D // 32), dtype=torch.int32, device=device) if residual else None,
                    torch.empty(n, dtype=torch.float32, device=device) if residual else None)


def empty_packed_pinned(shape, bits: int, residual: bool) -> PackedKV:
    """A packed cache in pinned host memory (target of asynchronous copies)."""
    D = int(shape[-1])
    n = math.prod(int(s) for s in shape[:-1])
    words = D // 32 if bits == 1 else D // 16
    e = lambda *sh, dt=torch.int32: torch.empty(sh, dtype=dt, pin_memory=True)  # noqa: E731
    return PackedKV(tuple(int(s) for s in shape), bits, e(n, words),
                    e(n, dt=torch.float32),
                    e(n, D // 32) if residual else None,
                    e(n, dt=torch.float32) if residual else None)


def _check_codebook(centroids: torch.Tensor) -> tuple[int, int]:
    n_c = centroids.numel()
    if n_c not in (2, 4):
        raise ValueError(f"codebook must have 2 or 4 levels, got {n_c}")
    return n_c, (1 if n_c == 2 else 2)


def compress(x: torch.Tensor, d, centroids, residual: bool = True,
             out: Optional[PackedKV] = None) -> PackedKV:
    """Fused compression of the rows x[..., D] (fp32 / fp16 / bf16, D in
    {128, 256}).  Replaces ``ultra_fused_full_fusion`` (KudaHitamCUDA.cu:197-231)."""
    dev = _require_cuda(x)
    if x.dtype not in _DTYPE_CODE:
        raise TypeError(f"unsupported dtype {x.dtype}")
    D = x.shape[-1]
    if D not in HEAD_DIMS:
        raise ValueError(f"head_dim must be 128 or 256, got {D}")
    dh, ch = _host_f32(d), _host_f32(centroids)
    _, bits = _check_codebook(ch)
    if out is None:
        r = ext().compress(x, dh, ch, residual)
        shape = tuple(int(s) for s in x.shape)
        if residual:
            return PackedKV(shape, bits, r[0], r[1], r[2], r[3])
        return PackedKV(shape, bits, r[0], r[1])
    ext().compress_out(x, dh, ch, residual, out.code, out.res, out.norms, out.rnorms)
    return out


class _HostPipe:
    """Per-device streams and double-buffered staging for compress_host."""

    def __init__(self, dev: torch.device):
        self.dev = dev
        self.h2d = torch.cuda.Stream(dev)
        self.comp = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.stage_in: list = [None, None]
        self.stage_out: list = [None, None]
        self.in_free = [None, None]   # compute done reading stage_in[slot]
        self.out_free = [None, None]  # D2H done reading stage_out[slot]

    def buffers(self, slot: int, rows: int, D: int, dtype, bits: int, residual: bool):
        need_in = rows * D
        b = self.stage_in[slot]
        o = self.stage_out[slot]
        grow_in = b is None or b.numel() < need_in or b.dtype != dtype
        grow_out = (o is None or o.n_rows < rows or o.head_dim != D or o.bits != bits
                    or o.residual != residual)
        if (grow_in and b is not None) or (grow_out and o is not None):
            torch.cuda.synchronize(self.dev)  # old buffers may still be in use on our streams
        if grow_in:
            self.stage_in[slot] = torch.empty(need_in, dtype=dtype, device=self.dev)
        if grow_out:
            self.stage_out[slot] = empty_packed((rows, D), bits, residual, self.dev)
        return self.stage_in[slot], self.stage_out[slot]


_pipes: dict = {}


def compress_host(xs: Sequence[torch.Tensor], d, centroids, residual: bool = True,
                  device=None, outs: Optional[Sequence[PackedKV]] = None,
                  chunk_rows: Optional[int] = None) -> list[PackedKV]:
    """Compress host-resident tensors into host-resident packed caches on the
    GPU, with the host-to-device copy of chunk k+1, the compression of chunk k
    and the device-to-host copy of chunk k-1 overlapped on three streams (a
    step costs about the larger copy instead of the sum of all three).

    xs are CPU tensors [..., D] (pinned memory for asynchronous copies; others
    are staged through pageable copies).  Returns pinned host PackedKVs (or
    fills ``outs``).  Work is enqueued; the caller's current stream waits for
    it, so synchronise that stream before reading the results."""
    if not xs:
        return []
    dev = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise ValueError("compress_host runs the compression on a CUDA device")
    dt = xs[0].dtype
    D = xs[0].shape[-1]
    if any(t.is_cuda or t.dtype != dt or t.shape[-1] != D for t in xs):
        raise ValueError("compress_host takes CPU tensors of one dtype and head_dim")
    if dt not in _DTYPE_CODE or D not in HEAD_DIMS:
        raise ValueError("unsupported dtype / head_dim")
    ch = _host_f32(centroids)
    _, bits = _check_codebook(ch)
    if outs is None:
        outs = [empty_packed_pinned(t.shape, bits, residual) for t in xs]
    if chunk_rows is None:
        chunk_rows = max(1024, (64 << 20) // (D * xs[0].element_size()))  # 64 MB chunks
    pipe = _pipes.get(dev)
    if pipe is None:
        pipe = _pipes[dev] = _HostPipe(dev)
    caller = torch.cuda.current_stream(dev)
    pipe.h2d.wait_stream(caller)
    fields = ("code", "res", "norms", "rnorms") if residual else ("code", "norms")
    k = 0
    last = None
    with _on(dev):
        for x, o in zip(xs, outs):
            rows = x.reshape(-1, D)
            if not rows.is_contiguous():
                rows = rows.contiguous()
            n = rows.shape[0]
            for a in range(0, n, chunk_rows):
                b = min(n, a + chunk_rows)
                m = b - a
                slot = k & 1
                sin, sout = pipe.buffers(slot, chunk_rows, D, dt, bits, residual)
                # host -> device
                if pipe.in_free[slot] is not None:
                    pipe.h2d.wait_event(pipe.in_free[slot])
                with torch.cuda.stream(pipe.h2d):
                    sin[: m * D].view(m, D).copy_(rows[a:b], non_blocking=True)
                    ready = torch.cuda.Event()
                    ready.record(pipe.h2d)
                # compress
                pipe.comp.wait_event(ready)
                if pipe.out_free[slot] is not None:
                    pipe.comp.wait_event(pipe.out_free[slot])
                with torch.cuda.stream(pipe.comp):
                    compress(sin[: m * D].view(m, D), d, ch, residual=residual,
                             out=sout.rows(0, m))
                    done = torch.cuda.Event()
                    done.record(pipe.comp)
                pipe.in_free[slot] = done
                # device -> host
                pipe.d2h.wait_event(done)
                with torch.cuda.stream(pipe.d2h):
                    dst = o.rows(a, b)
                    src = sout.rows(0, m)
                    for f in fields:
                        getattr(dst, f).copy_(getattr(src, f), non_blocking=True)
                    freed = torch.cuda.Event()
                    freed.record(pipe.d2h)
                pipe.out_free[slot] = freed
                last = freed
                k += 1
    if last is not None:
        caller.wait_event(last)
    return list(outs)


def compress_many(xs: Sequence[torch.Tensor], d, centroids, residual: bool = True,
                  outs: Optional[Sequence[PackedKV]] = None) -> list[PackedKV]:
    """Compress several tensors (same dtype and head_dim) in one launch per
    kh_max_segments() tensors."""
    if not xs:
        return []
    if not xs[0].is_cuda:
        raise ValueError("kudahitam ops run on CUDA tensors only (no CPU path)")
    # devices, dtypes, head dims and buffer sizes are checked by the operator
    dh, ch = _host_f32(d), _host_f32(centroids)
    if outs is None:
        _, bits = _check_codebook(ch)
        outs = [empty_packed(t.shape, bits, residual, xs[0].device) for t in xs]
    # one launch per kh_max_segments() tensors, inside the operator
    if residual:
        ext().compress_many_out(xs, dh, ch, True, [o.code for o in outs], [o.res for o in outs],
                                [o.norms for o in outs], [o.rnorms for o in outs])
    else:
        ext().compress_many_out(xs, dh, ch, False, [o.code for o in outs], [],
                                [o.norms for o in outs], [])
    return outs


def fwht_(x: torch.Tensor) -> torch.Tensor:
    """In-place orthonormal FWHT of contiguous float32 rows (the reference's
    ``cuda_ext.forward``, KudaHitamCUDA.cu:275-283)."""
    dev = _require_cuda(x)
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise ValueError("fwht_ needs a contiguous float32 tensor")
    return ext().fwht_(x)


def fwht(x: torch.Tensor) -> torch.Tensor:
    """Orthonormal FWHT along the last dim (returns a new float32 tensor)."""
    return fwht_(x.to(torch.float32).contiguous().clone())


def materialize(p: PackedKV, d, centroids, idx: bool = True, kmse: bool = True,
                signs: bool = True) -> dict:
    """Reference-layout tensors from a packed cache: idx uint8 [N, D],
    k_mse float32 [N, D], signs int8 [N, D]."""
    _require_cuda(p.code)
    dh, ch = _host_f32(d), _host_f32(centroids)
    o_idx, o_k, o_s = ext().materialize(p.code, p.res, p.norms, p.head_dim, dh, ch, idx, kmse,
                                        signs)
    return {"idx": o_idx if idx else None, "kmse": o_k if kmse else None,
            "signs": o_s if (signs and p.res is not None) else None}


def score(q: torch.Tensor, p: PackedKV, d, centroids, seq_len: Optional[int] = None
          ) -> torch.Tensor:
    """Asymmetric scores of q [G, nq, D] against G groups of seq_len cached
    rows each (rows of group g are rows [g*seq_len, (g+1)*seq_len) of p).
    Returns float32 [G, nq, seq_len]."""
    _require_cuda(q, p.norms)
    G, nq, D = q.shape
    if D != p.head_dim:
        raise ValueError("query head_dim does not match the cache")
    S = p.n_rows // max(G, 1) if seq_len is None else int(seq_len)
    if G * S != p.n_rows:
        raise ValueError(f"{p.n_rows} cached rows do not split into {G} groups of {S}")
    dh, ch = _host_f32(d), _host_f32(centroids)
    return ext().score(q, p.code, p.res, p.norms, p.rnorms, S, dh, ch)


def decode_workspace_bytes(n_groups: int, n_splits: int, head_dim: int) -> int:
    return int(_lib.lib().kh_decode_workspace_bytes(n_groups, n_splits, head_dim))


def default_splits(n_groups: int, seq_len: int, device, n_q: int = 1) -> int:
    """Records per query row for decode (the ``n_splits`` argument), for
    n_groups query rows (n_q per cache group) of seq_len cached rows.

    The decode kernel cuts the call's (cache group, row) pairs into equal
    ranges, one wave of CTAs at two per SM and no range under 8192 pairs,
    whatever the group count; a group spanning several ranges gets
    one record per range.  This rule returns how many records the longest
    group can need at that range length, so the kernel runs balanced.  (The
    earlier one-CTA-per-(row, split) grid ran 1.73 waves for 512 query rows
    on 148 SMs.)"""
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return splits_for(n_groups, seq_len, sms, n_q)


def splits_for(n_rows: int, seq_len: int, n_sms: int, n_q: int = 1) -> int:
    """The rule of ``default_splits`` for a GPU with n_sms SMs; mirrors the
    decode launcher's range length (kh_decode.cu: one wave of CTA sets of
    n_q CTAs at two CTAs per SM, at least 8192 pairs per range)."""
    if seq_len <= 0 or n_rows <= 0:
        return 1
    groups = max(1, n_rows // max(n_q, 1))
    total = groups * seq_len
    slots = max(1, 2 * n_sms // max(n_q, 1))
    sets = max(1, min(slots, -(-total // 8192)))
    w_bal = -(-total // sets)
    return int(min(1024, -(-seq_len // w_bal) + 1))


def decode_partial(q: torch.Tensor, k: PackedKV, v: PackedKV, dk, dv, centroids,
                   sm_scale: float, n_splits: int, partials: torch.Tensor,
                   part_stride: int, part_offset: int, seq_len: int,
                   seq_begin: int = 0, seq_end: Optional[int] = None) -> torch.Tensor:
    """Split-K partial records of decode attention.  q is [G, D] (one query
    per cache group) or [G, n_q, D] (grouped-query attention: n_q query heads
    share each cache group; records cover G * n_q query rows).  Rows of cache
    group g are rows [g * seq_len + seq_begin, g * seq_len + seq_end)."""
    _require_cuda(q, k.norms, v.norms, partials)
    if q.dim() == 2:
        G, D = q.shape
        n_q = 1
    else:
        G, n_q, D = q.shape
    seq_end = seq_len if seq_end is None else seq_end
    if not (k.residual and v.residual):
        raise ValueError("decode attention needs caches compressed with the residual plane")
    qf = q if (q.dtype == torch.float32 and q.is_contiguous()) else \
        q.to(torch.float32).contiguous()
    dkh, ch = _host_f32(dk), _host_f32(centroids)
    ext().decode_partial(qf, k.code, k.res, k.norms, k.rnorms, v.code, v.res, v.norms,
                         v.rnorms, seq_len, seq_begin, seq_end, dkh, ch, float(sm_scale),
                         n_splits, partials, part_stride, part_offset)
    return partials


def decode_combine(partials: torch.Tensor, n_parts: int, dv, out: torch.Tensor) -> torch.Tensor:
    """Merge split-K records into out ([R, D] or [G, n_q, D]: one row per
    query row of the records)."""
    _require_cuda(partials, out)
    D = out.shape[-1]
    R = out.numel() // D if D else 0
    ext().decode_combine(partials, R, n_parts, n_parts * (D + 2), D + 2, _host_f32(dv), out)
    return out


def _record_view(records: torch.Tensor, D: int):
    """(rows, parts, row stride, part stride) of a [R, P, D+2] float32 record
    view whose last dimension is contiguous."""
    if records.dtype != torch.float32 or records.dim() != 3 or records.shape[2] != D + 2:
        raise ValueError(f"records must be float32 [R, P, {D + 2}], got "
                         f"{records.dtype} {tuple(records.shape)}")
    if records.stride(2) != 1:
        raise ValueError("records must be contiguous in their last dimension")
    return records.shape[0], records.shape[1], records.stride(0), records.stride(1)


def decode_combine_records(records: torch.Tensor, dv, out: torch.Tensor) -> torch.Tensor:
    """decode_combine over a strided [R, P, D+2] record view (for example the
    transpose of records gathered as [world, R, D+2])."""
    _require_cuda(records, out)
    D = out.shape[-1]
    R, P, gs, ps = _record_view(records, D)
    if out.numel() != R * D:
        raise ValueError(f"out holds {out.numel()} values, records describe {R} x {D}")
    ext().decode_combine(records, R, P, gs, ps, _host_f32(dv), out)
    return out


def decode_merge(records: torch.Tensor, merged: torch.Tensor) -> torch.Tensor:
    """Merge the P records of each row of a [R, P, D+2] view into one record
    per row: merged [R, D+2], still in the rotated domain."""
    _require_cuda(records, merged)
    D = merged.shape[-1] - 2
    R, P, gs, ps = _record_view(records, D)
    if merged.numel() != R * (D + 2) or not merged.is_contiguous():
        raise ValueError(f"merged must be a contiguous float32 [{R}, {D + 2}]")
    if R:
        ext().decode_merge(records, R, P, gs, ps, merged)
    return merged


def decode_attention(q: torch.Tensor, k: PackedKV, v: PackedKV, dk, dv, centroids,
                     sm_scale: Optional[float] = None, n_splits: Optional[int] = None,
                     workspace: Optional[torch.Tensor] = None,
                     seq_len: Optional[int] = None, length: Optional[int] = None
                     ) -> torch.Tensor:
    """softmax(score * sm_scale) . V_hat.  q is [G, D] or [G, n_q, D]
    (n_q query heads per cache group, without expanding the cache).  The
    cache holds G groups of seq_len rows (default: all rows split evenly);
    the first `length` rows of each group (default seq_len) are attended.
    Returns float32 with q's shape."""
    dev = _require_cuda(q, k.norms, v.norms)
    G, D = q.shape[0], q.shape[-1]
    n_q = 1 if q.dim() == 2 else q.shape[1]
    S = k.n_rows // max(G, 1) if seq_len is None else int(seq_len)
    if G * S != k.n_rows or v.n_rows != k.n_rows:
        raise ValueError("K/V caches do not hold G * seq_len rows")
    L = S if length is None else int(length)
    if not 0 <= L <= S:
        raise ValueError("length must be within [0, seq_len]")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if n_splits is None:
        n_splits = default_splits(G * n_q, L, dev, n_q)
    if not (k.residual and v.residual):
        raise ValueError("decode attention needs caches compressed with the residual plane")
    if workspace is None:
        return ext().decode_attention(q, k.code, k.res, k.norms, k.rnorms, v.code, v.res,
                                      v.norms, v.rnorms, S, L, _host_f32(dk), _host_f32(dv),
                                      _host_f32(centroids), float(sm_scale), n_splits)
    need = decode_workspace_bytes(G * n_q, n_splits, D)
    if workspace.numel() * workspace.element_size() < need:
        raise ValueError(f"workspace holds fewer than the {need} bytes needed")
    out = torch.empty(q.shape, dtype=torch.float32, device=dev)
    decode_partial(q, k, v, dk, dv, centroids, sm_scale, n_splits, workspace, n_splits, 0, S,
                   0, L)
    return decode_combine(workspace, n_splits, dv, out)


def ultra_fused_full_fusion(x: torch.Tensor, d, centroids):
    """Compatibility op with the reference kernel's outputs
    (KudaHitamCUDA.cu:197-231): (idx uint8 [N, D], norms [N, 1],
    k_mse float32 [N, D], r_norms [N, 1], signs int8 [N, D]).  Accepts
    fp16 (like the reference) and also fp32 / bf16."""
    _require_cuda(x)
    if x.dtype not in _DTYPE_CODE:
        raise TypeError(f"unsupported dtype {x.dtype}")
    if x.shape[-1] not in HEAD_DIMS:
        raise ValueError(f"head_dim must be 128 or 256, got {x.shape[-1]}")
    return tuple(ext().ultra_fused_full_fusion(x, _host_f32(d), _host_f32(centroids)))


def ultra_fused_hbba_fusion(x: torch.Tensor, d, centroids_table: torch.Tensor,
                            mask: torch.Tensor, layer_id: int, active_mask: int):
    """The HBBA encoder with the reference binding's arguments and outputs
    (ultra_fused_hbba_fusion, KudaHitamCUDA.cu:397-420): x [N, D] (fp16 as in
    the reference; bf16 / fp32 accepted), d [D], centroids_table [D, 16],
    mask int32 [8].  Returns (packed uint8 [N, 128 or 32], norms [N, 1],
    r_norms [N], signs fp16 [N, D])."""
    dev = _require_cuda(x)
    if x.dim() != 2 or x.shape[-1] not in HEAD_DIMS:
        raise ValueError("x must be [N, D] with D in (128, 256)")
    if x.dtype not in _DTYPE_CODE:
        raise TypeError(f"unsupported dtype {x.dtype}")
    d = torch.as_tensor(d).to(dev)
    return tuple(ext().ultra_fused_hbba_fusion(x, d, centroids_table.to(dev), mask.to(dev),
                                               int(layer_id), int(active_mask)))


def hbba_calibrate(sample: torch.Tensor, n_map, layer_id: int, active_mask: int) -> torch.Tensor:
    """Per-dimension levels for the HBBA encoder (hbba_calibrate_cuda,
    KudaHitamCUDA.cu:498-516): sample [N, D] on the GPU, n_map [D] levels
    (2 or 16).  Returns float32 [D, 16]; zeros when bit layer_id of
    active_mask is clear, as the reference does."""
    _require_cuda(sample)
    return ext().hbba_calibrate_cuda(sample, torch.as_tensor(n_map).to(sample.device),
                                     int(layer_id), int(active_mask))


def fused_asymmetric_attention(q: torch.Tensor, k_packed: torch.Tensor, signs: torch.Tensor,
                               d_vec: torch.Tensor, k_norms: torch.Tensor,
                               r_norms: torch.Tensor, centroids: torch.Tensor,
                               layer_id: int, active_mask: int, scale: float) -> torch.Tensor:
    """The reference's packed-cache scorer, same arguments and result
    (fused_asymmetric_attention, KudaHitamCUDA.cu:774-797): q fp16 [H, D],
    k_packed uint8 [H, S, 32 or 128], signs fp16 [H, S, D], d_vec float32
    [D], k_norms / r_norms float32 [H, S], centroids float32 [D, 16].
    Returns float32 [H, S]:  sum_i q~_i c[i][v_i] k_norm + k_norm * scale *
    (q . signs) * r_norm  with q~ = H(q (.) d)/sqrt(D).  Inputs of another
    dtype are converted; non-contiguous inputs are copied."""
    _require_cuda(q, k_packed, signs, d_vec, k_norms, r_norms, centroids)
    H, D = q.shape
    S = k_norms.shape[1]
    nib = 0 <= layer_id < 8 and ((int(active_mask) & 0xFF) >> layer_id) & 1
    bpt = 128 if nib else 32
    if k_packed.shape[0] != H or k_packed.shape[1] != S or k_packed.shape[-1] != bpt:
        raise ValueError(f"k_packed must be [H, S, {bpt}] for this layer")
    if signs.shape != (H, S, D) or r_norms.shape != (H, S) or centroids.shape != (D, 16):
        raise ValueError("signs [H, S, D], r_norms [H, S] and centroids [D, 16] expected")

    return ext().fused_asymmetric_attention(q, k_packed, signs, d_vec, k_norms, r_norms,
                                            centroids, int(layer_id), int(active_mask),
                                            float(scale))

