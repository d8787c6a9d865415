"""The decode step with the record exchange fused into the partial kernel
(kh_decode_partial_to_peers, with its merge into the output either inside
the same kernel or by kh_decode_combine_peer_records), on one GPU through the
C ABI.

Two ranks are emulated in stream order: "rank" r holds rows
[r S/2, (r+1) S/2) of every group, and its partial kernel stores its split
records into slot [r] of both ranks' record buffers (two local allocations
standing in for the symmetric buffers) and raises its epoch flag in both flag
arrays.  The last "rank" (or a separate combine call) merges the records:
its flag wait covers its own flag, raised by its own last CTA, and the other
rank's, raised by a kernel that completed earlier in the stream.  The
result must match the all-gather path's arithmetic on the same two shards
(local partial kernels, per-rank merge, strided combine) within 1e-6
normwise (only the merge order differs), and the single-GPU decode of the
whole sequence within 1e-4, the tolerance of the multi-GPU decode tests (each
shard quantises its V histograms in its own segments), call after call with
alternating buffer sets, and leave the device error word clear."""
import ctypes
import math

import pytest
import torch

import khtest as K
from kudahitam import _lib, lloyd_max, ops, rademacher

pytestmark = pytest.mark.gpu


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("bits,n_q", [(1, 1), (1, 2), (2, 1)])
def test_fused_partial_to_peers_two_emulated_ranks(bits, n_q, fused):
    L = _lib.lib()
    D, G, S, n_splits, world = 128, 12, 6000, 3, 2
    dk, dv, c = rademacher(D, 5), rademacher(D, 6), lloyd_max(bits, D)
    g = torch.Generator(device="cuda").manual_seed(3)
    k = torch.randn(G, S, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(G, S, D, device="cuda", generator=g).to(torch.bfloat16)
    half = S // world
    shards = [(ops.compress(k[:, r * half:(r + 1) * half].contiguous(), dk, c),
               ops.compress(v[:, r * half:(r + 1) * half].contiguous(), dv, c))
              for r in range(world)]
    pk_all, pv_all = ops.compress(k, dk, c), ops.compress(v, dv, c)
    R = G * n_q
    rec_floats = world * R * n_splits * (D + 2)
    recs = [[torch.full((rec_floats,), float("nan"), device="cuda") for _ in range(world)]
            for _ in range(2)]  # [buffer set][rank]
    flags = [[torch.zeros(world, dtype=torch.int32, device="cuda") for _ in range(world)]
             for _ in range(2)]
    counters = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(world)]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dkh, dvh = dk.numpy(), dv.numpy()
    ch = c.numpy()
    sm = ctypes.c_float(1.0 / math.sqrt(D))
    for epoch in range(1, 5):
        par = epoch & 1
        q = torch.randn(G, n_q, D, device="cuda", generator=g)
        outs = [torch.full((R, D), float("nan"), device="cuda") for _ in range(world)]
        for r in range(world):
            pk, pv = shards[r]
            st = L.kh_decode_partial_to_peers(
                _vp(q), G, n_q, D, _vp(pk.code), _vp(pk.res), _vp(pk.norms), _vp(pk.rnorms),
                _vp(pv.code), _vp(pv.res), _vp(pv.norms), _vp(pv.rnorms), half, 0, half,
                dkh.ctypes.data_as(ctypes.c_void_p), dvh.ctypes.data_as(ctypes.c_void_p),
                ch.ctypes.data_as(ctypes.c_void_p), c.numel(), sm, n_splits,
                _ptrs(recs[par]), _ptrs(flags[par]), r, world, epoch, _vp(counters[r]),
                _vp(outs[r]) if (fused and r == world - 1) else None, stream)
            assert st == _lib.KH_OK, st
        out = outs[world - 1]
        if not fused:
            st = L.kh_decode_combine_peer_records(_vp(recs[par][0]), _vp(flags[par][0]), epoch,
                                                  R, n_splits, world, D,
                                                  dvh.ctypes.data_as(ctypes.c_void_p), _vp(out),
                                                  stream)
            assert st == _lib.KH_OK, st
        # the all-gather path's arithmetic on the same shards
        merged = torch.empty(world, R, D + 2, device="cuda")
        for r in range(world):
            pk, pv = shards[r]
            local = torch.empty(R, n_splits, D + 2, device="cuda")
            ops.decode_partial(q, pk, pv, dk, dv, c, 1 / math.sqrt(D), n_splits, local,
                               n_splits, 0, half)
            ops.decode_merge(local, merged[r])
        sharded = ops.decode_combine_records(merged.transpose(0, 1), dv,
                                             torch.empty(R, D, device="cuda"))
        want = ops.decode_attention(q, pk_all, pv_all, dk, dv, c, 1 / math.sqrt(D))
        torch.cuda.synchronize()
        assert _lib.device_error() == 0
        assert torch.isfinite(out).all(), epoch
        got = out.cpu().numpy()
        assert K.normwise(got, sharded.cpu().numpy()) < 1e-6, epoch
        assert K.normwise(got, want.reshape(R, D).cpu().numpy()) < 1e-4, epoch
        # both ranks' counters returned to zero; both flag arrays carry epoch
        assert all(int(cn.item()) == 0 for cn in counters)
        assert all(torch.equal(f.cpu(), torch.full((world,), epoch, dtype=torch.int32))
                   for f in flags[par])


def test_fused_partial_to_peers_rejects_the_direct_kernel_case():
    """D = 256 with the 4-level codebook runs the direct kernel, which has no
    peer mode: KH_ENOTSUP, and nothing is launched."""
    L = _lib.lib()
    D, G, S = 256, 2, 64
    dk, c = rademacher(D, 1), lloyd_max(2, D)
    x = torch.randn(G, S, D, device="cuda").to(torch.bfloat16)
    pk = ops.compress(x, dk, c)
    q = torch.randn(G, D, device="cuda")
    buf = torch.zeros(G * 2 * (D + 2), device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    dkh, ch = dk.numpy(), c.numpy()
    st = L.kh_decode_partial_to_peers(
        _vp(q), G, 1, D, _vp(pk.code), _vp(pk.res), _vp(pk.norms), _vp(pk.rnorms),
        _vp(pk.code), _vp(pk.res), _vp(pk.norms), _vp(pk.rnorms), S, 0, S,
        dkh.ctypes.data_as(ctypes.c_void_p), dkh.ctypes.data_as(ctypes.c_void_p),
        ch.ctypes.data_as(ctypes.c_void_p), 4, ctypes.c_float(0.1), 2, _ptrs([buf]),
        _ptrs([flag]), 0, 1, 1, _vp(cnt), None,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.KH_ENOTSUP
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
