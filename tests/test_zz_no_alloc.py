"""kh_decode_attn_static: decode attention for callers that cannot allocate
device memory when they call (a server whose memory is all reserved in its own
pool, a C/FFI caller holding only the buffers it was given).  Its split-K
scratch is a fixed array inside the library, so the call takes no workspace.

Checked through the C ABI against kh_decode_attn (which takes a caller
workspace) on two calls in a row, with different queries, so a stale record
left in the shared array by the first call would show up in the second.  This
file is named to be collected last."""
import ctypes
import math

import pytest
import torch

from kudahitam import _lib, lloyd_max, ops, rademacher

pytestmark = pytest.mark.gpu


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def _args(q, pk, pv, dk, dv, c, S):
    G, D = q.shape
    return [_vp(q), G, D, _vp(pk.code), _vp(pk.res), _vp(pk.norms), _vp(pk.rnorms),
            _vp(pv.code), _vp(pv.res), _vp(pv.norms), _vp(pv.rnorms), S, _vp(dk), _vp(dv),
            _vp(c), c.numel(), ctypes.c_float(1.0 / math.sqrt(D))]


def test_static_scratch_matches_workspace_entry_point():
    L = _lib.lib()
    D, G, S, n_splits = 128, 48, 3000, 8
    dk, dv = rademacher(D, 21), rademacher(D, 22)
    c = lloyd_max(1, D)
    g = torch.Generator(device="cuda").manual_seed(7)
    k = torch.randn(G, S, D, device="cuda", generator=g, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn(G, S, D, device="cuda", generator=g, dtype=torch.float32).to(torch.bfloat16)
    pk = ops.compress(k, dk, c)
    pv = ops.compress(v, dv, c)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    need = L.kh_decode_workspace_bytes(G, n_splits, D)
    assert 0 < need <= _lib.DECODE_STATIC_SCRATCH_BYTES
    for call in range(2):
        q = torch.randn(G, D, device="cuda", generator=g)
        ws = torch.empty(need // 4, device="cuda")
        ref = torch.empty(G, D, device="cuda")
        got = torch.full((G, D), float("nan"), device="cuda")
        a = _args(q, pk, pv, dk, dv, c, S)
        assert L.kh_decode_attn(*a, n_splits, _vp(ws), need, _vp(ref), stream) == 0
        assert L.kh_decode_attn_static(*a, n_splits, _vp(got), stream) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), call
        assert torch.allclose(got, ref, rtol=1e-4, atol=1e-6), call


def test_static_scratch_at_its_capacity_edge():
    """The largest request that fits the array (D = 128: 1613 groups x 5
    splits x 130 floats = 4,193,800 bytes, 504 bytes under the cap) matches
    the workspace entry point; one more group of records (8066 x 1 x 130
    floats = the cap + 16 bytes) is refused before any GPU work; zero groups
    is a no-op even with null pointers."""
    L = _lib.lib()
    cap = _lib.DECODE_STATIC_SCRATCH_BYTES
    D, S = 128, 64
    dk, dv = rademacher(D, 31), rademacher(D, 32)
    c = lloyd_max(1, D)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    G, n_splits = 1613, 5
    need = L.kh_decode_workspace_bytes(G, n_splits, D)
    assert need <= cap and L.kh_decode_workspace_bytes(G + 1, n_splits, D) > cap
    g = torch.Generator(device="cuda").manual_seed(11)
    k = torch.randn(G, S, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(G, S, D, device="cuda", generator=g).to(torch.bfloat16)
    pk, pv = ops.compress(k, dk, c), ops.compress(v, dv, c)
    q = torch.randn(G, D, device="cuda", generator=g)
    ws = torch.empty(need // 4, device="cuda")
    ref = torch.empty(G, D, device="cuda")
    got = torch.full((G, D), float("nan"), device="cuda")
    a = _args(q, pk, pv, dk, dv, c, S)
    assert L.kh_decode_attn(*a, n_splits, _vp(ws), need, _vp(ref), stream) == 0
    assert L.kh_decode_attn_static(*a, n_splits, _vp(got), stream) == 0
    torch.cuda.synchronize()
    assert torch.allclose(got, ref, rtol=1e-4, atol=1e-6)

    over = L.kh_decode_workspace_bytes(8066, 1, D)
    assert over == cap + 16
    before = got.clone()
    a8066 = [_vp(q), 8066] + a[2:]
    assert L.kh_decode_attn_static(*a8066, 1, _vp(got), stream) == _lib.KH_EINVAL
    a0 = [None, 0, D] + [None] * 8 + [S, _vp(dk), _vp(dv), _vp(c), 2,
                                       ctypes.c_float(1.0 / math.sqrt(D))]
    assert L.kh_decode_attn_static(*a0, 1, None, stream) == 0
    torch.cuda.synchronize()
    assert torch.equal(got, before)  # neither call touched the output


def test_static_scratch_rejects_oversized_requests():
    L = _lib.lib()
    D = 256
    c = lloyd_max(1, D)
    d = rademacher(D, 0)
    G = 4096
    n_splits = 64
    assert L.kh_decode_workspace_bytes(G, n_splits, D) > _lib.DECODE_STATIC_SCRATCH_BYTES
    dummy = torch.zeros(16, device="cuda")
    p = _vp(dummy)
    st = L.kh_decode_attn_static(p, G, D, p, p, p, p, p, p, p, p, 1000, _vp(d), _vp(d), _vp(c),
                                 2, ctypes.c_float(0.1), n_splits, p, None)
    assert st == _lib.KH_EINVAL
