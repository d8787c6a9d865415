"""Stream ordering of the programmatically launched kernels.

The compressors, the score-table kernel and the decode kernels are launched
with programmatic stream serialisation: their CTAs may start while the
previous kernel in the stream is still running, and each waits for that
kernel's completion before its first read of global memory.  These tests
chain dependent calls on one stream with no synchronisation in between (a
torch kernel writing the compressor's input, two compressions into the same
buffers, scores and decode attention reading the fresh cache) and require
results bitwise equal to the same calls run one at a time."""
import math

import pytest
import torch

from kudahitam import ops
from kudahitam.codebook import lloyd_max, rademacher

pytestmark = pytest.mark.gpu


def _same(a: ops.PackedKV, b: ops.PackedKV):
    assert torch.equal(a.code, b.code)
    assert torch.equal(a.norms, b.norms)
    if a.res is not None:
        assert torch.equal(a.res, b.res)
        assert torch.equal(a.rnorms, b.rnorms)


@pytest.mark.parametrize("dtype,D", [(torch.float16, 256), (torch.bfloat16, 128),
                                     (torch.float32, 128)])
def test_chained_compress_and_score_match_serial(dtype, D):
    G, S = 32, 8192
    d, c = rademacher(D, 3), lloyd_max(1, D)
    g = torch.Generator(device="cuda").manual_seed(11)
    x0 = torch.randn(G, S, D, device="cuda", generator=g).to(dtype)
    x1 = torch.randn(G, S, D, device="cuda", generator=g).to(dtype)
    q = torch.randn(G, 1, D, device="cuda", generator=g)
    ref1 = ops.compress(x1, d, c)
    torch.cuda.synchronize()
    s_ref = ops.score(q, ref1, d, c)
    torch.cuda.synchronize()
    for _ in range(3):
        y = torch.empty_like(x0)
        out = ops.empty_packed((G, S, D), 1, True, x0.device)
        y.copy_(x0)
        ops.compress(y, d, c, out=out)  # into the buffers the next call rewrites
        y.copy_(x1)                     # a torch kernel writes the next input
        ops.compress(y, d, c, out=out)
        s = ops.score(q, out, d, c)     # reads the fresh cache at once
        torch.cuda.synchronize()
        _same(out, ref1)
        assert torch.equal(s, s_ref)


def test_chained_compress_and_decode_match_serial():
    G, S, D = 64, 6000, 128
    dk, dv, c = rademacher(D, 10), rademacher(D, 11), lloyd_max(1, D)
    g = torch.Generator(device="cuda").manual_seed(12)
    k = torch.randn(G, S, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(G, S, D, device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn(G, D, device="cuda", generator=g)
    pk, pv = ops.compress(k, dk, c), ops.compress(v, dv, c)
    torch.cuda.synchronize()
    want = ops.decode_attention(q, pk, pv, dk, dv, c, 1 / math.sqrt(D), n_splits=3)
    torch.cuda.synchronize()
    for _ in range(3):
        ok = ops.empty_packed((G, S, D), 1, True, k.device)
        ov = ops.empty_packed((G, S, D), 1, True, k.device)
        ops.compress(k, dk, c, out=ok)
        ops.compress(v, dv, c, out=ov)
        got = ops.decode_attention(q, ok, ov, dk, dv, c, 1 / math.sqrt(D), n_splits=3)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
