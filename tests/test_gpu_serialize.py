"""KHPK file round trip of a cache compressed on the GPU: compress, save to a
file, read it back onto the device, and score and decode from the reloaded
cache -- bitwise equal to the same calls on the in-memory cache (the planes,
norms, d and centroids all survive the file exactly)."""
import pytest
import torch

from kudahitam import KudahitamCompressorV2, ops
from kudahitam import serialize as S

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (256, torch.float16)])
def test_khpk_round_trip_scores_and_decode_bitwise(tmp_path, D, dtype):
    G, Sq = 6, 3000
    comp = KudahitamCompressorV2(D, 1, seed=5)
    vcomp = KudahitamCompressorV2(D, 1, seed=6)
    g = torch.Generator(device="cuda").manual_seed(3)
    k = torch.randn(1, G, Sq, D, device="cuda", generator=g).to(dtype)
    v = torch.randn(1, G, Sq, D, device="cuda", generator=g).to(dtype)
    ck, cv = comp.compress(k), vcomp.compress(v)
    S.save(str(tmp_path / "k.khpk"), ck.packed, comp.d, comp.centroids)
    S.save(str(tmp_path / "v.khpk"), cv.packed, vcomp.d, vcomp.centroids)
    pk, dk, c = S.read(str(tmp_path / "k.khpk"), device="cuda")
    pv, dv, cv_c = S.read(str(tmp_path / "v.khpk"), device="cuda")
    for a, b in ((pk, ck.packed), (pv, cv.packed)):
        assert a.shape == b.shape and a.bits == b.bits
        for f in ("code", "res", "norms", "rnorms"):
            assert torch.equal(getattr(a, f), getattr(b, f)), f
    assert torch.equal(dk, comp.d.cpu()) and torch.equal(dv, vcomp.d.cpu())
    assert torch.equal(c.view(torch.int32), comp.centroids.cpu().view(torch.int32))

    q = torch.randn(G, 2, D, device="cuda", generator=g)
    s_mem = ops.score(q, ck.packed, comp.d, comp.centroids, seq_len=Sq)
    s_file = ops.score(q, pk, dk, c, seq_len=Sq)
    assert torch.equal(s_mem, s_file)
    o_mem = ops.decode_attention(q, ck.packed, cv.packed, comp.d, vcomp.d, comp.centroids,
                                 seq_len=Sq)
    o_file = ops.decode_attention(q, pk, pv, dk, dv, c, seq_len=Sq)
    assert torch.equal(o_mem, o_file)
