"""Scores and decode attention read from the packed cache, against the
oracle (the reference's score function, KudaHitamQuant_full.py:373-377) and
the reference-generated golden scores.  Tolerance: normwise per group
max|est - ref| / max|ref| <= 1e-3 (asserted tighter where the arithmetic
allows)."""
import math

import numpy as np
import pytest
import torch

import khtest as K
from kudahitam import KudahitamCompressorV2, fwht, load_cuda_ext, lloyd_max, ops, rademacher
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["d128_fp32_b1", "d128_fp32_b2", "d256_fp16_b1",
                                  "d256_fp16_b2"])
def test_scores_match_reference_golden(case):
    g = K.golden(f"compress_{case}.npz")
    B, H, S, D = g["x"].shape
    bits = 1 if len(g["c"]) == 2 else 2
    comp = KudahitamCompressorV2(D, bits, seed=7)
    out = comp.compress(torch.from_numpy(g["x"]).cuda())
    sc = comp.asymmetric_attention_scores(torch.from_numpy(g["q"]).cuda(), out)
    assert sc.shape == g["scores"].shape and sc.dtype == torch.float32
    got = sc.cpu().numpy().reshape(B * H, -1)
    ref = g["scores"].reshape(B * H, -1)
    for gi in range(B * H):
        assert K.normwise(got[gi], ref[gi]) < 1e-4


@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("bits", [1, 2])
@pytest.mark.parametrize("residual", [True, False])
def test_scores_match_oracle(D, bits, residual):
    if bits == 2 and not residual:
        pytest.skip("1-bit mode uses the 2-level codebook")
    G, S, nq = 6, 333, 3
    d = rademacher(D, 3).numpy()
    c = lloyd_max(bits, D).numpy()
    x = K.synth((1, G, S, D), dtype=torch.bfloat16, seed=9)
    q = torch.randn(G, nq, D, generator=torch.Generator().manual_seed(1))
    p = ops.compress(x.cuda(), d, c, residual=residual)
    got = ops.score(q.cuda(), p, d, c, seq_len=S).cpu().numpy()
    # the score kernel alone: the reference formula on this cache's own
    # materialised k_mse / signs
    m = ops.materialize(p, d, c)
    own = O.score(q.numpy(), m["kmse"].cpu().numpy().reshape(G, S, D),
                  m["signs"].cpu().numpy().reshape(G, S, D) if residual else None,
                  p.rnorms.cpu().numpy().reshape(G, S) if residual else None, d)
    errs = [K.normwise(got[gi], own[gi]) for gi in range(G)]
    assert max(errs) < 1e-4, f"score kernel vs its own cache: {errs}"
    # end to end against the oracle's own compression: rows holding an element
    # on a decision boundary (|y - b| <= 1e-6, where either rounding is
    # correct) may quantise differently, so they are left out here; the
    # check above covers every row
    ref = O.compress_v8(x, d, c)
    want = O.score(q.numpy(), ref["kmse"].reshape(G, S, D),
                   ref["signs"].reshape(G, S, D) if residual else None,
                   ref["rnorms"].reshape(G, S) if residual else None, d)
    y = K.projected(x.float().numpy().reshape(-1, D), d)
    decided = K.res_mask(y, ref["idx"].astype(np.int64), c).all(1).reshape(G, S)
    assert decided.mean() > 0.97  # bits=2 has three boundaries per element
    errs = [K.normwise(got[gi][:, decided[gi]], want[gi][:, decided[gi]]) for gi in range(G)]
    assert max(errs) < 1e-4, f"engine vs oracle: {errs}"


@pytest.mark.parametrize("bits,residual", [(1, True), (1, False), (2, True)])
def test_table_scores_span_several_ctas_and_equal_direct_kernel(bits, residual, monkeypatch):
    """Groups longer than one table CTA (8192 rows) with a ragged tail, two
    queries per group: the table-driven kernel (the 2-bit-plane variant for
    the bits=2 codebook) against the direct bit-select kernel and against
    the reference formula on the same cache."""
    D, G, S, nq = 128, 2, 2 * 8192 + 1234, 2
    d, c = rademacher(D, 4).numpy(), lloyd_max(bits, D).numpy()
    x = K.synth((1, G, S, D), dtype=torch.bfloat16, seed=12)
    q = torch.randn(G, nq, D, generator=torch.Generator().manual_seed(2)).cuda()
    p = ops.compress(x.cuda(), d, c, residual=residual)
    tab = ops.score(q, p, d, c, seq_len=S).cpu().numpy()
    monkeypatch.setenv("KUDAHITAM_SCORE_PATH", "direct")
    direct = ops.score(q, p, d, c, seq_len=S).cpu().numpy()
    m = ops.materialize(p, d, c)
    own = O.score(q.cpu().numpy(), m["kmse"].cpu().numpy().reshape(G, S, D),
                  m["signs"].cpu().numpy().reshape(G, S, D) if residual else None,
                  p.rnorms.cpu().numpy().reshape(G, S) if residual else None, d)
    for gi in range(G):
        assert K.normwise(tab[gi], own[gi]) < 1e-4
        assert K.normwise(tab[gi], direct[gi]) < 1e-5


def test_gqa_scores_share_kv_heads():
    D, S = 128, 200
    comp = KudahitamCompressorV2(D, 1, seed=0)
    k = torch.randn(2, 2, S, D, device="cuda", dtype=torch.float16)
    ck = comp.compress(k)
    q = torch.randn(2, 8, 1, D, device="cuda")   # 4 query heads per KV head
    sc = comp.asymmetric_attention_scores(q, ck)
    assert sc.shape == (2, 8, 1, S)
    for h in range(8):
        ck1 = comp.compress(k[:, h // 4:h // 4 + 1].contiguous())
        one = comp.asymmetric_attention_scores(q[:, h:h + 1], ck1)
        assert torch.allclose(sc[:, h:h + 1], one, rtol=0, atol=1e-5)


def test_fwht_matches_oracle_and_reference_forward():
    for D in (2, 4, 8, 64, 128, 256, 1024):
        x = torch.randn(37, D)
        got = fwht(x.cuda()).cpu().numpy()
        exact = x.double().numpy() @ K.hadamard(D).T / math.sqrt(D)
        assert K.normwise(got, exact) < 1e-6, D
        if D >= 8:  # the reference `forward` kernel needs D >= 8
            assert K.normwise(got, O.fwht_forward(x.numpy())) < 1e-6, D
    ext = load_cuda_ext()
    y = torch.randn(5, 128, device="cuda")
    y0 = y.clone()
    ext.forward(y)
    assert torch.allclose(y, torch.tensor(O.fwht_forward(y0.cpu().numpy()), device="cuda"),
                          atol=1e-6)


@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("bits", [1, 2])
def test_materialize_and_compat_op(D, bits):
    d = rademacher(D, 8).numpy()
    c = lloyd_max(bits, D).numpy()
    x = K.synth((1, 2, 50, D), dtype=torch.float16, seed=4)
    idx, norms, kmse, rn, signs = load_cuda_ext().ultra_fused_full_fusion(
        x.cuda().view(-1, D), torch.tensor(d).cuda(), torch.tensor(c).cuda())
    n = 100
    assert idx.shape == (n, D) and norms.shape == (n, 1) and kmse.shape == (n, D)
    assert rn.shape == (n, 1) and signs.shape == (n, D) and signs.dtype == torch.int8
    ref = O.compress_v8(x, d, c)
    y = K.projected(x.float().numpy().reshape(n, D), d)
    m = K.idx_mask(y, c)
    assert np.array_equal(idx.cpu().numpy()[m], ref["idx"][m])
    rm = K.res_mask(y, ref["idx"].astype(np.int64), c)
    assert np.array_equal(signs.cpu().numpy()[rm], ref["signs"][rm])
    assert K.normwise(kmse.cpu().numpy(), ref["kmse"]) < 1e-5
    assert K.rel_err(rn.cpu().numpy()[:, 0], ref["rnorms"]) < 1e-4


@pytest.fixture(params=["v3", "v2", "v1"])
def decode_path(request, monkeypatch):
    """Decode kernel: segment-exact table-driven (default), chunked
    table-driven, or the direct one."""
    monkeypatch.setenv("KUDAHITAM_DECODE_PATH", request.param)
    return request.param


def _caches(G, S, D, seed):
    dk = rademacher(D, 10).numpy()
    dv = rademacher(D, 11).numpy()
    c = lloyd_max(1, D).numpy()
    k = K.synth((1, G, S, D), dtype=torch.bfloat16, seed=seed)
    v = K.synth((1, G, S, D), dtype=torch.bfloat16, seed=seed + 1)
    return dk, dv, c, k, v


@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("S", [1, 7, 300, 1000, 5000])
def test_decode_attention_matches_oracle(D, S, decode_path):
    G = 5
    dk, dv, c, k, v = _caches(G, S, D, seed=S)
    q = torch.randn(G, D, generator=torch.Generator().manual_seed(S)).to(torch.bfloat16)
    pk = ops.compress(k.cuda(), dk, c)
    pv = ops.compress(v.cuda(), dv, c)
    sm = 1.0 / math.sqrt(D)
    rk = O.compress_v8(k, dk, c)
    rv = O.compress_v8(v, dv, c)
    want = O.decode(q.float().numpy(), rk["kmse"].reshape(G, S, D), rk["signs"].reshape(G, S, D),
                    rk["rnorms"].reshape(G, S), rv["kmse"].reshape(G, S, D),
                    rv["signs"].reshape(G, S, D), rv["rnorms"].reshape(G, S), dk, dv, sm)
    for n_splits in (1, 3, 16):
        got = ops.decode_attention(q.cuda(), pk, pv, dk, dv, c, sm, n_splits=n_splits)
        got = got.cpu().numpy()
        for gi in range(G):
            assert K.normwise(got[gi], want[gi]) < 1e-3, (n_splits, gi)


@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("S", [1, 300, 2000, 13000])
def test_decode_bits2_codebook_matches_oracle(D, S, monkeypatch):
    """The 4-level (bits=2) codebook: 2-bit code plane plus the residual
    plane, V reconstructed with c[idx] from four levels (the table kernel at
    D = 128, the direct kernel at D = 256), against the oracle's fp64 decode
    of its own compression; at D = 128 also against the direct kernel."""
    G = 4
    dk, dv = rademacher(D, 10).numpy(), rademacher(D, 11).numpy()
    c = lloyd_max(2, D).numpy()
    k = K.synth((1, G, S, D), dtype=torch.bfloat16, seed=S + 1)
    v = K.synth((1, G, S, D), dtype=torch.bfloat16, seed=S + 2)
    q = torch.randn(G, D, generator=torch.Generator().manual_seed(S)).to(torch.bfloat16)
    pk, pv = ops.compress(k.cuda(), dk, c), ops.compress(v.cuda(), dv, c)
    assert pk.bits == 2
    sm = 1.0 / math.sqrt(D)
    rk, rv = O.compress_v8(k, dk, c), O.compress_v8(v, dv, c)
    want = O.decode(q.float().numpy(), rk["kmse"].reshape(G, S, D), rk["signs"].reshape(G, S, D),
                    rk["rnorms"].reshape(G, S), rv["kmse"].reshape(G, S, D),
                    rv["signs"].reshape(G, S, D), rv["rnorms"].reshape(G, S), dk, dv, sm)
    for n_splits in (1, 3):
        got = ops.decode_attention(q.cuda(), pk, pv, dk, dv, c, sm, n_splits=n_splits)
        got = got.cpu().numpy()
        for gi in range(G):
            assert K.normwise(got[gi], want[gi]) < 1e-3, (n_splits, gi)
        if D == 128:
            monkeypatch.setenv("KUDAHITAM_DECODE_PATH", "v1")  # the direct kernel
            direct = ops.decode_attention(q.cuda(), pk, pv, dk, dv, c, sm, n_splits=n_splits)
            monkeypatch.delenv("KUDAHITAM_DECODE_PATH")
            for gi in range(G):
                assert K.normwise(got[gi], direct.cpu().numpy()[gi]) < 1e-4, (n_splits, gi)


@pytest.mark.parametrize("sm_mult", [1.0, 12.0])
def test_decode_long_splits_and_peaked_softmax(sm_mult, decode_path):
    """Splits longer than one 8192-row segment (online rescaling across
    segments) and a sharply peaked softmax (fixed-point weights dominated by
    a few rows)."""
    D, G, S = 128, 2, 20000
    dk, dv, c, k, v = _caches(G, S, D, seed=11)
    q = torch.randn(G, D, generator=torch.Generator().manual_seed(2)).to(torch.bfloat16)
    sm = sm_mult / math.sqrt(D)
    pk = ops.compress(k.cuda(), dk, c)
    pv = ops.compress(v.cuda(), dv, c)
    rk = O.compress_v8(k, dk, c)
    rv = O.compress_v8(v, dv, c)
    want = O.decode(q.float().numpy(), rk["kmse"].reshape(G, S, D), rk["signs"].reshape(G, S, D),
                    rk["rnorms"].reshape(G, S), rv["kmse"].reshape(G, S, D),
                    rv["signs"].reshape(G, S, D), rv["rnorms"].reshape(G, S), dk, dv, sm)
    for n_splits in (1, 2):
        got = ops.decode_attention(q.cuda(), pk, pv, dk, dv, c, sm, n_splits=n_splits)
        got = got.cpu().numpy()
        for gi in range(G):
            assert K.normwise(got[gi], want[gi]) < 1e-3, (n_splits, gi)


def test_decode_split_invariance_and_empty_splits(decode_path):
    D, G, S = 128, 3, 5
    dk, dv, c, k, v = _caches(G, S, D, seed=1)
    for seed in range(4):
        q = torch.randn(G, D, generator=torch.Generator().manual_seed(seed)).cuda()
        pk = ops.compress(k.cuda(), dk, c)
        pv = ops.compress(v.cuda(), dv, c)
        base = ops.decode_attention(q, pk, pv, dk, dv, c, n_splits=1).cpu().numpy()
        for n in (2, 5, 8, 64):  # 64 splits over 5 rows: most splits are empty
            got = ops.decode_attention(q, pk, pv, dk, dv, c, n_splits=n).cpu().numpy()
            # split-K reassociation only: normwise per group (elementwise
            # checks are meaningless for outputs near zero after the
            # D-term transform)
            for gi in range(G):
                assert K.normwise(got[gi], base[gi]) < 2e-6, (seed, n, gi)


def test_decode_grouped_query_heads_share_the_cache(decode_path):
    """q [G, n_q, D]: every query row reads its group's cache without any
    expansion, and equals the one-query decode of the same row bit for bit."""
    D, G, S, n_q = 128, 3, 2500, 4
    dk, dv, c, k, v = _caches(G, S, D, seed=7)
    pk = ops.compress(k.cuda(), dk, c)
    pv = ops.compress(v.cuda(), dv, c)
    q = torch.randn(G, n_q, D, generator=torch.Generator().manual_seed(5)).cuda()
    got = ops.decode_attention(q, pk, pv, dk, dv, c, n_splits=3)
    assert got.shape == (G, n_q, D)
    for j in range(n_q):
        one = ops.decode_attention(q[:, j].contiguous(), pk, pv, dk, dv, c, n_splits=3)
        assert torch.equal(got[:, j], one), j
    # the compressor API maps H_q = 2 H_kv query heads onto the KV heads
    ck = KudahitamCompressorV2(D, 1, seed=10)
    cv = KudahitamCompressorV2(D, 1, seed=11)
    kk = torch.randn(2, 2, 700, D, device="cuda", dtype=torch.bfloat16)
    vv = torch.randn(2, 2, 700, D, device="cuda", dtype=torch.bfloat16)
    qq = torch.randn(2, 4, D, device="cuda", dtype=torch.bfloat16)
    a = ck.decode_attention(qq, ck.compress(kk), cv.compress(vv), v_compressor=cv)
    b = ck.decode_attention(qq[:, 0::2].contiguous(), ck.compress(kk), cv.compress(vv),
                            v_compressor=cv)  # heads 0, 2 -> KV heads 0, 1
    assert a.shape == (2, 4, D) and torch.equal(a[:, 0::2], b)


def test_decode_capacity_stride_and_length(decode_path):
    """Groups laid out with a capacity stride larger than the filled length
    (an appendable cache): only the first `length` rows are attended."""
    D, G, S, cap = 128, 2, 900, 1500
    dk, dv, c, k, v = _caches(G, cap, D, seed=9)
    pk = ops.compress(k.cuda(), dk, c)
    pv = ops.compress(v.cuda(), dv, c)
    kk = k.view(G, cap, D)[:, :S].contiguous()
    vv = v.view(G, cap, D)[:, :S].contiguous()
    ref = ops.decode_attention(torch.ones(G, D).cuda(), ops.compress(kk.cuda(), dk, c),
                               ops.compress(vv.cuda(), dv, c), dk, dv, c, n_splits=2)
    got = ops.decode_attention(torch.ones(G, D).cuda(), pk, pv, dk, dv, c, n_splits=2,
                               seq_len=cap, length=S)
    assert torch.equal(got, ref)


def test_decode_seq_sharded_emulated_on_one_gpu(decode_path):
    """The multi-GPU combine, with the ranks' slots filled by one process:
    partial records of every S-shard in their own slots, merged once."""
    D, G, S, world, n_splits = 128, 4, 1000, 4, 2
    dk, dv, c, k, v = _caches(G, S, D, seed=3)
    q = torch.randn(G, D, device="cuda")
    kc, vc = k.cuda().view(G, S, D), v.cuda().view(G, S, D)
    parts = world * n_splits
    buf = torch.zeros(G, parts, D + 2, device="cuda")
    from kudahitam.dist import shard_range
    for r in range(world):
        a, b = shard_range(S, world, r)
        pk = ops.compress(kc[:, a:b].contiguous(), dk, c)
        pv = ops.compress(vc[:, a:b].contiguous(), dv, c)
        ops.decode_partial(q, pk, pv, dk, dv, c, 1 / math.sqrt(D), n_splits, buf,
                           part_stride=parts, part_offset=r * n_splits, seq_len=b - a)
    got = ops.decode_combine(buf, parts, dv, torch.empty(G, D, device="cuda"))
    pk = ops.compress(kc, dk, c)
    pv = ops.compress(vc, dv, c)
    want = ops.decode_attention(q, pk, pv, dk, dv, c, 1 / math.sqrt(D), n_splits=8)
    assert torch.allclose(got, want, rtol=1e-4, atol=1e-5)


def test_decode_merge_then_gathered_combine(decode_path):
    """The multi-GPU record path on one GPU: every emulated rank merges its
    own splits into one record per row (kh_decode_merge); the stacked
    [world, G, D+2] records are combined through a transposed, strided view
    (kh_decode_combine_strided).  The last rank owns no rows."""
    D, G, S, world, n_splits = 128, 4, 1000, 4, 3
    dk, dv, c, k, v = _caches(G, S, D, seed=4)
    q = torch.randn(G, D, device="cuda")
    kc, vc = k.cuda().view(G, S, D), v.cuda().view(G, S, D)
    from kudahitam.dist import shard_range
    a_last, _ = shard_range(S, world, world - 1)
    gathered = torch.empty(world, G, D + 2, device="cuda")
    for r in range(world):
        a, b = shard_range(S, world, r)
        if r == world - 1:
            a, b = 0, 0  # an empty shard: its records carry l = 0
        lo, hi = (a, b) if b > a else (0, 1)  # any valid cache for the empty shard
        local = torch.empty(G, n_splits, D + 2, device="cuda")
        pk = ops.compress(kc[:, lo:hi].contiguous(), dk, c)
        pv = ops.compress(vc[:, lo:hi].contiguous(), dv, c)
        ops.decode_partial(q, pk, pv, dk, dv, c, 1 / math.sqrt(D), n_splits, local,
                           part_stride=n_splits, part_offset=0, seq_len=hi - lo,
                           seq_begin=0, seq_end=b - a)
        ops.decode_merge(local, gathered[r])
    assert torch.all(gathered[world - 1, :, 1] == 0)
    got = ops.decode_combine_records(gathered.transpose(0, 1), dv,
                                     torch.empty(G, D, device="cuda"))
    pk = ops.compress(kc[:, :a_last].contiguous(), dk, c)
    pv = ops.compress(vc[:, :a_last].contiguous(), dv, c)
    want = ops.decode_attention(q, pk, pv, dk, dv, c, 1 / math.sqrt(D), n_splits=8)
    assert torch.allclose(got, want, rtol=1e-4, atol=1e-5)


def test_decode_combine_strided_matches_plain():
    """kh_decode_combine is kh_decode_combine_strided with the packed
    strides: bitwise the same output; merging first and combining the one
    merged record gives the same values."""
    D, G, P = 128, 6, 5
    g = torch.Generator(device="cuda").manual_seed(0)
    rec = torch.randn(G, P, D + 2, device="cuda", generator=g)
    rec[..., 1] = rec[..., 1].abs() + 0.1
    rec[2, 1, 1] = 0.0  # an empty split
    dv = torch.ones(D)
    a = ops.decode_combine(rec, P, dv, torch.empty(G, D, device="cuda"))
    b = ops.decode_combine_records(rec, dv, torch.empty(G, D, device="cuda"))
    assert torch.equal(a, b)
    merged = ops.decode_merge(rec, torch.empty(G, D + 2, device="cuda"))
    c = ops.decode_combine_records(merged.view(G, 1, D + 2), dv,
                                   torch.empty(G, D, device="cuda"))
    assert torch.allclose(a, c, rtol=1e-5, atol=1e-6)


def test_compressor_decode_api():
    D = 128
    ck = KudahitamCompressorV2(D, 1, seed=10)
    cv = KudahitamCompressorV2(D, 1, seed=11)
    k = torch.randn(2, 4, 500, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(2, 4, 500, D, device="cuda", dtype=torch.bfloat16)
    q = torch.randn(2, 4, D, device="cuda", dtype=torch.bfloat16)
    out = ck.decode_attention(q, ck.compress(k), cv.compress(v), v_compressor=cv)
    assert out.shape == (2, 4, D)
    # close to exact attention on the uncompressed cache
    att = torch.softmax((q.float().unsqueeze(2) @ k.float().transpose(-1, -2)) / math.sqrt(D), -1)
    exact = (att @ v.float()).squeeze(2)
    cos = torch.nn.functional.cosine_similarity(out.flatten(), exact.flatten(), dim=0)
    assert cos > 0.8
