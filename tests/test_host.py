"""Host-side logic of the Python layer (no GPU)."""
import numpy as np
import pytest
import torch

from kudahitam import KudahitamCompressorV2, lloyd_max, ops
from kudahitam.dist import shard_range


def test_shard_range_partitions():
    for n in (0, 1, 7, 1024, 1023):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            for (a, b), (c, _) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_compressor_signature_and_rejections():
    c = KudahitamCompressorV2(128, 1, seed=3)  # reference defaults
    assert c.d.shape == (128,) and set(c.d.unique().tolist()) <= {-1.0, 1.0}
    assert torch.equal(c.centroids, lloyd_max(1, 128))
    KudahitamCompressorV2(256, 2, 0, use_fractional=True, use_dynamic_codebook=True,
                          use_spectral=True, use_spaced=True, use_ultra=True)
    with pytest.raises(NotImplementedError):
        KudahitamCompressorV2(128, 1, 0, protected_dim_count=8)
    with pytest.raises(NotImplementedError):
        KudahitamCompressorV2(128, 1, 0, is_domain_layer=True)
    KudahitamCompressorV2(128, 1, 0, is_domain_layer=True, use_outlier=False)
    with pytest.raises(NotImplementedError):
        KudahitamCompressorV2(128, 1, 0, use_vwh=True)
    with pytest.raises(ValueError):
        KudahitamCompressorV2(96, 1, 0)
    with pytest.raises(ValueError):
        KudahitamCompressorV2(128, 2, 0, residual=False)


def test_no_cpu_path():
    c = KudahitamCompressorV2(128, 1, seed=0)
    with pytest.raises(ValueError, match="CUDA"):
        c.compress(torch.randn(1, 2, 8, 128))
    with pytest.raises(ValueError, match="CUDA"):
        ops.fwht(torch.randn(4, 128))


def test_packed_layout_shapes():
    p = ops.empty_packed((2, 3, 5, 128), bits=1, residual=True, device="cpu")
    assert p.code.shape == (30, 4) and p.res.shape == (30, 4)
    assert p.nbytes() == 30 * (16 + 16 + 4 + 4)
    p2 = ops.empty_packed((7, 256), bits=2, residual=False, device="cpu")
    assert p2.code.shape == (7, 16) and p2.res is None and p2.rnorms is None
    sub = p.rows(5, 10)
    assert sub.n_rows == 5 and sub.code.data_ptr() == p.code[5].data_ptr()


def test_lloyd_max_other_dims_sorted_symmetric():
    for D in (16, 64, 512):
        for bits in (1, 2, 3):
            c = lloyd_max(bits, D).numpy()
            assert np.all(np.diff(c) > 0)
            assert np.allclose(c, -c[::-1], atol=1e-9)


def test_decode_split_rule():
    """Records per query row on a 148-SM GPU: the kernel cuts (group, row)
    pairs into ranges over one wave of 296 CTAs, none under 8192 pairs; a
    group gets one record per range it touches."""
    from kudahitam.ops import splits_for
    assert [splits_for(512, s, 148) for s in (5000, 10000, 20000, 40000)] == [2, 2, 2, 2]
    assert splits_for(32, 40000, 148) == 6       # one sequence of 32 heads: 157 ranges
    assert splits_for(1024, 131072, 148) == 2
    assert splits_for(512, 100, 148) == 2 and splits_for(0, 0, 148) == 1
    assert splits_for(1, 10 ** 9, 148) == 297
    assert splits_for(64, 4096, 148, n_q=8) == 2  # 8 groups: 4 ranges of 8192
    # the launcher's range is never shorter than L / (n - 1): a group spans at most n ranges
    for R, L, nq in ((512, 40000, 1), (32, 40000, 1), (7, 12345, 1), (64, 9000, 4)):
        n = splits_for(R, L, 148, nq)
        total = (R // nq) * L
        sets = max(1, min(2 * 148 // nq, -(-total // 8192)))
        w = -(-total // sets)
        assert -(-L // w) + 1 <= n


def _launcher_ranges(G, nq, L, n_splits, sms):
    """kh_decode.cu launch_decode_partial: (W, CTA count) of the v3 split."""
    if L == 0:
        return 0, G * nq
    if n_splits == 1:
        return L, G * nq
    total = G * L
    slots = max(1, 2 * sms // nq)
    sets = max(1, min(slots, -(-total // 8192)))
    W = max(-(-total // sets), -(-L // (n_splits - 1)))
    return W, -(-total // W) * nq


def _kernel_writes(G, nq, L, seq_begin, n_splits, W, n_cta):
    """decode_v3_kernel / decode_b2_kernel: record slots written and the
    sequence intervals [s0, s1) each query row's pieces cover, from the
    kernel's index arithmetic."""
    writes, cover = {}, {}
    for b in range(n_cta):
        if W == 0:
            for p in range(n_splits):
                writes.setdefault((b, p), []).append("empty")
            continue
        jq, st = b % nq, b // nq
        wbeg, wend = st * W, min(st * W + W, G * L)
        gk = wbeg // L
        while gk * L < wend:
            g = gk * nq + jq
            s0, s1 = seq_begin + max(wbeg - gk * L, 0), seq_begin + min(wend - gk * L, L)
            assert s1 > s0
            rp = st - gk * L // W
            assert 0 <= rp < n_splits, (G, nq, L, n_splits, W)
            writes.setdefault((g, rp), []).append("rec")
            cover.setdefault(g, []).append((s0, s1))
            if s1 == seq_begin + L:
                for p in range(rp + 1, n_splits):
                    writes.setdefault((g, p), []).append("empty")
            gk += 1
    return writes, cover


def test_decode_work_split_covers_every_row_once():
    import random
    rng = random.Random(0)
    cases = [(512, 1, 40000, 2, 148), (512, 1, 5000, 2, 148), (32, 1, 40000, 6, 148),
             (6, 3, 3000, 2, 148), (48, 1, 3000, 8, 148), (1613, 1, 64, 5, 148),
             (2, 3, 17, 4, 148), (3, 1, 1, 1, 148), (5, 2, 0, 3, 148)]
    cases += [(rng.randint(1, 40), rng.choice([1, 2, 3, 4, 8]), rng.randint(0, 1500),
               rng.randint(1, 9), rng.choice([4, 7, 148])) for _ in range(300)]
    for G, nq, L, ns, sms in cases:
        W, n_cta = _launcher_ranges(G, nq, L, ns, sms)
        writes, cover = _kernel_writes(G, nq, L, 3, ns, W, n_cta)
        for g in range(G * nq):
            for p in range(ns):
                assert len(writes.get((g, p), [])) == 1, (G, nq, L, ns, sms, g, p)
            # the pieces of query row g tile [3, 3 + L) exactly once
            iv = sorted(cover.get(g, []))
            edges = [3] + [b for _, b in iv]
            assert [a for a, _ in iv] == edges[:-1] and edges[-1] == 3 + L, (G, nq, L, ns, g)
        assert all(g < G * nq and p < ns for g, p in writes)


def _prmt(a, b, sel):
    """prmt.b32 generic mode: result byte i = source byte (sel nibble i & 7) of
    (b:a), or that byte's sign bit replicated when the nibble's bit 3 is set."""
    src = [(a >> (8 * i)) & 255 for i in range(4)] + [(b >> (8 * i)) & 255 for i in range(4)]
    r = 0
    for i in range(4):
        n = (sel >> (4 * i)) & 15
        byte = src[n & 7]
        if n & 8:
            byte = 255 if byte & 128 else 0
        r |= byte << (8 * i)
    return r


def _xor_selectors(r):
    """kh_bytetab.cuh xor_selectors."""
    return [((8 | (4 + b)) << 12) | ((8 | (4 + b)) << 8) | ((b ^ (r & 3)) << 4) | (4 + b)
            for b in range(4)]


def _xor_slots(P, m, r, cp):
    """kh_bytetab.cuh xor_slots."""
    return sum((4 * (((4 * m + j) ^ r) + P * cp)) << (8 * j) for j in range(4))


def _xor_view(w, wx):
    """xor_plane<128> (two select stages) / xor_plane32 (halves swapped by the
    load addresses, then xor_plane<128> within each half)."""
    def x128(q):
        y = [q[2], q[3], q[0], q[1]] if wx & 2 else list(q)
        return [y[1], y[0], y[3], y[2]] if wx & 1 else y
    if len(w) == 4:
        return x128(w)
    hs = (wx >> 2) & 1
    return x128(w[4 * hs:4 * hs + 4]) + x128(w[4 * (hs ^ 1):4 * (hs ^ 1) + 4])


def test_xor_byte_order_addresses_and_banks():
    """The XOR byte order of the table kernels, restated from the device code:
    at step k lane l's byte-permute yields 256 * (plane byte k ^ r) + 4 * slot
    with slot = (k ^ r) + P (l / P), r = l mod P, and the 32 lanes of a warp
    touch 32 distinct banks (16-byte planes with two table copies, 32-byte
    planes with one; also the second V atomic's slots of the half-row layout)."""
    import random
    rng = random.Random(1)
    for nwords in (4, 8):
        P = 4 * nwords
        for _ in range(20):
            planes = [[rng.getrandbits(32) for _ in range(nwords)] for _ in range(32)]
            for k in range(P):
                banks, banks_y = set(), set()
                for lane in range(32):
                    r = lane % P
                    z = _xor_view(planes[lane], r >> 2)
                    slots = _xor_slots(P, k >> 2, r, lane // P)
                    a = _prmt(z[k >> 2], slots, _xor_selectors(r)[k & 3])
                    p = k ^ r
                    v = (planes[lane][p >> 2] >> (8 * (p & 3))) & 255
                    slot = p + P * (lane // P)
                    assert a == 256 * v + 4 * slot, (nwords, k, lane)
                    banks.add(slot % 32)
                    if P == 16:  # decode v3's second atomic: the other copy
                        a2 = _prmt(z[k >> 2], slots ^ 0x40404040, _xor_selectors(r)[k & 3])
                        assert a2 == 256 * v + 4 * (p + 16 * (1 - lane // 16))
                        banks_y.add((p + 16 * (1 - lane // 16)) % 32)
                assert len(banks) == 32 and (P != 16 or len(banks_y) == 32)
