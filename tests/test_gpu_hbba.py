"""The HBBA mixed-codebook path (KudaHitamCUDA.cu:285-518; the compressor
class of KudaHitamQuant_full-reasoning.py:467-560) against the oracle, and
the calibrator against the reference's own calibrator kernel.

Tolerances:
* calibrator: engine and oracle both sum in double in a fixed order, so the
  levels agree to 1e-6 absolute; the reference kernel adds with float
  atomics in unspecified order: 1e-4 of the sample's range;
* encoder: indices exact wherever the best level beats the second best by
  more than 1e-6 (ties may go either way, at most max(2, 1e-4 n)); norms
  1e-6 and residual norms 1e-5 relative; the fp16 residual transform within
  2 fp16 ulps plus 2e-6 of the row's largest magnitude: the engine sums
  ||x||^2 in float and the oracle in double, and a norm one float ulp apart
  moves every element of the transform by up to ~2.5e-7 of the row's scale
  (measured by nudging the oracle's norm), which is many fp16 ulps where an
  element cancels to near zero; bytes past the row's indices zero;
* scores through the packed-byte scorer: 1e-4 normwise against the
  oracle's scorer on the oracle's own encoding.
"""
import math

import numpy as np
import pytest
import torch

import khtest as K
from kudahitam import KudahitamCompressorHBBA, ops
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _levels(D, wide_dims, seed=0):
    """A [D, 16] table: sorted levels for the wide dimensions (16) and two
    levels elsewhere, scaled like the encoder's y ~ N(0, 1/D)."""
    rng = np.random.default_rng(seed)
    s = 1.0 / math.sqrt(D)
    c = np.zeros((D, 16), np.float32)
    for i in range(D):
        if i in wide_dims:
            c[i] = np.sort(rng.normal(0, 1.2 * s, 16)).astype(np.float32)
        else:
            c[i, :2] = np.array([-0.8 * s, 0.8 * s]) * (1 + 0.1 * rng.standard_normal())
    return c


def _mask(D, wide_dims):
    m = np.zeros(8, np.uint32)
    for i in wide_dims:
        m[i // 32] |= np.uint32(1 << (i % 32))
    return m


def _unpack(packed, D, nibble):
    p = packed.astype(np.uint32)
    if nibble:
        lo, hi = p[:, : D // 2] & 15, p[:, : D // 2] >> 4
        return np.stack([lo, hi], axis=2).reshape(p.shape[0], D)
    return np.unpackbits(packed[:, : D // 8], axis=1, bitorder="little")[:, :D]


def _decided(x, d, c, wide, D, tol=1e-6):
    """Elements whose nearest level beats the second nearest by > tol (in
    the encoder's float arithmetic restated in float64)."""
    xf = x.float().numpy().astype(np.float64).reshape(-1, D)
    n = np.sqrt((xf * xf).sum(1, keepdims=True) + 1e-8)
    y = (xf / n * d) @ K.hadamard(D).T / math.sqrt(D)
    ch = c.astype(np.float16).astype(np.float64)
    out = np.ones_like(y, dtype=bool)
    for i in range(D):
        nc = 16 if wide[i] else 2
        dist = np.sort(np.abs(y[:, i:i + 1] - ch[None, i, :nc]), axis=1)
        out[:, i] = (dist[:, 1] - dist[:, 0]) > tol
    return out


@pytest.mark.parametrize("D", [128, 256])
def test_calibrator_matches_oracle_and_reference_kernel(D):
    g = torch.Generator().manual_seed(D)
    smp = (torch.randn(4000, D, generator=g) * torch.linspace(0.02, 0.2, D)).float()
    n_map = torch.full((D,), 2, dtype=torch.int32)
    n_map[torch.randperm(D, generator=g)[: D // 4]] = 16
    got = ops.hbba_calibrate(smp.cuda(), n_map.cuda(), 0, 1).cpu().numpy()
    want = O.hbba_calibrate(smp.numpy(), n_map.numpy())
    assert np.max(np.abs(got - want)) <= 1e-6
    assert np.all(got[n_map.numpy() == 2][:, 2:] == 0)
    wide = got[n_map.numpy() == 16]
    assert np.all(np.diff(wide, axis=1) >= 0)  # levels stay sorted
    # inactive layer: zeros, as the reference binding returns
    assert torch.count_nonzero(ops.hbba_calibrate(smp.cuda(), n_map.cuda(), 3, 1)) == 0
    ref = O.reference_kernels()
    if ref is None:
        pytest.skip("the reference kernels were not built")
    r = ref.hbba_calibrate_cuda(smp.cuda(), n_map.cuda(), 0, 1).cpu().numpy()
    span = (smp.max(0).values - smp.min(0).values).numpy()[:, None]
    assert np.all(np.abs(got - r) <= 1e-4 * span), np.max(np.abs(got - r) / span)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("hbba_layer", [True, False])
def test_encoder_matches_oracle(dtype, D, hbba_layer):
    g = torch.Generator().manual_seed(D + 3)
    n = 3001
    x = K.synth((1, 3, n, D), dtype=dtype, seed=D).reshape(-1, D)
    wide_dims = set(torch.randperm(D, generator=g)[: D // 4].tolist())
    c = _levels(D, wide_dims)
    m = _mask(D, wide_dims)
    d = np.where(torch.randn(D, generator=g).numpy() > 0, 1.0, -1.0).astype(np.float32)
    layer, active = (2, 0b100) if hbba_layer else (2, 0b011)
    packed, norms, rn, signs = ops.ultra_fused_hbba_fusion(
        x.cuda(), torch.from_numpy(d), torch.from_numpy(c), torch.from_numpy(m.view(np.int32)),
        layer, active)
    torch.cuda.synchronize()
    ref = O.hbba_compress(x, d, c, m, hbba_layer)
    bpt = 128 if hbba_layer else 32
    assert packed.shape == (x.shape[0], bpt) and norms.shape == (x.shape[0], 1)
    assert signs.dtype == torch.float16 and signs.shape == x.shape
    pk = packed.cpu().numpy()
    used = D // 2 if hbba_layer else D // 8
    assert not pk[:, used:].any()  # bytes past the row's indices are zero
    wide = np.array([(i in wide_dims) and hbba_layer for i in range(D)])
    got_idx = _unpack(pk, D, hbba_layer)
    want_idx = _unpack(ref["packed"], D, hbba_layer)
    dec = _decided(x, d, c, wide, D)
    assert not ((got_idx != want_idx) & dec).any()
    assert (got_idx != want_idx).sum() <= max(2, 1e-4 * got_idx.size)
    assert K.rel_err(norms.cpu().numpy()[:, 0], ref["norms"]) < 1e-6
    rows = (got_idx == want_idx).all(1)
    assert K.rel_err(rn.cpu().numpy()[rows], ref["rnorms"][rows]) < 1e-5
    a = signs.cpu().numpy().astype(np.float32)[rows]
    b = ref["signs"].astype(np.float32)[rows]
    ulp = np.maximum(np.abs(b), 6.1e-5) * 2.0 ** -10
    row_scale = np.abs(b).max(1, keepdims=True)
    assert np.all(np.abs(a - b) <= 2 * ulp + 2e-6 * row_scale)


def test_compressor_class_end_to_end_scores():
    """KudahitamCompressorHBBA: calibrate (4 x 1000 staggered rows), compress
    and score with the packed-byte scorer, grouped-query heads in place,
    against the oracle's encoder and scorer on the same levels."""
    D, S = 128, 5000
    g = torch.Generator(device="cuda").manual_seed(4)
    k = (torch.randn(1, 2, S, D, device="cuda", generator=g)
         * torch.linspace(0.5, 2.0, D, device="cuda")).half()
    comp = KudahitamCompressorHBBA(D, 1, seed=3, layer_id=1, active_mask=0b10)
    assert comp.is_hbba
    out = comp.compress(k)
    assert comp.is_calibrated and out["indices"].shape == (2 * S, 128)
    assert int(comp.n_centroids_map.eq(16).sum()) == D // 4
    q = torch.randn(1, 4, 1, D, device="cuda", generator=g)  # 2 query heads per KV head
    sc = comp.asymmetric_attention_scores(q, out)
    assert sc.shape == (1, 4, 1, S)
    c = comp.centroids_table.cpu().numpy()
    m = comp.hbba_mask.cpu().numpy().view(np.uint32)
    d = comp.d.cpu().numpy()
    ref = O.hbba_compress(k.cpu(), d, c, m, True)
    for h in range(4):
        kv = h // 2
        rows = slice(kv * S, (kv + 1) * S)
        want = O.compat_score(q[0, h].half().cpu().numpy(), ref["packed"][rows][None],
                              ref["signs"][rows][None], d, ref["norms"][rows][None],
                              ref["rnorms"][rows][None], c, True, 1 / math.sqrt(D))
        got_idx = _unpack(out["indices"][rows].cpu().numpy(), D, True)
        ok = (got_idx == _unpack(ref["packed"][rows], D, True)).all(1)
        assert ok.mean() > 0.999
        assert K.normwise(sc[0, h, 0].cpu().numpy()[ok], want[0][ok]) < 1e-4
