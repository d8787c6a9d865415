"""The reference's packed-byte scorer (fused_asymmetric_attention,
KudaHitamCUDA.cu:695-797).

The oracle restates the kernel's own arithmetic (kh_oracle.c:
khx_compat_score) and is checked here against an independent float64
evaluation of the kernel's formula; the engine must equal the oracle bit for
bit (same per-lane fused multiply-add order, same butterfly reduction).
test_gpu_reference_kernels.py checks both against the reference kernel
itself on the GPU."""
import numpy as np
import pytest
import torch

import khtest as K
from oracle import oracle as O


def _inputs(H, S, D, nibble, seed=0, n_c=2):
    rng = np.random.default_rng(seed)
    q = (rng.standard_normal((H, D)) * 0.7).astype(np.float16)
    bpt = 128 if nibble else 32
    kp = rng.integers(0, 256, (H, S, bpt), dtype=np.uint8)
    sg = rng.standard_normal((H, S, D)).astype(np.float16)
    d = np.sign(rng.standard_normal(D)).astype(np.float32)
    d[d == 0] = 1
    kn = (rng.random((H, S)) + 0.1).astype(np.float32)
    rn = rng.random((H, S)).astype(np.float32)
    c = np.zeros((D, 16), np.float32)
    n_c = 16 if nibble else n_c
    c[:, :n_c] = np.sort(rng.standard_normal((D, n_c)), axis=1) / np.sqrt(D)
    return q, kp, sg, d, kn, rn, c


def _float64(q, kp, sg, d, kn, rn, c, nibble, scale):
    H, D = q.shape
    qf = q.astype(np.float64)
    qt = (qf * d) @ K.hadamard(D).T / np.sqrt(D)
    if nibble:
        lo, hi = kp & 15, kp >> 4
        v = np.stack([lo, hi], axis=-1).reshape(kp.shape[0], kp.shape[1], -1)[..., :D]
    else:
        v = np.unpackbits(kp, axis=-1, bitorder="little")[..., :D]
    kr = c[np.arange(D), v].astype(np.float64) * kn[..., None]
    s1 = np.einsum("hd,hsd->hs", qt, kr)
    s2 = np.einsum("hd,hsd->hs", qf, sg.astype(np.float64))
    return s1 + kn * scale * s2 * rn


@pytest.mark.parametrize("nibble", [False, True])
@pytest.mark.parametrize("D", [32, 128, 256])
def test_oracle_matches_float64(nibble, D):
    args = _inputs(3, 50, D, nibble, seed=D)
    scale = 1 / np.sqrt(D)
    got = O.compat_score(*args, nibble, scale)
    ref = _float64(*args, nibble, scale)
    assert np.abs(got - ref).max() <= 2e-6 * np.abs(ref).max()


@pytest.mark.gpu
@pytest.mark.parametrize("nibble", [False, True])
@pytest.mark.parametrize("D", [32, 64, 128, 256])
def test_engine_equals_oracle_bitwise(nibble, D):
    from kudahitam import load_cuda_ext
    H, S = 3, 2 * 1024 + 77  # three CTAs per head, ragged tail, odd row count
    q, kp, sg, d, kn, rn, c = _inputs(H, S, D, nibble, seed=1 + D)
    scale = 1 / np.sqrt(D)
    layer_id, mask = (3, 0b1000) if nibble else (3, 0b0111)
    ext = load_cuda_ext()
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    out = ext.fused_asymmetric_attention(t(q), t(kp), t(sg), t(d), t(kn), t(rn), t(c),
                                         layer_id, mask, scale)
    ref = O.compat_score(q, kp, sg, d, kn, rn, c, nibble, scale)
    got = out.cpu().numpy()
    assert got.shape == (H, S) and out.dtype == torch.float32
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), \
        np.abs(got - ref).max()


@pytest.mark.gpu
def test_layer_mask_selects_layout_and_edge_cases():
    from kudahitam import ops
    D, H, S = 128, 2, 300
    q, kp, sg, d, kn, rn, c = _inputs(H, S, D, False, seed=5)
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    ref = O.compat_score(q, kp, sg, d, kn, rn, c, False, 0.5)
    # layer 9 is outside the 8-bit mask: 1-bit layout whatever the mask
    out = ops.fused_asymmetric_attention(t(q), t(kp), t(sg), t(d), t(kn), t(rn), t(c), 9,
                                         0xFF, 0.5)
    assert np.array_equal(out.cpu().numpy(), ref)
    # a misaligned packed view (copied internally) gives the same result
    buf = torch.zeros(kp.size + 1, dtype=torch.uint8, device="cuda")
    kpm = buf[1:].view(kp.shape)
    kpm.copy_(t(kp))
    out = ops.fused_asymmetric_attention(t(q), kpm, t(sg), t(d), t(kn), t(rn), t(c), 0, 0, 0.5)
    assert np.array_equal(out.cpu().numpy(), ref)
    # wrong packed width for the layer's layout
    with pytest.raises(ValueError):
        ops.fused_asymmetric_attention(t(q), t(kp), t(sg), t(d), t(kn), t(rn), t(c), 0, 1, 0.5)
    # empty cache
    e = ops.fused_asymmetric_attention(t(q), t(kp[:, :0]), t(sg[:, :0]), t(d), t(kn[:, :0]),
                                       t(rn[:, :0]), t(c), 0, 0, 0.5)
    assert e.shape == (H, 0)
