"""The engine and the oracle against the reference's own CUDA kernels, run on
the GPU: kernel v8 (KudaHitamCUDA.cu:13-231, which the reference never
exports; oracle/ref_binding.cpp binds it), its FWHT `forward` (:233-283) and
its packed-byte scorer (:695-797), built from the reference source by
oracle/build_ref.py.

The reference kernels are run only on inputs they handle safely: kernel v8
and `forward` return early for threads past the last row and then use
full-warp shuffles and a block barrier, so every launch here covers whole
blocks (rows * D a multiple of 2048)."""
import numpy as np
import pytest
import torch

import khtest as K
from kudahitam import load_cuda_ext, lloyd_max, ops, rademacher
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REF = O.reference_kernels()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref/kh_ref.so not built")


def _fp16_rows(N, D, seed):
    x = K.synth((1, 1, N, D), dtype=torch.float16, seed=seed).reshape(N, D)
    assert (N * D) % 2048 == 0  # whole blocks only (see the module docstring)
    return x


@needs_ref
@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("bits", [1, 2])
def test_reference_kernel_v8_pins_oracle_and_engine(D, bits):
    N = 2048
    x = _fp16_rows(N, D, seed=D + bits)
    d = rademacher(D, 5)
    c = lloyd_max(bits, D)
    idx, norms, kmse, rn, signs = (t.cpu() for t in REF.ultra_fused_full_fusion(
        x.cuda().contiguous(), d.cuda().contiguous(), c.cuda().contiguous()))
    torch.cuda.synchronize()
    ref = {"idx": idx.numpy(), "norms": norms.numpy()[:, 0], "kmse": kmse.numpy(),
           "rnorms": rn.numpy()[:, 0], "signs": signs.numpy()}
    y = K.projected(x.float().numpy(), d.numpy().astype(np.float64))
    m_idx = K.idx_mask(y, c.numpy())
    m_res = K.res_mask(y, ref["idx"].astype(np.int64), c.numpy())
    # the oracle (fp32 restatement of the same kernel) against the kernel itself
    o = O.compress_v8(x, d.numpy(), c.numpy())
    assert not ((o["idx"] != ref["idx"]) & m_idx).any()
    assert not ((o["signs"] != ref["signs"]) & m_res).any()
    assert K.rel_err(o["norms"], ref["norms"]) < 1e-6
    assert K.normwise(o["kmse"], ref["kmse"]) < 1e-6
    assert K.rel_err(o["rnorms"], ref["rnorms"], floor=1e-30) < 1e-5
    # the engine against the kernel (the engine's tolerance contract)
    p = ops.compress(x.cuda(), d, c)
    mat = ops.materialize(p, d, c)
    code = mat["idx"].cpu().numpy()
    sg = mat["signs"].cpu().numpy()
    assert not ((code != ref["idx"]) & m_idx).any()
    assert (code != ref["idx"]).sum() <= max(2, 1e-4 * code.size)
    assert not ((sg != ref["signs"]) & m_res).any()
    assert K.rel_err(p.norms.cpu().numpy(), ref["norms"]) < 1e-5
    assert K.rel_err(p.rnorms.cpu().numpy(), ref["rnorms"], floor=1e-30) < 1e-4
    assert K.normwise(mat["kmse"].cpu().numpy(), ref["kmse"]) < 1e-5


@needs_ref
@pytest.mark.parametrize("D", [128, 256])
def test_reference_fwht_forward(D):
    N = 1024
    x = torch.randn(N, D, generator=torch.Generator().manual_seed(D)).cuda()
    want = x.clone()
    REF.forward(want)
    got = load_cuda_ext().forward(x.clone())
    torch.cuda.synchronize()
    assert K.normwise(got.cpu().numpy(), want.cpu().numpy()) < 1e-6


@needs_ref
@pytest.mark.parametrize("nibble", [False, True])
def test_reference_packed_scorer(nibble):
    """fused_asymmetric_attention: engine, oracle and reference kernel on the
    same inputs; the engine and the oracle follow the kernel's per-lane
    summation order."""
    from test_compat_score import _inputs
    D, H, S = 128, 3, 777
    q, kp, sg, d, kn, rn, c = _inputs(H, S, D, nibble, seed=21)
    scale = 1 / np.sqrt(D)
    layer_id, mask = (2, 0b100) if nibble else (2, 0)
    t = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    want = REF.fused_asymmetric_attention(t(q), t(kp), t(sg), t(d), t(kn), t(rn), t(c),
                                          layer_id, mask, float(scale)).cpu().numpy()
    got = ops.fused_asymmetric_attention(t(q), t(kp), t(sg), t(d), t(kn), t(rn), t(c),
                                         layer_id, mask, scale).cpu().numpy()
    orc = O.compat_score(q, kp, sg, d, kn, rn, c, nibble, scale)
    assert want.shape == (H, S)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))  # bit for bit
    assert np.array_equal(orc.view(np.uint32), want.view(np.uint32))
