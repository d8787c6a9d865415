"""Generate the golden fixtures in this folder from the reference itself.

    python tests/golden/make_golden.py REFERENCE_DIR
    KUDAHITAM_REFERENCE_DIR=... python tests/golden/make_golden.py

Runs where the reference is checked out (its location is the argument, or
the environment variable KUDAHITAM_REFERENCE_DIR); the fixtures it writes
are committed so that tests need no reference at run time.  What comes from
where:

* codebook.npz -- ``KudahitamCompressorV2(D, bits, seed).d`` and
  ``.centroids`` (KudaHitamQuant_full.py:256-275), for several D / bits / seeds.
* fwht.npz -- ``fwht_pytorch`` (KudaHitamQuant_full.py:231-239) on random rows.
* compress_*.npz -- ``KudahitamCompressorV2.compress`` executed by the
  reference's own code on CPU float32 input.  Two substitutions make it run
  here, because its GPU extension cannot be loaded: (1) the module-level
  ``fwht`` is bound to the orthonormal transform that its CUDA dispatch
  computes (``forward``, KudaHitamCUDA.cu:270-272; the CPU branch
  ``fwht_pytorch`` is unnormalised), so the fallback branch
  (KudaHitamQuant_full.py:337-353) computes the kernel's ``indices``,
  ``norms`` and ``k_mse``; (2) ``load_cuda_ext`` returns a stub whose
  ``ultra_fused_full_fusion`` (called at :356) takes those values from the
  caller's frame and completes the two outputs only the kernel produces,
  following KudaHitamCUDA.cu:141-194 (diff = x - k_mse, r_norm = ||diff||,
  signs = [fwht_pytorch(diff * d) >= 0]).  The reference's ``load_cuda_ext``
  is never called (it would JIT-build into the reference tree).
* score_*.npz -- ``KudahitamCompressorV2.asymmetric_attention_scores``
  (KudaHitamQuant_full.py:373-377) on those compressed dicts, with the same
  orthonormal ``fwht`` binding.
"""
from __future__ import annotations

import math
import pathlib
import sys
import types

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent


def load_reference(path: str):
    sys.path.insert(0, path)
    import KudaHitamQuant_full as R  # noqa: E402
    import torch

    R.fwht = lambda x: R.fwht_pytorch(x) / math.sqrt(x.shape[-1])

    def fused_from_fallback(flat, d, centroids):
        f = sys._getframe(1).f_locals
        indices, vec_norms, k_mse = f["indices"], f["vec_norms"], f["k_mse"]
        x = flat.float()
        diff = x - k_mse
        ss = (diff * diff).sum(-1, keepdim=True)
        r_norm = torch.where(ss > 0, ss.sqrt(), torch.full_like(ss, 1e-8))
        z = R.fwht_pytorch((diff * d).clone())
        signs = torch.where(z >= 0, 1, -1).to(torch.int8)
        return indices, vec_norms, k_mse, r_norm, signs

    stub = types.SimpleNamespace(ultra_fused_full_fusion=fused_from_fallback)
    R.load_cuda_ext = lambda: stub
    return R


def synth_rows(rng, B, H, S, D, kind):
    if kind == "outlier":   # N(0,1) with 3 channels per head x10
        x = rng.standard_normal((B, H, S, D)).astype(np.float32)
        for h in range(H):
            ch = rng.choice(D, 3, replace=False)
            x[:, h, :, ch] *= 10.0
    elif kind == "student":  # N(0,1) with 2% Student-t(3) channels
        x = rng.standard_normal((B, H, S, D)).astype(np.float32)
        n = max(1, round(0.02 * D))
        for h in range(H):
            for ch in rng.choice(D, n, replace=False):
                x[:, h, :, ch] = rng.standard_t(3, size=(B, S))
    else:
        raise ValueError(kind)
    # edge rows: all-zero, a single spike, tiny and huge magnitudes
    x[0, 0, 0] = 0.0
    x[0, 0, 1] = 0.0
    x[0, 0, 1, 5] = 3.0
    x[0, 0, 2] *= 1e-6
    x[0, 0, 3] *= 1e4
    return x


def main(ref: str | None = None) -> None:
    import os

    import torch

    ref = ref or os.environ.get("KUDAHITAM_REFERENCE_DIR")
    if not ref:
        raise SystemExit("usage: make_golden.py REFERENCE_DIR "
                         "(or set KUDAHITAM_REFERENCE_DIR)")

    R = load_reference(ref)

    cb = {}
    for D in (32, 64, 128, 256):
        for bits in (1, 2):
            c = R.KudahitamCompressorV2(D, bits, seed=0, use_outlier=False)
            cb[f"c_{D}_{bits}"] = c.centroids.numpy()
        for seed in range(8):
            cb[f"d_{D}_{seed}"] = R.KudahitamCompressorV2(D, 1, seed=seed,
                                                           use_outlier=False).d.numpy()
    np.savez_compressed(HERE / "codebook.npz", **cb)

    rng = np.random.default_rng(1234)
    fw = {}
    for D in (8, 128, 256):
        x = rng.standard_normal((6, D)).astype(np.float32)
        fw[f"x_{D}"] = x
        fw[f"y_{D}"] = R.fwht_pytorch(torch.from_numpy(x.copy())).numpy()
    np.savez_compressed(HERE / "fwht.npz", **fw)

    cases = [
        ("d128_fp32", 128, "outlier", np.float32, (1, 2, 48, 128)),
        ("d256_fp16", 256, "student", np.float16, (1, 2, 24, 256)),
    ]
    for name, D, kind, dt, shape in cases:
        x = synth_rows(rng, *shape, kind).astype(dt)
        x32 = torch.from_numpy(x.astype(np.float32))  # exact upcast
        q = rng.standard_normal((shape[0], shape[1], 2, D)).astype(np.float32)
        for bits in (1, 2):
            comp = R.KudahitamCompressorV2(D, bits, seed=7, use_outlier=False)
            out = comp.compress(x32, offload=False)
            sc = comp.asymmetric_attention_scores(torch.from_numpy(q), out)
            np.savez_compressed(
                HERE / f"compress_{name}_b{bits}.npz",
                x=x, q=q, d=comp.d.numpy(), c=comp.centroids.numpy(),
                indices=out["indices"].numpy(), norms=out["norms"].numpy(),
                k_mse=out["k_mse"].numpy(), r_norm=out["r_norm"].numpy(),
                signs=out["signs"].numpy(), scores=sc.numpy())
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main(*sys.argv[1:])
