"""Pin the CPU oracle (and the engine's host-side codebook) to golden vectors
produced by the reference itself (tests/golden/make_golden.py)."""
import math

import numpy as np
import pytest
import torch

import khtest as K
from oracle import oracle as O
from kudahitam.codebook import lloyd_max, rademacher

CASES = ["d128_fp32_b1", "d128_fp32_b2", "d256_fp16_b1", "d256_fp16_b2"]


def test_codebook_matches_reference_bitwise():
    g = K.golden("codebook.npz")
    for D in (32, 64, 128, 256):
        for bits in (1, 2):
            ref = g[f"c_{D}_{bits}"]
            got = lloyd_max(bits, D).numpy()
            assert got.view(np.uint32).tolist() == ref.view(np.uint32).tolist(), (D, bits)
        for seed in range(8):
            assert np.array_equal(rademacher(D, seed).numpy(), g[f"d_{D}_{seed}"]), (D, seed)


def test_oracle_fwht_is_sylvester_and_matches_reference():
    g = K.golden("fwht.npz")
    for D in (8, 128, 256):
        x, y = g[f"x_{D}"], g[f"y_{D}"]
        # exact Sylvester matrix, double precision
        exact = x.astype(np.float64) @ K.hadamard(D).T
        v8 = O.fwht_v8(x)
        assert np.max(np.abs(v8 - exact)) <= 4e-6 * np.max(np.abs(exact))
        assert np.max(np.abs(y - exact)) <= 4e-6 * np.max(np.abs(exact))
        fwd = O.fwht_forward(x)
        assert np.allclose(fwd, exact / math.sqrt(D), rtol=0, atol=1e-6)


def test_oracle_fwht_parseval():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((32, 256)).astype(np.float32)
    y = O.fwht_forward(x)
    assert np.allclose((y.astype(np.float64) ** 2).sum(1), (x.astype(np.float64) ** 2).sum(1),
                       rtol=1e-5)


@pytest.mark.parametrize("case", CASES)
def test_oracle_compress_matches_reference(case):
    g = K.golden(f"compress_{case}.npz")
    x, d, c = g["x"], g["d"], g["c"]
    D = x.shape[-1]
    out = O.compress_v8(torch.from_numpy(x), d, c)
    n = out["norms"].shape[0]
    live = g["norms"].reshape(-1) > 0  # the reference's CPU branch keeps 0 for a zero row
    # norms: same fp32 arithmetic up to summation order
    assert K.rel_err(out["norms"][live], g["norms"].reshape(-1)[live]) < 2e-6
    assert abs(out["norms"][~live]).max(initial=0) <= 1e-8
    # indices: exact wherever the decision is not within 1e-6 of a boundary
    y = K.projected(x.astype(np.float32), d)
    m = K.idx_mask(y, c)
    assert m[live].mean() > 0.999
    assert np.array_equal(out["idx"][m], g["indices"].reshape(n, D)[m])
    # the all-zero row sits exactly on the boundary: lowest index, sign +1
    tie = int(np.argmin(np.abs(c)))  # lowest index among the centroids nearest 0
    assert (out["idx"][~live] == tie).all() and (g["indices"].reshape(n, D)[~live] == tie).all()
    assert (out["signs"][~live] == 1).all() and (g["signs"].reshape(n, D)[~live] == 1).all()
    # k_mse
    assert K.normwise(out["kmse"][live], g["k_mse"].reshape(n, D)[live]) < 1e-5
    # residual signs: exact where decided
    rm = K.res_mask(y, g["indices"].reshape(n, D).astype(np.int64), c)
    assert np.array_equal(out["signs"][rm], g["signs"].reshape(n, D)[rm])
    # residual norm
    assert K.rel_err(out["rnorms"][live], g["r_norm"].reshape(-1)[live]) < 2e-5


@pytest.mark.parametrize("case", CASES)
def test_oracle_score_matches_reference(case):
    g = K.golden(f"compress_{case}.npz")
    B, H, S, D = g["x"].shape
    q = g["q"]  # [B, H, nq, D]
    nq = q.shape[2]
    sc = O.score(q.reshape(B * H, nq, D), g["k_mse"].reshape(B * H, S, D),
                 g["signs"].reshape(B * H, S, D), g["r_norm"].reshape(B * H, S), g["d"])
    ref = g["scores"].reshape(B * H, nq, S)
    for gi in range(B * H):
        assert K.normwise(sc[gi], ref[gi]) < 1e-5


def test_oracle_rotated_domain_identity():
    """H(d (.) (x - k_mse)) = sqrt(D) ||x|| (y - c[idx]): the identity the engine
    uses to replace the reference's 2nd and 3rd transforms."""
    g = K.golden("compress_d128_fp32_b2.npz")
    x = g["x"].reshape(-1, 128).astype(np.float64)
    d, c = g["d"].astype(np.float64), g["c"].astype(np.float64)
    out = O.compress_v8(torch.from_numpy(g["x"]), g["d"], g["c"])
    nrm = np.linalg.norm(x, axis=1, keepdims=True)
    keep = nrm[:, 0] > 0
    y = K.projected(x, d)
    lhs = ((x - out["kmse"]) * d) @ K.hadamard(128).T
    rhs = math.sqrt(128) * nrm * (y - c[out["idx"]])
    assert K.normwise(lhs[keep], rhs[keep]) < 1e-5
    assert K.rel_err(out["rnorms"][keep], (nrm[:, 0] * np.linalg.norm(y - c[out["idx"]], axis=1))[keep]) < 1e-5


def test_oracle_fidelity_matches_published_range():
    """Synthetic stand-in for the README's score-cosine table (README.md:22-37):
    the oracle reproduces ~0.996-0.997 (1-bit codebook + QJL) and ~0.999
    (2-bit) on N(0,1) keys with outlier channels."""
    x = K.synth((1, 4, 2048, 128), seed=11).numpy()
    q = x[:, :, -1:, :]  # the reference uses the last key as the query (full.py:625)
    cos = {}
    for bits in (1, 2):
        c = lloyd_max(bits, 128).numpy()
        d = rademacher(128, 0).numpy()
        out = O.compress_v8(torch.from_numpy(x), d, c)
        G = 4
        est = O.score(q.reshape(G, 1, 128), out["kmse"].reshape(G, 2048, 128),
                      out["signs"].reshape(G, 2048, 128), out["rnorms"].reshape(G, 2048), d)
        real = np.einsum("gqd,gsd->gqs", q.reshape(G, 1, 128), x.reshape(G, 2048, 128))
        e, r = est.ravel().astype(np.float64), real.ravel()
        cos[bits] = float(e @ r / np.linalg.norm(e) / np.linalg.norm(r))
    assert 0.990 < cos[1] < 0.9995
    assert 0.997 < cos[2] < 0.99995
    assert cos[2] > cos[1]
