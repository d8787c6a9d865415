"""Quantiser parameters: the Rademacher diagonal and the Lloyd-Max codebook.

Both must reproduce the reference's values exactly, since the packed bits
depend on them:

* ``rademacher(D, seed)`` is the reference's ``sign(randn(D))`` drawn from a
  CPU ``torch.Generator`` seeded with ``seed`` (KudaHitamQuant_full.py:257-258).
  The call is kept identical because the draw order defines the vector.
* ``lloyd_max(bits, D)`` is the Lloyd-Max quantiser of N(0, 1/D) with
  2**bits levels, started from the midpoints of 2**bits equal cells of
  [-3.5 sigma, 3.5 sigma], integrated over (-10.5 sigma, 10.5 sigma), stopped
  when no level moves by 1e-10 (keeping the iterate before that last move)
  or after 200 rounds (KudaHitamQuant_full.py:261-275).  The reference
  integrates with ``scipy.integrate.quad``; here the two Gaussian integrals
  are evaluated in closed form, int x phi = sigma^2 (phi(a) - phi(b)) and
  int phi = Phi(b) - Phi(a), which converges to the same fixed point.
"""
from __future__ import annotations

import functools
import math

import torch


def rademacher(head_dim: int, seed: int) -> torch.Tensor:
    gen = torch.Generator(device="cpu").manual_seed(seed)
    return torch.sign(torch.randn(head_dim, generator=gen))


@functools.lru_cache(maxsize=None)
def _lloyd_max_tuple(bits: int, head_dim: int) -> tuple[float, ...]:
    n = 1 << bits
    sigma = 1.0 / math.sqrt(head_dim)
    lo, hi = -3.5 * sigma, 3.5 * sigma
    inv = 1.0 / (sigma * math.sqrt(2.0 * math.pi))

    def pdf(x: float) -> float:
        return inv * math.exp(-x * x / (2.0 * sigma * sigma))

    def cdf(x: float) -> float:
        return 0.5 * (1.0 + math.erf(x / (sigma * math.sqrt(2.0))))

    cur = [lo + (hi - lo) * (i + 0.5) / n for i in range(n)]
    for _ in range(200):
        bounds = [(cur[i] + cur[i + 1]) / 2.0 for i in range(n - 1)]
        edges = [3.0 * lo] + bounds + [3.0 * hi]
        new = []
        for i in range(n):
            a, b = edges[i], edges[i + 1]
            num = sigma * sigma * (pdf(a) - pdf(b))
            den = cdf(b) - cdf(a)
            new.append(num / den if den > 1e-15 else cur[i])
        if max(abs(new[i] - cur[i]) for i in range(n)) < 1e-10:
            break
        cur = new
    return tuple(cur)


def lloyd_max(bits: int, head_dim: int) -> torch.Tensor:
    """float32 codebook, ascending, for ``bits`` in {1, 2} (any bits >= 1 works)."""
    if bits < 1:
        raise ValueError("bits must be >= 1")
    return torch.tensor(_lloyd_max_tuple(int(bits), int(head_dim)), dtype=torch.float32)
