"""Shared helpers for the test suite (synthetic inputs, masks, comparisons)."""
from __future__ import annotations

import math
import pathlib

import numpy as np
import torch

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def golden(name: str) -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


def hadamard(D: int) -> np.ndarray:
    H = np.array([[1.0]])
    while H.shape[0] < D:
        H = np.block([[H, H], [H, -H]])
    return H


def projected(x: np.ndarray, d: np.ndarray) -> np.ndarray:
    """y = H(d * x / ||x||) / sqrt(D) in float64 (the quantised value)."""
    x = np.asarray(x, dtype=np.float64).reshape(-1, x.shape[-1])
    D = x.shape[-1]
    n = np.linalg.norm(x, axis=1, keepdims=True)
    n = np.where(n > 0, n, 1e-8)
    return (x * d[None, :] / n) @ hadamard(D).T / math.sqrt(D)


def boundaries(c: np.ndarray) -> np.ndarray:
    c = np.asarray(c, dtype=np.float64)
    return (c[:-1] + c[1:]) / 2.0


def idx_mask(y: np.ndarray, c: np.ndarray, tol: float = 1e-6) -> np.ndarray:
    """Elements whose index is decided by more than tol (|y - boundary| > tol)."""
    b = boundaries(c)
    return np.all(np.abs(y[..., None] - b[None, None, :]) > tol, axis=-1)


def res_mask(y: np.ndarray, idx: np.ndarray, c: np.ndarray, tol: float = 1e-6) -> np.ndarray:
    """Residual-plane elements whose sign is decided: the index is decided and
    |y - c[idx]| > tol."""
    v = y - np.asarray(c, dtype=np.float64)[idx]
    return idx_mask(y, c, tol) & (np.abs(v) > tol)


def u32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().numpy().view(np.uint32)


def unpack_bits(words: np.ndarray, D: int) -> np.ndarray:
    w = np.ascontiguousarray(words, dtype=np.uint32)
    by = w.view(np.uint8).reshape(w.shape[0], -1)
    return np.unpackbits(by, axis=1, bitorder="little")[:, :D]


def unpack_idx2(words: np.ndarray, D: int) -> np.ndarray:
    w = np.ascontiguousarray(words, dtype=np.uint32)
    sh = (2 * np.arange(16, dtype=np.uint32))[None, None, :]
    return ((w[:, :, None] >> sh) & 3).reshape(w.shape[0], -1)[:, :D].astype(np.uint8)


def unpack_code(words: np.ndarray, D: int, bits: int) -> np.ndarray:
    return unpack_bits(words, D) if bits == 1 else unpack_idx2(words, D)


def rel_err(a, b, floor: float = 0.0) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), floor)))


def normwise(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def synth(shape, dtype=torch.float32, seed=0, outliers=3, scale=1.0, device="cpu"):
    """N(0, scale^2) rows with `outliers` channels per head scaled x10."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(*shape, generator=g) * scale
    if outliers and len(shape) >= 3:
        H = shape[-3]
        for h in range(H):
            ch = torch.randperm(shape[-1], generator=g)[:outliers]
            x[..., h, :, :][..., ch] *= 10.0
    return x.to(dtype).to(device)
