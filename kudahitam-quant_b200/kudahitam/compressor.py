"""Drop-in replacement for the reference's ``KudahitamCompressorV2``
(KudaHitamQuant_full.py:243-386).

Same constructor signature, same ``compress`` / ``asymmetric_attention_scores``
calls, same result keys.  Differences a caller can see:

* ``compress`` writes only the packed cache (code bits, residual sign bits and
  two norms: 40 B per row at D=128 instead of the reference's 6D+8 B).  The
  reference-layout tensors ``indices`` / ``k_mse`` / ``signs`` are
  materialised by a GPU kernel on first access of those keys.
* Inputs may be fp16, bf16 or fp32 (the reference kernel reads fp16 only,
  KudaHitamCUDA.cu:220); arithmetic is fp32 on the exact upcast.
* ``residual=False`` selects the 1-bit mode (norm + one sign plane, scores use
  the MSE term only).
* The options that feed the reference's outlier / whitening branches
  (protected dimensions > 0, ``use_vwh``) are not implemented and raise
  ``NotImplementedError``.  ``use_fractional``, ``use_dynamic_codebook``,
  ``use_ultra``, ``use_spaced`` and ``use_spectral`` are accepted: in the
  reference they only steer a fallback whose result is overwritten by the
  fused kernel's (KudaHitamQuant_full.py:333-356), or only act with
  protected dimensions.
"""
from __future__ import annotations

import math
from collections.abc import Mapping
from typing import Optional

import torch

from . import ops
from .codebook import lloyd_max, rademacher


class CompressedKV(Mapping):
    """Result of ``compress``: a read-only mapping with the reference's keys
    (KudaHitamQuant_full.py:358-370) plus the packed fields."""

    _LAZY = ("indices", "k_mse", "signs")

    def __init__(self, packed: ops.PackedKV, d_host: torch.Tensor,
                 centroids_host: torch.Tensor, is_domain: bool):
        self.packed = packed
        self._d = d_host
        self._c = centroids_host
        shape = tuple(packed.shape)
        self._eager = {
            "norms": packed.norms,
            "r_norm": packed.rnorms.view(shape[:-1]) if packed.rnorms is not None else None,
            "p_indices": None,
            "p_norms": None,
            "p_idx": None,
            "rank": len(shape),
            "shape": shape,
            "is_domain": is_domain,
            "code_bits": packed.code,
            "res_bits": packed.res,
        }
        self._cache: dict = {}

    def _materialize(self) -> None:
        m = ops.materialize(self.packed, self._d, self._c, idx=True, kmse=True,
                            signs=self.packed.residual)
        shape = tuple(self.packed.shape)
        self._cache["indices"] = m["idx"]
        self._cache["k_mse"] = m["kmse"].view(shape)
        self._cache["signs"] = m["signs"].view(shape) if m["signs"] is not None else None

    def __getitem__(self, key):
        if key in self._eager:
            return self._eager[key]
        if key in self._LAZY:
            if key not in self._cache:
                self._materialize()
            return self._cache[key]
        raise KeyError(key)

    def __iter__(self):
        yield from ("indices", "norms", "k_mse", "r_norm", "signs", "p_indices", "p_norms",
                    "p_idx", "rank", "shape", "is_domain", "code_bits", "res_bits")

    def __len__(self) -> int:
        return 13

    def nbytes(self) -> int:
        return self.packed.nbytes()


class KudahitamCompressorV2:
    def __init__(self, head_dim: int, bits: int, seed: int, device: str = "cpu",
                 outlier_threshold: Optional[float] = None,
                 protected_dim_count: int = 0,
                 is_domain_layer: bool = False,
                 use_outlier: bool = True,
                 domain_p_count: int = 64,
                 p_bits: int = 4,
                 use_spaced: bool = False,
                 use_spectral: bool = False, use_vwh: bool = False,
                 use_dynamic_codebook: bool = False, use_fractional: bool = False,
                 use_ultra: bool = False, *, residual: bool = True):
        if head_dim not in ops.HEAD_DIMS:
            raise ValueError(f"head_dim must be one of {ops.HEAD_DIMS}")
        if bits not in (1, 2):
            raise ValueError("bits must be 1 or 2")
        p_count = 0 if not use_outlier else (domain_p_count if is_domain_layer
                                             else protected_dim_count)
        if p_count > 0:
            raise NotImplementedError("outlier protection (protected dimensions) is not "
                                      "implemented by this engine")
        if use_vwh:
            raise NotImplementedError("variance whitening (use_vwh) is not implemented")
        if not residual and bits != 1:
            raise ValueError("residual=False (1-bit mode) needs bits=1")
        self.head_dim, self.bits, self.device = head_dim, bits, device
        self.outlier_threshold = outlier_threshold
        self.protected_dim_count = protected_dim_count
        self.is_domain_layer = is_domain_layer
        self.use_outlier = use_outlier
        self.domain_p_count, self.p_bits = domain_p_count, p_bits
        self.use_spaced, self.use_spectral, self.use_vwh = use_spaced, use_spectral, use_vwh
        self.use_dynamic_codebook, self.use_fractional = use_dynamic_codebook, use_fractional
        self.use_ultra = use_ultra
        self.residual = residual
        self.protected_indices = None
        self._d_host = rademacher(head_dim, seed)
        self._c_host = lloyd_max(bits, head_dim)
        self.d = self._d_host.to(device)
        self.centroids = self._c_host.to(device)

    @torch.no_grad()
    def compress(self, states, offload: bool = True) -> CompressedKV:
        """Compress states [..., S, D] (CUDA; fp16 / bf16 / fp32).  ``offload``
        is accepted and ignored, as in the reference."""
        if isinstance(states, (list, tuple)):
            states = states[0]
        packed = ops.compress(states, self._d_host, self._c_host, residual=self.residual)
        return CompressedKV(packed, self._d_host, self._c_host, self.is_domain_layer)

    def compress_to_host(self, states, device=None, outs=None) -> list:
        """Compress host-resident (pinned) tensors into host-resident packed
        caches, streaming them through the GPU with the uploads, the kernel
        and the downloads overlapped (``ops.compress_host``).  ``states`` is
        one CPU tensor or a list; returns a list of CompressedKV whose packed
        planes live in pinned host memory (``outs``: PackedKVs to fill
        instead).  Synchronise the current CUDA stream before reading them."""
        xs = list(states) if isinstance(states, (list, tuple)) else [states]
        dev = device if device is not None else (
            self.device if str(self.device).startswith("cuda") else None)
        packed = ops.compress_host(xs, self._d_host, self._c_host, residual=self.residual,
                                   device=dev, outs=outs)
        return [CompressedKV(p, self._d_host, self._c_host, self.is_domain_layer)
                for p in packed]

    @torch.no_grad()
    def asymmetric_attention_scores(self, queries: torch.Tensor, compressed) -> torch.Tensor:
        """queries [B, Hq, Lq, D] against a cache of shape [B, Hkv, S, D]
        (Hq a multiple of Hkv: grouped-query heads share their KV head
        without expanding the cache).  Returns float32 [B, Hq, Lq, S]."""
        packed = getattr(compressed, "packed", None)
        if packed is None:
            raise TypeError("asymmetric_attention_scores needs the result of this "
                            "engine's compress()")
        shape = tuple(packed.shape)
        S, D = shape[-2], shape[-1]
        B = shape[0] if len(shape) == 4 else 1
        Hkv = packed.n_rows // (B * S)
        q = queries
        if q.dim() == 3:
            q = q.unsqueeze(0)
        Bq, Hq, Lq, Dq = q.shape
        if Dq != D or Bq != B or Hq % Hkv != 0:
            raise ValueError(f"queries {tuple(queries.shape)} do not match cache {shape}")
        G = Hq // Hkv
        qg = q.reshape(B, Hkv, G * Lq, D).reshape(B * Hkv, G * Lq, D)
        out = ops.score(qg, packed, self._d_host, self._c_host, seq_len=S)
        return out.view(B, Hkv, G, Lq, S).view(Bq, Hq, Lq, S).view(*queries.shape[:-1], S)

    @torch.no_grad()
    def decode_attention(self, queries: torch.Tensor, k_compressed, v_compressed,
                         v_compressor: Optional["KudahitamCompressorV2"] = None,
                         sm_scale: Optional[float] = None,
                         n_splits: Optional[int] = None) -> torch.Tensor:
        """softmax(score / sqrt(D)) . V_hat for queries [B, H_q, D] or
        [B, H_q, 1, D] (one decode token) against compressed K and V caches
        [B, H_kv, S, D], H_q a multiple of H_kv (grouped-query heads share
        their KV head without expanding the cache).  V may use its own
        compressor (its own d); both must use bits=1 with the residual plane.
        Returns float32 [B, H_q, D]."""
        vc = v_compressor or self
        kp, vp = k_compressed.packed, v_compressed.packed
        B, Hq = queries.shape[0], queries.shape[1]
        Bk, Hk = kp.shape[0], kp.shape[1]
        if Bk != B or Hq % Hk:
            raise ValueError(f"{Hq} query heads do not map onto {Hk} KV heads (batch {B}/{Bk})")
        q = queries.reshape(B * Hk, Hq // Hk, self.head_dim)
        out = ops.decode_attention(q, kp, vp, self._d_host, vc._d_host, self._c_host,
                                   sm_scale=sm_scale or 1.0 / math.sqrt(self.head_dim),
                                   n_splits=n_splits)
        return out.view(B, Hq, self.head_dim)
