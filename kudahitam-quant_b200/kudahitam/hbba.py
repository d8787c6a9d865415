"""Drop-in replacement for the reference's ``KudahitamCompressorHBBA``
(KudaHitamQuant_full-reasoning.py:467-560): the mixed-codebook ("HBBA")
compressor whose packed cache ``fused_asymmetric_attention`` scores.

Per head dimension it keeps 16 Lloyd-Max levels for the ``hbba_4bit_ratio``
highest-variance rotated dimensions and 2 for the rest (an HBBA layer is one
whose bit ``layer_id`` of ``active_mask`` is set; other layers use 2 levels
everywhere).  ``calibrate`` samples the states, chooses the dimensions and
fits the levels on the GPU (``kh_hbba_calibrate``); ``compress`` runs the
encoder (``kh_compress_hbba``); ``asymmetric_attention_scores`` scores with
the packed-byte scorer (``kh_score_packed_compat``) without expanding
grouped-query heads.

The Python steps follow the reference line by line, including its d vector
(``randint(0, 2) * 2 - 1`` from the seed) and its calibration sample: rows
normalised, sign-flipped, passed through its orthonormal ``fwht`` and
divided by sqrt(D) once more (:506-509), while the encoder quantises
H(x / ||x|| (.) d) / sqrt(D).  The two scales differ by sqrt(D) in the
reference; this class keeps that, so a cache compressed here equals the
reference's encoder output on the reference's levels.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

from . import ops


class KudahitamCompressorHBBA:
    def __init__(self, head_dim: int, bits: int, seed: int, device: str = "cpu",
                 hbba_4bit_ratio: float = 0.25, layer_id: int = 0, active_mask: int = 0xFF):
        if head_dim not in ops.HEAD_DIMS:
            raise ValueError(f"head_dim must be one of {ops.HEAD_DIMS}")
        self.head_dim = head_dim
        self.bits = bits
        self.seed = seed
        self.device = device
        self.hbba_4bit_ratio = hbba_4bit_ratio
        self.layer_id = layer_id
        self.active_mask = active_mask
        g = torch.Generator().manual_seed(seed)
        self.d = (torch.randint(0, 2, (head_dim,), generator=g) * 2 - 1).float().to(device)
        self.centroids_table: Optional[torch.Tensor] = None
        self.n_centroids_map: Optional[torch.Tensor] = None
        self.hbba_mask: Optional[torch.Tensor] = None
        self.is_calibrated = False

    @property
    def is_hbba(self) -> bool:
        return bool(0 <= self.layer_id < 8 and ((self.active_mask & 0xFF) >> self.layer_id) & 1)

    def _calibrate_hbba(self, sample_rotated: torch.Tensor) -> None:
        """Levels per dimension from rotated samples [N, D]
        (KudaHitamQuant_full-reasoning.py:474-491)."""
        dev = sample_rotated.device
        D = self.head_dim
        variances = sample_rotated.var(0)
        num_4bit = int(D * self.hbba_4bit_ratio)
        top = torch.topk(variances, num_4bit).indices
        n_map = torch.full((D,), 2, dtype=torch.int32, device=dev)
        n_map[top] = 16
        mask_np = np.zeros(8, dtype=np.uint32)
        for idx in top.cpu().numpy():
            mask_np[idx // 32] |= np.uint32(1 << (int(idx) % 32))
        self.n_centroids_map = n_map
        self.hbba_mask = torch.from_numpy(mask_np.astype(np.int32)).to(dev)
        self.centroids_table = ops.hbba_calibrate(sample_rotated.float().contiguous(), n_map,
                                                  self.layer_id, self.active_mask)
        self.is_calibrated = True

    @torch.no_grad()
    def calibrate(self, states) -> None:
        """Sample 4 chunks of 1000 rows (staggered along S) and fit the
        levels (KudaHitamQuant_full-reasoning.py:494-510).  CUDA tensors."""
        if self.is_calibrated:
            return
        if isinstance(states, (list, tuple)):
            states = states[0]
        dev = states.device
        D, S = states.shape[-1], states.shape[-2]
        chunk, n_chunks = 1000, 4
        if S <= chunk * n_chunks:
            flat = states.reshape(-1, D)[: chunk * n_chunks].float()
        else:
            offsets = torch.linspace(0, S - chunk, n_chunks, dtype=torch.long)
            flat = torch.cat([states[:, int(o): int(o) + chunk, :].reshape(-1, D)
                              for o in offsets], dim=0).float()
        norm = torch.norm(flat, dim=-1, keepdim=True)
        rotated = ops.fwht((flat / (norm + 1e-8)) * self.d.to(dev)) / math.sqrt(D)
        self._calibrate_hbba(rotated)

    @torch.no_grad()
    def compress(self, states, offload: bool = True) -> dict:
        """Packed indices, norms, residual norms and fp16 residual transform
        (KudaHitamQuant_full-reasoning.py:513-531); ``offload`` is accepted
        and ignored, as in the reference."""
        if isinstance(states, (list, tuple)):
            states = states[0]
        shape = states.shape
        flat = states.reshape(-1, shape[-1])
        if not self.is_calibrated:
            self.calibrate(states)
        packed, norms, rnorms, signs = ops.ultra_fused_hbba_fusion(
            flat, self.d.to(states.device), self.centroids_table, self.hbba_mask,
            self.layer_id, self.active_mask)
        return {"indices": packed, "norms": norms.squeeze(-1), "r_norms": rnorms,
                "signs": signs.view(shape), "shape": tuple(shape)}

    @torch.no_grad()
    def asymmetric_attention_scores(self, queries: torch.Tensor, compressed: dict) -> torch.Tensor:
        """Scores of queries [B, H_q, 1, D] against the compressed [B, H_k, S, D]
        cache with the packed-byte scorer (KudaHitamQuant_full-reasoning.py:533-565),
        scale 1/sqrt(D).  Query head h reads KV head h // (H_q / H_k); the
        reference expands the cache to H_q heads first (:547-558), which
        gives the same numbers."""
        D = self.head_dim
        B, Hq = queries.shape[0], queries.shape[1]
        Bk, Hk, S, _ = compressed["shape"]
        if Bk != B or Hq % Hk:
            raise ValueError(f"{Hq} query heads / batch {B} do not map onto {Hk} KV heads")
        bpt = 128 if self.is_hbba else 32
        kp = compressed["indices"].view(Bk * Hk, S, bpt)
        sg = compressed["signs"].reshape(Bk * Hk, S, D)
        kn = compressed["norms"].float().reshape(Bk * Hk, S)
        rn = compressed["r_norms"].float().reshape(Bk * Hk, S)
        q = queries.reshape(B * Hq, D)
        rep = Hq // Hk
        d_vec = self.d.to(queries.device).float()
        scale = 1.0 / math.sqrt(D)
        if rep == 1:
            out = ops.fused_asymmetric_attention(q, kp, sg, d_vec, kn, rn, self.centroids_table,
                                                 self.layer_id, self.active_mask, scale)
        else:
            # one scorer call per query head within each KV group: the cache
            # is read in place, never expanded
            out = torch.empty(B * Hq, S, dtype=torch.float32, device=queries.device)
            qg = q.view(Bk * Hk, rep, D)
            ov = out.view(Bk * Hk, rep, S)
            for j in range(rep):
                ov[:, j] = ops.fused_asymmetric_attention(
                    qg[:, j].contiguous(), kp, sg, d_vec, kn, rn, self.centroids_table,
                    self.layer_id, self.active_mask, scale)
        return out.view(*queries.shape[:-1], S)
