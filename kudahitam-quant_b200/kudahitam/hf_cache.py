"""Hugging Face ``Cache`` adapter: a KV cache that stores every layer's keys
and values packed, compresses on append, and attends from the packed bytes.

The reference compresses a finished ``DynamicCache`` after prefill
(KudaHitamQuant_full.py:549-551, :654-668) and states that generation with a
compressed cache is not wired (:671, :676-677).  This module is that wiring:

* ``KudahitamLayer`` keeps a layer's K and V as packed planes in
  [batch * kv_heads, capacity] row groups; ``append`` compresses the new
  tokens in one launch and copies them into place (capacity doubles when
  full), so earlier tokens are never recompressed.
* ``attend(query)`` is one decode step straight from the packed cache
  (grouped-query heads share their KV head, nothing is expanded);
  ``scores(query)`` gives the reference's asymmetric scores.
* ``update`` implements the transformers cache contract.  On the first
  call (prefill into an empty layer) it returns the incoming K and V
  themselves: the prompt attends to itself exactly, and only the packed
  copy is kept.  On a one-token decode step of a cache made with
  ``packed_attention=True`` it returns a ``PackedAttention`` handle, and the
  attention function registered as ``attn_implementation="kudahitam"``
  (``register_attention``) attends from the packed bytes with the decode
  kernel: generation never dequantises the cache.  Otherwise (chunked
  prefill, or a model running its own attention) it returns dequantised K
  and V for every cached token, K as k_mse + r_norm / D * d (.) H sign (the
  reference's score estimator as a vector, so q . K_hat equals its scores)
  and V as k_mse + r_norm sqrt(2/pi) / D * d (.) H sign (the decode step's
  V_hat); that path trades the memory saving for compatibility.

The layer class derives from transformers' ``CacheLayerMixin`` when
transformers is installed (the cache container requires it); the packed
storage and ``attend`` work without it.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import ops
from .codebook import lloyd_max, rademacher

_SQRT_2_OVER_PI = math.sqrt(2.0 / math.pi)

try:  # transformers' layer base class, when transformers is installed
    from transformers.cache_utils import CacheLayerMixin as _LayerBase
except Exception:  # pragma: no cover
    _LayerBase = object


class PackedSeq:
    """Appendable packed storage of one tensor [B, H, S, D]: rows of group
    g = b * H + h live at [g * capacity, g * capacity + length)."""

    def __init__(self, B: int, H: int, D: int, device, capacity: int = 256):
        self.B, self.H, self.D = B, H, D
        self.device = torch.device(device)
        self.length = 0
        self.capacity = 0
        self.packed: Optional[ops.PackedKV] = None
        self._grow(max(1, capacity))

    @property
    def groups(self) -> int:
        return self.B * self.H

    def _grow(self, cap: int) -> None:
        new = ops.empty_packed((self.groups, cap, self.D), 1, True, self.device)
        if self.packed is not None and self.length:
            L = self.length
            for name in ("code", "res", "norms", "rnorms"):
                src = getattr(self.packed, name).view(self.groups, self.capacity, -1)
                dst = getattr(new, name).view(self.groups, cap, -1)
                dst[:, :L].copy_(src[:, :L])
        self.packed, self.capacity = new, cap

    def append(self, x: torch.Tensor, d, centroids) -> None:
        """Compress x [B, H, t, D] and append it."""
        B, H, t, D = x.shape
        if (B, H, D) != (self.B, self.H, self.D):
            raise ValueError(f"append of {tuple(x.shape)} to a [{self.B}, {self.H}, *, {self.D}] cache")
        if t == 0:
            return
        if self.length + t > self.capacity:
            self._grow(max(2 * self.capacity, self.length + t))
        new = ops.compress(x, d, centroids, residual=True)  # one launch, B*H*t rows
        L, cap, G = self.length, self.capacity, self.groups
        for name in ("code", "res", "norms", "rnorms"):
            dst = getattr(self.packed, name).view(G, cap, -1)
            dst[:, L:L + t].copy_(getattr(new, name).view(G, t, -1))
        self.length += t

    def truncate(self, length: int) -> None:
        self.length = max(0, min(self.length, int(length)))

    def dequantize(self, d, centroids, qjl_scale: float, dtype) -> torch.Tensor:
        """[B, H, length, D]: k_mse + r_norm * qjl_scale / D * d (.) H sign."""
        G, L, D = self.groups, self.length, self.D
        if L == 0:
            return torch.empty((self.B, self.H, 0, D), dtype=dtype, device=self.device)
        rows = self._first_rows()
        m = ops.materialize(rows, d, centroids, idx=False)
        s = ops.fwht_(m["signs"].to(torch.float32))  # H sign / sqrt(D)
        dd = torch.as_tensor(d, dtype=torch.float32, device=self.device)
        r = rows.rnorms.view(-1, 1) * (qjl_scale / math.sqrt(D))
        out = m["kmse"] + r * dd * s
        return out.view(self.B, self.H, L, D).to(dtype)

    def _first_rows(self) -> ops.PackedKV:
        """The filled rows as one contiguous PackedKV (copies when length <
        capacity)."""
        G, L, cap = self.groups, self.length, self.capacity
        if L == cap:
            return self.packed
        p = self.packed
        take = lambda t: t.view(G, cap, -1)[:, :L].reshape(G * L, -1)  # noqa: E731
        return ops.PackedKV((G * L, self.D), 1, take(p.code), take(p.norms).view(-1),
                            take(p.res), take(p.rnorms).view(-1))


class PackedAttention:
    """Returned by ``KudahitamLayer.update`` as both K and V on a one-token
    decode step of a cache with ``packed_attention=True``: the layer whose
    packed cache the attention function reads.  ``shape`` is that of the
    dequantised K it stands for ([B, H_kv, length, D])."""

    def __init__(self, layer: "KudahitamLayer"):
        self.layer = layer

    @property
    def shape(self):
        s = self.layer.k
        return (s.B, s.H, s.length, s.D)

    def dequantized(self) -> tuple[torch.Tensor, torch.Tensor]:
        return self.layer.dequantized()


def kudahitam_attention(module, query: torch.Tensor, key, value, attention_mask,
                        scaling: Optional[float] = None, dropout: float = 0.0, **kwargs):
    """transformers attention function (``attn_implementation="kudahitam"``).

    A ``PackedAttention`` key (a one-token decode step) runs the decode
    kernel over the layer's packed K and V: query [B, H_q, 1, D] ->
    [B, 1, H_q, D], no dequantisation, grouped-query heads read their KV
    head without expansion.  The packed path attends to every cached token,
    so a mask that hides some of them (left padding in a batch) falls back
    to dequantised K and V.  Tensor K and V (prefill) go to PyTorch's
    scaled-dot-product attention."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    if isinstance(key, PackedAttention):
        hides = attention_mask is not None and (
            (attention_mask.dtype == torch.bool and not bool(attention_mask.all())) or
            (attention_mask.dtype != torch.bool and bool((attention_mask < 0).any())))
        if query.shape[2] == 1 and not hides:
            out = key.layer.attend(query[:, :, 0], sm_scale=scaling)  # float32 [B, H_q, D]
            return out.to(query.dtype).unsqueeze(1), None
        key, value = key.dequantized()
    return sdpa_attention_forward(module, query, key, value, attention_mask, scaling=scaling,
                                  dropout=dropout, **kwargs)


def register_attention(name: str = "kudahitam") -> str:
    """Register ``kudahitam_attention`` (and PyTorch SDPA's mask builder) with
    transformers under ``name``; load a model with
    ``attn_implementation=name`` and give it ``KudahitamCache(...,
    packed_attention=True)``."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    AttentionInterface.register(name, kudahitam_attention)
    AttentionMaskInterface.register(name, sdpa_mask)
    return name


class KudahitamLayer(_LayerBase):
    """One layer's compressed K and V (transformers ``CacheLayerMixin``
    contract: update / get_seq_length / get_mask_sizes / ...)."""

    is_sliding = False
    is_compileable = False

    def __init__(self, head_dim: int, seed_k: int = 0, seed_v: int = 1,
                 initial_capacity: int = 256, packed_attention: bool = False):
        super().__init__()
        self.head_dim = head_dim
        self.packed_attention = packed_attention
        self.d_k, self.d_v = rademacher(head_dim, seed_k), rademacher(head_dim, seed_v)
        self.c = lloyd_max(1, head_dim)
        self.initial_capacity = initial_capacity
        self.k: Optional[PackedSeq] = None
        self.v: Optional[PackedSeq] = None
        self.keys = self.values = None  # transformers inspects these attributes
        self.is_initialized = False
        self.dtype = None
        self.device = None

    def __repr__(self):
        return f"KudahitamLayer(head_dim={self.head_dim}, length={self.get_seq_length()})"

    def lazy_initialization(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        B, H, _, D = key_states.shape
        if D != self.head_dim:
            raise ValueError(f"head_dim {D} != {self.head_dim}")
        self.dtype, self.device = key_states.dtype, key_states.device
        cap = max(self.initial_capacity, key_states.shape[-2])
        self.k = PackedSeq(B, H, D, self.device, cap)
        self.v = PackedSeq(B, value_states.shape[1], D, self.device, cap)
        self.is_initialized = True

    def append(self, key_states: torch.Tensor, value_states: torch.Tensor) -> None:
        if not self.is_initialized:
            self.lazy_initialization(key_states, value_states)
        self.k.append(key_states, self.d_k, self.c)
        self.v.append(value_states, self.d_v, self.c)

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, *args, **kwargs):
        """Append (compress) the new tokens, then return what the model's
        attention reads: the new K and V themselves when the layer was empty
        (prefill attends to itself), a ``PackedAttention`` handle on a
        one-token step with ``packed_attention``, else dequantised K and V
        of every cached token."""
        first = self.get_seq_length() == 0
        self.append(key_states, value_states)
        if first:
            return key_states, value_states
        if self.packed_attention and key_states.shape[-2] == 1:
            h = PackedAttention(self)
            return h, h
        return self.dequantized()

    def dequantized(self) -> tuple[torch.Tensor, torch.Tensor]:
        return (self.k.dequantize(self.d_k, self.c, 1.0, self.dtype),
                self.v.dequantize(self.d_v, self.c, _SQRT_2_OVER_PI, self.dtype))

    def attend(self, query: torch.Tensor, sm_scale: Optional[float] = None,
               n_splits: Optional[int] = None) -> torch.Tensor:
        """Decode attention of query [B, H_q, D] or [B, H_q, 1, D] over the
        cached tokens, from the packed bytes.  Returns float32 [B, H_q, D]."""
        B, Hq = query.shape[0], query.shape[1]
        Hk, D = self.k.H, self.head_dim
        if Hq % Hk or B != self.k.B:
            raise ValueError(f"{Hq} query heads / batch {B} do not map onto {Hk} KV heads")
        q = query.reshape(B * Hk, Hq // Hk, D)
        out = ops.decode_attention(q, self.k.packed, self.v.packed, self.d_k, self.d_v, self.c,
                                   sm_scale=sm_scale, n_splits=n_splits,
                                   seq_len=self.k.capacity, length=self.k.length)
        return out.view(B, Hq, D)

    def scores(self, query: torch.Tensor) -> torch.Tensor:
        """The reference's asymmetric scores (KudaHitamQuant_full.py:373-377)
        of query [B, H_q, n, D] against the cached keys: float32
        [B, H_q, n, length]."""
        B, Hq, n, D = query.shape
        Hk, L, cap = self.k.H, self.k.length, self.k.capacity
        q = query.reshape(B * Hk, (Hq // Hk) * n, D)
        sc = ops.score(q, self.k.packed, self.d_k, self.c, seq_len=cap)
        return sc[..., :L].reshape(B, Hq, n, L)

    def get_seq_length(self) -> int:
        return 0 if self.k is None else self.k.length

    def get_mask_sizes(self, query_length: int) -> tuple[int, int]:
        return self.get_seq_length() + query_length, 0

    def get_max_cache_shape(self) -> int:
        return -1

    def crop(self, max_length: int) -> None:
        if self.k is None:
            return
        if max_length < 0:
            max_length = self.get_seq_length() + max_length
        self.k.truncate(max_length)
        self.v.truncate(max_length)

    def reset(self) -> None:
        self.crop(0)

    def offload(self):  # packed planes stay on the device
        pass

    def prefetch(self):
        pass

    def nbytes(self) -> int:
        """Bytes of the filled part of the packed K and V."""
        if self.k is None:
            return 0
        per_row = self.head_dim // 32 * 8 + 8  # code + res words, 2 norms
        return per_row * (self.k.groups + self.v.groups) * self.k.length


def KudahitamCache(num_layers: Optional[int] = None, head_dim: int = 128, seed: int = 0,
                   initial_capacity: int = 256, packed_attention: bool = False):
    """A transformers ``Cache`` whose layers are ``KudahitamLayer``s (layer
    l uses seeds 2 seed + 2 l and 2 seed + 2 l + 1 for its K and V
    diagonals).  Pass it as ``past_key_values``.  With
    ``packed_attention=True`` (and a model loaded with the attention
    registered by ``register_attention``) decode steps attend from the
    packed bytes; ``cache.layers[l].attend(q)`` does the same directly."""
    from transformers.cache_utils import Cache

    class _KudahitamCache(Cache):
        def __init__(self):
            self._made = 0
            layers = None
            if num_layers is not None:
                layers = [self._new_layer() for _ in range(num_layers)]
            super().__init__(layers=layers,
                             layer_class_to_replicate=None if layers else self._new_layer)

        def _new_layer(self):
            l = self._made
            self._made += 1
            return KudahitamLayer(head_dim, 2 * seed + 2 * l, 2 * seed + 2 * l + 1,
                                  initial_capacity, packed_attention)

        def attend(self, layer_idx: int, query: torch.Tensor, **kw) -> torch.Tensor:
            return self.layers[layer_idx].attend(query, **kw)

        def nbytes(self) -> int:
            return sum(l.nbytes() for l in self.layers)

    return _KudahitamCache()


def from_dynamic_cache(dc, head_dim: Optional[int] = None, seed: int = 0):
    """Compress a filled transformers cache (``DynamicCache`` or anything
    with ``layers[l].keys / .values`` [B, H, S, D]) into a KudahitamCache,
    the reference's post-prefill step (KudaHitamQuant_full.py:654-668)."""
    src = [(l.keys, l.values) for l in dc.layers]
    D = head_dim or next(k.shape[-1] for k, _ in src if k is not None and k.numel())
    cache = KudahitamCache(num_layers=len(src), head_dim=D, seed=seed,
                           initial_capacity=max((k.shape[-2] for k, _ in src
                                                 if k is not None and k.numel()), default=1))
    for layer, (k, v) in zip(cache.layers, src):
        if k is not None and k.numel():
            layer.append(k, v)
    return cache
