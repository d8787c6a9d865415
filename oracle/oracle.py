"""CPU oracle for the KudaHitamQuant KV-compression path.

TEST INFRASTRUCTURE: only the tests, ``__graft_entry__.smoke()`` and the CPU
baseline leg of ``bench.py`` import this module, as the checker.  The engine
never calls it.

Wraps ``kh_oracle.c`` (a line-by-line fp32 restatement of the reference's
``ultra_fused_full_fusion_kernel_v8``, KudaHitamCUDA.cu:13-195, and of
``asymmetric_attention_scores``, KudaHitamQuant_full.py:373-377) and adds the
bit packing of the engine's cache layout in numpy.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import subprocess

import numpy as np

_DIR = pathlib.Path(__file__).resolve().parent
_SO = _DIR / "_build" / "libkh_oracle.so"
_lib = None

F32, F16, BF16 = 0, 1, 2

_fp = ctypes.POINTER(ctypes.c_float)
_vp = ctypes.c_void_p


def build() -> pathlib.Path:
    """Compile the oracle library (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", str(_DIR)], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not _SO.exists():
            build()
        L = ctypes.CDLL(str(_SO))
        L.khx_compress_v8.argtypes = [_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_int,
                                      ctypes.c_int64, _vp, _vp, ctypes.c_int, _vp, _vp,
                                      _vp, _vp, _vp, ctypes.c_int]
        L.khx_compress_v8.restype = None
        L.khx_fwht_v8.argtypes = [_vp, ctypes.c_int]
        L.khx_fwht_forward.argtypes = [_vp, ctypes.c_int64, ctypes.c_int]
        L.khx_score.argtypes = [_vp, ctypes.c_int64, ctypes.c_int, ctypes.c_int, _vp, _vp,
                                _vp, ctypes.c_int64, _vp, _vp]
        L.khx_decode.argtypes = [_vp, ctypes.c_int64, ctypes.c_int, _vp, _vp, _vp, _vp, _vp,
                                 _vp, ctypes.c_int64, _vp, _vp, ctypes.c_float, _vp]
        L.khx_compat_score.argtypes = [_vp, ctypes.c_int64, ctypes.c_int, ctypes.c_int64, _vp,
                                       ctypes.c_int, _vp, _vp, _vp, _vp, _vp, ctypes.c_float,
                                       _vp]
        L.khx_hbba_compress.argtypes = [_vp, ctypes.c_int, ctypes.c_int64, ctypes.c_int, _vp,
                                        _vp, _vp, ctypes.c_int, _vp, _vp, _vp, _vp]
        L.khx_hbba_calibrate.argtypes = [_vp, ctypes.c_int64, ctypes.c_int, _vp, _vp]
        L.khx_num_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def num_threads() -> int:
    return int(lib().khx_num_threads())


def as_raw(x) -> tuple[np.ndarray, int]:
    """(numpy view of the raw elements, dtype code) for a torch tensor or numpy
    array; bf16 travels as its 16-bit pattern."""
    try:
        import torch
        if isinstance(x, torch.Tensor):
            x = x.detach().cpu().contiguous()
            if x.dtype == torch.bfloat16:
                return x.view(torch.int16).numpy().view(np.uint16), BF16
            if x.dtype == torch.float16:
                return x.numpy(), F16
            return x.float().numpy(), F32
    except ImportError:  # pragma: no cover
        pass
    x = np.ascontiguousarray(x)
    if x.dtype == np.float16:
        return x, F16
    return x.astype(np.float32, copy=False), F32


def compress_v8(x, d, c, *, want=("idx", "norms", "kmse", "rnorms", "signs"),
                n_threads: int = 0) -> dict:
    """Reference kernel outputs for rows x[..., D] (any float dtype, upcast
    exactly as the kernel does at KudaHitamCUDA.cu:41-42)."""
    raw, code = as_raw(x)
    D = raw.shape[-1]
    raw = raw.reshape(-1, D)
    n = raw.shape[0]
    d = np.ascontiguousarray(np.asarray(d, dtype=np.float32))
    c = np.ascontiguousarray(np.asarray(c, dtype=np.float32))
    out = {
        "idx": np.empty((n, D), np.uint8) if "idx" in want else None,
        "norms": np.empty(n, np.float32) if "norms" in want else None,
        "kmse": np.empty((n, D), np.float32) if "kmse" in want else None,
        "rnorms": np.empty(n, np.float32) if "rnorms" in want else None,
        "signs": np.empty((n, D), np.int8) if "signs" in want else None,
    }
    lib().khx_compress_v8(_ptr(raw), code, n, D, D, _ptr(d), _ptr(c), len(c),
                          _ptr(out["idx"]), _ptr(out["norms"]), _ptr(out["kmse"]),
                          _ptr(out["rnorms"]), _ptr(out["signs"]), int(n_threads))
    return {k: v for k, v in out.items() if v is not None}


def fwht_forward(x) -> np.ndarray:
    """x <- H x / sqrt(D) per row (the GPU ``forward`` op)."""
    a = np.array(x, dtype=np.float32, copy=True, order="C")
    D = a.shape[-1]
    lib().khx_fwht_forward(_ptr(a), a.size // D, D)
    return a


def fwht_v8(x) -> np.ndarray:
    """Unnormalised Sylvester transform in the v8 butterfly order."""
    a = np.array(x, dtype=np.float32, copy=True, order="C")
    D = a.shape[-1]
    flat = a.reshape(-1, D)
    for i in range(flat.shape[0]):
        lib().khx_fwht_v8(_ptr(flat[i]), D)
    return a


def pack_bits(b: np.ndarray) -> np.ndarray:
    """bool/0-1 [N, D] -> uint32 [N, D/32], element i at bit i&31 of word i>>5."""
    b = np.ascontiguousarray(b, dtype=np.uint8)
    n, D = b.shape
    packed = np.packbits(b, axis=1, bitorder="little")  # [N, D/8] bytes
    return packed.view("<u4").reshape(n, D // 32).astype(np.uint32)


def pack_idx2(idx: np.ndarray) -> np.ndarray:
    """2-bit indices [N, D] -> uint32 [N, D/16], element i at bits 2*(i&15) of
    word i>>4."""
    idx = np.ascontiguousarray(idx, dtype=np.uint32)
    n, D = idx.shape
    g = idx.reshape(n, D // 16, 16)
    sh = (2 * np.arange(16, dtype=np.uint32))[None, None, :]
    return np.bitwise_or.reduce(g << sh, axis=2).astype(np.uint32)


def unpack_bits(w: np.ndarray, D: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint32)
    by = w.view(np.uint8).reshape(w.shape[0], -1)
    return np.unpackbits(by, axis=1, bitorder="little")[:, :D]


def unpack_idx2(w: np.ndarray, D: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint32)
    sh = (2 * np.arange(16, dtype=np.uint32))[None, None, :]
    return ((w[:, :, None] >> sh) & 3).reshape(w.shape[0], -1)[:, :D].astype(np.uint8)


def packed_from_v8(out: dict, n_c: int) -> dict:
    """The engine's packed cache built from the reference outputs."""
    code = pack_bits(out["idx"]) if n_c == 2 else pack_idx2(out["idx"])
    res = pack_bits(out["signs"] > 0) if "signs" in out else None
    return {"code": code, "res": res, "norms": out["norms"],
            "rnorms": out.get("rnorms")}


def score(q, kmse, signs, rnorms, d) -> np.ndarray:
    """Reference scores.  q [G, nq, D]; kmse/signs [G, S, D]; rnorms [G, S]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    G, nq, D = q.shape
    S = kmse.shape[1]
    kmse = np.ascontiguousarray(kmse, dtype=np.float32)
    signs = None if signs is None else np.ascontiguousarray(signs, dtype=np.int8)
    rn = None if rnorms is None else np.ascontiguousarray(rnorms, dtype=np.float32)
    d = np.ascontiguousarray(d, dtype=np.float32)
    out = np.empty((G, nq, S), np.float32)
    lib().khx_score(_ptr(q), G, nq, D, _ptr(kmse), _ptr(signs), _ptr(rn), S, _ptr(d),
                    _ptr(out))
    return out


def decode(q, k_kmse, k_signs, k_rnorms, v_kmse, v_signs, v_rnorms, dk, dv,
           sm_scale: float) -> np.ndarray:
    """Softmax(score * sm_scale) . V_hat in double.  q [G, D]; caches [G, S, D]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    G, D = q.shape
    S = k_kmse.shape[1]
    arrs = [np.ascontiguousarray(a, dtype=t) for a, t in
            ((k_kmse, np.float32), (k_signs, np.int8), (k_rnorms, np.float32),
             (v_kmse, np.float32), (v_signs, np.int8), (v_rnorms, np.float32),
             (dk, np.float32), (dv, np.float32))]
    out = np.empty((G, D), np.float32)
    lib().khx_decode(_ptr(q), G, D, *[_ptr(a) for a in arrs[:6]], S, _ptr(arrs[6]),
                     _ptr(arrs[7]), float(sm_scale), _ptr(out))
    return out


def compat_score(q, k_packed, signs, d, k_norms, r_norms, centroids, nibble: bool,
                 scale: float) -> np.ndarray:
    """The reference's packed-byte scorer (KudaHitamCUDA.cu:695-772).
    q fp16 [H, D]; k_packed uint8 [H, S, 32 or 128]; signs fp16 [H, S, D];
    k_norms, r_norms [H, S]; centroids [D, 16].  Returns float32 [H, S]."""
    q = np.ascontiguousarray(q, dtype=np.float16)
    H, D = q.shape
    kp = np.ascontiguousarray(k_packed, dtype=np.uint8)
    S = kp.shape[1]
    sg = np.ascontiguousarray(signs, dtype=np.float16)
    arrs = [np.ascontiguousarray(a, dtype=np.float32) for a in (d, k_norms, r_norms, centroids)]
    out = np.empty((H, S), np.float32)
    lib().khx_compat_score(_ptr(q), H, D, S, _ptr(kp), int(bool(nibble)), _ptr(sg),
                           *[_ptr(a) for a in arrs], float(scale), _ptr(out))
    return out


def hbba_compress(x, d, centroids, mask, is_hbba: bool) -> dict:
    """The HBBA encoder (KudaHitamCUDA.cu:285-395, whole-row reductions):
    x [..., D]; centroids [D, 16]; mask [8] uint32.  Returns packed uint8
    [N, 128 or 32], norms [N], r_norms [N], signs float16 [N, D]."""
    raw, code = as_raw(x)
    D = raw.shape[-1]
    raw = np.ascontiguousarray(raw.reshape(-1, D))
    n = raw.shape[0]
    d = np.ascontiguousarray(np.asarray(d, dtype=np.float32))
    cen = np.ascontiguousarray(np.asarray(centroids, dtype=np.float32).reshape(D, 16))
    m = np.ascontiguousarray(np.asarray(mask).astype(np.int64).astype(np.uint32).reshape(8))
    bpt = 128 if is_hbba else 32
    out = {"packed": np.zeros((n, bpt), np.uint8), "norms": np.empty(n, np.float32),
           "rnorms": np.empty(n, np.float32), "signs": np.empty((n, D), np.float16)}
    lib().khx_hbba_compress(_ptr(raw), code, n, D, _ptr(d), _ptr(cen), _ptr(m), int(is_hbba),
                            _ptr(out["packed"]), _ptr(out["norms"]), _ptr(out["rnorms"]),
                            _ptr(out["signs"]))
    return out


def hbba_calibrate(sample, n_map) -> np.ndarray:
    """The HBBA calibrator (KudaHitamCUDA.cu:423-496): sample [N, D] float;
    n_map [D] levels per dimension.  Returns centroids [D, 16]."""
    smp = np.ascontiguousarray(np.asarray(sample, dtype=np.float32))
    n, D = smp.shape
    nm = np.ascontiguousarray(np.asarray(n_map, dtype=np.int32).reshape(D))
    out = np.zeros((D, 16), np.float32)
    lib().khx_hbba_calibrate(_ptr(smp), n, D, _ptr(nm), _ptr(out))
    return out


def merge_partials(parts: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Split-K merge of (m, l, acc[D]) records [G, P, D+2] -> (m, l, acc) with
    empty records (l == 0) ignored."""
    parts = np.asarray(parts, dtype=np.float64)
    m, l, acc = parts[..., 0], parts[..., 1], parts[..., 2:]
    live = l > 0
    M = np.where(live, m, -np.inf).max(axis=1)
    e = np.where(live, np.exp(m - np.where(np.isfinite(M), M, 0.0)[:, None]), 0.0)
    return M, (l * e).sum(axis=1), (acc * e[..., None]).sum(axis=1)


_ref_mod = None


def reference_kernels():
    """The reference's own CUDA kernels (KudaHitamCUDA.cu, built for sm_100a
    by build_ref.py into _ref/kh_ref.so), or None when that build is absent.
    Exposes ultra_fused_full_fusion (kernel v8), forward (FWHT) and
    fused_asymmetric_attention, with the reference's argument conventions."""
    global _ref_mod
    if _ref_mod is None:
        so = _DIR / "_ref" / "kh_ref.so"
        if not so.exists():
            return None
        import importlib.util

        import torch  # noqa: F401  (the module links against torch)
        spec = importlib.util.spec_from_file_location("kh_ref", so)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        _ref_mod = mod
    return _ref_mod
