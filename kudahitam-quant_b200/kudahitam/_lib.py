"""ctypes binding of ``libkudahitam.so`` (declared in ``include/kudahitam.h``).

The library is the only compute path: when it is missing every op raises
``NativeLibraryError``; there is no CPU or pure-PyTorch fallback.
"""
from __future__ import annotations

import ctypes
import os
import pathlib
import threading

_SO = pathlib.Path(__file__).resolve().parent / "_lib" / "libkudahitam.so"

KH_OK, KH_EINVAL, KH_EALIGN, KH_ELAUNCH, KH_ECUDA, KH_ENOTSUP = range(6)
KH_F32, KH_F16, KH_BF16 = 0, 1, 2

_c_i = ctypes.c_int
_c_i64 = ctypes.c_int64
_c_f = ctypes.c_float
_vp = ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/kudahitam.h one to one.
SIGNATURES = {
    "kh_status_string": (ctypes.c_char_p, [_c_i]),
    "kh_version": (_c_i, []),
    "kh_device_error": (_c_i, [ctypes.POINTER(ctypes.c_uint32)]),
    "kh_clear_device_error": (_c_i, []),
    "kh_max_segments": (_c_i, []),
    "kh_compress": (_c_i, [_vp, _c_i, _c_i64, _c_i, _c_i64, _vp, _vp, _c_i, _c_i,
                           _vp, _vp, _vp, _vp, _vp]),
    "kh_compress_batched": (_c_i, [_c_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _c_i, _c_i,
                                   _vp, _vp, _c_i, _c_i, _vp]),
    "kh_fwht_inplace": (_c_i, [_vp, _c_i64, _c_i, _vp]),
    "kh_materialize": (_c_i, [_vp, _vp, _vp, _c_i64, _c_i, _vp, _vp, _c_i, _vp, _vp,
                              _vp, _vp]),
    "kh_score": (_c_i, [_vp, _c_i64, _c_i, _c_i, _vp, _vp, _vp, _vp, _c_i64, _vp, _vp,
                        _c_i, _vp, _vp]),
    "kh_score_packed_compat": (_c_i, [_vp, _c_i64, _c_i, _c_i64, _vp, _vp, _vp, _vp, _vp,
                                      _vp, _c_i, _c_i, _c_f, _vp, _vp]),
    "kh_compress_hbba": (_c_i, [_vp, _c_i, _c_i64, _c_i, _c_i64, _vp, _vp, _vp, _c_i, _c_i,
                                _vp, _vp, _vp, _vp, _vp]),
    "kh_hbba_calibrate": (_c_i, [_vp, _c_i64, _c_i, _vp, _vp, _vp]),
    "kh_decode_workspace_bytes": (_c_i64, [_c_i64, _c_i, _c_i]),
    "kh_decode_partial": (_c_i, [_vp, _c_i64, _c_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                 _vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, _c_i, _c_f,
                                 _c_i, _vp, _c_i64, _c_i64, _vp]),
    "kh_decode_partial_gqa": (_c_i, [_vp, _c_i64, _c_i, _c_i, _vp, _vp, _vp, _vp, _vp, _vp,
                                     _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, _c_i,
                                     _c_f, _c_i, _vp, _c_i64, _c_i64, _vp]),
    "kh_decode_combine": (_c_i, [_vp, _c_i64, _c_i, _c_i, _vp, _vp, _vp]),
    "kh_decode_combine_strided": (_c_i, [_vp, _c_i64, _c_i, _c_i64, _c_i64, _c_i, _vp, _vp,
                                         _vp]),
    "kh_decode_merge": (_c_i, [_vp, _c_i64, _c_i, _c_i64, _c_i64, _c_i, _vp, _vp]),
    "kh_decode_merge_to_peers": (_c_i, [_vp, _c_i64, _c_i, _c_i64, _c_i64, _c_i, _vp, _vp,
                                        _c_i, _c_i, ctypes.c_uint32, _vp, _vp]),
    "kh_decode_combine_from_peers": (_c_i, [_vp, _vp, ctypes.c_uint32, _c_i64, _c_i, _c_i,
                                            _vp, _vp, _vp]),
    "kh_decode_partial_to_peers": (_c_i, [_vp, _c_i64, _c_i, _c_i, _vp, _vp, _vp, _vp, _vp,
                                          _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp,
                                          _c_i, _c_f, _c_i, _vp, _vp, _c_i, _c_i,
                                          ctypes.c_uint32, _vp, _vp, _vp]),
    "kh_decode_combine_peer_records": (_c_i, [_vp, _vp, ctypes.c_uint32, _c_i64, _c_i, _c_i,
                                              _c_i, _vp, _vp, _vp]),
    "kh_decode_attn": (_c_i, [_vp, _c_i64, _c_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                              _c_i64, _vp, _vp, _vp, _c_i, _c_f, _c_i, _vp, _c_i64, _vp,
                              _vp]),
    "kh_decode_attn_static": (_c_i, [_vp, _c_i64, _c_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                     _vp, _c_i64, _vp, _vp, _vp, _c_i, _c_f, _c_i, _vp,
                                     _vp]),
}

# Size of the library's fixed scratch array used by kh_decode_attn_static.
DECODE_STATIC_SCRATCH_BYTES = 4 * 1024 * 1024


class NativeLibraryError(RuntimeError):
    """The compiled engine is missing or failed to load."""


class KHError(RuntimeError):
    """A C-ABI call returned a non-zero kh_status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed: {msg} (kh_status={status})")
        self.status = status


_lock = threading.Lock()
_lib = None


def library_path() -> pathlib.Path:
    return pathlib.Path(os.environ.get("KUDAHITAM_LIB", str(_SO)))


def lib() -> ctypes.CDLL:
    """Load the engine (once).  Raises NativeLibraryError if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not path.exists():
                raise NativeLibraryError(
                    f"{path} not found: build it with `python kudahitam-quant_b200/build.py`")
            try:
                L = ctypes.CDLL(str(path))
            except OSError as e:  # pragma: no cover
                raise NativeLibraryError(f"cannot load {path}: {e}") from e
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(fn: str, status: int) -> None:
    if status != KH_OK:
        msg = lib().kh_status_string(status).decode()
        raise KHError(fn, status, msg)


def call(fn: str, *args) -> None:
    check(fn, getattr(lib(), fn)(*args))


def device_error() -> int:
    v = ctypes.c_uint32(0)
    check("kh_device_error", lib().kh_device_error(ctypes.byref(v)))
    return int(v.value)
