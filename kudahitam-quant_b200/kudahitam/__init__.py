"""kudahitam -- B200 (sm_100a) engine for KudaHitamQuant's KV-cache
compression hot path, behind the reference's Python API
(KudaHitamQuant_full.py: ``KudahitamCompressorV2``, ``fwht``,
``load_cuda_ext``)."""
from __future__ import annotations

import types

from . import ops
from ._lib import KHError, NativeLibraryError, library_path
from .codebook import lloyd_max, rademacher
from .compressor import CompressedKV, KudahitamCompressorV2
from .hbba import KudahitamCompressorHBBA
from .ops import PackedKV

__all__ = ["KudahitamCompressorV2", "KudahitamCompressorHBBA", "CompressedKV", "PackedKV", "fwht", "fwht_",
           "load_cuda_ext", "lloyd_max", "rademacher", "ops", "KHError",
           "NativeLibraryError", "library_path"]


def fwht(x):
    """Orthonormal Walsh-Hadamard transform along the last dim of a CUDA
    tensor (the reference's ``fwht``, KudaHitamQuant_full.py:207-215; its CPU
    branch is unnormalised, this engine has no CPU branch)."""
    return ops.fwht(x)


fwht_ = ops.fwht_


def load_cuda_ext():
    """The reference's extension handle (KudaHitamQuant_full.py:43-98, module
    KudaHitamCUDA.cu:799-804): an object with ``forward`` (in-place
    orthonormal FWHT of [N, D] float32 rows), ``ultra_fused_full_fusion``
    (the fused compressor with the reference kernel's five outputs, defined
    but never bound by the reference), ``ultra_fused_hbba_fusion`` and
    ``hbba_calibrate_cuda`` (the HBBA encoder and calibrator) and
    ``fused_asymmetric_attention`` (the packed-byte scorer,
    KudaHitamCUDA.cu:695-797).  Raises NativeLibraryError when the engine is
    not built, instead of returning None."""
    from . import _lib
    _lib.lib()
    ops.ext()
    return types.SimpleNamespace(forward=ops.fwht_,
                                 ultra_fused_full_fusion=ops.ultra_fused_full_fusion,
                                 ultra_fused_hbba_fusion=ops.ultra_fused_hbba_fusion,
                                 hbba_calibrate_cuda=ops.hbba_calibrate,
                                 fused_asymmetric_attention=ops.fused_asymmetric_attention)
