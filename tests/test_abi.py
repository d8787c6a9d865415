"""The C ABI: the library loads, exports exactly what include/kudahitam.h
declares, and validates arguments without touching a GPU."""
import ctypes
import pathlib
import re

import pytest

from kudahitam import _lib

HEADER = pathlib.Path(__file__).resolve().parents[1] / "include" / "kudahitam.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kh_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declaration():
    L = _lib.lib()
    names = declared()
    assert len(names) >= 14
    for n in names:
        assert hasattr(L, n), n
        assert n in _lib.SIGNATURES, n
    assert sorted(_lib.SIGNATURES) == names


def test_status_strings_and_version():
    L = _lib.lib()
    assert L.kh_version() >= 100
    assert L.kh_status_string(0) == b"ok"
    assert b"aligned" in L.kh_status_string(_lib.KH_EALIGN)
    assert L.kh_status_string(99) == b"unknown status"


def _f(vals):
    return (ctypes.c_float * len(vals))(*vals)


D128 = _f([1.0, -1.0] * 64)
C2 = _f([-0.07, 0.07])
FAKE = ctypes.c_void_p(0x10000)  # never dereferenced: validation fails first


@pytest.mark.parametrize("kw,status", [
    (dict(head_dim=64), _lib.KH_EINVAL),
    (dict(dtype=7), _lib.KH_EINVAL),
    (dict(n_centroids=3), _lib.KH_EINVAL),
    (dict(centroids=_f([0.07, -0.07])), _lib.KH_EINVAL),
    (dict(d=_f([0.5] * 128)), _lib.KH_EINVAL),
    (dict(residual=2), _lib.KH_EINVAL),
    (dict(x=ctypes.c_void_p(0x10008)), _lib.KH_EALIGN),
    (dict(row_stride=100), _lib.KH_EINVAL),
    (dict(row_stride=132, dtype=_lib.KH_BF16), _lib.KH_EALIGN),
    (dict(res=None), _lib.KH_EINVAL),
    (dict(n_rows=-1), _lib.KH_EINVAL),
    (dict(n_rows=1 << 31), _lib.KH_EINVAL),
    (dict(n_rows=0), _lib.KH_OK),
])
def test_compress_validation(kw, status):
    a = dict(x=FAKE, dtype=_lib.KH_F32, n_rows=10, head_dim=128, row_stride=128, d=D128,
             centroids=C2, n_centroids=2, residual=1, code=FAKE, res=FAKE, norms=FAKE,
             rnorms=FAKE)
    a.update(kw)
    st = _lib.lib().kh_compress(a["x"], a["dtype"], a["n_rows"], a["head_dim"], a["row_stride"],
                                a["d"], a["centroids"], a["n_centroids"], a["residual"],
                                a["code"], a["res"], a["norms"], a["rnorms"], None)
    assert st == status


def test_batched_validation():
    L = _lib.lib()
    assert L.kh_max_segments() == 64
    assert L.kh_compress_batched(65, None, None, None, None, None, None, None, 0, 128, D128,
                                 C2, 2, 1, None) == _lib.KH_EINVAL
    assert L.kh_compress_batched(0, None, None, None, None, None, None, None, 0, 128, D128,
                                 C2, 2, 1, None) == _lib.KH_OK


def test_other_entry_points_validate():
    L = _lib.lib()
    assert L.kh_fwht_inplace(FAKE, 4, 100, None) == _lib.KH_EINVAL
    assert L.kh_fwht_inplace(FAKE, 0, 128, None) == _lib.KH_OK
    assert L.kh_materialize(FAKE, None, FAKE, 4, 96, D128, C2, 2, None, None, None,
                            None) == _lib.KH_EINVAL
    assert L.kh_materialize(FAKE, None, FAKE, 4, 128, D128, C2, 2, None, None, FAKE,
                            None) == _lib.KH_EINVAL  # signs need res_bits
    assert L.kh_score(FAKE, 2, 1, 128, FAKE, FAKE, FAKE, None, 16, D128, C2, 2, FAKE,
                      None) == _lib.KH_EINVAL  # res_bits without r_norms
    assert L.kh_decode_workspace_bytes(10, 4, 128) == 10 * 4 * 130 * 4
    assert L.kh_decode_workspace_bytes(10, 0, 128) == -1
    assert L.kh_decode_partial(FAKE, 2, 128, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE,
                               100, 50, 10, D128, D128, C2, 2, 0.1, 2, FAKE, 2, 0,
                               None) == _lib.KH_EINVAL  # seq_end < seq_begin
    assert L.kh_decode_partial(FAKE, 2, 128, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE,
                               100, 0, 100, D128, D128, _f([-0.1, 0.05, -0.05, 0.1]), 4, 0.1,
                               2, FAKE, 2, 0, None) == _lib.KH_EINVAL  # unsorted codebook
    assert L.kh_decode_attn(FAKE, 2, 128, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 100,
                            D128, D128, C2, 2, 0.1, 4, FAKE, 16, FAKE,
                            None) == _lib.KH_EINVAL  # workspace too small
    assert L.kh_decode_merge(FAKE, 2, 0, 260, 130, 128, FAKE, None) == _lib.KH_EINVAL
    assert L.kh_decode_merge(FAKE, 2, 2, 260, 130, 96, FAKE, None) == _lib.KH_EINVAL
    assert L.kh_decode_merge(FAKE, 2, 2, -1, 130, 128, FAKE, None) == _lib.KH_EINVAL
    assert L.kh_decode_merge(FAKE, 0, 2, 260, 130, 128, FAKE, None) == _lib.KH_OK
    assert L.kh_decode_merge(FAKE, 2, 2, 260, 130, 128, None, None) == _lib.KH_EINVAL
    assert L.kh_decode_merge(ctypes.c_void_p(0x10002), 2, 2, 260, 130, 128, FAKE,
                             None) == _lib.KH_EALIGN
    assert L.kh_decode_combine_strided(FAKE, 2, 2, 260, -130, 128, D128, FAKE,
                                       None) == _lib.KH_EINVAL
    assert L.kh_decode_combine_strided(FAKE, 2, 2, 260, 130, 128, None, FAKE,
                                       None) == _lib.KH_EINVAL  # no d vector
    two = (ctypes.c_void_p * 2)(0x10000, 0x20000)
    P2 = ctypes.cast(two, ctypes.c_void_p)
    assert L.kh_decode_merge_to_peers(FAKE, 2, 2, 260, 130, 128, P2, P2, 0, 9, 1, FAKE,
                                      None) == _lib.KH_EINVAL  # world > 8
    assert L.kh_decode_merge_to_peers(FAKE, 2, 2, 260, 130, 128, P2, P2, 2, 2, 1, FAKE,
                                      None) == _lib.KH_EINVAL  # rank >= world
    assert L.kh_decode_merge_to_peers(FAKE, 2, 2, 260, 130, 128, P2, P2, 0, 2, 0, FAKE,
                                      None) == _lib.KH_EINVAL  # epoch 0
    assert L.kh_decode_merge_to_peers(FAKE, 2, 2, 260, 130, 128, P2, P2, 0, 2, 1, None,
                                      None) == _lib.KH_EINVAL  # no counter
    assert L.kh_decode_merge_to_peers(FAKE, 0, 2, 260, 130, 128, P2, P2, 0, 2, 1, FAKE,
                                      None) == _lib.KH_OK
    assert L.kh_decode_combine_from_peers(FAKE, FAKE, 0, 2, 2, 128, D128, FAKE,
                                          None) == _lib.KH_EINVAL  # epoch 0
    assert L.kh_decode_combine_from_peers(FAKE, FAKE, 1, 2, 2, 128, None, FAKE,
                                          None) == _lib.KH_EINVAL  # no d vector
    assert L.kh_decode_combine_from_peers(FAKE, FAKE, 1, 0, 2, 128, D128, FAKE,
                                          None) == _lib.KH_OK
    assert L.kh_decode_combine_peer_records(FAKE, FAKE, 1, 2, 0, 2, 128, D128, FAKE,
                                            None) == _lib.KH_EINVAL  # no parts
    assert L.kh_decode_combine_peer_records(FAKE, FAKE, 1, 2, 3, 9, 128, D128, FAKE,
                                            None) == _lib.KH_EINVAL  # world > 8
    assert L.kh_decode_combine_peer_records(FAKE, FAKE, 1, 0, 3, 2, 128, D128, FAKE,
                                            None) == _lib.KH_OK

    def to_peers(rank, world, epoch, counter, n_groups=2, records=P2):
        return L.kh_decode_partial_to_peers(
            FAKE, n_groups, 1, 128, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 100, 0, 100,
            D128, D128, C2, 2, 0.1, 2, records, P2, rank, world, epoch, counter, None, None)
    assert to_peers(0, 9, 1, FAKE) == _lib.KH_EINVAL  # world > 8
    assert to_peers(2, 2, 1, FAKE) == _lib.KH_EINVAL  # rank >= world
    assert to_peers(0, 2, 0, FAKE) == _lib.KH_EINVAL  # epoch 0
    assert to_peers(0, 2, 1, None) == _lib.KH_EINVAL  # no counter
    assert to_peers(0, 2, 1, FAKE, records=None) == _lib.KH_EINVAL
    odd = ctypes.cast((ctypes.c_void_p * 2)(0x10002, 0x20000), ctypes.c_void_p)
    assert to_peers(0, 2, 1, FAKE, records=odd) == _lib.KH_EALIGN
    assert to_peers(0, 2, 1, FAKE, n_groups=0) == _lib.KH_OK


def test_gqa_decode_and_compat_scorer_validate():
    L = _lib.lib()
    args = (FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 100, 0, 100, D128, D128, C2, 2,
            0.1, 2, FAKE, 2, 0, None)
    assert L.kh_decode_partial_gqa(FAKE, 2, 0, 128, *args) == _lib.KH_EINVAL  # n_q < 1
    assert L.kh_decode_partial_gqa(FAKE, 16384, 4, 128, *args) == _lib.KH_EINVAL  # grid.y
    assert L.kh_decode_partial_gqa(FAKE, 0, 4, 128, *args) == _lib.KH_OK  # nothing to do
    assert L.kh_decode_partial_gqa(FAKE, 2, 2, 96, *args) == _lib.KH_EINVAL  # head_dim
    ok = dict(q=FAKE, H=2, D=128, S=10, kp=FAKE, sg=FAKE, d=FAKE, kn=FAKE, rn=FAKE, c=FAKE,
              layer=0, mask=0)

    def compat(**kw):
        a = dict(ok)
        a.update(kw)
        return L.kh_score_packed_compat(a["q"], a["H"], a["D"], a["S"], a["kp"], a["sg"],
                                        a["d"], a["kn"], a["rn"], a["c"], a["layer"],
                                        a["mask"], 0.1, FAKE, None)
    assert compat(D=96) == _lib.KH_EINVAL
    assert compat(layer=-1) == _lib.KH_EINVAL
    assert compat(H=0) == _lib.KH_OK
    assert compat(S=0) == _lib.KH_OK
    assert compat(kp=ctypes.c_void_p(0x10002)) == _lib.KH_EALIGN
    assert compat(q=ctypes.c_void_p(0x10001)) == _lib.KH_EALIGN
    assert compat(c=None) == _lib.KH_EINVAL


TORCH_OPS = ["compress", "compress_out", "compress_many_out", "fwht_", "materialize", "score",
             "score_out", "decode_partial", "decode_combine", "decode_merge", "decode_attention",
             "decode_merge_to_peers", "decode_combine_from_peers", "ultra_fused_full_fusion",
             "ultra_fused_hbba_fusion", "hbba_calibrate_cuda", "fused_asymmetric_attention"]


def test_torch_extension_registers_every_operator():
    """torch.ops.kudahitam.* (the thin torch extension over this ABI) loads,
    registers every operator, and has no CPU kernel: CPU tensors fail in the
    dispatcher."""
    import torch

    from kudahitam import ops
    K = ops.ext()
    for name in TORCH_OPS:
        assert hasattr(K, name), name
    assert "Tensor(a!) code" in str(K.compress_out.default._schema)
    with pytest.raises(NotImplementedError):
        K.compress(torch.randn(4, 128), torch.ones(128), torch.tensor([-0.1, 0.1]), True)
