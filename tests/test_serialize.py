"""The packed-cache file format (KHPK): exact round trips, corruption checks."""
import io

import numpy as np
import pytest
import torch

from kudahitam import lloyd_max, ops, rademacher, serialize


def _random_packed(shape, bits, residual, seed=0):
    g = torch.Generator().manual_seed(seed)
    p = ops.empty_packed(shape, bits, residual, "cpu")
    p.code.copy_(torch.randint(-2**31, 2**31 - 1, p.code.shape, generator=g, dtype=torch.int64).to(torch.int32))
    p.norms.copy_(torch.rand(p.norms.shape, generator=g) * 10)
    if residual:
        p.res.copy_(torch.randint(-2**31, 2**31 - 1, p.res.shape, generator=g, dtype=torch.int64).to(torch.int32))
        p.rnorms.copy_(torch.rand(p.rnorms.shape, generator=g))
    return p


@pytest.mark.parametrize("shape,bits,residual", [((2, 3, 17, 128), 1, True),
                                                 ((5, 256), 2, True),
                                                 ((1, 4, 9, 128), 1, False)])
def test_round_trip_exact(shape, bits, residual, tmp_path):
    D = shape[-1]
    p = _random_packed(shape, bits, residual)
    d, c = rademacher(D, 3), lloyd_max(bits, D)
    path = tmp_path / "cache.khpk"
    n = serialize.save(str(path), p, d, c)
    assert path.stat().st_size == n
    q, d2, c2 = serialize.read(str(path))
    assert q.shape == p.shape and q.bits == bits and q.residual == residual
    assert torch.equal(q.code, p.code) and torch.equal(q.norms, p.norms)
    if residual:
        assert torch.equal(q.res, p.res) and torch.equal(q.rnorms, p.rnorms)
    assert torch.equal(d2, d)
    assert c2.numpy().view(np.uint32).tolist() == c.numpy().view(np.uint32).tolist()
    # arrays are 16-byte aligned in the file
    raw = path.read_bytes()
    assert raw[:4] == b"KHPK"


def test_bytes_round_trip_and_errors():
    p = _random_packed((3, 128), 1, True)
    d, c = rademacher(128, 0), lloyd_max(1, 128)
    blob = serialize.to_bytes(p, d, c)
    q, _, _ = serialize.from_bytes(blob)
    assert torch.equal(q.code, p.code)
    with pytest.raises(ValueError, match="KHPK"):
        serialize.from_bytes(b"XXXX" + blob[4:])
    with pytest.raises(ValueError, match="truncated"):
        serialize.from_bytes(blob[:-3])
    bad = bytearray(blob)
    bad[4] = 9
    with pytest.raises(ValueError, match="version"):
        serialize.from_bytes(bytes(bad))
    with pytest.raises(ValueError):
        serialize.to_bytes(p, torch.zeros(128), c)
