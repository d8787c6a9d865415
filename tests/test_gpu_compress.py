"""Parity of the fused compression kernel with the CPU oracle and with the
reference-generated golden vectors.

Tolerances (the engine's contract):
* code / residual sign bits: bit-exact on every element whose decision is
  not within 1e-6 of a boundary (|y - boundary| > 1e-6, y the orthonormal
  projection of x/||x||, i.e. |v| > 1e-6 ||x|| in unnormalised units); the
  residual plane additionally needs |y - c[idx]| > 1e-6;
* norms: 1e-5 relative; residual norms: 1e-4 relative (fp32 accumulate).
"""
import numpy as np
import pytest
import torch

import khtest as K
from kudahitam import KudahitamCompressorV2, lloyd_max, ops, rademacher
from kudahitam import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]


def check_against_oracle(x_cpu: torch.Tensor, p: ops.PackedKV, d, c, residual=True):
    D = x_cpu.shape[-1]
    bits = 1 if len(c) == 2 else 2
    ref = O.compress_v8(x_cpu, d, c)
    n = ref["norms"].shape[0]
    xf = x_cpu.float().numpy().reshape(n, D)
    y = K.projected(xf, np.asarray(d, np.float64))
    m = K.idx_mask(y, c)
    code = K.unpack_code(K.u32(p.code), D, bits)
    assert code.shape == (n, D)
    bad = (code != ref["idx"]) & m
    assert not bad.any(), f"{bad.sum()} decided index mismatches"
    # undecided elements (inside the 1e-6 band) may go either way; they are
    # rare (|y| < 1e-6 has probability ~1e-5 per element)
    assert (code != ref["idx"]).sum() <= max(2, 1e-4 * code.size)
    assert K.rel_err(p.norms.cpu().numpy(), ref["norms"]) < 1e-5
    if residual:
        rm = K.res_mask(y, ref["idx"].astype(np.int64), c)
        sg = K.unpack_bits(K.u32(p.res), D).astype(np.int8) * 2 - 1
        bad = (sg != ref["signs"]) & rm
        assert not bad.any(), f"{bad.sum()} decided sign mismatches"
        assert K.rel_err(p.rnorms.cpu().numpy(), ref["rnorms"], floor=1e-30) < 1e-4
    return ref


@pytest.fixture(params=["simt", "tensor"])
def path(request, monkeypatch):
    """Datapath of the 16-bit compressor (fp32 always takes the SIMT one)."""
    monkeypatch.setenv("KUDAHITAM_COMPRESS_PATH", request.param)
    return request.param


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("bits", [1, 2])
def test_compress_matches_oracle(dtype, D, bits, path):
    d = rademacher(D, 1).numpy()
    c = lloyd_max(bits, D).numpy()
    x = K.synth((2, 3, 171, D), dtype=dtype, seed=D + bits)
    p = ops.compress(x.cuda(), d, c, residual=True)
    torch.cuda.synchronize()
    check_against_oracle(x, p, d, c)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("D", [128, 256])
def test_one_bit_mode(dtype, D, path):
    d = rademacher(D, 2).numpy()
    c = lloyd_max(1, D).numpy()
    x = K.synth((1, 2, 77, D), dtype=dtype, seed=3)
    p = ops.compress(x.cuda(), d, c, residual=False)
    assert p.res is None and p.rnorms is None
    check_against_oracle(x, p, d, c, residual=False)
    full = ops.compress(x.cuda(), d, c, residual=True)
    assert torch.equal(full.code, p.code) and torch.equal(full.norms, p.norms)


@pytest.mark.parametrize("n", [1, 2, 3, 15, 16, 17, 31, 32, 33, 63, 65, 129, 1000])
@pytest.mark.parametrize("D", [128, 256])
def test_tails(n, D, path):
    d = rademacher(D, 4).numpy()
    c = lloyd_max(1, D).numpy()
    x = torch.randn(n, D, generator=torch.Generator().manual_seed(n)).to(torch.bfloat16)
    xg = x.cuda()
    p = ops.empty_packed(x.shape, 1, True, "cuda")
    # poison the outputs: rows past n must never be written, rows < n always
    for t in (p.code, p.res):
        t.fill_(0x5A5A5A5A)
    p.norms.fill_(-7.0)
    p.rnorms.fill_(-7.0)
    ops.compress(xg, d, c, out=p)
    check_against_oracle(x, p, d, c)


def test_edge_rows(path):
    D = 128
    d = rademacher(D, 0).numpy()
    for bits in (1, 2):
        c = lloyd_max(bits, D).numpy()
        x = torch.zeros(6, D)
        x[1, 5] = 3.0                      # single spike
        x[2] = torch.randn(D) * 1e-6       # tiny
        x[3] = torch.randn(D) * 1e4        # huge
        x[4] = torch.arange(D).float()     # structured, exact zeros after H
        x[5] = 1.0                          # constant row
        p = ops.compress(x.cuda(), d, c)
        torch.cuda.synchronize()
        ref = O.compress_v8(x, d, c)
        # all-zero row: norm 1e-8, lowest tie index, every residual sign +1
        assert p.norms[0].item() == pytest.approx(1e-8)
        code = K.unpack_code(K.u32(p.code), D, bits)
        assert (code[0] == int(np.argmin(np.abs(c)))).all()
        assert (K.unpack_bits(K.u32(p.res), D)[0] == 1).all()
        assert p.rnorms[0].item() == pytest.approx(ref["rnorms"][0], rel=1e-5)
        check_against_oracle(x, p, d, c)


def _dc(seed=5, D=128):
    return rademacher(D, seed).numpy(), lloyd_max(1, D).numpy()


def test_row_pitch_wider_than_head_dim(path):
    D = 128
    d, c = _dc()
    base = torch.randn(64, D + 8, dtype=torch.float16, device="cuda")
    x = base[:, :D]                         # row pitch D+8 elements (272 B), read in place
    p = ops.compress(x, d, c)
    check_against_oracle(x.cpu(), p, d, c)


def test_unaligned_base_is_copied():
    D = 128
    d, c = _dc()
    flat = torch.randn(64 * D + 1, dtype=torch.bfloat16, device="cuda")
    xu = flat[1:].view(64, D)               # 2-byte offset
    p = ops.compress(xu, d, c)
    check_against_oracle(xu.cpu(), p, d, c)


def test_non_uniform_rows_are_copied():
    D = 128
    d, c = _dc()
    big = torch.randn(2, 4, 40, D, device="cuda")
    xs = big[:, :, 5:30]
    p = ops.compress(xs, d, c)
    check_against_oracle(xs.cpu(), p, d, c)


def test_batched_equals_single(path):
    D = 128
    d = rademacher(D, 6).numpy()
    c = lloyd_max(1, D).numpy()
    xs = [torch.randn(n, D, device="cuda", dtype=torch.bfloat16) for n in (5, 100, 33, 0, 64)]
    many = ops.compress_many(xs, d, c)
    for x, pm in zip(xs, many):
        ps = ops.compress(x, d, c)
        assert torch.equal(pm.code, ps.code) and torch.equal(pm.res, ps.res)
        assert torch.equal(pm.norms, ps.norms) and torch.equal(pm.rnorms, ps.rnorms)
    # more tensors than one launch takes
    xs = [torch.randn(3, D, device="cuda") for _ in range(70)]
    many = ops.compress_many(xs, d, c)
    for x, pm in zip(xs, many):
        assert torch.equal(pm.code, ops.compress(x, d, c).code)


@pytest.mark.parametrize("case", ["d128_fp32_b1", "d128_fp32_b2", "d256_fp16_b1",
                                  "d256_fp16_b2"])
def test_matches_reference_golden(case):
    g = K.golden(f"compress_{case}.npz")
    x, d, c = g["x"], g["d"], g["c"]
    B, H, S, D = x.shape
    bits = 1 if len(c) == 2 else 2
    comp = KudahitamCompressorV2(D, bits, seed=7)
    assert np.array_equal(comp.d.numpy(), d) and np.array_equal(comp.centroids.numpy(), c)
    out = comp.compress(torch.from_numpy(x).cuda())
    n = B * H * S
    live = g["norms"].reshape(-1) > 0
    y = K.projected(x.astype(np.float32), d)
    m = K.idx_mask(y, c)
    assert np.array_equal(out["indices"].cpu().numpy()[m], g["indices"].reshape(n, D)[m])
    assert K.rel_err(out["norms"].cpu().numpy()[live], g["norms"].reshape(-1)[live]) < 1e-5
    assert K.normwise(out["k_mse"].cpu().numpy().reshape(n, D)[live],
                      g["k_mse"].reshape(n, D)[live]) < 1e-5
    rm = K.res_mask(y, g["indices"].reshape(n, D).astype(np.int64), c)
    assert np.array_equal(out["signs"].cpu().numpy().reshape(n, D)[rm],
                          g["signs"].reshape(n, D)[rm])
    assert K.rel_err(out["r_norm"].cpu().numpy().reshape(-1)[live],
                     g["r_norm"].reshape(-1)[live]) < 1e-4
    # reference dict layout (KudaHitamQuant_full.py:358-370)
    assert out["indices"].shape == (n, D) and out["indices"].dtype == torch.uint8
    assert out["norms"].shape == (n,)
    assert out["k_mse"].shape == (B, H, S, D) and out["k_mse"].dtype == torch.float32
    assert out["r_norm"].shape == (B, H, S)
    assert out["signs"].shape == (B, H, S, D) and out["signs"].dtype == torch.int8
    assert out["rank"] == 4 and out["shape"] == (B, H, S, D) and out["p_indices"] is None


def test_full_size_fp16_d256_properties(path):
    """40000-token fp16 D=256 K tensor (the 2-bit-mode workload): sampled rows
    against the oracle, and on every row the residual identity
    sign(H(d (.) (x - k_mse))) == residual bits, r_norm == ||x - k_mse||."""
    D = 256
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(1, 16, 40000, D, device="cuda", generator=g).half()
    d = rademacher(D, 1).numpy()
    c = lloyd_max(1, D).numpy()
    p = ops.compress(x, d, c)
    rows = torch.arange(0, 640000, 997, device="cuda")
    sub = ops.PackedKV((len(rows), D), 1, p.code[rows], p.norms[rows], p.res[rows],
                       p.rnorms[rows])
    check_against_oracle(x.view(-1, D)[rows].cpu(), sub, d, c)
    m = ops.materialize(p, d, c, idx=False, kmse=True, signs=False)["kmse"]
    Hm = torch.tensor(K.hadamard(D), dtype=torch.float32, device="cuda")
    dd = torch.tensor(d, device="cuda")
    for r0 in range(0, 640000, 160000):
        xs = x.view(-1, D)[r0:r0 + 160000].float()
        diff = xs - m[r0:r0 + 160000]
        z = (diff * dd) @ Hm
        bits = torch.tensor(K.unpack_bits(K.u32(p.res[r0:r0 + 160000]), D), device="cuda")
        decided = z.abs() > 1e-4 * xs.norm(dim=1, keepdim=True)
        assert ((z >= 0).to(torch.uint8) == bits)[decided].all()
        rn = diff.norm(dim=1)
        assert torch.allclose(p.rnorms[r0:r0 + 160000], rn, rtol=1e-4, atol=1e-6)


def test_cuda_graph_capture():
    D = 128
    d = rademacher(D, 1).numpy()
    c = lloyd_max(1, D).numpy()
    x = torch.randn(4096, D, device="cuda", dtype=torch.bfloat16)
    out = ops.empty_packed(x.shape, 1, True, "cuda")
    ops.compress(x, d, c, out=out)  # warm-up outside capture
    ref_code = out.code.clone()
    out.code.zero_()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            ops.compress(x, d, c, out=out)
    torch.cuda.current_stream().wait_stream(s)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out.code, ref_code)


def test_no_device_errors_recorded():
    torch.cuda.synchronize()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("residual", [True, False])
def test_host_streamed_compression_equals_device(residual):
    """compress_host (uploads, kernels and downloads overlapped over chunks)
    produces the same packed bytes as compressing on the device."""
    D = 256
    d, c = rademacher(D, 3).numpy(), lloyd_max(1, D).numpy()
    g = torch.Generator().manual_seed(4)
    xs = [torch.randn(n, D, generator=g).to(torch.float16) for n in (2500, 1, 777)]
    xs[0] = xs[0].pin_memory()  # pinned and pageable inputs alike
    outs = ops.compress_host(xs, d, c, residual=residual, device="cuda", chunk_rows=1000)
    torch.cuda.current_stream().synchronize()
    for x, o in zip(xs, outs):
        ref = ops.compress(x.cuda(), d, c, residual=residual)
        assert not o.code.is_cuda and o.code.is_pinned()
        assert torch.equal(o.code, ref.code.cpu())
        assert torch.equal(o.norms, ref.norms.cpu())
        if residual:
            assert torch.equal(o.res, ref.res.cpu()) and torch.equal(o.rnorms, ref.rnorms.cpu())
    # the public method, repeated into the same buffers
    comp = KudahitamCompressorV2(D, 1, seed=3)
    a = comp.compress_to_host([xs[2]])
    b = comp.compress_to_host([xs[2]], outs=[a[0].packed])
    torch.cuda.current_stream().synchronize()
    assert torch.equal(b[0].packed.code, comp.compress(xs[2].cuda()).packed.code.cpu())
