// kh_torch.cpp -- the engine's PyTorch operators: torch.ops.kudahitam.*
//
// A thin layer over the C ABI (include/kudahitam.h): each operator checks
// its tensors, turns them into raw pointers, allocates outputs with the
// caching allocator and calls kh_* on the tensors' device and its current
// stream.  It replaces the reference's pybind11 extension
// (KudaHitamCUDA.cu:799-804, loaded by load_cuda_ext, KudaHitamQuant_full.py:43-98):
// the operators are registered with the dispatcher (TORCH_LIBRARY), so they
// show under their own names in the profiler and in torch.library, and a
// call costs a few microseconds of host time.  Only the CUDA backend is
// registered: a call with CPU tensors only fails in the dispatcher, there is
// no CPU path.
//
// Host arrays: d (the +-1 diagonal) and the centroids are float32 CPU
// tensors; kh_* reads them during the call (except for
// fused_asymmetric_attention, whose reference binding takes them on the
// device).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <vector>

#include "kudahitam.h"

namespace {

using at::Tensor;

void check(int st, const char* fn) {
  TORCH_CHECK(st == KH_OK, fn, " failed: ", kh_status_string(st), " (kh_status=", st, ")");
}

const float* host_f32(const Tensor& t, int64_t n, const char* what) {
  TORCH_CHECK(t.device().is_cpu() && t.scalar_type() == at::kFloat && t.is_contiguous() &&
                  t.numel() == n,
              what, " must be a contiguous float32 CPU tensor of ", n, " values");
  return t.data_ptr<float>();
}

const float* host_c(const Tensor& c) {
  TORCH_CHECK(c.numel() == 2 || c.numel() == 4, "the codebook must have 2 or 4 levels, got ",
              c.numel());
  return host_f32(c, c.numel(), "centroids");
}

int bits_of(const Tensor& c) { return c.numel() == 2 ? 1 : 2; }

void* stream_of(const Tensor& t) {
  return c10::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

void require_cuda(const Tensor& t, const char* what) {
  TORCH_CHECK(t.is_cuda(), what, " must be a CUDA tensor (kudahitam has no CPU path)");
}

int dtype_code(at::ScalarType s) {
  switch (s) {
    case at::kFloat: return KH_F32;
    case at::kHalf: return KH_F16;
    case at::kBFloat16: return KH_BF16;
    default: TORCH_CHECK(false, "unsupported dtype ", s, " (float32, float16, bfloat16)");
  }
  return -1;
}

// The rows of x as the C ABI reads them: N rows of D elements with unit
// inner stride and a 16-byte row pitch.  x itself when its layout allows
// (no tensor is created on this common path), else an aligned contiguous
// copy kept alive in `keep`.
struct Rows {
  const void* ptr;
  int64_t n, pitch;
  Tensor keep;
};
Rows rows_of(const Tensor& x) {
  const int64_t D = x.size(-1);
  const int64_t elt = x.element_size();
  const auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (x.is_contiguous() && aligned(x.data_ptr()) && (D * elt) % 16 == 0)
    return {x.data_ptr(), D ? x.numel() / D : 0, D, Tensor()};
  Tensor r = x.reshape({-1, D});
  const bool ok = r.stride(-1) == 1 && aligned(r.data_ptr()) &&
                  (r.size(0) <= 1 || (r.stride(0) * elt) % 16 == 0);
  if (!ok) r = at::empty(r.sizes(), r.options()).copy_(r);  // fresh: 256-byte aligned
  return {r.data_ptr(), r.size(0), r.size(0) > 1 ? r.stride(0) : D, r};
}

int64_t code_words(int64_t D, int bits) { return bits == 1 ? D / 32 : D / 16; }

// float32 elements addressable from t.data_ptr() to the end of its storage.
int64_t floats_from_ptr(const Tensor& t) {
  return (int64_t)(t.storage().nbytes() / 4) - t.storage_offset();
}

// An output (or input) buffer the kernels address as a flat array: on the
// launching device and contiguous.
void check_buf(const Tensor& t, const c10::Device& dev, const char* what) {
  TORCH_CHECK(t.device() == dev, what, " is on ", t.device(), ", expected ", dev);
  TORCH_CHECK(t.is_contiguous(), what, " must be contiguous");
}
void check_buf(const c10::optional<Tensor>& t, const c10::Device& dev, const char* what) {
  if (t && t->defined()) check_buf(*t, dev, what);
}

uint32_t* u32(const Tensor& t) { return reinterpret_cast<uint32_t*>(t.data_ptr()); }
const uint32_t* cu32(const Tensor& t) {
  return reinterpret_cast<const uint32_t*>(t.data_ptr());
}
const uint32_t* opt_u32(const c10::optional<Tensor>& t) {
  return t && t->defined() ? cu32(*t) : nullptr;
}
const float* opt_f32(const c10::optional<Tensor>& t) {
  return t && t->defined() ? t->data_ptr<float>() : nullptr;
}

// ---------------------------------------------------------------- compress

void compress_out(const Tensor& x, const Tensor& d, const Tensor& c, bool residual,
                  const Tensor& code, const c10::optional<Tensor>& res, const Tensor& norms,
                  const c10::optional<Tensor>& rnorms) {
  require_cuda(x, "x");
  const int64_t D = x.size(-1);
  const int dt = dtype_code(x.scalar_type());
  const float* ch = host_c(c);
  const float* dh = host_f32(d, D, "d");
  const Rows r = rows_of(x);
  const int64_t n = r.n;
  TORCH_CHECK(code.numel() == n * code_words(D, bits_of(c)) && norms.numel() == n,
              "output buffers do not match ", n, " rows");
  check_buf(code, x.device(), "code");
  check_buf(norms, x.device(), "norms");
  check_buf(res, x.device(), "res");
  check_buf(rnorms, x.device(), "rnorms");
  if (residual)
    TORCH_CHECK(res && res->defined() && rnorms && rnorms->defined() &&
                    res->numel() == n * (D / 32) && rnorms->numel() == n,
                "2-bit mode needs res [N, D/32] and rnorms [N]");
  c10::cuda::CUDAGuard guard(x.device());
  check(kh_compress(r.ptr, dt, n, (int)D, r.pitch, dh, ch, (int)c.numel(), residual ? 1 : 0,
                    u32(code), residual ? u32(*res) : nullptr, norms.data_ptr<float>(),
                    residual ? rnorms->data_ptr<float>() : nullptr, stream_of(x)),
        "kh_compress");
}

std::vector<Tensor> compress(const Tensor& x, const Tensor& d, const Tensor& c, bool residual) {
  require_cuda(x, "x");
  const int64_t D = x.size(-1);
  const int64_t n = D ? x.numel() / D : 0;
  auto i32 = x.options().dtype(at::kInt);
  auto f32 = x.options().dtype(at::kFloat);
  host_c(c);
  Tensor code = at::empty({n, code_words(D, bits_of(c))}, i32);
  Tensor norms = at::empty({n}, f32);
  if (!residual) {
    compress_out(x, d, c, false, code, c10::nullopt, norms, c10::nullopt);
    return {code, norms};
  }
  Tensor res = at::empty({n, D / 32}, i32);
  Tensor rnorms = at::empty({n}, f32);
  compress_out(x, d, c, true, code, res, norms, rnorms);
  return {code, norms, res, rnorms};
}

void compress_many_out(at::TensorList xs, const Tensor& d, const Tensor& c, bool residual,
                       at::TensorList code, at::TensorList res, at::TensorList norms,
                       at::TensorList rnorms) {
  const size_t n = xs.size();
  if (n == 0) return;
  TORCH_CHECK(code.size() == n && norms.size() == n, "one code and norms buffer per tensor");
  TORCH_CHECK(!residual || (res.size() == n && rnorms.size() == n),
              "2-bit mode needs one res and rnorms buffer per tensor");
  require_cuda(xs[0], "xs");
  const auto dev = xs[0].device();
  const auto st = xs[0].scalar_type();
  const int64_t D = xs[0].size(-1);
  const float* ch = host_c(c);
  const float* dh = host_f32(d, D, "d");
  const int bits = bits_of(c);
  std::vector<Tensor> keep(n);  // aligned copies (if any) alive for the call
  std::vector<const void*> xp(n);
  std::vector<int64_t> rows(n), pitch(n);
  std::vector<uint32_t*> cp(n), rp(n, nullptr);
  std::vector<float*> np_(n), rnp(n, nullptr);
  for (size_t i = 0; i < n; ++i) {
    TORCH_CHECK(xs[i].device() == dev && xs[i].scalar_type() == st && xs[i].size(-1) == D,
                "compress_many needs tensors of one device, dtype and head_dim");
    const Rows r = rows_of(xs[i]);
    keep[i] = r.keep;
    xp[i] = r.ptr;
    rows[i] = r.n;
    pitch[i] = r.pitch;
    TORCH_CHECK(code[i].numel() == rows[i] * code_words(D, bits) && norms[i].numel() == rows[i],
                "output buffers of tensor ", i, " do not match its rows");
    check_buf(code[i], dev, "code");
    check_buf(norms[i], dev, "norms");
    cp[i] = u32(code[i]);
    np_[i] = norms[i].data_ptr<float>();
    if (residual) {
      TORCH_CHECK(res[i].numel() == rows[i] * (D / 32) && rnorms[i].numel() == rows[i],
                  "residual buffers of tensor ", i, " do not match its rows");
      check_buf(res[i], dev, "res");
      check_buf(rnorms[i], dev, "rnorms");
      rp[i] = u32(res[i]);
      rnp[i] = rnorms[i].data_ptr<float>();
    }
  }
  c10::cuda::CUDAGuard guard(dev);
  void* s = stream_of(xs[0]);
  const int maxseg = kh_max_segments();
  for (size_t a = 0; a < n; a += maxseg) {
    const int m = (int)std::min<size_t>(maxseg, n - a);
    check(kh_compress_batched(m, xp.data() + a, rows.data() + a, pitch.data() + a, cp.data() + a,
                              rp.data() + a, np_.data() + a, rnp.data() + a,
                              dtype_code(st), (int)D, dh, ch, (int)c.numel(), residual ? 1 : 0, s),
          "kh_compress_batched");
  }
}

// ------------------------------------------------------ transform / expand

Tensor& fwht_(Tensor& x) {
  require_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == at::kFloat && x.is_contiguous(),
              "fwht_ needs a contiguous float32 tensor");
  const int64_t D = x.size(-1);
  c10::cuda::CUDAGuard guard(x.device());
  check(kh_fwht_inplace(x.data_ptr<float>(), D ? x.numel() / D : 0, (int)D, stream_of(x)),
        "kh_fwht_inplace");
  return x;
}

std::vector<Tensor> materialize(const Tensor& code, const c10::optional<Tensor>& res,
                                const Tensor& norms, int64_t head_dim, const Tensor& d,
                                const Tensor& c, bool want_idx, bool want_kmse,
                                bool want_signs) {
  require_cuda(code, "code");
  const int64_t n = norms.numel();
  check_buf(code, code.device(), "code");
  check_buf(norms, code.device(), "norms");
  check_buf(res, code.device(), "res");
  TORCH_CHECK(code.numel() == n * code_words(head_dim, bits_of(c)),
              "code does not hold ", n, " rows of head_dim ", head_dim);
  if (res && res->defined())
    TORCH_CHECK(res->numel() == n * (head_dim / 32), "res does not hold ", n, " rows");
  const float* ch = host_c(c);
  const float* dh = host_f32(d, head_dim, "d");
  auto o = code.options();
  const bool has_res = res && res->defined();
  Tensor idx = want_idx ? at::empty({n, head_dim}, o.dtype(at::kByte)) : at::empty({0}, o.dtype(at::kByte));
  Tensor kmse = want_kmse ? at::empty({n, head_dim}, o.dtype(at::kFloat)) : at::empty({0}, o.dtype(at::kFloat));
  Tensor signs = (want_signs && has_res) ? at::empty({n, head_dim}, o.dtype(at::kChar))
                                         : at::empty({0}, o.dtype(at::kChar));
  c10::cuda::CUDAGuard guard(code.device());
  check(kh_materialize(cu32(code), opt_u32(res), norms.data_ptr<float>(), n, (int)head_dim, dh, ch,
                       (int)c.numel(), want_idx ? idx.data_ptr<uint8_t>() : nullptr,
                       want_kmse ? kmse.data_ptr<float>() : nullptr,
                       (want_signs && has_res) ? signs.data_ptr<int8_t>() : nullptr,
                       stream_of(code)),
        "kh_materialize");
  return {idx, kmse, signs};
}

// ------------------------------------------------------------------- score

void score_out(const Tensor& q, const Tensor& code, const c10::optional<Tensor>& res,
               const Tensor& norms, const c10::optional<Tensor>& rnorms, int64_t seq_len,
               const Tensor& d, const Tensor& c, const Tensor& out) {
  require_cuda(q, "q");
  TORCH_CHECK(q.dim() == 3 && q.scalar_type() == at::kFloat && q.is_contiguous(),
              "q must be a contiguous float32 [G, n_q, D] tensor");
  const int64_t G = q.size(0), nq = q.size(1), D = q.size(2);
  TORCH_CHECK(G * seq_len == norms.numel(), norms.numel(), " cached rows do not split into ", G,
              " groups of ", seq_len);
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() &&
                  out.numel() == G * nq * seq_len,
              "out must be a contiguous float32 tensor of G * n_q * seq_len values");
  const auto dev = q.device();
  check_buf(out, dev, "out");
  check_buf(code, dev, "code");
  check_buf(norms, dev, "norms");
  check_buf(res, dev, "res");
  check_buf(rnorms, dev, "rnorms");
  TORCH_CHECK(code.numel() == norms.numel() * code_words(D, bits_of(c)),
              "code does not match the cached rows");
  if (res && res->defined())
    TORCH_CHECK(res->numel() == norms.numel() * (D / 32) && rnorms && rnorms->defined() &&
                    rnorms->numel() == norms.numel(),
                "res / rnorms do not match the cached rows");
  const float* ch = host_c(c);
  const float* dh = host_f32(d, D, "d");
  c10::cuda::CUDAGuard guard(q.device());
  check(kh_score(q.data_ptr<float>(), G, (int)nq, (int)D, cu32(code), opt_u32(res),
                 norms.data_ptr<float>(), opt_f32(rnorms), seq_len, dh, ch, (int)c.numel(),
                 out.data_ptr<float>(), stream_of(q)),
        "kh_score");
}

Tensor score(const Tensor& q, const Tensor& code, const c10::optional<Tensor>& res,
             const Tensor& norms, const c10::optional<Tensor>& rnorms, int64_t seq_len,
             const Tensor& d, const Tensor& c) {
  require_cuda(q, "q");
  Tensor qf = q.scalar_type() == at::kFloat && q.is_contiguous() ? q
                                                                 : q.to(at::kFloat).contiguous();
  Tensor out = at::empty({qf.size(0), qf.size(1), seq_len}, qf.options());
  score_out(qf, code, res, norms, rnorms, seq_len, d, c, out);
  return out;
}

// ------------------------------------------------------------------ decode

struct Cache {
  const uint32_t *code, *res;
  const float *norms, *rnorms;
};

Cache cache_of(const Tensor& code, const Tensor& res, const Tensor& norms, const Tensor& rnorms) {
  return {cu32(code), cu32(res), norms.data_ptr<float>(), rnorms.data_ptr<float>()};
}

void decode_partial(const Tensor& q, const Tensor& kc, const Tensor& kr, const Tensor& kn,
                    const Tensor& krn, const Tensor& vc, const Tensor& vr, const Tensor& vn,
                    const Tensor& vrn, int64_t seq_len, int64_t seq_begin, int64_t seq_end,
                    const Tensor& dk, const Tensor& c, double sm_scale, int64_t n_splits,
                    const Tensor& partials, int64_t part_stride, int64_t part_offset) {
  require_cuda(q, "q");
  TORCH_CHECK(q.scalar_type() == at::kFloat && q.is_contiguous() && (q.dim() == 2 || q.dim() == 3),
              "q must be a contiguous float32 [G, D] or [G, n_q, D] tensor");
  const int64_t G = q.size(0), nq = q.dim() == 3 ? q.size(1) : 1, D = q.size(-1);
  TORCH_CHECK(partials.scalar_type() == at::kFloat, "partials must be float32");
  const auto dev = q.device();
  check_buf(partials, dev, "partials");
  TORCH_CHECK(floats_from_ptr(partials) >= G * nq * part_stride * (D + 2),
              "partials holds fewer than G * n_q * part_stride records");
  for (const Tensor* t : {&kc, &kr, &kn, &krn, &vc, &vr, &vn, &vrn}) check_buf(*t, dev, "cache");
  const int64_t rows = kn.numel();
  TORCH_CHECK(G * seq_len <= rows && vn.numel() == rows && krn.numel() == rows &&
                  vrn.numel() == rows && kc.numel() == rows * code_words(D, bits_of(c)) &&
                  vc.numel() == kc.numel() && kr.numel() == rows * (D / 32) &&
                  vr.numel() == kr.numel(),
              "K / V caches do not hold G * seq_len rows of head_dim ", D);
  const float* ch = host_c(c);
  const float* dh = host_f32(dk, D, "dk");
  const Cache K = cache_of(kc, kr, kn, krn), V = cache_of(vc, vr, vn, vrn);
  c10::cuda::CUDAGuard guard(q.device());
  check(kh_decode_partial_gqa(q.data_ptr<float>(), G, (int)nq, (int)D, K.code, K.res, K.norms,
                              K.rnorms, V.code, V.res, V.norms, V.rnorms, seq_len, seq_begin,
                              seq_end, dh, dh, ch, (int)c.numel(), (float)sm_scale, (int)n_splits,
                              partials.data_ptr<float>(), part_stride, part_offset, stream_of(q)),
        "kh_decode_partial_gqa");
}

// decode_partial with the records stored into slot [rank] of every rank's
// record buffer (peer_records: device addresses, one per rank) and the
// epoch raised in every rank's flag array (peer_flags) by the last CTA.
void decode_partial_to_peers(const Tensor& q, const Tensor& kc, const Tensor& kr,
                             const Tensor& kn, const Tensor& krn, const Tensor& vc,
                             const Tensor& vr, const Tensor& vn, const Tensor& vrn,
                             int64_t seq_len, int64_t seq_begin, int64_t seq_end,
                             const Tensor& dk, const Tensor& c, double sm_scale, int64_t n_splits,
                             c10::IntArrayRef peer_records, c10::IntArrayRef peer_flags,
                             int64_t rank, int64_t epoch, const Tensor& counter,
                             const c10::optional<Tensor>& dv, const c10::optional<Tensor>& out) {
  require_cuda(q, "q");
  TORCH_CHECK(q.scalar_type() == at::kFloat && q.is_contiguous() && (q.dim() == 2 || q.dim() == 3),
              "q must be a contiguous float32 [G, D] or [G, n_q, D] tensor");
  const int64_t G = q.size(0), nq = q.dim() == 3 ? q.size(1) : 1, D = q.size(-1);
  const auto dev = q.device();
  for (const Tensor* t : {&kc, &kr, &kn, &krn, &vc, &vr, &vn, &vrn}) check_buf(*t, dev, "cache");
  const int64_t rows = kn.numel();
  TORCH_CHECK(G * seq_len <= rows && vn.numel() == rows && krn.numel() == rows &&
                  vrn.numel() == rows && kc.numel() == rows * code_words(D, bits_of(c)) &&
                  vc.numel() == kc.numel() && kr.numel() == rows * (D / 32) &&
                  vr.numel() == kr.numel(),
              "K / V caches do not hold G * seq_len rows of head_dim ", D);
  const size_t world = peer_records.size();
  TORCH_CHECK(world >= 1 && world <= 8 && peer_flags.size() == world,
              "one record buffer and flag array per rank, at most 8 ranks");
  TORCH_CHECK(epoch > 0 && epoch <= 0xFFFFFFFFll, "epoch must be in [1, 2^32)");
  std::vector<float*> recs(world);
  std::vector<uint32_t*> flags(world);
  for (size_t i = 0; i < world; ++i) {
    recs[i] = reinterpret_cast<float*>(static_cast<uintptr_t>(peer_records[i]));
    flags[i] = reinterpret_cast<uint32_t*>(static_cast<uintptr_t>(peer_flags[i]));
  }
  const float* ch = host_c(c);
  const float* dh = host_f32(dk, D, "dk");
  float* op = nullptr;
  std::vector<float> dvh(D, 1.f);
  if (out.has_value()) {
    TORCH_CHECK(dv.has_value(), "out needs dv");
    TORCH_CHECK(out->scalar_type() == at::kFloat && out->is_contiguous() &&
                    out->numel() == G * nq * D && out->device() == dev,
                "out must be a contiguous float32 tensor of G * n_q * D values on q's device");
    const float* d2 = host_f32(*dv, D, "dv");
    std::copy(d2, d2 + D, dvh.begin());
    op = out->data_ptr<float>();
  }
  const Cache K = cache_of(kc, kr, kn, krn), V = cache_of(vc, vr, vn, vrn);
  c10::cuda::CUDAGuard guard(q.device());
  check(kh_decode_partial_to_peers(q.data_ptr<float>(), G, (int)nq, (int)D, K.code, K.res,
                                   K.norms, K.rnorms, V.code, V.res, V.norms, V.rnorms, seq_len,
                                   seq_begin, seq_end, dh, dvh.data(), ch, (int)c.numel(),
                                   (float)sm_scale, (int)n_splits, recs.data(), flags.data(),
                                   (int)rank, (int)world, (uint32_t)epoch, u32(counter), op,
                                   stream_of(q)),
        "kh_decode_partial_to_peers");
}

// records: merged (m, l, acc) records of n_rows query rows, record p of row
// g at offset g * group_stride + p * part_stride floats.
void decode_combine(const Tensor& records, int64_t n_rows, int64_t n_parts, int64_t group_stride,
                    int64_t part_stride, const Tensor& dv, const Tensor& out) {
  require_cuda(records, "records");
  const int64_t D = out.size(-1);
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == n_rows * D,
              "out must be a contiguous float32 tensor of n_rows * D values");
  check_buf(out, records.device(), "out");
  TORCH_CHECK(records.device() == out.device() && records.scalar_type() == at::kFloat,
              "records must be float32 on out's device");
  TORCH_CHECK(n_rows == 0 || (n_rows - 1) * group_stride + (n_parts - 1) * part_stride + D + 2 <=
                                 floats_from_ptr(records),
              "records too small for the strides");
  const float* dh = host_f32(dv, D, "dv");
  c10::cuda::CUDAGuard guard(records.device());
  check(kh_decode_combine_strided(records.data_ptr<float>(), n_rows, (int)n_parts, group_stride,
                                  part_stride, (int)D, dh, out.data_ptr<float>(),
                                  stream_of(records)),
        "kh_decode_combine_strided");
}

void decode_merge(const Tensor& records, int64_t n_rows, int64_t n_parts, int64_t group_stride,
                  int64_t part_stride, const Tensor& merged) {
  require_cuda(records, "records");
  TORCH_CHECK(merged.scalar_type() == at::kFloat && merged.is_contiguous() && n_rows > 0 &&
                  merged.numel() % n_rows == 0,
              "merged must be a contiguous float32 [n_rows, D + 2] tensor");
  const int64_t D = merged.numel() / n_rows - 2;
  check_buf(merged, records.device(), "merged");
  TORCH_CHECK(records.scalar_type() == at::kFloat &&
                  (n_rows - 1) * group_stride + (n_parts - 1) * part_stride + D + 2 <=
                      floats_from_ptr(records),
              "records must be float32 and large enough for the strides");
  c10::cuda::CUDAGuard guard(records.device());
  check(kh_decode_merge(records.data_ptr<float>(), n_rows, (int)n_parts, group_stride, part_stride,
                        (int)D, merged.data_ptr<float>(), stream_of(records)),
        "kh_decode_merge");
}

Tensor decode_attention(const Tensor& q, const Tensor& kc, const Tensor& kr, const Tensor& kn,
                        const Tensor& krn, const Tensor& vc, const Tensor& vr, const Tensor& vn,
                        const Tensor& vrn, int64_t seq_len, int64_t length, const Tensor& dk,
                        const Tensor& dv, const Tensor& c, double sm_scale, int64_t n_splits) {
  require_cuda(q, "q");
  Tensor qf = q.scalar_type() == at::kFloat && q.is_contiguous() ? q
                                                                 : q.to(at::kFloat).contiguous();
  const int64_t D = qf.size(-1);
  const int64_t R = D ? qf.numel() / D : 0;  // query rows G * n_q
  const int64_t need = kh_decode_workspace_bytes(R, (int)n_splits, (int)D);
  TORCH_CHECK(need >= 0, "bad decode shape: ", R, " query rows, ", n_splits, " splits, D = ", D);
  Tensor ws = at::empty({std::max<int64_t>(need / 4, 1)}, qf.options());
  Tensor out = at::empty(qf.sizes(), qf.options());
  decode_partial(qf, kc, kr, kn, krn, vc, vr, vn, vrn, seq_len, 0, length, dk, c, sm_scale,
                 n_splits, ws, n_splits, 0);
  decode_combine(ws, R, n_splits, n_splits * (D + 2), D + 2, dv, out);
  return out;
}

// Sequence-sharded decode, record exchange over peer memory.  peer_records
// and peer_flags are the device addresses of every rank's record buffer and
// flag array (symmetric memory); buf is this rank's own allocation holding
// its record buffer at rec_offset and its flags at flag_offset bytes.
void decode_merge_to_peers(const Tensor& partials, int64_t n_rows, int64_t n_parts,
                           int64_t group_stride, int64_t part_stride, int64_t head_dim,
                           c10::IntArrayRef peer_records, c10::IntArrayRef peer_flags,
                           int64_t rank, int64_t epoch, const Tensor& counter) {
  require_cuda(partials, "partials");
  const size_t world = peer_records.size();
  TORCH_CHECK(world >= 1 && world <= 8 && peer_flags.size() == world,
              "one record buffer and flag array per rank, at most 8 ranks");
  TORCH_CHECK(epoch > 0 && epoch <= 0xFFFFFFFFll, "epoch must be in [1, 2^32)");
  std::vector<float*> recs(world);
  std::vector<uint32_t*> flags(world);
  for (size_t i = 0; i < world; ++i) {
    recs[i] = reinterpret_cast<float*>(static_cast<uintptr_t>(peer_records[i]));
    flags[i] = reinterpret_cast<uint32_t*>(static_cast<uintptr_t>(peer_flags[i]));
  }
  c10::cuda::CUDAGuard guard(partials.device());
  check(kh_decode_merge_to_peers(partials.data_ptr<float>(), n_rows, (int)n_parts, group_stride,
                                 part_stride, (int)head_dim, recs.data(), flags.data(), (int)rank,
                                 (int)world, (uint32_t)epoch, u32(counter), stream_of(partials)),
        "kh_decode_merge_to_peers");
}

void decode_combine_from_peers(const Tensor& buf, int64_t rec_offset, int64_t flag_offset,
                               int64_t epoch, int64_t n_rows, int64_t world, const Tensor& dv,
                               const Tensor& out, int64_t n_parts) {
  require_cuda(buf, "buf");
  const int64_t D = out.size(-1);
  TORCH_CHECK(n_parts >= 1, "n_parts must be at least 1");
  TORCH_CHECK(rec_offset >= 0 && flag_offset >= 0 && flag_offset + 4 * world <= buf.nbytes() &&
                  rec_offset + world * n_rows * n_parts * (D + 2) * 4 <= buf.nbytes(),
              "record buffer or flags outside buf");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == n_rows * D,
              "out must be a contiguous float32 tensor of n_rows * D values");
  TORCH_CHECK(epoch > 0 && epoch <= 0xFFFFFFFFll, "epoch must be in [1, 2^32)");
  const float* dh = host_f32(dv, D, "dv");
  char* base = static_cast<char*>(buf.data_ptr());
  c10::cuda::CUDAGuard guard(buf.device());
  check(kh_decode_combine_peer_records(reinterpret_cast<const float*>(base + rec_offset),
                                       reinterpret_cast<const uint32_t*>(base + flag_offset),
                                       (uint32_t)epoch, n_rows, (int)n_parts, (int)world, (int)D,
                                       dh, out.data_ptr<float>(), stream_of(buf)),
        "kh_decode_combine_peer_records");
}

// ------------------------------------------------------------------ HBBA

std::tuple<Tensor, Tensor, Tensor, Tensor> ultra_fused_hbba_fusion(
    const Tensor& x, const Tensor& d, const Tensor& centroids_table, const Tensor& mask,
    int64_t layer_id, int64_t active_mask) {
  require_cuda(x, "x");
  TORCH_CHECK(x.dim() == 2, "x must be [N, D]");
  const int64_t N = x.size(0), D = x.size(1);
  const auto dev = x.device();
  const auto prep = [&](const Tensor& t, at::ScalarType s, int64_t n, const char* what) {
    TORCH_CHECK(t.numel() == n, what, " must hold ", n, " values");
    Tensor u = t.to(dev, s).contiguous();
    return u;
  };
  Tensor xr = x.stride(-1) == 1 ? x : x.contiguous();
  Tensor dd = prep(d, at::kFloat, D, "d");
  Tensor cb = prep(centroids_table, at::kFloat, D * 16, "centroids_table");
  Tensor mk = prep(mask, at::kInt, 8, "mask");
  const bool hbba = layer_id >= 0 && layer_id < 8 && (((active_mask & 0xFF) >> layer_id) & 1);
  auto o = x.options();
  Tensor packed = at::empty({N, hbba ? 128 : 32}, o.dtype(at::kByte));
  Tensor norms = at::empty({N, 1}, o.dtype(at::kFloat));
  Tensor rnorms = at::empty({N}, o.dtype(at::kFloat));
  Tensor signs = at::empty({N, D}, o.dtype(at::kHalf));
  c10::cuda::CUDAGuard guard(dev);
  check(kh_compress_hbba(xr.data_ptr(), dtype_code(x.scalar_type()), N, (int)D,
                         N > 1 ? xr.stride(0) : D, dd.data_ptr<float>(), cb.data_ptr<float>(),
                         reinterpret_cast<const uint32_t*>(mk.data_ptr<int>()), (int)layer_id,
                         (int)(active_mask & 0xFF), packed.data_ptr<uint8_t>(),
                         norms.data_ptr<float>(), rnorms.data_ptr<float>(), signs.data_ptr(),
                         stream_of(x)),
        "kh_compress_hbba");
  return {packed, norms, rnorms, signs};
}

Tensor hbba_calibrate_cuda(const Tensor& sample, const Tensor& n_map, int64_t layer_id,
                           int64_t active_mask) {
  require_cuda(sample, "sample");
  TORCH_CHECK(sample.dim() == 2, "sample must be [N, D]");
  const int64_t D = sample.size(1);
  auto o = sample.options().dtype(at::kFloat);
  Tensor out = at::zeros({D, 16}, o);
  const bool hbba = layer_id >= 0 && layer_id < 8 && (((active_mask & 0xFF) >> layer_id) & 1);
  if (!hbba || sample.size(0) == 0) return out;  // the reference returns zeros too (:499)
  Tensor smp = sample.to(at::kFloat).contiguous();
  TORCH_CHECK(n_map.numel() == D, "n_map must hold D values");
  Tensor nm = n_map.to(sample.device(), at::kInt).contiguous();
  c10::cuda::CUDAGuard guard(sample.device());
  check(kh_hbba_calibrate(smp.data_ptr<float>(), smp.size(0), (int)D, nm.data_ptr<int>(),
                          out.data_ptr<float>(), stream_of(sample)),
        "kh_hbba_calibrate");
  return out;
}

// ------------------------------------------------- reference-layout compat

std::tuple<Tensor, Tensor, Tensor, Tensor, Tensor> ultra_fused_full_fusion(const Tensor& x,
                                                                            const Tensor& d,
                                                                            const Tensor& c) {
  auto p = compress(x, d, c, true);
  const int64_t D = x.size(-1);
  auto m = materialize(p[0], p[2], p[1], D, d, c, true, true, true);
  return {m[0], p[1].view({-1, 1}), m[1], p[3].view({-1, 1}), m[2]};
}

Tensor fused_asymmetric_attention(const Tensor& q, const Tensor& k_packed, const Tensor& signs,
                                  const Tensor& d_vec, const Tensor& k_norms,
                                  const Tensor& r_norms, const Tensor& centroids,
                                  int64_t layer_id, int64_t active_mask, double scale) {
  require_cuda(q, "q");
  TORCH_CHECK(q.dim() == 2 && k_norms.dim() == 2, "q [H, D] and k_norms [H, S] expected");
  const int64_t H = q.size(0), D = q.size(1), S = k_norms.size(1);
  const bool nib = layer_id >= 0 && layer_id < 8 && (((active_mask & 0xFF) >> layer_id) & 1);
  const int64_t bpt = nib ? 128 : 32;
  TORCH_CHECK(k_packed.dim() == 3 && k_packed.size(0) == H && k_packed.size(1) == S &&
                  k_packed.size(2) == bpt,
              "k_packed must be [H, S, ", bpt, "] for this layer");
  TORCH_CHECK(signs.dim() == 3 && signs.size(0) == H && signs.size(1) == S && signs.size(2) == D &&
                  r_norms.sizes() == k_norms.sizes() && centroids.numel() == D * 16,
              "signs [H, S, D], r_norms [H, S] and centroids [D, 16] expected");
  const auto prep = [](const Tensor& t, at::ScalarType s) {
    Tensor u = t.to(s).contiguous();
    if ((reinterpret_cast<uintptr_t>(u.data_ptr()) & 15) != 0)
      u = at::empty(u.sizes(), u.options()).copy_(u);
    return u;
  };
  Tensor qh = prep(q, at::kHalf), sg = prep(signs, at::kHalf), kp = prep(k_packed, at::kByte);
  Tensor dvv = prep(d_vec, at::kFloat), kn = prep(k_norms, at::kFloat),
         rn = prep(r_norms, at::kFloat), cb = prep(centroids, at::kFloat);
  Tensor out = at::empty({H, S}, q.options().dtype(at::kFloat));
  c10::cuda::CUDAGuard guard(q.device());
  check(kh_score_packed_compat(qh.data_ptr(), H, (int)D, S, kp.data_ptr<uint8_t>(), sg.data_ptr(),
                               dvv.data_ptr<float>(), kn.data_ptr<float>(), rn.data_ptr<float>(),
                               cb.data_ptr<float>(), (int)layer_id, (int)(active_mask & 0xFF),
                               (float)scale, out.data_ptr<float>(), stream_of(q)),
        "kh_score_packed_compat");
  return out;
}

}  // namespace

TORCH_LIBRARY(kudahitam, m) {
  m.def("compress(Tensor x, Tensor d, Tensor centroids, bool residual=True) -> Tensor[]");
  m.def("compress_out(Tensor x, Tensor d, Tensor centroids, bool residual, Tensor(a!) code, "
        "Tensor(b!)? res, Tensor(c!) norms, Tensor(d!)? rnorms) -> ()");
  m.def("compress_many_out(Tensor[] xs, Tensor d, Tensor centroids, bool residual, "
        "Tensor(a!)[] code, Tensor(b!)[] res, Tensor(c!)[] norms, Tensor(d!)[] rnorms) -> ()");
  m.def("fwht_(Tensor(a!) x) -> Tensor(a!)");
  m.def("materialize(Tensor code, Tensor? res, Tensor norms, int head_dim, Tensor d, "
        "Tensor centroids, bool idx=True, bool kmse=True, bool signs=True) -> Tensor[]");
  m.def("score(Tensor q, Tensor code, Tensor? res, Tensor norms, Tensor? rnorms, int seq_len, "
        "Tensor d, Tensor centroids) -> Tensor");
  m.def("score_out(Tensor q, Tensor code, Tensor? res, Tensor norms, Tensor? rnorms, "
        "int seq_len, Tensor d, Tensor centroids, Tensor(a!) out) -> ()");
  m.def("decode_partial(Tensor q, Tensor k_code, Tensor k_res, Tensor k_norms, Tensor k_rnorms, "
        "Tensor v_code, Tensor v_res, Tensor v_norms, Tensor v_rnorms, int seq_len, "
        "int seq_begin, int seq_end, Tensor dk, Tensor centroids, float sm_scale, int n_splits, "
        "Tensor(a!) partials, int part_stride, int part_offset) -> ()");
  m.def("decode_combine(Tensor records, int n_rows, int n_parts, int group_stride, "
        "int part_stride, Tensor dv, Tensor(a!) out) -> ()");
  m.def("decode_merge(Tensor records, int n_rows, int n_parts, int group_stride, "
        "int part_stride, Tensor(a!) merged) -> ()");
  m.def("decode_attention(Tensor q, Tensor k_code, Tensor k_res, Tensor k_norms, "
        "Tensor k_rnorms, Tensor v_code, Tensor v_res, Tensor v_norms, Tensor v_rnorms, "
        "int seq_len, int length, Tensor dk, Tensor dv, Tensor centroids, float sm_scale, "
        "int n_splits) -> Tensor");
  m.def("decode_merge_to_peers(Tensor partials, int n_rows, int n_parts, int group_stride, "
        "int part_stride, int head_dim, int[] peer_records, int[] peer_flags, int rank, "
        "int epoch, Tensor(a!) counter) -> ()");
  m.def("decode_combine_from_peers(Tensor buf, int rec_offset, int flag_offset, int epoch, "
        "int n_rows, int world, Tensor dv, Tensor(a!) out, int n_parts=1) -> ()");
  m.def("decode_partial_to_peers(Tensor q, Tensor k_code, Tensor k_res, Tensor k_norms, "
        "Tensor k_rnorms, Tensor v_code, Tensor v_res, Tensor v_norms, Tensor v_rnorms, "
        "int seq_len, int seq_begin, int seq_end, Tensor dk, Tensor centroids, float sm_scale, "
        "int n_splits, int[] peer_records, int[] peer_flags, int rank, int epoch, "
        "Tensor(a!) counter, Tensor? dv=None, Tensor(b!)? out=None) -> ()");
  m.def("ultra_fused_hbba_fusion(Tensor x, Tensor d, Tensor centroids_table, Tensor mask, "
        "int layer_id, int active_mask) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("hbba_calibrate_cuda(Tensor sample, Tensor n_map, int layer_id, int active_mask) "
        "-> Tensor");
  m.def("ultra_fused_full_fusion(Tensor x, Tensor d, Tensor centroids) "
        "-> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def("fused_asymmetric_attention(Tensor q, Tensor k_packed, Tensor signs, Tensor d_vec, "
        "Tensor k_norms, Tensor r_norms, Tensor centroids, int layer_id, int active_mask, "
        "float scale) -> Tensor");
}

TORCH_LIBRARY_IMPL(kudahitam, CUDA, m) {
  m.impl("compress", &compress);
  m.impl("compress_out", &compress_out);
  m.impl("compress_many_out", &compress_many_out);
  m.impl("fwht_", &fwht_);
  m.impl("materialize", &materialize);
  m.impl("score", &score);
  m.impl("score_out", &score_out);
  m.impl("decode_partial", &decode_partial);
  m.impl("decode_combine", &decode_combine);
  m.impl("decode_merge", &decode_merge);
  m.impl("decode_attention", &decode_attention);
  m.impl("decode_merge_to_peers", &decode_merge_to_peers);
  m.impl("decode_combine_from_peers", &decode_combine_from_peers);
  m.impl("decode_partial_to_peers", &decode_partial_to_peers);
  m.impl("ultra_fused_hbba_fusion", &ultra_fused_hbba_fusion);
  m.impl("hbba_calibrate_cuda", &hbba_calibrate_cuda);
  m.impl("ultra_fused_full_fusion", &ultra_fused_full_fusion);
  m.impl("fused_asymmetric_attention", &fused_asymmetric_attention);
}
