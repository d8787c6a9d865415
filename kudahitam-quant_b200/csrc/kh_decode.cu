// kh_decode.cu -- split-K decode attention over a compressed K/V cache.
//
// The reference has no softmax.V step (it stops at the scores,
// KudaHitamQuant_full.py:373-386).  Definition used here, per group g
// (one (batch, head) pair, one query):
//   logit_s = score_s * sm_scale      (score_s as in kh_score)
//   p_s     = softmax(logit)_s
//   V_hat_s = d_v (.) H( a_s c[idx_s] + b_s sign_s ),
//             a_s = ||v_s|| / sqrt(D)            (MSE part, KudaHitamCUDA.cu:141-149)
//             b_s = r_norm_s sqrt(2/pi) / D      (QJL residual, E|z| = sqrt(2/pi) sigma)
//   out     = sum_s p_s V_hat_s = d_v (.) H(acc) / l,
//             acc_i = sum_s e^{logit_s - m} (a_s c[idx_si] + b_s sign_si)
// Accumulation stays in the rotated domain; one FWHT per group in the
// combine step.  A partial record is (m, l, acc[0..D-1]).
#include <cmath>

#include "kh_common.cuh"
#include "kh_internal.h"

namespace kh {
namespace {

struct alignas(16) DecodeParams {
  const float* q;
  const uint32_t *k_code, *k_res, *v_code, *v_res;
  const float *k_norms, *k_rnorms, *v_norms, *v_rnorms;
  float* partials;
  int64_t seq_len, seq_begin, seq_end, part_stride, part_offset;
  float sm_scale;
  int n_splits;
  float c0, c1;
  float dk[256];
};

template <int D>
__device__ __forceinline__ float block_reduce(float v, float* red, bool is_max) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < D / 32; ++i) r = is_max ? fmaxf(r, red[i]) : r + red[i];
  return r;
}

// Block of D threads: thread t scores row (blk + t) and owns accumulator t.
template <int D>
__global__ void __launch_bounds__(D)
    decode_partial_kernel(const __grid_constant__ DecodeParams P) {
  constexpr int W = D / 32;
  __shared__ float qt[D];
  __shared__ float w1[D], w2[D];
  __shared__ uint32_t vc[D][W + 1], vr[D][W + 1];
  __shared__ float red[32];

  const int t = threadIdx.x;
  const int64_t g = blockIdx.y;
  const int split = blockIdx.x;
  const int64_t len = P.seq_end - P.seq_begin;
  const int64_t s0 = P.seq_begin + len * split / P.n_splits;
  const int64_t s1 = P.seq_begin + len * (split + 1) / P.n_splits;
  const float inv_sqrt_d = 1.0f / sqrtf((float)D);
  const float qjl = 0.7978845608028654f / (float)D;  // sqrt(2/pi) / D

  // q~ = H(q (.) d) / sqrt(D)
  qt[t] = P.q[g * D + t] * P.dk[t];
  __syncthreads();
  for (int h = 1; h < D; h <<= 1) {
    if (t < D / 2) {
      const int lo = (t / h) * 2 * h + (t % h);
      const float a = qt[lo], c = qt[lo + h];
      qt[lo] = a + c;
      qt[lo + h] = a - c;
    }
    __syncthreads();
  }
  qt[t] *= inv_sqrt_d;
  __syncthreads();
  const float Q = block_reduce<D>(qt[t], red, false);

  float m_run = -INFINITY, l_run = 0.f, acc = 0.f;
  for (int64_t blk = s0; blk < s1; blk += D) {
    const int64_t s = blk + t;
    const bool valid = s < s1;
    float logit = -INFINITY;
    float va = 0.f, vb = 0.f;
    if (valid) {
      const int64_t row = g * P.seq_len + s;
      float m1 = 0.f, m2 = 0.f;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        const uint32_t c = P.k_code[row * W + w];
        const uint32_t r = P.k_res[row * W + w];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const float qv = qt[32 * w + k];
          m1 += ((c >> k) & 1u) ? qv : 0.f;
          m2 += ((r >> k) & 1u) ? qv : 0.f;
        }
      }
      const float score =
          P.k_norms[row] * (P.c0 * Q + (P.c1 - P.c0) * m1) +
          inv_sqrt_d * (2.f * m2 - Q) * P.k_rnorms[row];
      logit = score * P.sm_scale;
      va = P.v_norms[row] * inv_sqrt_d;
      vb = P.v_rnorms[row] * qjl;
#pragma unroll
      for (int w = 0; w < W; ++w) {
        vc[t][w] = P.v_code[row * W + w];
        vr[t][w] = P.v_res[row * W + w];
      }
    } else {
#pragma unroll
      for (int w = 0; w < W; ++w) vc[t][w] = vr[t][w] = 0u;
    }
    const float m_blk = block_reduce<D>(logit, red, true);
    const float m_new = fmaxf(m_run, m_blk);
    const float alpha = expf(m_run - m_new);  // 0 on the first block
    const float p = valid ? expf(logit - m_new) : 0.f;
    const float l_blk = block_reduce<D>(p, red, false);
    // constant part: sum_s p (a c0 - b)
    const float base = block_reduce<D>(p * (va * P.c0 - vb), red, false);
    w1[t] = p * va * (P.c1 - P.c0);
    w2[t] = 2.f * p * vb;
    __syncthreads();
    float a = acc * alpha + base;
    const int wi = t >> 5, bi = t & 31;
    const int nrow = (int)(s1 - blk < D ? s1 - blk : D);
    for (int j = 0; j < nrow; ++j) {
      a += ((vc[j][wi] >> bi) & 1u) ? w1[j] : 0.f;
      a += ((vr[j][wi] >> bi) & 1u) ? w2[j] : 0.f;
    }
    acc = a;
    l_run = l_run * alpha + l_blk;
    m_run = m_new;
    __syncthreads();
  }
  float* rec = P.partials + (g * P.part_stride + P.part_offset + split) * (D + 2);
  if (t == 0) {
    rec[0] = m_run;
    rec[1] = l_run;
  }
  rec[2 + t] = acc;
}

template <int D>
__global__ void __launch_bounds__(D)
    decode_combine_kernel(const float* __restrict__ parts, int n_parts,
                          float* __restrict__ out, const float* __restrict__ dv_unused,
                          const __grid_constant__ DecodeParams P) {
  (void)dv_unused;
  __shared__ float sh[D];
  const int t = threadIdx.x;
  const int64_t g = blockIdx.x;
  const float* base = parts + g * (int64_t)n_parts * (D + 2);
  float M = -INFINITY;
  for (int r = 0; r < n_parts; ++r) {
    const float* rec = base + (int64_t)r * (D + 2);
    if (rec[1] > 0.f) M = fmaxf(M, rec[0]);
  }
  float L = 0.f, a = 0.f;
  for (int r = 0; r < n_parts; ++r) {
    const float* rec = base + (int64_t)r * (D + 2);
    if (rec[1] > 0.f) {
      const float e = expf(rec[0] - M);
      L += rec[1] * e;
      a += rec[2 + t] * e;
    }
  }
  sh[t] = a;
  __syncthreads();
  for (int h = 1; h < D; h <<= 1) {
    if (t < D / 2) {
      const int lo = (t / h) * 2 * h + (t % h);
      const float x = sh[lo], y = sh[lo + h];
      sh[lo] = x + y;
      sh[lo + h] = x - y;
    }
    __syncthreads();
  }
  out[g * D + t] = L > 0.f ? sh[t] * P.dk[t] / L : 0.f;
}

}  // namespace

kh_status launch_decode_partial(const DecodeRequest& r, cudaStream_t stream) {
  DecodeParams P;
  memset(&P, 0, sizeof(P));
  P.q = r.q;
  P.k_code = r.k_code; P.k_res = r.k_res; P.v_code = r.v_code; P.v_res = r.v_res;
  P.k_norms = r.k_norms; P.k_rnorms = r.k_rnorms;
  P.v_norms = r.v_norms; P.v_rnorms = r.v_rnorms;
  P.partials = r.partials;
  P.seq_len = r.seq_len; P.seq_begin = r.seq_begin; P.seq_end = r.seq_end;
  P.part_stride = r.part_stride; P.part_offset = r.part_offset;
  P.sm_scale = r.sm_scale;
  P.n_splits = r.n_splits;
  P.c0 = r.cb.c[0];
  P.c1 = r.cb.c[1];
  for (int i = 0; i < r.D; ++i) P.dk[i] = r.dk[i];
  const dim3 grid((unsigned)r.n_splits, (unsigned)r.n_groups);
  if (r.D == 128) decode_partial_kernel<128><<<grid, 128, 0, stream>>>(P);
  else decode_partial_kernel<256><<<grid, 256, 0, stream>>>(P);
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

kh_status launch_decode_combine(const float* partials, int64_t n_groups,
                                int n_parts, int D, const float* dv,
                                float* out, cudaStream_t stream) {
  DecodeParams P;
  memset(&P, 0, sizeof(P));
  for (int i = 0; i < D; ++i) P.dk[i] = dv[i];
  if (n_groups > 0x7fffffff) return KH_EINVAL;
  if (D == 128)
    decode_combine_kernel<128><<<(unsigned)n_groups, 128, 0, stream>>>(
        partials, n_parts, out, nullptr, P);
  else
    decode_combine_kernel<256><<<(unsigned)n_groups, 256, 0, stream>>>(
        partials, n_parts, out, nullptr, P);
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

}  // namespace kh
