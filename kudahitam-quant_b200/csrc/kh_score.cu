// kh_score.cu -- asymmetric attention scores read straight from the packed
// cache (no k_mse / int8 signs materialised).
//
// Reference (KudaHitamQuant_full.py:373-377):
//   score = q . k_mse + (1/sqrt(D)) <fwht(q (.) d), signs> r_norm
// With k_mse = norm d (.) H c[idx] / sqrt(D) and q~ = H(q (.) d)/sqrt(D):
//   q . k_mse = norm <q~, c[idx]>
// so for a two-level codebook, with M1 = sum_{idx_i=1} q~_i,
// M2 = sum_{sign_i=+1} q~_i and Q = sum_i q~_i:
//   score = norm (c0 Q + (c1 - c0) M1) + r_norm / sqrt(D) (2 M2 - Q).
#include <cmath>

#include "kh_common.cuh"
#include "kh_internal.h"

namespace kh {
namespace {

constexpr int kScoreThreads = 256;
constexpr int kQChunk = 8;  // queries projected per shared-memory pass

struct alignas(16) ScoreParams {
  const float* q;
  const uint32_t* code;
  const uint32_t* res;
  const float* norms;
  const float* rnorms;
  float* out;
  int64_t seq_len;
  int n_q;
  Codebook cb;
  float d[256];
};

template <int D, int NC>
__global__ void __launch_bounds__(kScoreThreads)
    score_kernel(const __grid_constant__ ScoreParams P) {
  constexpr int kCodeW = (NC == 2) ? D / 32 : D / 16;
  constexpr int kResW = D / 32;
  __shared__ float qt[kQChunk][D];
  __shared__ float qsum[kQChunk];

  const int64_t g = blockIdx.y;
  const int64_t s = (int64_t)blockIdx.x * kScoreThreads + threadIdx.x;
  const bool valid = s < P.seq_len;
  const int64_t row = g * P.seq_len + (valid ? s : 0);
  const bool has_res = P.res != nullptr;

  uint32_t cw[kCodeW], rw[kResW];
  float nrm = 0.f, rn = 0.f;
  if (valid) {
#pragma unroll
    for (int i = 0; i < kCodeW; i += 4)
      *reinterpret_cast<uint4*>(&cw[i]) =
          *reinterpret_cast<const uint4*>(P.code + row * kCodeW + i);
    nrm = P.norms[row];
    if (has_res) {
#pragma unroll
      for (int i = 0; i < kResW; i += 4)
        *reinterpret_cast<uint4*>(&rw[i]) =
            *reinterpret_cast<const uint4*>(P.res + row * kResW + i);
      rn = P.rnorms[row];
    }
  }
  const float inv_sqrt_d = 1.0f / sqrtf((float)D);

  for (int j0 = 0; j0 < P.n_q; j0 += kQChunk) {
    const int nq = min(kQChunk, P.n_q - j0);
    __syncthreads();
    for (int i = threadIdx.x; i < nq * D; i += kScoreThreads) {
      const int j = i / D, e = i % D;
      qt[j][e] = P.q[(g * P.n_q + j0 + j) * D + e] * P.d[e];
    }
    __syncthreads();
    for (int h = 1; h < D; h <<= 1) {
      for (int b = threadIdx.x; b < nq * D / 2; b += kScoreThreads) {
        const int j = b / (D / 2), k = b % (D / 2);
        const int lo = (k / h) * 2 * h + (k % h);
        const float a = qt[j][lo], c = qt[j][lo + h];
        qt[j][lo] = a + c;
        qt[j][lo + h] = a - c;
      }
      __syncthreads();
    }
    for (int i = threadIdx.x; i < nq * D; i += kScoreThreads)
      qt[i / D][i % D] *= inv_sqrt_d;
    __syncthreads();
    if (threadIdx.x < 32 * nq) {
      const int j = threadIdx.x >> 5, l = threadIdx.x & 31;
      float a = 0.f;
      for (int e = l; e < D; e += 32) a += qt[j][e];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (l == 0) qsum[j] = a;
    }
    __syncthreads();
    if (!valid) continue;

    for (int j = 0; j < nq; ++j) {
      const float* qv = qt[j];
      float t1;
      if (NC == 2) {
        float m1 = 0.f;
#pragma unroll
        for (int w = 0; w < kCodeW; ++w) {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            m1 += ((cw[w] >> k) & 1u) ? qv[32 * w + k] : 0.f;
        }
        t1 = nrm * (P.cb.c[0] * qsum[j] + (P.cb.c[1] - P.cb.c[0]) * m1);
      } else {
        float a = 0.f;
#pragma unroll
        for (int w = 0; w < kCodeW; ++w) {
#pragma unroll
          for (int k = 0; k < 16; ++k)
            a = fmaf(qv[16 * w + k], P.cb.c[(cw[w] >> (2 * k)) & 3u], a);
        }
        t1 = nrm * a;
      }
      float t2 = 0.f;
      if (has_res) {
        float m2 = 0.f;
#pragma unroll
        for (int w = 0; w < kResW; ++w) {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            m2 += ((rw[w] >> k) & 1u) ? qv[32 * w + k] : 0.f;
        }
        t2 = inv_sqrt_d * (2.f * m2 - qsum[j]) * rn;
      }
      P.out[(g * P.n_q + j0 + j) * P.seq_len + s] = t1 + t2;
    }
  }
}

}  // namespace

kh_status launch_score(const float* q, int64_t n_groups, int n_q, int D,
                       const uint32_t* code, const uint32_t* res,
                       const float* norms, const float* rnorms,
                       int64_t seq_len, const float* d, const Codebook& cb,
                       float* out, cudaStream_t stream) {
  ScoreParams P;
  P.q = q;
  P.code = code;
  P.res = res;
  P.norms = norms;
  P.rnorms = rnorms;
  P.out = out;
  P.seq_len = seq_len;
  P.n_q = n_q;
  P.cb = cb;
  for (int i = 0; i < D; ++i) P.d[i] = d[i];
  const int64_t bx = (seq_len + kScoreThreads - 1) / kScoreThreads;
  if (bx > 0x7fffffff) return KH_EINVAL;
  const dim3 grid((unsigned)bx, (unsigned)n_groups);
  if (D == 128) {
    if (cb.n_c == 2) score_kernel<128, 2><<<grid, kScoreThreads, 0, stream>>>(P);
    else score_kernel<128, 4><<<grid, kScoreThreads, 0, stream>>>(P);
  } else {
    if (cb.n_c == 2) score_kernel<256, 2><<<grid, kScoreThreads, 0, stream>>>(P);
    else score_kernel<256, 4><<<grid, kScoreThreads, 0, stream>>>(P);
  }
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

}  // namespace kh
