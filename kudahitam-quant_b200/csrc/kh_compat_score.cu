// kh_compat_score.cu -- the reference's packed-cache scorer, argument for
// argument (fused_asymmetric_attention_packed_kernel + its binding,
// KudaHitamCUDA.cu:695-797).
//
// For head h and cached row s:
//   q~   = H(q_h (.) d) / sqrt(D)      H = unnormalised Sylvester Hadamard,
//                                      butterfly strides 1, 2, 4, ... (:723-735)
//   sum1 = sum_i q~_i * (centroids[i][v_i] * k_norm)          (:758-760)
//   sum2 = sum_i q_i * signs[h][s][i]   (unrotated q, raw values, :761)
//   out  = sum1 + k_norm * scale * sum2 * r_norm              (:771)
// v_i is bit (i & 7) of byte (i >> 3) of the row's packed bytes, or, for a
// layer whose bit is set in active_mask, nibble (i & 1) of byte (i >> 1)
// (:751-757); a row holds 32 resp. 128 packed bytes (:407, :745).
//
// The summation order is the reference's: lane l of a warp accumulates
// elements l, l + 32, ... with one fused multiply-add each, then a butterfly
// shuffle reduction, so the result is the reference kernel's to the bit.
//
// B200 layout: one warp per row as in the reference, but each warp keeps two
// rows in flight, the packed bytes are read as 32-bit words (one broadcast
// load per 32 elements in the 1-bit layout), and the centroid table sits in
// shared memory transposed ([value][element]) so that the 32 lanes of a
// lookup hit 32 distinct banks (the reference's [element][16] layout puts
// lane l and lane l + 2 in the same bank).  A CTA serves 1024 rows of one
// head, so the per-CTA set-up (query transform, 16*D-entry table) is read
// once per 1024 rows.
#include <cuda_fp16.h>

#include <cstdint>

#include "kh_internal.h"

namespace kh {
namespace {

constexpr int kCompatThreads = 256;
constexpr int kCompatRowsPerCta = 1024;

struct CompatParams {
  const __half* q;
  const uint8_t* k_packed;
  const __half* signs;
  const float* d;
  const float* k_norms;
  const float* r_norms;
  const float* centroids;
  float* out;
  int64_t seq_len;
  float scale;
  int nibble;  // 1: 4-bit layout (128 bytes per row), 0: 1-bit (32 bytes per row)
};

template <int D>
__global__ void __launch_bounds__(kCompatThreads)
    compat_score_kernel(const __grid_constant__ CompatParams P) {
  constexpr int kJ = D / 32;  // elements per lane
  __shared__ float s_q[D];
  __shared__ float s_qp[D];
  __shared__ float s_c[16 * D];  // [value][element]
  const int t = threadIdx.x;
  const int64_t h = blockIdx.y;

  for (int i = t; i < D; i += kCompatThreads) {
    const float qv = __half2float(P.q[h * D + i]);
    s_q[i] = qv;
    s_qp[i] = qv * P.d[i];
  }
  for (int e = t; e < 16 * D; e += kCompatThreads) {
    const int i = e >> 4, v = e & 15;  // coalesced read of [D][16]
    s_c[v * D + i] = P.centroids[e];
  }
  __syncthreads();
  for (int len = 1; len < D; len <<= 1) {
    for (int b = t; b < D / 2; b += kCompatThreads) {
      const int lo = (b / len) * 2 * len + (b % len);
      const float a = s_qp[lo], c = s_qp[lo + len];
      s_qp[lo] = a + c;
      s_qp[lo + len] = a - c;
    }
    __syncthreads();
  }
  const float inv = 1.0f / sqrtf((float)D);
  for (int i = t; i < D; i += kCompatThreads) s_qp[i] *= inv;
  __syncthreads();

  const int lane = t & 31, warp = t >> 5;
  const int bpt = P.nibble ? 128 : 32;
  const int64_t r_begin = (int64_t)blockIdx.x * kCompatRowsPerCta;
  int64_t r_end = r_begin + kCompatRowsPerCta;
  if (r_end > P.seq_len) r_end = P.seq_len;

  for (int64_t r0 = r_begin + 2 * warp; r0 < r_end; r0 += 2 * (kCompatThreads / 32)) {
    float s1[2] = {0.f, 0.f}, s2[2] = {0.f, 0.f}, kn[2], rn[2];
    const int nr = (r0 + 1 < r_end) ? 2 : 1;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (u >= nr) break;
      const int64_t row = h * P.seq_len + r0 + u;
      const uint32_t* kw = reinterpret_cast<const uint32_t*>(P.k_packed + row * bpt);
      const __half* sg = P.signs + row * D;
      kn[u] = __ldg(P.k_norms + row);
      rn[u] = __ldg(P.r_norms + row);
#pragma unroll
      for (int j = 0; j < kJ; ++j) {
        const int i = lane + 32 * j;
        int v;
        if (P.nibble) {
          v = (int)((__ldg(kw + (i >> 3)) >> (4 * (i & 7))) & 15u);
        } else {
          v = (int)((__ldg(kw + j) >> lane) & 1u);  // word j = elements 32j .. 32j+31
        }
        const float k_recon = s_c[v * D + i] * kn[u];
        s1[u] = __fmaf_rn(s_qp[i], k_recon, s1[u]);
        s2[u] = __fmaf_rn(s_q[i], __half2float(sg[i]), s2[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        s1[u] += __shfl_xor_sync(0xffffffffu, s1[u], o);
        s2[u] += __shfl_xor_sync(0xffffffffu, s2[u], o);
      }
    }
    if (lane == 0) {
      for (int u = 0; u < nr; ++u) {
        const float t2 = kn[u] * P.scale * s2[u];
        P.out[h * P.seq_len + r0 + u] = __fmaf_rn(t2, rn[u], s1[u]);
      }
    }
  }
}

}  // namespace

kh_status launch_score_packed_compat(const void* q, int64_t n_heads, int D, int64_t seq_len,
                                     const uint8_t* k_packed, const void* signs,
                                     const float* d, const float* k_norms,
                                     const float* r_norms, const float* centroids,
                                     int nibble, float scale, float* out,
                                     cudaStream_t stream) {
  CompatParams P;
  P.q = static_cast<const __half*>(q);
  P.k_packed = k_packed;
  P.signs = static_cast<const __half*>(signs);
  P.d = d;
  P.k_norms = k_norms;
  P.r_norms = r_norms;
  P.centroids = centroids;
  P.out = out;
  P.seq_len = seq_len;
  P.scale = scale;
  P.nibble = nibble;
  const int64_t bx = (seq_len + kCompatRowsPerCta - 1) / kCompatRowsPerCta;
  if (bx > 0x7fffffff) return KH_EINVAL;
  const dim3 grid((unsigned)bx, (unsigned)n_heads);
  switch (D) {
    case 32: compat_score_kernel<32><<<grid, kCompatThreads, 0, stream>>>(P); break;
    case 64: compat_score_kernel<64><<<grid, kCompatThreads, 0, stream>>>(P); break;
    case 128: compat_score_kernel<128><<<grid, kCompatThreads, 0, stream>>>(P); break;
    case 256: compat_score_kernel<256><<<grid, kCompatThreads, 0, stream>>>(P); break;
    default: return KH_EINVAL;
  }
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

}  // namespace kh
