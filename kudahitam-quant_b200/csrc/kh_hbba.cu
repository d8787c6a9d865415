// kh_hbba.cu -- the HBBA mixed-codebook encoder and its calibrator.
//
// The reference's HBBA path (KudaHitamCUDA.cu:285-518, driven by
// KudahitamCompressorHBBA in KudaHitamQuant_full-reasoning.py:467-560) gives
// every element of a row its own codebook from a [D][16] table: 16 levels
// for the high-variance elements chosen by a mask (when the layer is an
// HBBA layer), 2 levels for the rest.  Its output is the packed-byte cache
// that fused_asymmetric_attention reads (kh_score_packed_compat here): the
// indices packed as nibbles (HBBA layer, 128 bytes per row) or single bits
// (32 bytes per row), the row norm, a residual norm, and the residual's
// unnormalised Hadamard transform in fp16.
//
// Encoder (one warp per row, rows strided over a persistent grid; lane l
// holds elements l + 32 j):
//   norm   = sqrt(sum x^2 + 1e-8) over the whole row
//   y      = H(x / norm (.) d) / sqrt(D)       (butterflies: shuffles for
//            element bits 0..4, registers above)
//   idx_i  = argmin_c |y_i - c_i[c]| over the element's 2 or 16 levels
//            (strict <, lowest index; levels rounded to fp16 as the
//            reference's shared table holds them)
//   diff_i = y_i - c_i[idx_i];  r_norm = sqrt(sum diff^2 * D + 1e-8)
//   signs  = fp16(H diff)
// The reference reduces both sums of squares within a warp only while 256
// threads hold the row (:312-314, :377), so for D > 32 each warp divides
// its 32 elements by its own partial norm; here the sums cover the row, the
// computation the code describes.  Packed words are assembled in registers
// (a ballot per 32 one-bit indices, shuffles per 8 nibbles) and stored
// whole; the reference ORs bytes into shared memory and copies them out
// from thread 0 with no barrier after the other warps' atomics (:356-381).
//
// Calibrator (hbba_calibrate_cuda_kernel, :423-496): per dimension, levels
// start uniform between the sample's min and max and take 10 Lloyd rounds
// (nearest level, then the mean of its samples; a level with no samples
// keeps its value).  One lane per dimension, 4 warps striding over the
// samples; sums accumulate in double in a fixed order, so the result does
// not depend on scheduling (the reference adds with float atomics).
#include <algorithm>
#include <cmath>
#include <type_traits>

#include "kh_common.cuh"
#include "kh_internal.h"

namespace kh {
namespace {

struct alignas(16) HbbaParams {
  const void* x;
  int64_t n_rows, row_stride;
  const float* d;        // device [D]
  const float* cent;     // device [D][16]
  const uint32_t* mask;  // device [8]
  uint8_t* packed;       // [n][128 or 32]
  float* norms;
  float* rnorms;
  __half* signs;         // [n][D]
  int is_hbba;
};

template <typename T>
__device__ __forceinline__ float to_f32(T v) {
  if constexpr (std::is_same<T, float>::value) return v;
  else if constexpr (std::is_same<T, __half>::value) return __half2float(v);
  else return __bfloat162float(v);
}

// Unnormalised Sylvester transform of the warp's row held as element
// lane + 32 j in r[j].
template <int J>
__device__ __forceinline__ void warp_fwht(float (&r)[J], int lane) {
#pragma unroll
  for (int h = 1; h < 32; h <<= 1) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const float o = __shfl_xor_sync(0xffffffffu, r[j], h);
      r[j] = (lane & h) ? (o - r[j]) : (r[j] + o);
    }
  }
#pragma unroll
  for (int h = 1; h < J; h <<= 1) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if ((j & h) == 0) {
        const float a = r[j], b = r[j + h];
        r[j] = a + b;
        r[j + h] = a - b;
      }
    }
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T, int D>
__global__ void __launch_bounds__(256)
    hbba_compress_kernel(const __grid_constant__ HbbaParams P) {
  constexpr int J = D / 32;
  __shared__ float cen[16][D];  // level-major: lanes read consecutive elements
  const int t = threadIdx.x, lane = t & 31;
  for (int i = t; i < D * 16; i += blockDim.x)
    cen[i & 15][i >> 4] = __half2float(__float2half_rn(P.cent[i]));
  __syncthreads();
  float dv[J];
  bool wide[J];  // the element uses 16 levels
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int e = lane + 32 * j;
    dv[j] = P.d[e];
    wide[j] = P.is_hbba && ((P.mask[e >> 5] >> (e & 31)) & 1u);
  }
  const float f_scale = 1.0f / sqrtf((float)D);
  const int bpt = P.is_hbba ? 128 : 32;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (t >> 5); row < P.n_rows;
       row += warps) {  // uniform per warp
    const T* xr = static_cast<const T*>(P.x) + row * P.row_stride;
    float r[J];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      r[j] = to_f32(xr[lane + 32 * j]);
      ss = fmaf(r[j], r[j], ss);
    }
    ss = warp_sum(ss);
    const float norm = sqrtf(ss + 1e-8f);
    const float inv = 1.0f / norm;
#pragma unroll
    for (int j = 0; j < J; ++j) r[j] = (r[j] * inv) * dv[j];
    warp_fwht<J>(r, lane);
    uint32_t idx[J];
    float rs = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int e = lane + 32 * j;
      const float y = r[j] * f_scale;
      const int n_c = wide[j] ? 16 : 2;
      int best = 0;
      float md = 1e18f;
      for (int c = 0; c < n_c; ++c) {
        const float dist = fabsf(y - cen[c][e]);
        if (dist < md) {
          md = dist;
          best = c;
        }
      }
      idx[j] = (uint32_t)best;
      const float diff = y - cen[best][e];
      rs = fmaf(diff, diff, rs);
      r[j] = diff;
    }
    rs = warp_sum(rs);
    // packed indices, whole words
    uint8_t* pk = P.packed + row * bpt;
    if (P.is_hbba) {
      // nibble (e & 1) of byte e >> 1: word w holds elements 8 w .. 8 w + 7,
      // which sit in 8 consecutive lanes for each j
#pragma unroll
      for (int j = 0; j < J; ++j) {
        uint32_t w = (idx[j] & 15u) << (4 * (lane & 7));
        w |= __shfl_xor_sync(0xffffffffu, w, 1);
        w |= __shfl_xor_sync(0xffffffffu, w, 2);
        w |= __shfl_xor_sync(0xffffffffu, w, 4);
        if ((lane & 7) == 0) reinterpret_cast<uint32_t*>(pk)[(32 * j + lane) >> 3] = w;
      }
      if (lane < (128 - D / 2) / 4) reinterpret_cast<uint32_t*>(pk)[D / 8 + lane] = 0u;
    } else {
      // bit (e & 7) of byte e >> 3: word j holds elements 32 j .. 32 j + 31
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const uint32_t w = __ballot_sync(0xffffffffu, idx[j] & 1u);
        if (lane == 0) reinterpret_cast<uint32_t*>(pk)[j] = w;
      }
      if (lane >= J && lane < 8) reinterpret_cast<uint32_t*>(pk)[lane] = 0u;
    }
    if (lane == 0) {
      P.norms[row] = norm;
      P.rnorms[row] = sqrtf(rs * (float)D + 1e-8f);
    }
    warp_fwht<J>(r, lane);
#pragma unroll
    for (int j = 0; j < J; ++j) P.signs[row * D + lane + 32 * j] = __float2half_rn(r[j]);
  }
}

struct alignas(16) CalParams {
  const float* sample;  // [n][D]
  int64_t n;
  int D;
  const int* n_map;     // device [D]
  float* out;           // [D][16]
};

// Block of kCalWarps warps serves 32 dimensions (lane = dimension); warp w
// takes samples w, w + kCalWarps, ...
constexpr int kCalWarps = 4;

__global__ void __launch_bounds__(kCalWarps * 32)
    hbba_calibrate_kernel(const __grid_constant__ CalParams P) {
  __shared__ float s_min[kCalWarps][32], s_max[kCalWarps][32];
  __shared__ double s_sum[kCalWarps][16][32];
  __shared__ int s_cnt[kCalWarps][16][32];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int d = blockIdx.x * 32 + lane;
  const bool live = d < P.D;
  const int n_c = live ? min(16, max(1, P.n_map[d])) : 1;
  float mn = 1e18f, mx = -1e18f;
  for (int64_t i = w; i < P.n; i += kCalWarps) {
    if (live) {
      const float v = P.sample[i * P.D + d];
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
  }
  s_min[w][lane] = mn;
  s_max[w][lane] = mx;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kCalWarps; ++k) {
    mn = fminf(mn, s_min[k][lane]);
    mx = fmaxf(mx, s_max[k][lane]);
  }
  float c[16];
#pragma unroll
  for (int k = 0; k < 16; ++k)
    c[k] = k < n_c ? mn + (float)k * (mx - mn) / fmaxf(1.0f, (float)(n_c - 1)) : 0.f;
  for (int it = 0; it < 10; ++it) {
    double sum[16];
    int cnt[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      sum[k] = 0.0;
      cnt[k] = 0;
    }
    if (live) {
      for (int64_t i = w; i < P.n; i += kCalWarps) {
        const float v = P.sample[i * P.D + d];
        int best = 0;
        float md = 1e18f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float dist = fabsf(v - c[k]);
          if (k < n_c && dist < md) {
            md = dist;
            best = k;
          }
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) {  // register arrays: no dynamic index
          sum[k] += best == k ? (double)v : 0.0;
          cnt[k] += best == k;
        }
      }
    }
    __syncthreads();  // the previous round's partials are read
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      s_sum[w][k][lane] = sum[k];
      s_cnt[w][k][lane] = cnt[k];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      double sm = 0.0;
      long long cn = 0;
#pragma unroll
      for (int ww = 0; ww < kCalWarps; ++ww) {
        sm += s_sum[ww][k][lane];
        cn += s_cnt[ww][k][lane];
      }
      if (k < n_c && cn > 0) c[k] = (float)(sm / (double)cn);
    }
  }
  if (live && w == 0) {
#pragma unroll
    for (int k = 0; k < 16; ++k) P.out[d * 16 + k] = k < n_c ? c[k] : 0.f;
  }
}

}  // namespace

kh_status launch_hbba_compress(const void* x, int dtype, int64_t n_rows, int D,
                               int64_t row_stride, const float* d, const float* cent,
                               const uint32_t* mask, int is_hbba, uint8_t* packed,
                               float* norms, float* rnorms, void* signs, cudaStream_t stream) {
  HbbaParams P;
  P.x = x;
  P.n_rows = n_rows;
  P.row_stride = row_stride;
  P.d = d;
  P.cent = cent;
  P.mask = mask;
  P.packed = packed;
  P.norms = norms;
  P.rnorms = rnorms;
  P.signs = static_cast<__half*>(signs);
  P.is_hbba = is_hbba;
  const int64_t blocks = std::min<int64_t>((n_rows + 7) / 8, (int64_t)sm_count() * 8);
  if (blocks <= 0) return KH_OK;
  const dim3 g((unsigned)blocks);
  auto go = [&](auto kern) { kern<<<g, 256, 0, stream>>>(P); };
  if (D == 128) {
    if (dtype == KH_F32) go(hbba_compress_kernel<float, 128>);
    else if (dtype == KH_F16) go(hbba_compress_kernel<__half, 128>);
    else go(hbba_compress_kernel<__nv_bfloat16, 128>);
  } else {
    if (dtype == KH_F32) go(hbba_compress_kernel<float, 256>);
    else if (dtype == KH_F16) go(hbba_compress_kernel<__half, 256>);
    else go(hbba_compress_kernel<__nv_bfloat16, 256>);
  }
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

kh_status launch_hbba_calibrate(const float* sample, int64_t n, int D, const int* n_map,
                                float* out, cudaStream_t stream) {
  CalParams P;
  P.sample = sample;
  P.n = n;
  P.D = D;
  P.n_map = n_map;
  P.out = out;
  hbba_calibrate_kernel<<<(unsigned)((D + 31) / 32), kCalWarps * 32, 0, stream>>>(P);
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

}  // namespace kh
