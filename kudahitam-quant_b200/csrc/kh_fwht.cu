// kh_fwht.cu -- standalone orthonormal FWHT (the query projection) and the
// packed-cache materialiser (reference-layout idx / k_mse / signs).
#include <algorithm>
#include <cmath>

#include "kh_common.cuh"
#include "kh_internal.h"

namespace kh {
namespace {

// In-place x <- H x / sqrt(D) for rows of D floats, D a power of two <= 1024.
// Same semantics as fwht_cuda_forward_kernel (KudaHitamCUDA.cu:233-273):
// unnormalised Sylvester butterflies, then one multiply by 1/sqrt(D)
// (:270-272).  A block stages kRowsPerBlock rows in shared memory.
__global__ void __launch_bounds__(256)
    fwht_rows_kernel(float* __restrict__ x, int64_t n_rows, int D,
                     int rows_per_block) {
  extern __shared__ float sh[];
  const int64_t row0 = (int64_t)blockIdx.x * rows_per_block;
  const int nr = (int)(n_rows - row0 < rows_per_block ? n_rows - row0 : rows_per_block);
  const int n = nr * D;
  float* g = x + row0 * D;
  for (int i = threadIdx.x; i < n; i += blockDim.x) sh[i] = g[i];
  __syncthreads();
  for (int h = 1; h < D; h <<= 1) {
    // n/2 butterflies per stage
    for (int b = threadIdx.x; b < n / 2; b += blockDim.x) {
      const int row = b / (D / 2);
      const int k = b % (D / 2);
      const int lo = row * D + (k / h) * 2 * h + (k % h);
      const float a = sh[lo], c = sh[lo + h];
      sh[lo] = a + c;
      sh[lo + h] = a - c;
    }
    __syncthreads();
  }
  const float scale = 1.0f / sqrtf((float)D);
  for (int i = threadIdx.x; i < n; i += blockDim.x) g[i] = sh[i] * scale;
}

struct alignas(16) MatParams {
  const uint32_t* code;
  const uint32_t* res;
  const float* norms;
  uint8_t* idx;
  float* kmse;
  int8_t* signs;
  int64_t n_rows;
  Codebook cb;
  float d[256];
};

// One warp per row, rows strided over a persistent grid; lane l holds
// elements l + 32 j, j < D/32, for the transform (coalesced 128-byte kmse
// stores).  A row's code and residual words are read once per row, one word
// per lane, and broadcast with shuffles; the next row's words are loaded
// before this row is processed, so the loads overlap the work.  The lane's
// d values and the centroids come from the kernel parameters once per
// thread (indexing the parameter bank with a lane-dependent index
// serialises the warp).  Butterfly stages on element bits 0..4 exchange
// across lanes, stages on bits 5.. stay in registers.
template <int D, int NC>
__global__ void __launch_bounds__(256)
    materialize_kernel(const __grid_constant__ MatParams P) {
  constexpr int J = D / 32;
  constexpr int E = D / 32;  // bytes of idx / signs a lane writes per row
  constexpr int kWords = (NC == 2) ? D / 32 : D / 16;
  const int lane = threadIdx.x & 31;
  float dv[J];
#pragma unroll
  for (int j = 0; j < J; ++j) dv[j] = P.d[lane + 32 * j];
  const float c0 = P.cb.c[0], c1 = P.cb.c[1];
  const float c2 = NC == 4 ? P.cb.c[2] : 0.f, c3 = NC == 4 ? P.cb.c[3] : 0.f;
  const float inv_sqrt_d = 1.0f / sqrtf((float)D);
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const bool want_res = P.signs != nullptr;
  const bool want_norm = P.kmse != nullptr;
  int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  uint32_t cw = 0, rw = 0;  // lane l: word l of the row's code / residual plane
  float nrm = 0.f;
  auto load = [&](int64_t r) {
    if (r < P.n_rows) {
      cw = lane < kWords ? __ldg(P.code + r * kWords + lane) : 0u;
      rw = (want_res && lane < D / 32) ? __ldg(P.res + r * (D / 32) + lane) : 0u;
      nrm = want_norm ? __ldg(P.norms + r) : 0.f;
    }
  };
  load(row);
  for (; row < P.n_rows; row += warps) {  // uniform per warp
    const uint32_t cwr = cw, rwr = rw;
    const float nr = nrm;
    load(row + warps);  // next row, in flight while this one is written
    if (P.idx) {
      // lane l writes elements [E l, E (l + 1)) as one 4- or 8-byte store
      uint32_t w[E / 4];
      if (NC == 2) {
        const uint32_t word = __shfl_sync(0xffffffffu, cwr, (E * lane) >> 5);
        const uint32_t bits = (word >> ((E * lane) & 31)) & ((1u << E) - 1);
#pragma unroll
        for (int h = 0; h < E / 4; ++h)  // 4 bits -> 4 bytes of 0 / 1 (no carries)
          w[h] = (((bits >> (4 * h)) & 0xFu) * 0x00204081u) & 0x01010101u;
      } else {
        const uint32_t word = __shfl_sync(0xffffffffu, cwr, (E * lane) >> 4);
        const uint32_t f = word >> (2 * ((E * lane) & 15));
#pragma unroll
        for (int h = 0; h < E / 4; ++h)
          w[h] = ((f >> (8 * h)) & 3u) | (((f >> (8 * h + 2)) & 3u) << 8) |
                 (((f >> (8 * h + 4)) & 3u) << 16) | (((f >> (8 * h + 6)) & 3u) << 24);
      }
      uint8_t* dst = P.idx + row * D + E * lane;
      if constexpr (E == 4) *reinterpret_cast<uint32_t*>(dst) = w[0];
      else *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
    }
    if (P.signs) {
      const uint32_t word = __shfl_sync(0xffffffffu, rwr, (E * lane) >> 5);
      const uint32_t bits = (word >> ((E * lane) & 31)) & ((1u << E) - 1);
      uint32_t w[E / 4];
#pragma unroll
      for (int h = 0; h < E / 4; ++h) {
        const uint32_t e = (((bits >> (4 * h)) & 0xFu) * 0x00204081u) & 0x01010101u;
        w[h] = 0xFFFFFFFFu ^ (e * 0xFEu);  // per byte: bit 1 -> +1, bit 0 -> -1 (0xFF)
      }
      int8_t* dst = P.signs + row * D + E * lane;
      if constexpr (E == 4) *reinterpret_cast<uint32_t*>(dst) = w[0];
      else *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
    }
    if (P.kmse) {
      float r[J];
#pragma unroll
      for (int j = 0; j < J; ++j) {
        if (NC == 2) {
          const uint32_t word = __shfl_sync(0xffffffffu, cwr, j);
          r[j] = ((word >> lane) & 1u) ? c1 : c0;
        } else {
          const uint32_t word = __shfl_sync(0xffffffffu, cwr, 2 * j + (lane >> 4));
          const uint32_t idx = (word >> (2 * (lane & 15))) & 3u;
          r[j] = idx < 2 ? (idx ? c1 : c0) : (idx == 2 ? c2 : c3);
        }
      }
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
      // k_mse = r * m_base * d, m_base = (1/sqrt(D)) * norm (KudaHitamCUDA.cu:142-148)
      const float m_base = inv_sqrt_d * nr;
#pragma unroll
      for (int j = 0; j < J; ++j) P.kmse[row * D + lane + 32 * j] = r[j] * m_base * dv[j];
    }
  }
}

}  // namespace

kh_status launch_fwht(float* x, int64_t n_rows, int D, cudaStream_t stream) {
  const int rows_per_block = D >= 2048 ? 1 : 2048 / D;
  const int64_t blocks = (n_rows + rows_per_block - 1) / rows_per_block;
  if (blocks > 0x7fffffff) return KH_EINVAL;
  const size_t smem = (size_t)rows_per_block * D * sizeof(float);
  fwht_rows_kernel<<<(unsigned)blocks, 256, smem, stream>>>(x, n_rows, D,
                                                            rows_per_block);
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

kh_status launch_materialize(const uint32_t* code, const uint32_t* res,
                             const float* norms, int64_t n_rows, int D,
                             const float* d, const Codebook& cb, uint8_t* idx,
                             float* kmse, int8_t* signs, cudaStream_t stream) {
  MatParams P;
  P.code = code;
  P.res = res;
  P.norms = norms;
  P.idx = idx;
  P.kmse = kmse;
  P.signs = signs;
  P.n_rows = n_rows;
  P.cb = cb;
  for (int i = 0; i < D; ++i) P.d[i] = d[i];
  // persistent grid: 8 blocks of 8 warps per SM, each warp striding over rows
  const int64_t blocks = std::min<int64_t>((n_rows + 7) / 8, (int64_t)sm_count() * 8);
  if (blocks <= 0) return KH_OK;
  const unsigned g = (unsigned)blocks;
  if (D == 128) {
    if (cb.n_c == 2) materialize_kernel<128, 2><<<g, 256, 0, stream>>>(P);
    else materialize_kernel<128, 4><<<g, 256, 0, stream>>>(P);
  } else {
    if (cb.n_c == 2) materialize_kernel<256, 2><<<g, 256, 0, stream>>>(P);
    else materialize_kernel<256, 4><<<g, 256, 0, stream>>>(P);
  }
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

}  // namespace kh
