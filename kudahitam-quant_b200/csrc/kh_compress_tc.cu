// kh_compress_tc.cu -- fused compression with the Walsh-Hadamard transform on
// the 5th-generation tensor cores (tcgen05), for fp16 / bf16 rows.
//
// u = X . B with B[k][n] = d_k H_128[k][n] (+-1, exact in fp16/bf16) turns the
// d-flip and the unnormalised transform into one MMA chain per 128-row tile;
// products are exact and accumulate in fp32 in tensor memory.  D = 256 uses
// H_256 = [[H_128, H_128], [H_128, -H_128]]: two 128-column accumulators
// a = X_lo B_lo and b = X_hi B_hi give u_lo = a + b and u_hi = a - b, half
// the tensor work of a full 256x256 product.  ||x||^2 follows from Parseval:
// sum of all accumulator squares = 128 ||x||^2 for both head dims.
//
// Roles (one CTA per SM, persistent over tiles):
//   warp 0      TMA producer: 128 x D tile -> shared memory ring (128B swizzle)
//   warp 1      allocates tensor memory; one lane issues tcgen05.mma
//   warps 2..9  two epilogue warpgroups; warpgroup g drains accumulator buffer
//               g (tiles alternate), thread = tensor-memory lane = row; at
//               D = 256 a thread reads its 256 values in two passes of 128
// All mbarrier waits are bounded (kh::mbar_wait); a timeout records an error
// bit and every role leaves its loop.  Every TMA load is a plain per-CTA load.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "kh_common.cuh"
#include "kh_internal.h"
#include "kh_quant.cuh"

namespace kh {
namespace {

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_u32(dst)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
               ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, kind::f16, fp32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc,
                                         uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
      ::"r"(smem_u32(bar)) : "memory");
}
// 32 consecutive fp32 columns of this thread's tensor-memory lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand stored as 128-byte rows
// with the 128B swizzle (the layout TMA SWIZZLE_128B writes), 8-row groups
// 1024 B apart, descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulator, A and B of the same
// 16-bit type (both K-major), M x N.
__host__ __device__ constexpr uint32_t make_idesc(bool bf16, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int MAXSEG>
struct alignas(64) TcParams {
  CUtensorMap tmap[MAXSEG];
  uint32_t* code[MAXSEG];
  uint32_t* res[MAXSEG];
  float* norms[MAXSEG];
  float* rnorms[MAXSEG];
  int64_t n_rows[MAXSEG];
  int64_t tile_begin[MAXSEG + 1];
  uint32_t* err;
  int n_seg;
  Codebook cb;
  float dsign[256];
};

template <int D>
struct TcCfg {
  static constexpr int kM = 128;                 // rows per tile
  static constexpr int kNB = D / 128;            // 128-column chunks per tile
  static constexpr int kBoxBytes = kM * 128;     // one 64-column K-block of a chunk
  static constexpr int kChunkBytes = 2 * kBoxBytes;  // 128 rows x 128 columns, 32 KB
  static constexpr int kStages = (D == 128) ? 5 : 4;  // chunk ring depth
  static constexpr int kBMatBytes = 2 * kBoxBytes;
  static constexpr int kAccCols = D;             // tensor-memory columns per tile
  static constexpr uint32_t kTmemCols = 2 * kAccCols;
  static constexpr int kThreads = 320;
  static constexpr int kBarOff = kStages * kChunkBytes + kNB * kBMatBytes;
  // then the barriers and the tensor-memory slot; 1024 bytes of slack align
  // the stage ring to the 128B swizzle's 1024-byte atom
  static constexpr int kEndOff = kBarOff + (2 * kStages + 4) * 8 + 16;
  static constexpr int kSmem = 1024 + kEndOff;
  static_assert(kSmem <= 232448, "exceeds the 227 KB of shared memory a CTA can use");
};

// Store this row's packed words w[0..n) at dst (16-byte vectors when possible).
template <int N>
__device__ __forceinline__ void store_words(uint32_t* dst, const uint32_t* w) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int k = 0; k < N / 4; ++k)
      reinterpret_cast<uint4*>(dst)[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  } else {
#pragma unroll
    for (int k = 0; k < N / 2; ++k)
      reinterpret_cast<uint2*>(dst)[k] = make_uint2(w[2 * k], w[2 * k + 1]);
  }
}

// Quantise NG groups of 32 values: the interleaved fast path for the
// symmetric codebook, the per-group generic code otherwise.
template <int CK, bool RES, int NG, class P>
__device__ __forceinline__ void quant_groups(const float (&u)[NG][32], float rs, const P& prm,
                                             uint32_t* code, uint32_t* resw, float2& acc,
                                             bool nonzero_row) {
  if constexpr (CK == kCbSym2) {
    quant_sym2_groups<NG, RES>(u, rs, prm.cb.c[1], code, resw, acc,
                               nonzero_row ? 0xffffffffu : 0u);
  } else {
    using Q = Quant<CK, RES>;
#pragma unroll
    for (int g = 0; g < NG; ++g) Q::run(u[g], rs, prm, &code[g * Q::kCodeWords], resw[g], acc);
  }
}

template <typename T, int D, int CK, bool RES, int MAXSEG>
__global__ void __launch_bounds__(320, 1)
    compress_tc_kernel(const __grid_constant__ TcParams<MAXSEG> P) {
  using C = TcCfg<D>;
  using Q = Quant<CK, RES>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdesc = make_idesc(kBF16, 128, 128);
  constexpr uint16_t kOne = kBF16 ? 0x3F80 : 0x3C00;
  constexpr int kCW = Q::kCodeWords;  // code words per 32 elements

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* g = smem_raw + (base - raw);
  uint8_t* stages = g;
  uint8_t* bmat = g + C::kStages * C::kChunkBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(g + C::kBarOff);
  uint64_t* empty = full + C::kStages;
  uint64_t* tfull = empty + C::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- B = diag(d) H_128 per 128-column chunk, K-major, 128B-swizzled -----
  for (int i = threadIdx.x; i < C::kNB * 2 * 128 * 8; i += C::kThreads) {
    const int mat = i / 2048, rem = i % 2048;
    const int kb = rem / 1024, n = (rem / 8) % 128, c = rem % 8;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      uint32_t h2 = 0;
#pragma unroll
      for (int f = 0; f < 2; ++f) {
        const int k = kb * 64 + c * 8 + e + f;
        const bool neg = ((__popc(k & n) & 1) != 0) != (P.dsign[mat * 128 + k] < 0.f);
        h2 |= (uint32_t)(kOne | (neg ? 0x8000u : 0u)) << (16 * f);
      }
      w[e / 2] = h2;
    }
    *reinterpret_cast<uint4*>(bmat + mat * C::kBMatBytes + kb * C::kBoxBytes + n * 128 +
                              ((c ^ (n & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);  // the 4 warps of one warpgroup
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int64_t total = P.tile_begin[P.n_seg];
  // Segment of tile t.  Each role visits its tiles in increasing order, so
  // the search resumes from the previous answer (amortised O(1) per tile
  // instead of a scan of the segment table per tile).
  auto seg_of = [&](int64_t t, int& sg) {
#pragma unroll 1
    while (sg + 1 < P.n_seg && t >= P.tile_begin[sg + 1]) ++sg;
    return sg;
  };

  if (warp == 0) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t policy = l2_policy_evict_first();
      // The set-up above reads only kernel parameters, so with a programmatic
      // launch it overlaps the previous kernel in the stream; rows are read
      // (and hence outputs written) only after that kernel has completed.
      grid_dependency_wait();
      int c = 0;  // chunk counter
      int sg_cur = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const int sg = seg_of(t, sg_cur);
        const int32_t row0 = (int32_t)((t - P.tile_begin[sg]) * C::kM);
#pragma unroll 1
        for (int h = 0; h < C::kNB; ++h, ++c) {
          const int s = c % C::kStages;
          const uint32_t ph = (uint32_t)((c / C::kStages) & 1);
          if (!mbar_wait(&empty[s], ph ^ 1u, P.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], C::kChunkBytes);
          uint8_t* dst = stages + s * C::kChunkBytes;
          tma_load_2d(dst, &P.tmap[sg], h * 128, row0, &full[s], policy);
          tma_load_2d(dst + C::kBoxBytes, &P.tmap[sg], h * 128 + 64, row0, &full[s], policy);
        }
      }
      // this CTA has issued its last row loads: the next kernel in the stream
      // may start its set-up on SMs as they free up
      grid_dependents_launch();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int i = 0, c = 0;
      bool ok = true;
      const uint32_t b0 = smem_u32(bmat);
      for (int64_t t = blockIdx.x; t < total && ok; t += gridDim.x, ++i) {
        const int b = i & 1;
        const uint32_t jb = (uint32_t)((i >> 1) & 1);
        if (!mbar_wait(&tempty[b], jb ^ 1u, P.err)) break;
        tc_fence_after();
#pragma unroll 1
        for (int h = 0; h < C::kNB; ++h, ++c) {
          const int s = c % C::kStages;
          const uint32_t ph = (uint32_t)((c / C::kStages) & 1);
          if (!mbar_wait(&full[s], ph, P.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a0 = smem_u32(stages + s * C::kChunkBytes);
          const uint32_t dt = tmem + b * C::kAccCols + h * 128;
#pragma unroll
          for (int kb = 0; kb < 2; ++kb) {
            const uint64_t ad = sw128_desc(a0 + kb * C::kBoxBytes);
            const uint64_t bd = sw128_desc(b0 + h * C::kBMatBytes + kb * C::kBoxBytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)  // K = 16 per MMA: 32 B along the row
              umma_f16(dt, ad + 2 * kk, bd + 2 * kk, kIdesc, (kb | kk) != 0);
          }
          umma_commit(&empty[s]);  // frees the chunk stage once these MMAs finish
        }
        if (ok) umma_commit(&tfull[b]);
      }
    }
  } else {
    // ------------------------------------------------------ epilogue
    const int wg = (warp - 2) >> 2;  // warpgroup 0 or 1
    const int q = warp & 3;          // tensor-memory lane quarter of this warp
    const int r = 32 * q + lane;     // row within the tile
    int i = 0;
    int sg_cur = 0;
    for (int64_t t = blockIdx.x; t < total; t += gridDim.x, ++i) {
      if ((i & 1) != wg) continue;  // warpgroups alternate tiles (and buffers)
      const int b = i & 1;
      const uint32_t jb = (uint32_t)((i >> 1) & 1);
      // warp-uniform outcome: tcgen05.ld below is a warp-collective
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[b], jb, P.err));
      if (!ok) break;
      tc_fence_after();
      const int sg = seg_of(t, sg_cur);
      const int64_t row = (t - P.tile_begin[sg]) * C::kM + r;
      const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + b * C::kAccCols;
      constexpr int kRowCW = (D / 32) * kCW;
      uint32_t code[kRowCW];
      uint32_t resw[D / 32];
      float2 acc = make_float2(0.f, 0.f);
      float norm;

      if constexpr (D == 128) {
        float u[4][32];
        float2 s2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int gq = 0; gq < 4; ++gq) tmem_ld32(ta + 32 * gq, u[gq]);
        tmem_wait_ld();
        // accumulator in registers: hand the buffer back to the MMA issuer
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
#pragma unroll
        for (int gq = 0; gq < 4; ++gq)
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 p = make_float2(u[gq][e], u[gq][e + 1]);
            s2[gq & 1] = __ffma2_rn(p, p, s2[gq & 1]);
          }
        const float ss = (s2[0].x + s2[0].y) + (s2[1].x + s2[1].y);  // = 128 ||x||^2
        norm = ss > 0.f ? sqrtf(ss * (1.0f / 128.0f)) : 1e-8f;
        const float rs = 1.0f / (norm * 11.313708498984761f);
        quant_groups<CK, RES, 4>(u, rs, P, code, resw, acc, ss > 0.f);
      } else {
        // D = 256: a = X_lo B in columns [0,128), b = X_hi B in [128,256);
        // u_lo = a + b, u_hi = a - b.  The thread owns the whole row and
        // reads its 256 values twice, 128 at a time: sums of squares first
        // (sum a^2 + b^2 = 128 ||x||^2), then the butterfly and quantisation
        // of 64 columns of a and b (words 2h, 2h+1 of u_lo, 4+2h, 5+2h of u_hi).
        float2 s2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float v[4][32];
#pragma unroll
          for (int gq = 0; gq < 4; ++gq) tmem_ld32(ta + 128 * h + 32 * gq, v[gq]);
          tmem_wait_ld();
#pragma unroll
          for (int gq = 0; gq < 4; ++gq)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 p = make_float2(v[gq][e], v[gq][e + 1]);
              s2[gq & 1] = __ffma2_rn(p, p, s2[gq & 1]);
            }
        }
        const float ss = (s2[0].x + s2[0].y) + (s2[1].x + s2[1].y);
        norm = ss > 0.f ? sqrtf(ss * (1.0f / 128.0f)) : 1e-8f;
        const float rs = 1.0f / (norm * 16.0f);
        const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float u[4][32];  // a cols 64h.., 64h+32.., then b cols 64h.., 64h+32..
          tmem_ld32(ta + 64 * h, u[0]);
          tmem_ld32(ta + 64 * h + 32, u[1]);
          tmem_ld32(ta + 128 + 64 * h, u[2]);
          tmem_ld32(ta + 128 + 64 * h + 32, u[3]);
          tmem_wait_ld();
          if (h == 1) {  // every read of this buffer done: hand it back
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
          }
#pragma unroll
          for (int gq = 0; gq < 2; ++gq)
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const float2 pa = make_float2(u[gq][e], u[gq][e + 1]);
              const float2 pb = make_float2(u[2 + gq][e], u[2 + gq][e + 1]);
              const float2 lo = __fadd2_rn(pa, pb);
              const float2 hi = __ffma2_rn(pb, neg1, pa);
              u[gq][e] = lo.x; u[gq][e + 1] = lo.y;
              u[2 + gq][e] = hi.x; u[2 + gq][e + 1] = hi.y;
            }
          uint32_t ch[4 * kCW], rh[4];
          quant_groups<CK, RES, 4>(u, rs, P, ch, rh, acc, ss > 0.f);
#pragma unroll
          for (int w = 0; w < 2 * kCW; ++w) {
            code[2 * h * kCW + w] = ch[w];
            code[(4 + 2 * h) * kCW + w] = ch[2 * kCW + w];
          }
          resw[2 * h] = rh[0];
          resw[2 * h + 1] = rh[1];
          resw[4 + 2 * h] = rh[2];
          resw[5 + 2 * h] = rh[3];
        }
      }
      const float a = acc.x + acc.y;
      const float rn = a > 0.f ? norm * sqrtf(a) : 1e-8f;

      if (row < P.n_rows[sg]) {
        store_words<kRowCW>(P.code[sg] + row * kRowCW, code);
        if (RES) store_words<D / 32>(P.res[sg] + row * (D / 32), resw);
        P.norms[sg][row] = norm;
        if (RES) P.rnorms[sg][row] = rn;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host
template <typename T, int D, int CK, bool RES, int MAXSEG>
kh_status launch_tc_typed(const CompressRequest& req, cudaStream_t stream) {
  using C = TcCfg<D>;
  auto kern = compress_tc_kernel<T, D, CK, RES, MAXSEG>;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KH_ECUDA;
  static std::once_flag attr_once[64];
  std::call_once(attr_once[dev & 63], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  });

  TcParams<MAXSEG> P;
  memset(&P, 0, sizeof(P));
  const CUtensorMapDataType dt = std::is_same<T, __half>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int64_t tiles = 0;
  P.n_seg = req.n_seg;
  for (int i = 0; i < req.n_seg; ++i) {
    const CompressSegHost& s = req.seg[i];
    P.tile_begin[i] = tiles;
    tiles += (s.n_rows + C::kM - 1) / C::kM;
    P.code[i] = s.code;
    P.res[i] = s.res;
    P.norms[i] = s.norms;
    P.rnorms[i] = s.rnorms;
    P.n_rows[i] = s.n_rows;
    if (s.n_rows > 0) {
      const CUresult cr = encode_tensor_map_2d(
          &P.tmap[i], dt, const_cast<void*>(s.x), (uint64_t)D, (uint64_t)s.n_rows,
          (uint64_t)(s.row_stride * 2), 64u, (uint32_t)C::kM, CU_TENSOR_MAP_SWIZZLE_128B);
      if (cr != CUDA_SUCCESS) return KH_ECUDA;
    }
  }
  P.tile_begin[req.n_seg] = tiles;
  if (tiles == 0) return KH_OK;
  P.err = device_error_ptr();
  P.cb = req.cb;
  for (int e = 0; e < D; ++e) P.dsign[e] = req.dflip[e] ? -1.f : 1.f;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, sm_count()));
  // Programmatic dependent launch: this grid may start while the previous
  // kernel in the stream finishes; its producer waits for that kernel's
  // completion before the first row load.
  if (launch_programmatic(kern, dim3((unsigned)grid), dim3(C::kThreads), C::kSmem, stream, P) !=
      cudaSuccess)
    return KH_ELAUNCH;
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

template <typename T, int D, int MAXSEG>
kh_status tc_dispatch_cb(const CompressRequest& req, cudaStream_t s) {
  const bool res = req.residual != 0;
  switch (req.cb.kind) {
    case kCbSym2:
      return res ? launch_tc_typed<T, D, kCbSym2, true, MAXSEG>(req, s)
                 : launch_tc_typed<T, D, kCbSym2, false, MAXSEG>(req, s);
    case kCbGen2:
      return res ? launch_tc_typed<T, D, kCbGen2, true, MAXSEG>(req, s)
                 : launch_tc_typed<T, D, kCbGen2, false, MAXSEG>(req, s);
    case kCbGen4:
      return res ? launch_tc_typed<T, D, kCbGen4, true, MAXSEG>(req, s)
                 : launch_tc_typed<T, D, kCbGen4, false, MAXSEG>(req, s);
  }
  return KH_EINVAL;
}

template <int MAXSEG>
kh_status tc_dispatch(const CompressRequest& req, cudaStream_t s) {
  if (req.dtype == KH_F16)
    return req.head_dim == 128 ? tc_dispatch_cb<__half, 128, MAXSEG>(req, s)
                               : tc_dispatch_cb<__half, 256, MAXSEG>(req, s);
  return req.head_dim == 128 ? tc_dispatch_cb<__nv_bfloat16, 128, MAXSEG>(req, s)
                             : tc_dispatch_cb<__nv_bfloat16, 256, MAXSEG>(req, s);
}

}  // namespace

kh_status launch_compress_tc(const CompressRequest& req, cudaStream_t stream) {
  if (req.dtype != KH_F16 && req.dtype != KH_BF16) return KH_ENOTSUP;
  if (req.n_seg <= 2) return tc_dispatch<2>(req, stream);
  return tc_dispatch<kMaxSegments>(req, stream);
}

}  // namespace kh
