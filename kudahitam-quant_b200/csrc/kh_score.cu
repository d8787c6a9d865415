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
// Two-level codebooks take the table-driven kernel (score_tab_kernel), the
// 4-level codebook at D = 128 its 2-bit-plane variant (score_tab2b_kernel);
// the 4-level codebook at D = 256 (and KUDAHITAM_SCORE_PATH=direct) the
// direct one.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "kh_bytetab.cuh"
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
  int64_t chunk;  // cached rows per CTA (table path)
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

// Table-driven scores for the two-level codebook.  M1 and M2 are both
// sums of q~ over the set bits of a plane, so one byte table serves both:
// T[v][slot] = sum of q~ over the set bits of byte value v at the slot's byte
// position.  A row costs D/8 lookups per plane instead of D bit-selects.
// One CTA serves one query row (query j of cache group g) and P.chunk cached
// rows, so the query transform and the table are built once per chunk.  The
// host picks chunks like the decode splits: about three waves of CTAs at two
// per SM, no chunk shorter than 4096 rows, equal chunk lengths.  With 512
// query rows this matches fixed 8192-row chunks (160 us at 40000 rows on one
// B200); with few query rows (one sequence of 32 heads) it fills the GPU
// where 8192-row chunks would launch under one wave.
// Table rows are 256 bytes apart (slots 0..31 used) so that one byte-permute
// forms each lookup address (see tab_addr).
template <int D>
struct ScoreTabCfg {
  static constexpr int kP = D / 8;
  static constexpr int kThreads = 256;
  static constexpr int kBatch = 2;  // rows per thread per batch
  // batches in the register ring: kRing - 1 batches are loading while one
  // is scored
  static constexpr int kRing = D == 128 ? 4 : 2;
  // table [256][64] (entries 0..31 of each row used) | q~ [D] | reduction
  // scratch [32]: 65 KB, so two CTAs per SM fit the 132 KB shared-memory
  // carveout and leave the rest of the 256 KB to the L1 that holds the
  // in-flight row loads
  static constexpr int kSmem = (256 * 64 + D + 32) * 4;
};

template <int D, bool RES>
__global__ void __launch_bounds__(256, 2)
    score_tab_kernel(const __grid_constant__ ScoreParams P) {
  grid_dependency_wait();  // q and the cache may come from the previous kernel
  using C = ScoreTabCfg<D>;
  constexpr int kP = C::kP;
  constexpr int kW = D / 32;
  constexpr int NT = C::kThreads;
  constexpr int B = C::kBatch;
  extern __shared__ __align__(16) unsigned char smem_s[];
  unsigned char* tabb = smem_s;
  float* qt = reinterpret_cast<float*>(smem_s) + 256 * 64;
  float* red = qt + D;

  const int t = threadIdx.x;
  const int lane = t & 31;
  const int64_t y = blockIdx.y;      // query row: cache group y / n_q
  const int64_t gk = y / P.n_q;
  const int64_t s0 = (int64_t)blockIdx.x * P.chunk;
  const int n = (int)min(P.chunk, P.seq_len - s0);
  const int64_t row0 = gk * P.seq_len + s0;
  const float inv_sqrt_d = 1.0f / sqrtf((float)D);
  const float c0 = P.cb.c[0], dc = P.cb.c[1] - P.cb.c[0];

  for (int i = t; i < D; i += NT) qt[i] = P.q[y * D + i] * P.d[i];
  __syncthreads();
  for (int h = 1; h < D; h <<= 1) {
    for (int b = t; b < D / 2; b += NT) {
      const int lo = (b / h) * 2 * h + (b % h);
      const float a = qt[lo], c = qt[lo + h];
      qt[lo] = a + c;
      qt[lo + h] = a - c;
    }
    __syncthreads();
  }
  float qpart = 0.f;
  for (int i = t; i < D; i += NT) {
    qt[i] *= inv_sqrt_d;
    qpart += qt[i];
  }
  const float Q = block_sum<NT>(qpart, red);  // (its barriers also publish qt)
  build_byte_table<D>(reinterpret_cast<float*>(tabb), qt, t);
  __syncthreads();

  // D = 128: XOR byte order (at step k this lane reads plane byte k ^ rr, in
  // slot (k ^ rr) + kP (lane / kP)); D = 256 keeps the rotated order (plane
  // byte (k + rr) mod kP), which needs fewer registers with its 8-word planes
  constexpr bool kX = D == 128;
  const int rr = lane % kP;
  const int wr = rr >> 2, bs = 8 * (rr & 3);
  const XorSel xs = xor_selectors(rr);
  uint32_t slot4[kP / 4];  // byte (k & 3) of slot4[k >> 2] = 4 * slot(k)
  static_for<kP / 4>([&](auto mc) {
    constexpr int m = decltype(mc)::value;
    if constexpr (kX) {
      slot4[m] = xor_slots<kP>(m, rr, lane / kP);
    } else {
      uint32_t w = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        w |= (4u * (uint32_t)(((4 * m + j + lane) % kP) + kP * (lane / kP))) << (8 * j);
      slot4[m] = w;
    }
  });

  struct Row {
    uint32_t c[kW], r[RES ? kW : 1];
    float n, rn;
  };
  const int nb = (n + NT * B - 1) / (NT * B);
  auto load_batch = [&](Row (&dst)[B], int bi) {
#pragma unroll
    for (int u = 0; u < B; ++u) {
      const int ii = t + (bi * B + u) * NT;
      const int64_t row = row0 + (ii < n ? ii : 0);
      if constexpr (kX)
        load_plane_xg<D>(P.code + row * kW, wr, dst[u].c);
      else
        load_plane<D>(P.code + row * kW, wr, dst[u].c);
      dst[u].n = __ldg(P.norms + row);
      if constexpr (RES) {
        if constexpr (kX)
          load_plane_xg<D>(P.res + row * kW, wr, dst[u].r);
        else
          load_plane<D>(P.res + row * kW, wr, dst[u].r);
        dst[u].rn = __ldg(P.rnorms + row);
      }
    }
  };
  auto score_batch = [&](const Row (&src)[B], int bi) {
#pragma unroll
    for (int u = 0; u < B; ++u) {
      float2 m = make_float2(0.f, 0.f);
      uint32_t rc[kW], rs[RES ? kW : 1];
      if constexpr (kX) {
        xor_plane<D>(src[u].c, wr, rc);
        if constexpr (RES) xor_plane<D>(src[u].r, wr, rs);
      } else {
        rotate_plane<D>(src[u].c, wr, bs, rc);
        if constexpr (RES) rotate_plane<D>(src[u].r, wr, bs, rs);
      }
      static_for<kP>([&](auto kc) {
        constexpr int k = decltype(kc)::value;
        const uint32_t a1 = kX ? tab_addr_x(rc[k >> 2], slot4[k >> 2], xs.s[k & 3])
                               : tab_addr<k & 3>(rc[k >> 2], slot4[k >> 2]);
        const float x1 = *reinterpret_cast<const float*>(tabb + a1);
        float x2 = 0.f;
        if constexpr (RES) {
          const uint32_t a2 = kX ? tab_addr_x(rs[k >> 2], slot4[k >> 2], xs.s[k & 3])
                                 : tab_addr<k & 3>(rs[k >> 2], slot4[k >> 2]);
          x2 = *reinterpret_cast<const float*>(tabb + a2);
        }
        m = __fadd2_rn(m, make_float2(x1, x2));
      });
      float sc = src[u].n * (c0 * Q + dc * m.x);
      if constexpr (RES) sc += inv_sqrt_d * (2.f * m.y - Q) * src[u].rn;
      const int ii = t + (bi * B + u) * NT;
      if (ii < n) P.out[y * P.seq_len + s0 + ii] = sc;
    }
  };
  Row a[C::kRing][B];
  static_for<C::kRing - 1>([&](auto jc) { load_batch(a[decltype(jc)::value], decltype(jc)::value); });
  for (int bi = 0; bi < nb; bi += C::kRing) {
    static_for<C::kRing>([&](auto jc) {
      constexpr int j = decltype(jc)::value;
      if (bi + j < nb) {
        load_batch(a[(j + C::kRing - 1) % C::kRing], bi + j + C::kRing - 1);
        score_batch(a[j], bi + j);
      }
    });
  }
}

// Table-driven scores for the 4-level (bits=2) codebook at D = 128.  The
// code plane holds 2-bit indices, 4 elements per byte (32 bytes per row), so
// its table folds the centroids in: T2[v][p] = sum_{k<4} q~[4p+k]
// c[(v >> 2k) & 3], and a row's  <q~, c[idx]>  is 32 lookups.  The residual
// plane keeps the 1-bit table (sum of q~ over set bits, 16 positions in two
// copies).  Both tables share the 64-word table rows: T2 in entries 0..31
// (one copy, lane l looks up position (k + l) mod 32 at step k), the
// residual table in entries 32..63.  score = norm * M_code +
// r_norm / sqrt(D) (2 M_res - Q).
template <bool RES>
__global__ void __launch_bounds__(256, 2)
    score_tab2b_kernel(const __grid_constant__ ScoreParams P) {
  grid_dependency_wait();  // q and the cache may come from the previous kernel
  constexpr int D = 128;
  constexpr int kPC = 32, kWC = 8;  // code plane: byte positions, words
  constexpr int kPR = 16, kWR = 4;  // residual plane
  constexpr int NT = 256;
  constexpr int B = 2;
  constexpr int kRing = 3;
  extern __shared__ __align__(16) unsigned char smem_s[];
  unsigned char* tabb = smem_s;
  float* tab = reinterpret_cast<float*>(smem_s);
  float* qt = tab + 256 * 64;
  float* red = qt + D;

  const int t = threadIdx.x;
  const int lane = t & 31;
  const int64_t y = blockIdx.y;
  const int64_t gk = y / P.n_q;
  const int64_t s0 = (int64_t)blockIdx.x * P.chunk;
  const int n = (int)min(P.chunk, P.seq_len - s0);
  const int64_t row0 = gk * P.seq_len + s0;
  const float inv_sqrt_d = 1.0f / sqrtf((float)D);

  for (int i = t; i < D; i += NT) qt[i] = P.q[y * D + i] * P.d[i];
  __syncthreads();
  for (int h = 1; h < D; h <<= 1) {
    for (int b = t; b < D / 2; b += NT) {
      const int lo = (b / h) * 2 * h + (b % h);
      const float a = qt[lo], c = qt[lo + h];
      qt[lo] = a + c;
      qt[lo + h] = a - c;
    }
    __syncthreads();
  }
  float qpart = 0.f;
  for (int i = t; i < D; i += NT) {
    qt[i] *= inv_sqrt_d;
    qpart += qt[i];
  }
  const float Q = block_sum<NT>(qpart, red);  // (its barriers also publish qt)
  {
    // T2: thread (position p = t mod 32, w = t / 32) fills the byte values
    // v = w + 8 kk: low nibble w + 8 (kk & 1), high nibble kk >> 1
    const int p = t & 31, w = t >> 5;
    const float c[4] = {P.cb.c[0], P.cb.c[1], P.cb.c[2], P.cb.c[3]};
    const float q0 = qt[4 * p], q1 = qt[4 * p + 1], q2 = qt[4 * p + 2], q3 = qt[4 * p + 3];
    float lo[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int v = w + 8 * h;
      lo[h] = q0 * c[v & 3] + q1 * c[(v >> 2) & 3];
    }
    static_for<32>([&](auto kc) {
      constexpr int kk = decltype(kc)::value, hv = kk >> 1;
      const float hi = q2 * c[hv & 3] + q3 * c[(hv >> 2) & 3];
      tab[(w + 8 * kk) * 64 + p] = lo[kk & 1] + hi;
    });
  }
  if constexpr (RES) build_byte_table<D>(tab + 32, qt, t);
  __syncthreads();

  // XOR byte order.  Code plane: at step k byte k ^ lane (of 32), slot
  // k ^ lane.  Residual plane: byte k ^ (lane mod 16), two copies (slots 32 +
  // (k ^ (lane mod 16)) + 16 (lane / 16)).  The selectors depend on lane mod
  // 4 only, so both planes share them.
  const int wrc = lane >> 2;
  const XorSel xs = xor_selectors(lane);
  uint32_t slotc[kPC / 4];
  static_for<kPC / 4>([&](auto mc) {
    constexpr int m = decltype(mc)::value;
    slotc[m] = xor_slots<kPC>(m, lane, 0);
  });
  const int rr = lane % kPR;
  const int wrr = rr >> 2;
  uint32_t slotr[kPR / 4];
  static_for<kPR / 4>([&](auto mc) {
    constexpr int m = decltype(mc)::value;
    slotr[m] = xor_slots<kPR>(m, rr, lane / kPR);
  });
  const unsigned char* tabr = tabb + 128;  // entries 32..63 of each table row

  struct Row {
    uint32_t c[kWC], r[RES ? kWR : 1];
    float n, rn;
  };
  const int nb = (n + NT * B - 1) / (NT * B);
  auto load_batch = [&](Row (&dst)[B], int bi) {
#pragma unroll
    for (int u = 0; u < B; ++u) {
      const int ii = t + (bi * B + u) * NT;
      const int64_t row = row0 + (ii < n ? ii : 0);
      load_plane32_xg(P.code + row * kWC, wrc, dst[u].c);  // 32-byte plane
      dst[u].n = __ldg(P.norms + row);
      if constexpr (RES) {
        load_plane_xg<128>(P.res + row * kWR, wrr, dst[u].r);
        dst[u].rn = __ldg(P.rnorms + row);
      }
    }
  };
  auto score_batch = [&](const Row (&src)[B], int bi) {
#pragma unroll
    for (int u = 0; u < B; ++u) {
      float2 m = make_float2(0.f, 0.f);
      uint32_t rc[kWC];
      xor_plane32(src[u].c, wrc, rc);
      static_for<kPC / 2>([&](auto jc) {  // (x = even steps, y = odd steps)
        constexpr int k = 2 * decltype(jc)::value;
        const float x0 = *reinterpret_cast<const float*>(
            tabb + tab_addr_x(rc[k >> 2], slotc[k >> 2], xs.s[k & 3]));
        const float x1 = *reinterpret_cast<const float*>(
            tabb + tab_addr_x(rc[k >> 2], slotc[k >> 2], xs.s[(k + 1) & 3]));
        m = __fadd2_rn(m, make_float2(x0, x1));
      });
      float sc = src[u].n * (m.x + m.y);
      if constexpr (RES) {
        uint32_t rs[kWR];
        xor_plane<128>(src[u].r, wrr, rs);
        float2 mr = make_float2(0.f, 0.f);
        static_for<kPR / 2>([&](auto jc) {
          constexpr int k = 2 * decltype(jc)::value;
          const float x0 = *reinterpret_cast<const float*>(
              tabr + tab_addr_x(rs[k >> 2], slotr[k >> 2], xs.s[k & 3]));
          const float x1 = *reinterpret_cast<const float*>(
              tabr + tab_addr_x(rs[k >> 2], slotr[k >> 2], xs.s[(k + 1) & 3]));
          mr = __fadd2_rn(mr, make_float2(x0, x1));
        });
        sc += inv_sqrt_d * (2.f * (mr.x + mr.y) - Q) * src[u].rn;
      }
      const int ii = t + (bi * B + u) * NT;
      if (ii < n) P.out[y * P.seq_len + s0 + ii] = sc;
    }
  };
  Row a[kRing][B];
  static_for<kRing - 1>([&](auto jc) { load_batch(a[decltype(jc)::value], decltype(jc)::value); });
  for (int bi = 0; bi < nb; bi += kRing) {
    static_for<kRing>([&](auto jc) {
      constexpr int j = decltype(jc)::value;
      if (bi + j < nb) {
        load_batch(a[(j + kRing - 1) % kRing], bi + j + kRing - 1);
        score_batch(a[j], bi + j);
      }
    });
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
  const char* env = getenv("KUDAHITAM_SCORE_PATH");
  const bool direct = env && strcmp(env, "direct") == 0;
  if (!direct && (cb.n_c == 2 || D == 128)) {
    // table-driven path: one CTA per (chunk of cached rows, query row)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KH_ECUDA;
    const int64_t rows_q = n_groups * (int64_t)n_q;
    if (rows_q >= 65536) return KH_EINVAL;
    const int64_t fill = (6 * (int64_t)sm_count() + rows_q - 1) / rows_q;
    const int64_t chunks = std::max<int64_t>(1, std::min(fill, seq_len / 4096));
    // equal chunks, rounded up to whole batches of rows (256 threads x 2)
    P.chunk = ((seq_len + chunks - 1) / chunks + 511) / 512 * 512;
    if (P.chunk > 0x7fffffff) return KH_EINVAL;  // a CTA's row count is an int
    const int64_t bxt = (seq_len + P.chunk - 1) / P.chunk;
    if (bxt > 0x7fffffff) return KH_EINVAL;
    const dim3 gridt((unsigned)bxt, (unsigned)rows_q);
    static std::once_flag once[6][64];
    auto launch = [&](auto kern, int slot, int smem) {
      std::call_once(once[slot][dev & 63], [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      });
      launch_programmatic(kern, gridt, dim3(256), smem, stream, P);
    };
    const bool r = res != nullptr;
    if (cb.n_c == 4) {  // D == 128
      if (r) launch(score_tab2b_kernel<true>, 4, ScoreTabCfg<128>::kSmem);
      else launch(score_tab2b_kernel<false>, 5, ScoreTabCfg<128>::kSmem);
    } else if (D == 128) {
      if (r) launch(score_tab_kernel<128, true>, 0, ScoreTabCfg<128>::kSmem);
      else launch(score_tab_kernel<128, false>, 1, ScoreTabCfg<128>::kSmem);
    } else {
      if (r) launch(score_tab_kernel<256, true>, 2, ScoreTabCfg<256>::kSmem);
      else launch(score_tab_kernel<256, false>, 3, ScoreTabCfg<256>::kSmem);
    }
    return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
  }
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
