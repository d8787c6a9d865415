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
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <utility>

#include "kh_bytetab.cuh"
#include "kh_common.cuh"
#include "kh_internal.h"

namespace kh {
namespace {

constexpr int kMaxPeers = 8;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

struct alignas(16) DecodeParams {
  const float* q;
  const uint32_t *k_code, *k_res, *v_code, *v_res;
  const float *k_norms, *k_rnorms, *v_norms, *v_rnorms;
  float* partials;
  int64_t seq_len, seq_begin, seq_end, part_stride, part_offset;
  float sm_scale;
  int n_splits;
  int n_q;  // queries per cache group (grouped-query attention); blockIdx.y = query row
  float c0, c1;
  float cb[4];  // the codebook (2 or 4 levels)
  // decode v3 work split: CTA b serves query j = b mod n_q of every cache
  // group in the flattened range [set W, (set + 1) W) of (cache group,
  // sequence row), set = b / n_q; W = 0: the sequence range is empty
  int64_t W;
  int64_t n_groups_kv;
  // peer mode (world > 0): records go to slot [rank] of every rank's buffer
  // [world][n_rows_q][n_splits][D+2] instead of `partials`; the last CTA
  // raises epoch in slot [rank] of every rank's flag array
  int world, rank;
  uint32_t epoch;
  uint32_t* counter;
  int64_t n_rows_q;
  float* peer_rec[kMaxPeers];
  uint32_t* peer_flag[kMaxPeers];
  // peer mode with the combine fused (fuse = 1; every CTA of the launch is
  // resident at once): after the count-out, every CTA waits for all ranks'
  // flags and merges its share of the query rows into out
  int fuse;
  float* out;
  uint32_t* err;
  float dk[256];
  float dv[256];
};

// Record (m, l, acc) of query row g, slot p: into the caller's partials, or
// in peer mode into this rank's slot of every rank's record buffer.  Thread
// t < D writes acc[t] (when with_acc), thread 0 writes m and l.
template <int D>
__device__ __forceinline__ void put_record(const DecodeParams& P, int64_t g, int64_t p, int t,
                                           float m, float l, float a, bool with_acc) {
  if (P.world == 0) {
    float* rec = P.partials + (g * P.part_stride + P.part_offset + p) * (D + 2);
    if (with_acc && t < D) rec[2 + t] = a;
    if (t == 0) {
      rec[0] = m;
      rec[1] = l;
    }
    return;
  }
  const int64_t off = (((int64_t)P.rank * P.n_rows_q + g) * P.n_splits + p) * (D + 2);
  for (int r = 0; r < P.world; ++r) {
    float* rec = P.peer_rec[r] + off;
    if (with_acc && t < D) rec[2 + t] = a;
    if (t == 0) {
      rec[0] = m;
      rec[1] = l;
    }
  }
}

// Peer mode, once per CTA after its last record: every thread fences its
// peer stores at system scope before the CTA's count; the last CTA to count
// raises this call's epoch in every rank's flag array.
__device__ __forceinline__ void peers_count_out(const DecodeParams& P) {
  if (P.world == 0) return;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(P.counter, 1u) == gridDim.x - 1) {
      atomicExch(P.counter, 0u);  // ready for the next call
      __threadfence_system();
      for (int r = 0; r < P.world; ++r) st_release_sys(P.peer_flag[r] + P.rank, P.epoch);
    }
  }
}

// Called by one warp: lane r < world polls rank r's flag (relaxed) until it
// carries epoch, all flags at once; one acquire fence by lane 0 after the
// last one arrived orders the record reads that follow a CTA barrier.  Each
// wait gives up after about a second (2^31 cycles) and reports false; lane 0
// then sets the peer-timeout bit of the error word.
__device__ __forceinline__ bool wait_peer_flags(const uint32_t* flags, int world,
                                                uint32_t epoch, uint32_t* err, int lane) {
  bool good = true;
  if (lane < world) {
    const long long t0 = clock64();
    while (ld_relaxed_sys(flags + lane) != epoch) {
      if (clock64() - t0 > (1ll << 31)) {
        good = false;
        break;
      }
    }
  }
  const bool all = __all_sync(0xffffffffu, good);
  if (lane == 0) {
    if (!all) flag_error(err, kErrPeerTimeout);
    fence_acq_rel_sys();
  }
  __syncwarp();
  return all;
}

// One warp merges the world x n_parts records of query row g (records
// [world][n_rows][n_parts][D+2], in (rank, part) order) and writes
// out[g] = d (.) H(acc) / l, or zeros when !ok.  Element lane + 32 j; the
// transform runs stage by stage in the order of the other combine kernels.
template <int D>
__device__ __forceinline__ void combine_peer_row(const float* __restrict__ recs, int64_t n_rows,
                                                 int n_parts, int world, int64_t g,
                                                 const float* dvec, float* __restrict__ out,
                                                 int lane, bool ok) {
  constexpr int kJ = D / 32;
  float* o = out + g * D;
  if (!ok) {
#pragma unroll
    for (int j = 0; j < kJ; ++j) o[lane + 32 * j] = 0.f;
    return;
  }
  // records arrived over NVLink into this GPU's L2: read them there
  const int64_t rs = (int64_t)n_parts * (D + 2);  // one rank's records of a row
  const int64_t ws = n_rows * rs;                  // one rank's block
  const float* base = recs + g * rs;
  float M = -INFINITY;
  for (int r = 0; r < world; ++r)
    for (int p = 0; p < n_parts; ++p) {
      const float* rec = base + r * ws + (int64_t)p * (D + 2);
      if (__ldcg(rec + 1) > 0.f) M = fmaxf(M, __ldcg(rec));
    }
  float L = 0.f, acc[kJ];
#pragma unroll
  for (int j = 0; j < kJ; ++j) acc[j] = 0.f;
  for (int r = 0; r < world; ++r)
    for (int p = 0; p < n_parts; ++p) {
      const float* rec = base + r * ws + (int64_t)p * (D + 2);
      const float l = __ldcg(rec + 1);
      if (l > 0.f) {
        const float e = expf(__ldcg(rec) - M);
        L += l * e;
#pragma unroll
        for (int j = 0; j < kJ; ++j) acc[j] += __ldcg(rec + 2 + lane + 32 * j) * e;
      }
    }
#pragma unroll
  for (int h = 1; h < 32; h <<= 1)
#pragma unroll
    for (int j = 0; j < kJ; ++j) {
      const float x = __shfl_xor_sync(0xffffffffu, acc[j], h);
      acc[j] = (lane & h) ? (x - acc[j]) : (acc[j] + x);
    }
#pragma unroll
  for (int h = 1; h < kJ; h <<= 1)
#pragma unroll
    for (int j = 0; j < kJ; ++j)
      if ((j & h) == 0) {
        const float x = acc[j], y = acc[j + h];
        acc[j] = x + y;
        acc[j + h] = x - y;
      }
#pragma unroll
  for (int j = 0; j < kJ; ++j)
    o[lane + 32 * j] = L > 0.f ? acc[j] * dvec[lane + 32 * j] / L : 0.f;
}

// End of a partial kernel in peer mode: count out (the last CTA raises the
// flags); with the combine fused, every CTA then waits for all ranks' flags
// and its warps merge query rows blockIdx.x * warps + w, stepping by the
// grid's warps.  Every CTA of the launch must reach this point.
template <int D>
__device__ __forceinline__ void peers_finish(const DecodeParams& P) {
  if (P.world == 0) return;
  peers_count_out(P);
  if (!P.fuse) return;
  __shared__ int s_ok;
  const int t = threadIdx.x;
  if (t < 32) {
    const bool all = wait_peer_flags(P.peer_flag[P.rank], P.world, P.epoch, P.err, t);
    if (t == 0) s_ok = all ? 1 : 0;
  }
  __syncthreads();
  const bool ok = s_ok != 0;
  const int warps = blockDim.x / 32;
  for (int64_t g = (int64_t)blockIdx.x * warps + (t >> 5); g < P.n_rows_q;
       g += (int64_t)gridDim.x * warps)
    combine_peer_row<D>(P.peer_rec[P.rank], P.n_rows_q, P.n_splits, P.world, g, P.dv, P.out,
                        t & 31, ok);
}

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
// NC = 2: the bits=1 codebook (one bit per element); NC = 4: the bits=2
// codebook, 2-bit indices, element e at bits 2 (e & 15) of word e >> 4.
// This direct kernel is the datapath of the 4-level codebook.
template <int D, int NC>
__global__ void __launch_bounds__(D)
    decode_partial_kernel(const __grid_constant__ DecodeParams P) {
  constexpr int W = D / 32;                      // residual-plane words
  constexpr int WC = NC == 2 ? D / 32 : D / 16;  // code-plane words
  __shared__ float qt[D];
  __shared__ float w1[D], w2[D];
  __shared__ uint32_t vc[D][WC + 1], vr[D][W + 1];
  __shared__ float red[32];

  const int t = threadIdx.x;
  const int64_t g = blockIdx.y;      // query row (q, partial records)
  const int64_t gk = g / P.n_q;      // cache group it reads
  const int split = blockIdx.x;
  const int64_t len = P.seq_end - P.seq_begin;
  const int64_t s0 = P.seq_begin + len * split / P.n_splits;
  const int64_t s1 = P.seq_begin + len * (split + 1) / P.n_splits;
  const float inv_sqrt_d = 1.0f / sqrtf((float)D);
  const float qjl = 0.7978845608028654f / (float)D;  // sqrt(2/pi) / D
  const float cv0 = P.cb[0], cv1 = P.cb[1], cv2 = P.cb[2], cv3 = P.cb[3];
  auto cval = [=](uint32_t idx) -> float {  // c[idx] without dynamic indexing
    return idx < 2 ? (idx ? cv1 : cv0) : (idx == 2 ? cv2 : cv3);
  };

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
      const int64_t row = gk * P.seq_len + s;
      float m1 = 0.f, m2 = 0.f;
      if constexpr (NC == 2) {
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
        m1 = P.c0 * Q + (P.c1 - P.c0) * m1;  // <q~, c[idx]>
      } else {
#pragma unroll 1
        for (int w = 0; w < WC; ++w) {
          const uint32_t c = P.k_code[row * WC + w];
#pragma unroll
          for (int k = 0; k < 16; ++k) m1 += qt[16 * w + k] * cval((c >> (2 * k)) & 3u);
        }
#pragma unroll 1
        for (int w = 0; w < W; ++w) {
          const uint32_t r = P.k_res[row * W + w];
#pragma unroll
          for (int k = 0; k < 32; ++k) m2 += ((r >> k) & 1u) ? qt[32 * w + k] : 0.f;
        }
      }
      const float score = P.k_norms[row] * m1 + inv_sqrt_d * (2.f * m2 - Q) * P.k_rnorms[row];
      logit = score * P.sm_scale;
      va = P.v_norms[row] * inv_sqrt_d;
      vb = P.v_rnorms[row] * qjl;
#pragma unroll
      for (int w = 0; w < WC; ++w) vc[t][w] = P.v_code[row * WC + w];
#pragma unroll
      for (int w = 0; w < W; ++w) vr[t][w] = P.v_res[row * W + w];
    } else {
#pragma unroll
      for (int w = 0; w < WC; ++w) vc[t][w] = 0u;
#pragma unroll
      for (int w = 0; w < W; ++w) vr[t][w] = 0u;
    }
    const float m_blk = block_reduce<D>(logit, red, true);
    const float m_new = fmaxf(m_run, m_blk);
    const float alpha = expf(m_run - m_new);  // 0 on the first block
    const float p = valid ? expf(logit - m_new) : 0.f;
    const float l_blk = block_reduce<D>(p, red, false);
    // constant part: sum_s p (a c0 - b) (NC = 2), sum_s -p b (NC = 4)
    const float base = block_reduce<D>(p * ((NC == 2 ? va * P.c0 : 0.f) - vb), red, false);
    w1[t] = NC == 2 ? p * va * (P.c1 - P.c0) : p * va;
    w2[t] = 2.f * p * vb;
    __syncthreads();
    float a = acc * alpha + base;
    const int wi = t >> 5, bi = t & 31;
    const int nrow = (int)(s1 - blk < D ? s1 - blk : D);
    for (int j = 0; j < nrow; ++j) {
      if constexpr (NC == 2)
        a += ((vc[j][wi] >> bi) & 1u) ? w1[j] : 0.f;
      else
        a += cval((vc[j][t >> 4] >> (2 * (t & 15))) & 3u) * w1[j];
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

// Merges n_parts split-K records per query row; record p of row g is at
// parts + g * gs + p * ps (floats).  Records with l = 0 (empty splits) are
// skipped.  kRecord: writes the merged record (m, l, acc) at
// out + g * (D + 2), still in the rotated domain (the multi-GPU path gathers
// these); otherwise out[g] = d (.) H(acc) / l.
template <int D, bool kRecord>
__global__ void __launch_bounds__(D)
    decode_combine_kernel(const float* __restrict__ parts, int n_parts, int64_t gs,
                          int64_t ps, float* __restrict__ out,
                          const __grid_constant__ DecodeParams P) {
  grid_dependency_wait();  // the records come from the partial kernel
  __shared__ float sh[D];
  const int t = threadIdx.x;
  const int64_t g = blockIdx.x;
  const float* base = parts + g * gs;
  float M = -INFINITY;
  for (int r = 0; r < n_parts; ++r) {
    const float* rec = base + (int64_t)r * ps;
    if (rec[1] > 0.f) M = fmaxf(M, rec[0]);
  }
  float L = 0.f, a = 0.f;
  for (int r = 0; r < n_parts; ++r) {
    const float* rec = base + (int64_t)r * ps;
    if (rec[1] > 0.f) {
      const float e = expf(rec[0] - M);
      L += rec[1] * e;
      a += rec[2 + t] * e;
    }
  }
  if constexpr (kRecord) {
    float* rec = out + g * (D + 2);
    rec[2 + t] = a;
    if (t == 0) {
      rec[0] = M;
      rec[1] = L;
    }
    return;
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


// ---------------------------------------------------------------------------
// Sequence-sharded decode: the record exchange fused into the merge, over
// peer memory.  Every rank's merge kernel stores its merged record of each
// query row straight into slot [rank] of every rank's record buffer (plain
// stores to peer addresses over NVLink), fences, and the last CTA to finish
// raises this call's epoch in slot [rank] of every rank's flag array.  The
// combine kernel waits (bounded) until all world flags carry the epoch, then
// merges the world records of its row from local memory.
struct PeerParams {
  float* rec[kMaxPeers];     // rank r's record buffer [world][n_rows][D+2]
  uint32_t* flag[kMaxPeers]; // rank r's flag array [world]
};

template <int D>
__global__ void __launch_bounds__(D)
    decode_merge_to_peers_kernel(const float* __restrict__ parts, int n_parts, int64_t gs,
                                 int64_t ps, int64_t n_rows, int rank, int world,
                                 uint32_t epoch, uint32_t* counter,
                                 const __grid_constant__ PeerParams Q) {
  const int t = threadIdx.x;
  const int64_t g = blockIdx.x;
  const float* base = parts + g * gs;
  float M = -INFINITY;
  for (int r = 0; r < n_parts; ++r) {
    const float* rec = base + (int64_t)r * ps;
    if (rec[1] > 0.f) M = fmaxf(M, rec[0]);
  }
  float L = 0.f, a = 0.f;
  for (int r = 0; r < n_parts; ++r) {
    const float* rec = base + (int64_t)r * ps;
    if (rec[1] > 0.f) {
      const float e = expf(rec[0] - M);
      L += rec[1] * e;
      a += rec[2 + t] * e;
    }
  }
  const int64_t off = ((int64_t)rank * n_rows + g) * (D + 2);
  for (int p = 0; p < world; ++p) {
    float* dst = Q.rec[p] + off;
    dst[2 + t] = a;
    if (t == 0) {
      dst[0] = M;
      dst[1] = L;
    }
  }
  __threadfence_system();  // this thread's peer stores before the count below
  __syncthreads();
  if (t == 0) {
    const uint32_t done = atomicAdd(counter, 1u);
    if (done == (uint32_t)(n_rows - 1)) {  // the last CTA: every row is stored
      atomicExch(counter, 0u);             // ready for the next call
      __threadfence_system();
      for (int p = 0; p < world; ++p) st_release_sys(Q.flag[p] + rank, epoch);
    }
  }
}

// Combine step of the peer exchange: waits (bounded) until all world flags
// carry epoch, then merges the world x n_parts records of each query row
// (records [world][n_rows][n_parts][D+2], stored into this GPU's memory by
// the ranks' merge or partial kernels) and writes out[g] = d (.) H(acc) / l.
// One warp per row, eight rows per CTA; lane r of warp 0 polls rank r's flag.
// The records are merged in (rank, part) order and the transform runs stage
// by stage in the order of the other combine kernels.
template <int D>
__global__ void __launch_bounds__(256)
    decode_combine_peer_records_kernel(const float* __restrict__ recs, const uint32_t* flags,
                                       uint32_t epoch, int64_t n_rows, int n_parts, int world,
                                       float* __restrict__ out, uint32_t* err,
                                       const __grid_constant__ DecodeParams P) {
  __shared__ int ok;
  const int t = threadIdx.x;
  if (t < 32) {
    const bool all = wait_peer_flags(flags, world, epoch, err, t);
    if (t == 0) ok = all ? 1 : 0;
  }
  __syncthreads();
  const int64_t g = (int64_t)blockIdx.x * 8 + (t >> 5);
  if (g < n_rows) combine_peer_row<D>(recs, n_rows, n_parts, world, g, P.dk, out, t & 31, ok != 0);
}

// ---------------------------------------------------------------------------
// Decode v2: table-driven.  Both planes of a row are read as bytes.
//
// K side: per CTA (one query) a table holds, for every byte position p of a
// plane and byte value v, the partial sum  sum_{k<8, bit k of v} q~[8p+k];
// a row's masked sums M1, M2 are 2 * D/8 table lookups.
// V side: instead of touching D accumulators per row, each row adds its
// softmax weight into a histogram per byte position, H_p[byte] += w; after a
// chunk of rows the histograms are folded into the D accumulators
// (acc[8p+b] = sum over v with bit b set of H_p[v]).
// Tables and histograms use the bank-conflict-free slot rotation described
// in kh_bytetab.cuh (entry (slot j, value v) at float index 32 v + j).

template <int D>
struct V2Cfg {
  static constexpr int kP = D / 8;          // byte positions per plane
  static constexpr int kW = D / 32;         // words per plane
  static constexpr int kThreads = 256;      // thread = row in both passes
  static constexpr int kRPT = 8;            // rows per thread per chunk (registers)
  static constexpr int kChunk = kRPT * kThreads;
  static constexpr int kTab = 256 * 32;     // entries per K table / V histogram plane
  // lut | hist (int32 fixed point, 2 planes) | q~ | reduction scratch | folded sums [4][D]
  static constexpr int kSmem = (3 * kTab + D + 64 + 4 * D) * 4;
};


template <int D>
struct RowK {
  uint32_t c[D / 32], r[D / 32];
  float n, rn;
};

template <int D>
__global__ void __launch_bounds__(256)
    decode_v2_kernel(const __grid_constant__ DecodeParams P) {
  using C = V2Cfg<D>;
  constexpr int kP = C::kP;
  constexpr int kW = C::kW;
  constexpr int NT = C::kThreads;
  extern __shared__ float sm[];
  float* lut = sm;                                         // [256][32]
  int* hist = reinterpret_cast<int*>(sm + C::kTab);        // [2][256][32], fixed point
  float* qt = sm + 3 * C::kTab;                            // [D]
  float* red = qt + D;                                     // [64]
  int* fsum = reinterpret_cast<int*>(red + 64);            // [plane * copies][D]

  const int t = threadIdx.x;
  const int lane = t & 31;
  const int64_t g = blockIdx.y;      // query row (q, partial records)
  const int64_t gk = g / P.n_q;      // cache group it reads
  const int split = blockIdx.x;
  const int64_t len = P.seq_end - P.seq_begin;
  const int64_t s0 = P.seq_begin + len * split / P.n_splits;
  const int64_t s1 = P.seq_begin + len * (split + 1) / P.n_splits;
  const float inv_sqrt_d = 1.0f / sqrtf((float)D);
  const float qjl = 0.7978845608028654f / (float)D;  // sqrt(2/pi) / D
  const float dc = P.c1 - P.c0;

  // q~ = H(q (.) d) / sqrt(D)
  for (int i = t; i < D; i += NT) qt[i] = P.q[g * D + i] * P.dk[i];
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
  const float Q = block_sum<NT>(qpart, red);

  // K table (every copy) and zeroed histograms
  for (int e = t; e < kP * 256; e += NT) {
    const int pos = e % kP, v = e / kP;
    float sum = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += ((v >> k) & 1) ? qt[8 * pos + k] : 0.f;
#pragma unroll
    for (int c = 0; c < 32 / kP; ++c) lut[v * 32 + pos + kP * c] = sum;
  }
  for (int e = t; e < 2 * C::kTab; e += NT) hist[e] = 0;
  __syncthreads();

  // lane-constant addressing: slot(k) = ((k + lane) mod P) + P (lane / P)
  const int rr = lane % kP;
  const int wr = rr >> 2, bs = 8 * (rr & 3);
  const int copy_off = kP * (lane / kP);
  const char* lutb = reinterpret_cast<const char*>(lut);
  char* h1b = reinterpret_cast<char*>(hist);
  char* h2b = reinterpret_cast<char*>(hist + C::kTab);
  int slot4[kP];  // byte offset of slot(k) in a table / histogram row
  static_for<kP>([&](auto kc) {
    constexpr int k = decltype(kc)::value;
    slot4[k] = 4 * (((k + lane) % kP) + copy_off);
  });

  float m_run = -INFINITY, l_run = 0.f, c_run = 0.f;
  // accumulators of the elements this thread folds: element t (D <= NT)
  float acc = 0.f;

  constexpr int R = C::kRPT;
  for (int64_t c0 = s0; c0 < s1; c0 += C::kChunk) {
    const int n = (int)min((int64_t)C::kChunk, s1 - c0);
    const int64_t row0 = gk * P.seq_len + c0;
    // this thread's rows of the chunk: t + r * NT, r < R
    float lg[R];
    // ---------------- pass 1: scores -> logits (two rows in flight)
    float mloc = -INFINITY;
    static_for<R / 2>([&](auto rc) {
      constexpr int r0 = 2 * decltype(rc)::value;
      RowK<D> a[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int ii = t + (r0 + u) * NT;
        const int64_t row = row0 + (ii < n ? ii : 0);
        load_rotated<D>(P.k_code + row * kW, wr, bs, a[u].c);
        load_rotated<D>(P.k_res + row * kW, wr, bs, a[u].r);
        a[u].n = __ldg(P.k_norms + row);
        a[u].rn = __ldg(P.k_rnorms + row);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        float m1 = 0.f, m2 = 0.f;
        const RowK<D>& ar = a[u];
        static_for<kP>([&](auto kc) {
          constexpr int k = decltype(kc)::value;
          const uint32_t b1 = __byte_perm(ar.c[k >> 2], 0u, 0x4440u + (k & 3));
          const uint32_t b2 = __byte_perm(ar.r[k >> 2], 0u, 0x4440u + (k & 3));
          m1 += *reinterpret_cast<const float*>(lutb + b1 * 128 + slot4[k]);
          m2 += *reinterpret_cast<const float*>(lutb + b2 * 128 + slot4[k]);
        });
        const float score = ar.n * (P.c0 * Q + dc * m1) + inv_sqrt_d * (2.f * m2 - Q) * ar.rn;
        const bool ok = t + (r0 + u) * NT < n;
        lg[r0 + u] = ok ? score * P.sm_scale : -INFINITY;
        mloc = fmaxf(mloc, lg[r0 + u]);
      }
    });
    const float m_c = block_max<NT>(mloc, red);
    const float m_new = fmaxf(m_run, m_c);
    const float alpha = expf(m_run - m_new);  // rescales earlier chunks (0 on the first)
    m_run = m_new;

    // ---------------- pass 2a: softmax weights of this thread's rows
    float w1[R], w2[R];
    float lsum = 0.f, wmax = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int ii = t + r * NT;
      const bool ok = ii < n;
      const int64_t row = row0 + (ok ? ii : 0);
      const float p = ok ? expf(lg[r] - m_new) : 0.f;
      const float va = __ldg(P.v_norms + row) * inv_sqrt_d;
      const float vb = __ldg(P.v_rnorms + row) * qjl;
      lsum += p;
      w1[r] = p * va * dc;
      w2[r] = 2.f * p * vb;
      wmax = fmaxf(wmax, fmaxf(w1[r], w2[r]));
    }
    const float l_c = block_sum<NT>(lsum, red);
    const float w_max = block_max<NT>(wmax, red);
    // Fixed point: the bins of one (plane, copy) sum a subset of the chunk's
    // rows, so a bin stays below n * w_max * scale_inv <= 2^30.  The constant
    // term sum_s p (a c0 - b) = -sum_s (w1 + w2) / 2 (c0 = -c1) is built from
    // the same quantised weights, so a row rounded to zero drops out of every
    // output element alike instead of biasing their sum.
    const float scale_inv = w_max > 0.f ? 1073741824.0f / (w_max * (float)n) : 0.f;
    const float scale = w_max > 0.f ? (w_max * (float)n) / 1073741824.0f : 0.f;
    float csum = 0.f;  // constant term in units of the quantum

    // ---------------- pass 2b: scatter the V bytes into the histograms
    static_for<R / 2>([&](auto rc) {
      constexpr int r0 = 2 * decltype(rc)::value;
      RowK<D> a[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int ii = t + (r0 + u) * NT;
        const int64_t row = row0 + (ii < n ? ii : 0);
        load_rotated<D>(P.v_code + row * kW, wr, bs, a[u].c);
        load_rotated<D>(P.v_res + row * kW, wr, bs, a[u].r);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const RowK<D>& ar = a[u];
        const int f1 = __float2int_rn(w1[r0 + u] * scale_inv);  // 0 for rows past n
        const int f2 = __float2int_rn(w2[r0 + u] * scale_inv);
        csum += (float)f1 * (P.c0 / dc) - 0.5f * (float)f2;
        static_for<kP>([&](auto kc) {
          constexpr int k = decltype(kc)::value;
          const uint32_t b1 = __byte_perm(ar.c[k >> 2], 0u, 0x4440u + (k & 3));
          const uint32_t b2 = __byte_perm(ar.r[k >> 2], 0u, 0x4440u + (k & 3));
          atomicAdd(reinterpret_cast<int*>(h1b + b1 * 128 + slot4[k]), f1);
          atomicAdd(reinterpret_cast<int*>(h2b + b2 * 128 + slot4[k]), f2);
        });
      }
    });

    const float c_c = block_sum<NT>(csum, red) * scale;  // also fences the histograms
    // ---------------- fold: acc[8 pos + b] = sum over bins v with bit b set.
    // Thread t takes (plane, slot) = t / 4 and bins [64 q, 64 q + 64), q = t % 4:
    // each bin is read once; bits 0..5 of v are compile-time, bits 6..7 are q.
    {
      const int combo = t >> 2, q = t & 3;
      const int pl = combo >> 5, slot = combo & 31;
      const int* hb = hist + pl * C::kTab + slot;
      int sb[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int tot = 0;
      static_for<64>([&](auto jc) {
        constexpr int j = decltype(jc)::value;
        const int h = hb[(64 * q + j) * 32];
        tot += h;
        if (j & 1) sb[0] += h;
        if (j & 2) sb[1] += h;
        if (j & 4) sb[2] += h;
        if (j & 8) sb[3] += h;
        if (j & 16) sb[4] += h;
        if (j & 32) sb[5] += h;
      });
      sb[6] = (q & 1) ? tot : 0;
      sb[7] = (q & 2) ? tot : 0;
#pragma unroll
      for (int bb = 0; bb < 8; ++bb) {
        sb[bb] += __shfl_xor_sync(0xffffffffu, sb[bb], 1);
        sb[bb] += __shfl_xor_sync(0xffffffffu, sb[bb], 2);
      }
      if (q == 0) {
        // slot = pos + P * copy; element 8 pos + b of plane pl, copy class pl * copies + copy
        const int pos = slot % kP, cp = slot / kP;
#pragma unroll
        for (int bb = 0; bb < 8; ++bb) fsum[(pl * (32 / kP) + cp) * D + 8 * pos + bb] = sb[bb];
      }
    }
    __syncthreads();
    if (t < D) {
      float a = 0.f;
#pragma unroll
      for (int k = 0; k < 2 * (32 / kP); ++k) a += (float)fsum[k * D + t];
      acc = acc * alpha + a * scale;
    }
    l_run = l_run * alpha + l_c;
    c_run = c_run * alpha + c_c;
    __syncthreads();
    for (int e = t; e < 2 * C::kTab; e += NT) hist[e] = 0;
    __syncthreads();
  }

  float* rec = P.partials + (g * P.part_stride + P.part_offset + split) * (D + 2);
  if (t < D) rec[2 + t] = c_run + acc;
  if (t == 0) {
    rec[0] = m_run;
    rec[1] = l_run;
  }
}

// ---------------------------------------------------------------------------
// Decode v3: segment-exact softmax, one-instruction table addressing.
//
// A split's rows are processed in segments of up to kSeg rows:
//   phase 1  K scores through the byte table -> logits (log2 units) kept in
//            shared memory for the whole segment; per-thread online sums of
//            p and of the V weights (for the fixed-point range); block max
//            and block sums;
//   phase 2b V bytes scattered into int32 histograms with the segment's
//            fixed-point scale 2^30 / sum(weights) (any bin <= 2^30 + n/2);
//   fold     histograms -> D accumulators, rescaled online across segments.
// Table and histograms share one array of 256 rows (one per byte value) of
// 64 32-bit entries; row v starts at byte 256 v, so one byte-permute of
// (plane word, lane slot offset) yields the byte address 256 v + 4 slot.
// Slots follow the XOR byte order of kh_bytetab.cuh (lane l visits byte
// k ^ (l mod D/8) at step k; 32 distinct banks per warp instruction).
//   D = 128 (half-row layout): the K table (two copies of 16 positions) and
//     the two V histograms (one copy each: code plane slots 0..15, residual
//     plane 16..31) use entries 0..31; half the lanes scatter the residual
//     plane first, so each atomic instruction of a warp still covers 32
//     banks.  Entries 32..63 hold the segment's 8192 logits during phases 1
//     and 2, then the fold partials.  65 KB of shared memory per CTA leaves
//     two CTAs per SM with the L1 room their in-flight row loads need (the
//     same kernel with 109 KB of shared memory ran 20 % slower).
//   D = 256: the K table uses entries 0..31, the V histograms 0..31 (code
//     plane) and 32..63 (residual plane, the same address + 128).
// The K table is rebuilt from q~ for every segment, since phase 2 overwrites
// it.  Each thread keeps kRing batches of rows in a register ring: the
// plane words of the next kRing - 1 batches load while one batch is scored
// or scattered.  (Bulk L2 prefetches of the rows a few batches ahead were
// measured slower.)
// Build-time tuning knobs of decode v3 (defaults are the measured best).
#ifndef KH_DECODE_SEG
#define KH_DECODE_SEG 4096
#endif
#ifndef KH_DECODE_BATCH128
#define KH_DECODE_BATCH128 2
#endif

template <int D>
struct V3Cfg {
  static constexpr int kP = D / 8;
  static constexpr int kCopies = 32 / kP;  // K-table copies (bank-conflict-free slots)
  static_assert(kCopies * kP == 32, "32 slots per table row");
  static constexpr int kThreads = 256;
  // D = 128: the K table and both V histograms fit in words 0..31 of every
  // 64-word table row (half-row layout); words 32..63 of the 256 rows hold
  // the segment's logits (8192) in phase 1 and the fold partials after
  // phase 2.  D = 256 needs all 64 words for its two V histograms.
  static constexpr bool kHalf = D == 128;
  static constexpr int kSeg = kHalf ? 8192 : KH_DECODE_SEG;
  static constexpr int kBatch = D == 128 ? KH_DECODE_BATCH128 : 1;  // rows per thread per batch
  // batches in the register ring: kRing - 1 batches are loading while one
  // is scored or scattered
  static constexpr int kRing = D == 128 ? 3 : 2;
  // tab [256][64] | (D = 256: logits [kSeg] | fold partials [2][4][32][8]) |
  // q~ [D] | reduction scratch [64]
  static constexpr int kTabWords = 256 * 64;
  static constexpr int kSmem = (kTabWords + (kHalf ? 0 : kSeg + 2048) + D + 64) * 4;
};


template <int D>
struct RowKV {
  uint32_t c[D / 32], r[D / 32];
  float n, rn, vn, vrn;
};


// One segment's rows of the six arrays phase 1 reads, as bases at the
// segment's first row: a row is then addressed by a 32-bit index (one
// multiply-add per load instead of 64-bit index arithmetic).
template <int D>
struct SegK {
  const uint32_t *code, *res;
  const float *n, *rn, *vn, *vrn;
  __device__ __forceinline__ SegK(const DecodeParams& P, int64_t row0)
      : code(P.k_code + row0 * (D / 32)), res(P.k_res + row0 * (D / 32)),
        n(P.k_norms + row0), rn(P.k_rnorms + row0), vn(P.v_norms + row0),
        vrn(P.v_rnorms + row0) {}
};

// Phase-1 loads: K planes and norms are read once (evict-first); the V
// norms are read again by phase 2 of the same segment (evict-last).
template <int D>
__device__ __forceinline__ void load_k_row(const SegK<D>& S, uint32_t i, int wr,
                                           uint64_t once, uint64_t again, RowKV<D>& a) {
  constexpr uint32_t kW = D / 32;
  load_plane_x<D>(S.code + i * kW, wr, once, a.c);
  load_plane_x<D>(S.res + i * kW, wr, once, a.r);
  a.n = ldg_policy(S.n + i, once);
  a.rn = ldg_policy(S.rn + i, once);
  a.vn = ldg_policy(S.vn + i, again);
  a.vrn = ldg_policy(S.vrn + i, again);
}

template <int NT>
__device__ __forceinline__ float2 block_sum2(float2 v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
    v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    red[2 * (threadIdx.x >> 5)] = v.x;
    red[2 * (threadIdx.x >> 5) + 1] = v.y;
  }
  __syncthreads();
  float2 r = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) {
    r.x += red[2 * i];
    r.y += red[2 * i + 1];
  }
  return r;
}

template <int D>
__global__ void __launch_bounds__(256, 2)
    decode_v3_kernel(const __grid_constant__ DecodeParams P) {
  grid_dependency_wait();  // q and the cache may come from the previous kernel
  using C = V3Cfg<D>;
  constexpr int kP = C::kP;
  constexpr int NT = C::kThreads;
  constexpr int B = C::kBatch;
  constexpr float kLog2e = 1.4426950408889634f;
  constexpr float kLn2 = 0.6931471805599453f;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* tabb = smem_raw;                                    // [256][64] words
  float* lg = reinterpret_cast<float*>(smem_raw) + C::kTabWords;    // [kSeg] (D = 256)
  int* part = reinterpret_cast<int*>(lg + (C::kHalf ? 0 : C::kSeg));  // [2048] (D = 256)
  float* qt = reinterpret_cast<float*>(part + (C::kHalf ? 0 : 2048));  // [D]
  // element e of the logits / fold partials: half-row layout puts it in word
  // 32 + (e mod 32) of table row e / 32 (a warp's 32 consecutive elements
  // fill one half row: conflict-free)
  auto upper = [&](int e) -> int* {
    if constexpr (C::kHalf)
      return reinterpret_cast<int*>(tabb + 256 * (e >> 5) + 128 + 4 * (e & 31));
    else
      return part + e;
  };
  float* red = qt + D;                                               // [64]

  const int t = threadIdx.x;
  const int lane = t & 31;
  const float inv_sqrt_d = 1.0f / sqrtf((float)D);
  const float qjl = 0.7978845608028654f / (float)D;  // sqrt(2/pi) / D
  const float dc = P.c1 - P.c0;
  const float lscale = P.sm_scale * kLog2e;
  const float c0dc = P.c0 / dc;
  const float wa = inv_sqrt_d * dc, wb = 2.f * qjl;  // V weight = p (wa |v| + wb r_norm)

  // lane constants: at step k this lane reads plane byte k ^ rr (XOR order),
  // looked up in slot (k ^ rr) + kP (lane / kP)
  const int rr = lane % kP;
  const int wr = rr >> 2;
  const XorSel xs = xor_selectors(rr);
  uint32_t slot4[kP / 4];  // byte (k & 3) of slot4[k >> 2] = 4 * slot(k)
  static_for<kP / 4>([&](auto mc) {
    constexpr int m = decltype(mc)::value;
    slot4[m] = xor_slots<kP>(m, rr, lane / kP);
  });

  // phase-2 plane order.  Half-row layout: the code-plane histogram is slots
  // pos, the residual one slots 16 + pos (one copy each); lanes 0..15
  // scatter the code plane with the first atomic of each byte step and lanes
  // 16..31 the residual plane, then the other way round, so every atomic
  // instruction of a warp touches 32 distinct banks.  D = 256: all lanes
  // code plane first (slots 0..31), residual plane second (slots 32..63).
  const bool swap = C::kHalf && lane >= 16;
  const uint32_t* vx = swap ? P.v_res : P.v_code;
  const uint32_t* vy = swap ? P.v_code : P.v_res;
  const float* vxn = swap ? P.v_rnorms : P.v_norms;
  const float* vyn = swap ? P.v_norms : P.v_rnorms;
  uint32_t slot4y[kP / 4];  // slots of the second atomic (half-row layout)
  static_for<kP / 4>([&](auto mc) {
    constexpr int m = decltype(mc)::value;
    slot4y[m] = slot4[m] ^ 0x40404040u;  // 4 * (slot +- 16) in every byte
  });

  // Work split.  The (cache group, sequence row) pairs of the call are laid
  // out group after group, L rows each, and cut into ranges of W pairs, one
  // per CTA set (n_q CTAs: one per query of the group, running side by side
  // so the group's rows are read from L2 after the first).  A CTA takes the
  // pieces of its range one group at a time; a group's pieces are its
  // records, numbered from the first set that covers it, and the set that
  // ends the group marks its unused record slots empty (l = 0).  Every CTA
  // gets the same number of rows whatever the group count, so no wave of
  // CTAs runs part-full.
  const int64_t L = P.seq_end - P.seq_begin;
  if (P.W == 0) {  // empty range: every record of query row blockIdx.x is empty
    if (t == 0)
      for (int p = 0; p < P.n_splits; ++p)
        put_record<D>(P, blockIdx.x, p, 0, -INFINITY, 0.f, 0.f, false);
    peers_finish<D>(P);
    return;
  }
  const int jq = (int)(blockIdx.x % (unsigned)P.n_q);
  const int64_t set = blockIdx.x / (unsigned)P.n_q;
  const int64_t wbeg = set * P.W;
  const int64_t wend = min(wbeg + P.W, P.n_groups_kv * L);
  for (int64_t gk = wbeg / L; gk * L < wend; ++gk) {
  const int64_t g = gk * P.n_q + jq;  // query row (q, partial records)
  const int64_t s0 = P.seq_begin + max(wbeg - gk * L, (int64_t)0);
  const int64_t s1 = P.seq_begin + min(wend - gk * L, L);
  const int64_t rpart = set - gk * L / P.W;  // this piece's record slot

  // q~ = H(q (.) d) / sqrt(D)
  for (int i = t; i < D; i += NT) qt[i] = P.q[g * D + i] * P.dk[i];
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

  float m_run = -INFINITY, l_run = 0.f, c_run = 0.f, acc = 0.f;
  const uint64_t pol_once = l2_policy_evict_first(), pol_again = l2_policy_evict_last();

  for (int64_t c0 = s0; c0 < s1; c0 += C::kSeg) {
    const int n = (int)min((int64_t)C::kSeg, s1 - c0);
    const int64_t row0 = gk * P.seq_len + c0;
    const int nb = (n + NT * B - 1) / (NT * B);  // batches of B rows per thread
    const uint32_t last = (uint32_t)n - 1;        // loads past the segment read this row
    // half-row layout: this thread's logit of batch row k (= bi B + u) sits
    // k (NT / 32) table rows below its first one
    float* const lgt = reinterpret_cast<float*>(upper(t));

    // K table into entries 0..31 of every row
    build_byte_table<D>(reinterpret_cast<float*>(tabb), qt, t);
    __syncthreads();

    // ---------------- phase 1: logits (log2 units) of the segment, online
    // per-thread sums of p and of the V weights relative to the running max mt
    float mt = -INFINITY;
    float2 sums = make_float2(0.f, 0.f);
    {
      RowKV<D> a[C::kRing][B];
      const SegK<D> seg(P, row0);
      auto load_batch = [&](RowKV<D>(&dst)[B], int bi) {
#pragma unroll
        for (int u = 0; u < B; ++u) {
          const uint32_t ii = min((uint32_t)(t + (bi * B + u) * NT), last);
          load_k_row<D>(seg, ii, wr, pol_once, pol_again, dst[u]);
        }
      };
      auto score_batch = [&](const RowKV<D>(&src)[B], int bi) {
        float l2[B];
        float mb = mt;
#pragma unroll
        for (int u = 0; u < B; ++u) {
          float2 m = make_float2(0.f, 0.f);
          uint32_t rc[D / 32], rs[D / 32];
          xor_plane<D>(src[u].c, wr, rc);
          xor_plane<D>(src[u].r, wr, rs);
          static_for<kP>([&](auto kc) {
            constexpr int k = decltype(kc)::value;
            const float x1 = *reinterpret_cast<const float*>(
                tabb + tab_addr_x(rc[k >> 2], slot4[k >> 2], xs.s[k & 3]));
            const float x2 = *reinterpret_cast<const float*>(
                tabb + tab_addr_x(rs[k >> 2], slot4[k >> 2], xs.s[k & 3]));
            m = __fadd2_rn(m, make_float2(x1, x2));
          });
          const float score = src[u].n * (P.c0 * Q + dc * m.x) +
                              inv_sqrt_d * (2.f * m.y - Q) * src[u].rn;
          const int ii = t + (bi * B + u) * NT;
          l2[u] = ii < n ? score * lscale : -INFINITY;
          // every ii < nb B NT <= kSeg has a slot: rows past n store -inf,
          // which phase 2 turns into a zero weight
          if constexpr (C::kHalf)
            lgt[(bi * B + u) * (NT / 32) * 64] = l2[u];
          else
            lg[ii] = l2[u];
          mb = fmaxf(mb, l2[u]);
        }
        if (mb > -INFINITY) {
          const float sc = ex2_approx(mt - mb);  // 0 while mt is -inf
          sums.x *= sc;
          sums.y *= sc;
#pragma unroll
          for (int u = 0; u < B; ++u) {
            const float p = ex2_approx(l2[u] - mb);  // 0 for rows past n
            sums.x += p;
            sums.y += p * (src[u].vn * wa + src[u].vrn * wb);
          }
          mt = mb;
        }
      };
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
    // phase 2's first V rows, loaded now so that their latency overlaps the
    // block reductions below
    RowK<D> va[C::kRing][B];
    const uint32_t* const vxs = vx + row0 * (D / 32);
    const uint32_t* const vys = vy + row0 * (D / 32);
    const float* const vxns = vxn + row0;
    const float* const vyns = vyn + row0;
    auto load_vbatch = [&](RowK<D>(&dst)[B], int bi) {
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const uint32_t ii = min((uint32_t)(t + (bi * B + u) * NT), last);
        load_plane_x<D>(vxs + ii * (uint32_t)(D / 32), wr, pol_once, dst[u].c);
        load_plane_x<D>(vys + ii * (uint32_t)(D / 32), wr, pol_once, dst[u].r);
        dst[u].n = ldg_policy(vxns + ii, pol_once);
        dst[u].rn = ldg_policy(vyns + ii, pol_once);
      }
    };
    static_for<C::kRing - 1>([&](auto jc) { load_vbatch(va[decltype(jc)::value], decltype(jc)::value); });
    const float m_seg = block_max<NT>(mt, red);  // also: phase-1 table reads done
    const float m_new = fmaxf(m_run, m_seg);
    const float alpha = ex2_approx(m_run - m_new);  // 0 on the first segment
    m_run = m_new;

    // zero both histograms (D = 128: words 0..31 of every row, keeping the
    // logits; D = 256: all 64 words)
    {
      int4* z = reinterpret_cast<int4*>(tabb);
      if constexpr (C::kHalf) {
        for (int e = t; e < C::kTabWords / 8; e += NT) z[(e >> 3) * 16 + (e & 7)] = make_int4(0, 0, 0, 0);
      } else {
        for (int e = t; e < C::kTabWords / 4; e += NT) z[e] = make_int4(0, 0, 0, 0);
      }
    }
    {
      const float r = mt > -INFINITY ? ex2_approx(mt - m_new) : 0.f;
      sums.x *= r;
      sums.y *= r;
    }
    const float2 tot = block_sum2<NT>(sums, red);  // barriers also order the zeroing
    const float l_c = tot.x;
    const float scale_inv = tot.y > 0.f ? 1073741824.0f / tot.y : 0.f;
    const float scale = tot.y / 1073741824.0f;

    // ---------------- phase 2b: scatter V bytes with fixed-point weights
    float csum = 0.f;  // constant term in quanta
    const float k1 = wa * scale_inv, k2 = wb * scale_inv;
    const float kx = swap ? k2 : k1, ky = swap ? k1 : k2;           // (x, y) = this lane's
    const float cx = swap ? -0.5f : c0dc, cy = swap ? c0dc : -0.5f;  // plane order
    {
      auto scatter_batch = [&](const RowK<D>(&src)[B], int bi) {
#pragma unroll
        for (int u = 0; u < B; ++u) {
          float l2;  // -inf past n: weight 0
          if constexpr (C::kHalf)
            l2 = lgt[(bi * B + u) * (NT / 32) * 64];
          else
            l2 = lg[t + (bi * B + u) * NT];
          const float p = ex2_approx(l2 - m_new);
          const int fx = __float2int_rn(p * src[u].n * kx);
          const int fy = __float2int_rn(p * src[u].rn * ky);
          csum += (float)fx * cx + (float)fy * cy;
          uint32_t rx[D / 32], ry[D / 32];
          xor_plane<D>(src[u].c, wr, rx);
          xor_plane<D>(src[u].r, wr, ry);
          static_for<kP>([&](auto kc) {
            constexpr int k = decltype(kc)::value;
            atomicAdd(reinterpret_cast<int*>(
                          tabb + tab_addr_x(rx[k >> 2], slot4[k >> 2], xs.s[k & 3])),
                      fx);
            if constexpr (C::kHalf)
              atomicAdd(reinterpret_cast<int*>(
                            tabb + tab_addr_x(ry[k >> 2], slot4y[k >> 2], xs.s[k & 3])),
                        fy);
            else
              atomicAdd(reinterpret_cast<int*>(
                            tabb + 128 + tab_addr_x(ry[k >> 2], slot4[k >> 2], xs.s[k & 3])),
                        fy);
          });
        }
      };
      for (int bi = 0; bi < nb; bi += C::kRing) {
        static_for<C::kRing>([&](auto jc) {
          constexpr int j = decltype(jc)::value;
          if (bi + j < nb) {
            load_vbatch(va[(j + C::kRing - 1) % C::kRing], bi + j + C::kRing - 1);
            scatter_batch(va[j], bi + j);
          }
        });
      }
    }
    const float c_c = block_sum<NT>(csum, red) * scale;  // also fences the histograms

    // ---------------- fold.  Half-row layout: thread (group of 32 byte
    // values, slot) sums its 32 bins per bit of the byte value; bits 5..7 of
    // v are the group's bits.
    if constexpr (C::kHalf) {
      const int slot = t & 31, grp = t >> 5;
      const int* hb = reinterpret_cast<const int*>(tabb) + slot;
      int sb[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int tt = 0;
      static_for<32>([&](auto jc) {
        constexpr int j = decltype(jc)::value;
        const int h = hb[(32 * grp + j) * 64];
        tt += h;
        if (j & 1) sb[0] += h;
        if (j & 2) sb[1] += h;
        if (j & 4) sb[2] += h;
        if (j & 8) sb[3] += h;
        if (j & 16) sb[4] += h;
      });
      sb[5] = (grp & 1) ? tt : 0;
      sb[6] = (grp & 2) ? tt : 0;
      sb[7] = (grp & 4) ? tt : 0;
      int4* pp = reinterpret_cast<int4*>(upper((grp * 32 + slot) * 8));
      pp[0] = make_int4(sb[0], sb[1], sb[2], sb[3]);
      pp[1] = make_int4(sb[4], sb[5], sb[6], sb[7]);
    } else {
      // D = 256: thread (plane, quarter, slot) sums its 64 bins; bits 6, 7
      // of v are the quarter's bits
      const int slot = t & 31, pl = (t >> 5) & 1, q = t >> 6;
      const int* hb = reinterpret_cast<const int*>(tabb) + 32 * pl + slot;
      int sb[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      int tt = 0;
      static_for<64>([&](auto jc) {
        constexpr int j = decltype(jc)::value;
        const int h = hb[(64 * q + j) * 64];
        tt += h;
        if (j & 1) sb[0] += h;
        if (j & 2) sb[1] += h;
        if (j & 4) sb[2] += h;
        if (j & 8) sb[3] += h;
        if (j & 16) sb[4] += h;
        if (j & 32) sb[5] += h;
      });
      sb[6] = (q & 1) ? tt : 0;
      sb[7] = (q & 2) ? tt : 0;
      int4* pp = reinterpret_cast<int4*>(part + ((pl * 4 + q) * 32 + slot) * 8);
      pp[0] = make_int4(sb[0], sb[1], sb[2], sb[3]);
      pp[1] = make_int4(sb[4], sb[5], sb[6], sb[7]);
    }
    __syncthreads();
    if (t < D) {
      const int pos = t >> 3, bb = t & 7;
      float a = 0.f;
      if constexpr (C::kHalf) {
        int sc = 0, sr = 0;  // one plane each: a subset sum of one histogram, < 2^31
#pragma unroll
        for (int grp = 0; grp < 8; ++grp) {
          sc += *upper((grp * 32 + pos) * 8 + bb);
          sr += *upper((grp * 32 + 16 + pos) * 8 + bb);
        }
        a = (float)sc + (float)sr;
      } else {
#pragma unroll
        for (int pl = 0; pl < 2; ++pl) {
          int s = 0;  // one plane: a subset sum of one histogram, < 2^31
#pragma unroll
          for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int cp = 0; cp < C::kCopies; ++cp)
              s += part[((pl * 4 + q) * 32 + pos + kP * cp) * 8 + bb];
          a += (float)s;
        }
      }
      acc = acc * alpha + a * scale;
    }
    l_run = l_run * alpha + l_c;
    c_run = c_run * alpha + c_c;
    __syncthreads();  // fold reads done before the next segment's table
  }

  if (rpart < P.n_splits)  // the host sizes W so that it always is
    // m in natural-log units for the combine step
    put_record<D>(P, g, rpart, t, m_run * kLn2, l_run, c_run + acc, true);
  if (s1 == P.seq_end && t == 0)  // this set ends the group: empty the unused slots
    for (int64_t p = rpart + 1; p < P.n_splits; ++p)
      put_record<D>(P, g, p, 0, -INFINITY, 0.f, 0.f, false);
  __syncthreads();  // q~ and the reduction scratch are rewritten by the next piece
  }
  peers_finish<D>(P);
}

// ---------------------------------------------------------------------------
// Decode for the 4-level (bits=2) codebook at D = 128: the v3 scheme (same
// work ranges, segments, logits, fixed-point V histograms) with a 2-bit code
// plane of 32 bytes per row (4 elements per byte, element 4p + k at bits 2k
// of byte p).
//   K table  entries 0..31 of each 64-word row: T2[v][p] =
//            sum_{k<4} q~[4p + k] c[(v >> 2k) & 3] (one copy; lane l looks up
//            position k ^ l at step k); entries 32..63: the 1-bit
//            residual table (16 positions, two copies).
//   score    norm * sum_p T2 + r_norm / sqrt(D) (2 M_res - Q).
//   V        the code plane's histogram H2[v][p] takes w = p_s |v_s| / sqrt(D)
//            per row (entries 0..31), the residual plane's as in v3
//            (entries 32..63, two copies); the fold gives, per element,
//            the four sums S_val = sum over byte values whose field is val,
//            and acc_e = sum_val c[val] S_val + the residual plane's share.
// Logits live in their own array; after phase 2 it holds the fold partials.
struct B2Cfg {
  static constexpr int kD = 128;
  static constexpr int kPC = 32, kWC = 8;  // code plane: byte positions, words
  static constexpr int kPR = 16, kWR = 4;  // residual plane
  static constexpr int kThreads = 256;
  static constexpr int kSeg = 6144;        // rows per segment (24 KB of logits)
  static constexpr int kRing = 3;          // batches (one row each) in the register ring
  static constexpr int kTabWords = 256 * 64;
  static constexpr int kFoldCode = 8 * 32 * 16;  // [bin group][position][field][value]
  static constexpr int kFoldRes = 8 * 32 * 8;    // [bin group][slot][bit]
  static_assert(kFoldCode + kFoldRes <= kSeg, "fold partials overlay the logits");
  // tab [256][64] | logits / fold [kSeg] | q~ [128] | reduction scratch [64]
  static constexpr int kSmem = (kTabWords + kSeg + kD + 64) * 4;
};

struct RowB2 {
  uint32_t c[B2Cfg::kWC], r[B2Cfg::kWR];
  float n, rn;
};

__global__ void __launch_bounds__(256, 2)
    decode_b2_kernel(const __grid_constant__ DecodeParams P) {
  grid_dependency_wait();  // q and the cache may come from the previous kernel
  using C = B2Cfg;
  constexpr int D = C::kD;
  constexpr int NT = C::kThreads;
  constexpr float kLog2e = 1.4426950408889634f;
  constexpr float kLn2 = 0.6931471805599453f;
  extern __shared__ __align__(16) unsigned char smem_b2[];
  unsigned char* tabb = smem_b2;
  float* tab = reinterpret_cast<float*>(smem_b2);
  float* lg = tab + C::kTabWords;                       // [kSeg] logits, then fold partials
  int* cf = reinterpret_cast<int*>(lg);                 // [8][32][16]
  int* rf = cf + C::kFoldCode;                          // [8][32][8]
  float* qt = lg + C::kSeg;                             // [D]
  float* red = qt + D;                                  // [64]

  const int t = threadIdx.x;
  const int lane = t & 31;
  const float inv_sqrt_d = 1.0f / sqrtf((float)D);
  const float qjl = 0.7978845608028654f / (float)D;  // sqrt(2/pi) / D
  const float lscale = P.sm_scale * kLog2e;
  const float wb = 2.f * qjl;  // V weight = p (|v| / sqrt(D) + wb r_norm)
  const float cv0 = P.cb[0], cv1 = P.cb[1], cv2 = P.cb[2], cv3 = P.cb[3];

  // lane constants (XOR byte order): at step k the code plane's byte k ^ lane
  // (of 32), slot k ^ lane; the residual plane's byte k ^ (lane mod 16), slot
  // 32 + (k ^ (lane mod 16)) + 16 (lane / 16).  Both share the selectors
  // (they depend on lane mod 4 only).
  const int wrc = lane >> 2;
  const XorSel xs = xor_selectors(lane);
  uint32_t slotc[C::kPC / 4];
  static_for<C::kPC / 4>([&](auto mc) {
    constexpr int m = decltype(mc)::value;
    slotc[m] = xor_slots<C::kPC>(m, lane, 0);
  });
  const int rr = lane % C::kPR;
  const int wrr = rr >> 2;
  uint32_t slotr[C::kPR / 4];
  static_for<C::kPR / 4>([&](auto mc) {
    constexpr int m = decltype(mc)::value;
    slotr[m] = xor_slots<C::kPR>(m, rr, lane / C::kPR);
  });
  const unsigned char* tabr = tabb + 128;  // entries 32..63 of each table row

  // work split: as decode_v3_kernel
  const int64_t L = P.seq_end - P.seq_begin;
  if (P.W == 0) {
    if (t == 0)
      for (int p = 0; p < P.n_splits; ++p)
        put_record<D>(P, blockIdx.x, p, 0, -INFINITY, 0.f, 0.f, false);
    peers_finish<D>(P);
    return;
  }
  const int jq = (int)(blockIdx.x % (unsigned)P.n_q);
  const int64_t set = blockIdx.x / (unsigned)P.n_q;
  const int64_t wbeg = set * P.W;
  const int64_t wend = min(wbeg + P.W, P.n_groups_kv * L);
  const uint64_t pol_once = l2_policy_evict_first(), pol_again = l2_policy_evict_last();
  for (int64_t gk = wbeg / L; gk * L < wend; ++gk) {
    const int64_t g = gk * P.n_q + jq;
    const int64_t s0 = P.seq_begin + max(wbeg - gk * L, (int64_t)0);
    const int64_t s1 = P.seq_begin + min(wend - gk * L, L);
    const int64_t rpart = set - gk * L / P.W;

    for (int i = t; i < D; i += NT) qt[i] = P.q[g * D + i] * P.dk[i];
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

    float m_run = -INFINITY, l_run = 0.f, c_run = 0.f, acc = 0.f;
    for (int64_t c0 = s0; c0 < s1; c0 += C::kSeg) {
      const int n = (int)min((int64_t)C::kSeg, s1 - c0);
      const int64_t row0 = gk * P.seq_len + c0;
      const int nb = (n + NT - 1) / NT;  // batches of one row per thread

      // K tables: T2 (thread (position t mod 32, group t / 32) fills the byte
      // values t / 32 + 8 kk), then the residual table in entries 32..63
      {
        const int p = t & 31, w = t >> 5;
        const float q0 = qt[4 * p], q1 = qt[4 * p + 1], q2 = qt[4 * p + 2], q3 = qt[4 * p + 3];
        auto cvv = [&](int i) {  // c[i] without a local array
          return i < 2 ? (i ? cv1 : cv0) : (i == 2 ? cv2 : cv3);
        };
        float lo[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int v = w + 8 * h;
          lo[h] = q0 * cvv(v & 3) + q1 * cvv((v >> 2) & 3);
        }
        static_for<32>([&](auto kc) {
          constexpr int kk = decltype(kc)::value, hv = kk >> 1;
          const float hi = q2 * cvv(hv & 3) + q3 * cvv((hv >> 2) & 3);
          tab[(w + 8 * kk) * 64 + p] = lo[kk & 1] + hi;
        });
      }
      build_byte_table<D>(tab + 32, qt, t);
      __syncthreads();

      // ---------------- phase 1: logits and online sums of p and V weights
      float mt = -INFINITY;
      float2 sums = make_float2(0.f, 0.f);
      {
        struct RowK2 {
          RowB2 k;
          float vn, vrn;
        };
        RowK2 a[C::kRing];
        auto load = [&](RowK2& dst, int bi) {
          const int ii = t + bi * NT;
          const int64_t row = row0 + (ii < n ? ii : 0);
          load_plane32_x(P.k_code + row * C::kWC, wrc, pol_once, dst.k.c);  // 32-byte plane
          load_plane_x<128>(P.k_res + row * C::kWR, wrr, pol_once, dst.k.r);
          dst.k.n = ldg_policy(P.k_norms + row, pol_once);
          dst.k.rn = ldg_policy(P.k_rnorms + row, pol_once);
          dst.vn = ldg_policy(P.v_norms + row, pol_again);
          dst.vrn = ldg_policy(P.v_rnorms + row, pol_again);
        };
        auto score = [&](const RowK2& src, int bi) {
          uint32_t rc[C::kWC], rs[C::kWR];
          xor_plane32(src.k.c, wrc, rc);
          xor_plane<128>(src.k.r, wrr, rs);
          // (x = even steps, y = odd steps)
          float2 mc = make_float2(0.f, 0.f), mr = make_float2(0.f, 0.f);
          static_for<C::kPC / 2>([&](auto jc) {
            constexpr int k = 2 * decltype(jc)::value;
            const float x0 = *reinterpret_cast<const float*>(
                tabb + tab_addr_x(rc[k >> 2], slotc[k >> 2], xs.s[k & 3]));
            const float x1 = *reinterpret_cast<const float*>(
                tabb + tab_addr_x(rc[k >> 2], slotc[k >> 2], xs.s[(k + 1) & 3]));
            mc = __fadd2_rn(mc, make_float2(x0, x1));
          });
          static_for<C::kPR / 2>([&](auto jc) {
            constexpr int k = 2 * decltype(jc)::value;
            const float x0 = *reinterpret_cast<const float*>(
                tabr + tab_addr_x(rs[k >> 2], slotr[k >> 2], xs.s[k & 3]));
            const float x1 = *reinterpret_cast<const float*>(
                tabr + tab_addr_x(rs[k >> 2], slotr[k >> 2], xs.s[(k + 1) & 3]));
            mr = __fadd2_rn(mr, make_float2(x0, x1));
          });
          const float sc = src.k.n * (mc.x + mc.y) +
                           inv_sqrt_d * (2.f * (mr.x + mr.y) - Q) * src.k.rn;
          const int ii = t + bi * NT;
          const float l2 = ii < n ? sc * lscale : -INFINITY;
          if (ii < n) lg[ii] = l2;
          if (l2 > -INFINITY) {
            const float mb = fmaxf(mt, l2);
            const float scl = exp2f(mt - mb);  // 0 while mt is -inf
            const float p = exp2f(l2 - mb);
            sums.x = sums.x * scl + p;
            sums.y = sums.y * scl + p * (src.vn * inv_sqrt_d + src.vrn * wb);
            mt = mb;
          }
        };
        static_for<C::kRing - 1>([&](auto jc) { load(a[decltype(jc)::value], decltype(jc)::value); });
        for (int bi = 0; bi < nb; bi += C::kRing) {
          static_for<C::kRing>([&](auto jc) {
            constexpr int j = decltype(jc)::value;
            if (bi + j < nb) {
              load(a[(j + C::kRing - 1) % C::kRing], bi + j + C::kRing - 1);
              score(a[j], bi + j);
            }
          });
        }
      }
      RowB2 va[C::kRing];
      auto load_v = [&](RowB2& dst, int bi) {
        const int ii = t + bi * NT;
        const int64_t row = row0 + (ii < n ? ii : 0);
        load_plane32_x(P.v_code + row * C::kWC, wrc, pol_once, dst.c);
        load_plane_x<128>(P.v_res + row * C::kWR, wrr, pol_once, dst.r);
        dst.n = ldg_policy(P.v_norms + row, pol_once);
        dst.rn = ldg_policy(P.v_rnorms + row, pol_once);
      };
      static_for<C::kRing - 1>([&](auto jc) { load_v(va[decltype(jc)::value], decltype(jc)::value); });
      const float m_seg = block_max<NT>(mt, red);  // also: phase-1 table reads done
      const float m_new = fmaxf(m_run, m_seg);
      const float alpha = exp2f(m_run - m_new);  // 0 on the first segment
      m_run = m_new;
      {
        int4* z = reinterpret_cast<int4*>(tabb);
        for (int e = t; e < C::kTabWords / 4; e += NT) z[e] = make_int4(0, 0, 0, 0);
      }
      {
        const float r = mt > -INFINITY ? exp2f(mt - m_new) : 0.f;
        sums.x *= r;
        sums.y *= r;
      }
      const float2 tot = block_sum2<NT>(sums, red);  // barriers also order the zeroing
      const float l_c = tot.x;
      const float scale_inv = tot.y > 0.f ? 1073741824.0f / tot.y : 0.f;
      const float scale = tot.y / 1073741824.0f;

      // ---------------- phase 2: scatter V bytes with fixed-point weights
      float csum = 0.f;  // the residual plane's constant term, in quanta
      const float k1 = inv_sqrt_d * scale_inv, k2 = wb * scale_inv;
      {
        auto scatter = [&](const RowB2& src, int bi) {
          const int ii = t + bi * NT;
          const bool ok = ii < n;
          const float p = ok ? exp2f(lg[ok ? ii : 0] - m_new) : 0.f;
          const int fx = __float2int_rn(p * src.n * k1);
          const int fy = __float2int_rn(p * src.rn * k2);
          csum += -0.5f * (float)fy;
          uint32_t rc[C::kWC], rs[C::kWR];
          xor_plane32(src.c, wrc, rc);
          xor_plane<128>(src.r, wrr, rs);
          static_for<C::kPC>([&](auto kc) {
            constexpr int k = decltype(kc)::value;
            atomicAdd(reinterpret_cast<int*>(
                          tabb + tab_addr_x(rc[k >> 2], slotc[k >> 2], xs.s[k & 3])),
                      fx);
          });
          static_for<C::kPR>([&](auto kc) {
            constexpr int k = decltype(kc)::value;
            atomicAdd(reinterpret_cast<int*>(const_cast<unsigned char*>(tabr) +
                                             tab_addr_x(rs[k >> 2], slotr[k >> 2], xs.s[k & 3])),
                      fy);
          });
        };
        for (int bi = 0; bi < nb; bi += C::kRing) {
          static_for<C::kRing>([&](auto jc) {
            constexpr int j = decltype(jc)::value;
            if (bi + j < nb) {
              load_v(va[(j + C::kRing - 1) % C::kRing], bi + j + C::kRing - 1);
              scatter(va[j], bi + j);
            }
          });
        }
      }
      const float c_c = block_sum<NT>(csum, red) * scale;  // also fences the histograms

      // ---------------- fold (the logits are no longer needed: partials
      // overlay them)
      {
        const int* hi = reinterpret_cast<const int*>(tabb);
        const int slot = t & 31, w = t >> 5;
        // code plane: position slot, byte values 32 w + j
        int s0[4] = {0, 0, 0, 0}, s1[4] = {0, 0, 0, 0}, lo16 = 0, hi16 = 0;
        static_for<32>([&](auto jc) {
          constexpr int j = decltype(jc)::value;
          const int h = hi[(32 * w + j) * 64 + slot];
          s0[j & 3] += h;
          s1[(j >> 2) & 3] += h;
          if constexpr (j < 16) lo16 += h; else hi16 += h;
        });
        const int T = lo16 + hi16;
        int4* o = reinterpret_cast<int4*>(cf + (w * 32 + slot) * 16);
        o[0] = make_int4(s0[0], s0[1], s0[2], s0[3]);  // field 0 (bits 0-1)
        o[1] = make_int4(s1[0], s1[1], s1[2], s1[3]);  // field 1 (bits 2-3)
        const int v2 = 2 * (w & 1);                    // field 2: bit 4 of j, bit 5 of v
        o[2] = make_int4(v2 == 0 ? lo16 : 0, v2 == 0 ? hi16 : 0, v2 == 2 ? lo16 : 0,
                         v2 == 2 ? hi16 : 0);
        const int v3 = w >> 1;                         // field 3: bits 6-7 of v
        o[3] = make_int4(v3 == 0 ? T : 0, v3 == 1 ? T : 0, v3 == 2 ? T : 0, v3 == 3 ? T : 0);
        // residual plane: slot (position slot mod 16, copy slot / 16), subset
        // sums per bit of the byte value
        int sb[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int tt = 0;
        static_for<32>([&](auto jc) {
          constexpr int j = decltype(jc)::value;
          const int h = hi[(32 * w + j) * 64 + 32 + slot];
          tt += h;
          if (j & 1) sb[0] += h;
          if (j & 2) sb[1] += h;
          if (j & 4) sb[2] += h;
          if (j & 8) sb[3] += h;
          if (j & 16) sb[4] += h;
        });
        sb[5] = (w & 1) ? tt : 0;
        sb[6] = (w & 2) ? tt : 0;
        sb[7] = (w & 4) ? tt : 0;
        int4* rp = reinterpret_cast<int4*>(rf + (w * 32 + slot) * 8);
        rp[0] = make_int4(sb[0], sb[1], sb[2], sb[3]);
        rp[1] = make_int4(sb[4], sb[5], sb[6], sb[7]);
      }
      __syncthreads();
      if (t < D) {
        const int p = t >> 2, k = t & 3;
        int sv[4] = {0, 0, 0, 0};
#pragma unroll
        for (int w = 0; w < 8; ++w)
#pragma unroll
          for (int v = 0; v < 4; ++v) sv[v] += cf[(w * 32 + p) * 16 + 4 * k + v];
        float a = cv0 * (float)sv[0] + cv1 * (float)sv[1] + cv2 * (float)sv[2] +
                  cv3 * (float)sv[3];
        const int pos = t >> 3, b = t & 7;
        int sr = 0;  // one plane: a subset sum of one histogram, < 2^31
#pragma unroll
        for (int w = 0; w < 8; ++w) sr += rf[(w * 32 + pos) * 8 + b] + rf[(w * 32 + 16 + pos) * 8 + b];
        a += (float)sr;
        acc = acc * alpha + a * scale;
      }
      l_run = l_run * alpha + l_c;
      c_run = c_run * alpha + c_c;
      __syncthreads();  // fold reads done before the next segment's table and logits
    }

    if (rpart < P.n_splits)  // m in natural-log units for the combine step
      put_record<D>(P, g, rpart, t, m_run * kLn2, l_run, c_run + acc, true);
    if (s1 == P.seq_end && t == 0)
      for (int64_t p = rpart + 1; p < P.n_splits; ++p)
        put_record<D>(P, g, p, 0, -INFINITY, 0.f, 0.f, false);
    __syncthreads();
  }
  peers_finish<D>(P);
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
  P.n_q = r.n_q;
  P.c0 = r.cb.c[0];
  P.c1 = r.cb.c[1];
  for (int i = 0; i < 4; ++i) P.cb[i] = r.cb.c[i];
  for (int i = 0; i < r.D; ++i) P.dk[i] = r.dk[i];
  P.world = r.world;
  if (r.world > 0) {
    if (r.world > kMaxPeers) return KH_EINVAL;
    P.out = r.out;
    P.err = device_error_ptr();
    for (int i = 0; i < r.D; ++i) P.dv[i] = r.dv[i];
    P.rank = r.rank;
    P.epoch = r.epoch;
    P.counter = r.counter;
    P.n_rows_q = r.n_groups * r.n_q;
    for (int i = 0; i < r.world; ++i) {
      P.peer_rec[i] = r.peer_records[i];
      P.peer_flag[i] = r.peer_flags[i];
    }
  }
  const dim3 grid((unsigned)r.n_splits, (unsigned)(r.n_groups * r.n_q));
  const char* env = getenv("KUDAHITAM_DECODE_PATH");
  int path = (env && strcmp(env, "v1") == 0) ? 1 : (env && strcmp(env, "v2") == 0) ? 2 : 3;
  // the 4-level codebook: the table kernel at D = 128, the direct one at D = 256
  if (r.cb.n_c == 4 && (r.D == 256 || path != 3)) path = 1;
  // v3 work split (see decode_v3_kernel): ranges of W (cache group, row)
  // pairs, one CTA set of n_q CTAs each.  W cuts the pairs into one wave of
  // CTAs at two per SM, but no range under 8192 pairs (a range pays the
  // query transform and one table build per segment); and W is at least
  // L / (n_splits - 1) so that no group spans more than n_splits ranges
  // (its record slots).  With one record per row, one range per group.
  // (Four waves of shorter ranges measured 4 % slower on 512 x 40000 pairs
  // and 16 % slower on 1024 x 131072.)
  const int64_t L = r.seq_end - r.seq_begin;
  P.n_groups_kv = r.n_groups;
  int64_t n_cta = 0;
  if (L == 0) {
    P.W = 0;
    n_cta = r.n_groups * r.n_q;
  } else if (r.n_splits == 1) {
    P.W = L;
    n_cta = r.n_groups * r.n_q;
  } else {
    const int64_t total = r.n_groups * L;
    const int64_t slots = std::max<int64_t>(1, 2 * (int64_t)sm_count() / r.n_q);
    const int64_t sets = std::max<int64_t>(1, std::min<int64_t>(slots, (total + 8191) / 8192));
    const int64_t w_bal = (total + sets - 1) / sets;
    const int64_t w_min = (L + r.n_splits - 2) / (r.n_splits - 1);
    P.W = std::max(w_bal, w_min);
    n_cta = (total + P.W - 1) / P.W * r.n_q;
  }
  if (n_cta > 0x7fffffff) return KH_EINVAL;
  if (r.world > 0 && path < 3) return KH_ENOTSUP;  // peer mode: table kernels only
  const dim3 grid3((unsigned)n_cta);
  if (path == 1) {
    if (r.cb.n_c == 4) {
      if (r.D == 128) decode_partial_kernel<128, 4><<<grid, 128, 0, stream>>>(P);
      else decode_partial_kernel<256, 4><<<grid, 256, 0, stream>>>(P);
    } else {
      if (r.D == 128) decode_partial_kernel<128, 2><<<grid, 128, 0, stream>>>(P);
      else decode_partial_kernel<256, 2><<<grid, 256, 0, stream>>>(P);
    }
  } else {
    // the shared-memory opt-in is a per-device function attribute
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KH_ECUDA;
    static std::once_flag once[5][64];
    static int resident[5][64];  // CTAs of the kernel one SM holds at once
    auto launch = [&](auto kern, int slot, int smem, int threads) {
      std::call_once(once[slot][dev & 63], [&] {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        int nb = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, threads, smem) !=
            cudaSuccess)
          nb = 0;
        resident[slot][dev & 63] = nb;
      });
      // the combine is fused only when every CTA of the launch is resident at
      // once (the CTAs wait for each other's flag); else it runs as a
      // separate kernel after this one
      P.fuse = (r.world > 0 && r.out &&
                n_cta <= (int64_t)resident[slot][dev & 63] * sm_count()) ? 1 : 0;
      if (path == 3)  // v3 waits for the previous kernel before its first read
        launch_programmatic(kern, grid3, dim3(threads), smem, stream, P);
      else
        kern<<<grid, threads, smem, stream>>>(P);
    };
    if (path == 2) {
      if (r.D == 128) launch(decode_v2_kernel<128>, 0, V2Cfg<128>::kSmem, V2Cfg<128>::kThreads);
      else launch(decode_v2_kernel<256>, 1, V2Cfg<256>::kSmem, V2Cfg<256>::kThreads);
    } else if (r.cb.n_c == 4) {
      launch(decode_b2_kernel, 4, B2Cfg::kSmem, B2Cfg::kThreads);
    } else {
      if (r.D == 128) launch(decode_v3_kernel<128>, 2, V3Cfg<128>::kSmem, V3Cfg<128>::kThreads);
      else launch(decode_v3_kernel<256>, 3, V3Cfg<256>::kSmem, V3Cfg<256>::kThreads);
    }
  }
  if (cudaGetLastError() != cudaSuccess) return KH_ELAUNCH;
  if (r.world > 0 && r.out && !P.fuse)
    return launch_decode_combine_from_peers(P.peer_rec[r.rank], P.peer_flag[r.rank], r.epoch,
                                            r.n_groups * r.n_q, r.n_splits, r.world, r.D, r.dv,
                                            r.out, stream);
  return KH_OK;
}

kh_status launch_decode_combine(const float* partials, int64_t n_groups, int n_parts,
                                int64_t group_stride, int64_t part_stride, int D,
                                const float* dv, bool records, float* out,
                                cudaStream_t stream) {
  DecodeParams P;
  memset(&P, 0, sizeof(P));
  if (dv)
    for (int i = 0; i < D; ++i) P.dk[i] = dv[i];
  if (n_groups > 0x7fffffff) return KH_EINVAL;
  const dim3 grid((unsigned)n_groups);
  auto go = [&](auto kern, int threads) {
    launch_programmatic(kern, grid, dim3(threads), 0, stream, partials, n_parts, group_stride,
                        part_stride, out, P);
  };
  if (D == 128) {
    if (records) go(decode_combine_kernel<128, true>, 128);
    else go(decode_combine_kernel<128, false>, 128);
  } else {
    if (records) go(decode_combine_kernel<256, true>, 256);
    else go(decode_combine_kernel<256, false>, 256);
  }
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

kh_status launch_decode_merge_to_peers(const float* partials, int64_t n_rows, int n_parts,
                                      int64_t group_stride, int64_t part_stride, int D,
                                      float* const* peer_records, uint32_t* const* peer_flags,
                                      int rank, int world, uint32_t epoch, uint32_t* counter,
                                      cudaStream_t stream) {
  if (world < 1 || world > kMaxPeers || n_rows > 0x7fffffff) return KH_EINVAL;
  PeerParams Q;
  memset(&Q, 0, sizeof(Q));
  for (int p = 0; p < world; ++p) {
    Q.rec[p] = peer_records[p];
    Q.flag[p] = peer_flags[p];
  }
  const dim3 grid((unsigned)n_rows);
  if (D == 128)
    decode_merge_to_peers_kernel<128><<<grid, 128, 0, stream>>>(
        partials, n_parts, group_stride, part_stride, n_rows, rank, world, epoch, counter, Q);
  else
    decode_merge_to_peers_kernel<256><<<grid, 256, 0, stream>>>(
        partials, n_parts, group_stride, part_stride, n_rows, rank, world, epoch, counter, Q);
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

kh_status launch_decode_combine_from_peers(const float* records, const uint32_t* flags,
                                           uint32_t epoch, int64_t n_rows, int n_parts,
                                           int world, int D, const float* dv, float* out,
                                           cudaStream_t stream) {
  if (world < 1 || world > kMaxPeers || n_parts < 1 || n_rows > 0x3ffffffffll) return KH_EINVAL;
  DecodeParams P;
  memset(&P, 0, sizeof(P));
  for (int i = 0; i < D; ++i) P.dk[i] = dv[i];
  const dim3 grid((unsigned)((n_rows + 7) / 8));
  uint32_t* err = device_error_ptr();
  if (D == 128)
    decode_combine_peer_records_kernel<128><<<grid, 256, 0, stream>>>(
        records, flags, epoch, n_rows, n_parts, world, out, err, P);
  else
    decode_combine_peer_records_kernel<256><<<grid, 256, 0, stream>>>(
        records, flags, epoch, n_rows, n_parts, world, out, err, P);
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

}  // namespace kh
