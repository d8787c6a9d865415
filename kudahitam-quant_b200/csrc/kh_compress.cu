// kh_compress.cu -- fused single-pass KV-row compression (SIMT datapath).
//
// One pass over HBM per row:  load (TMA, 128B-swizzled tiles) -> ||x|| ->
// d-flip -> Walsh-Hadamard in registers -> Lloyd-Max index -> residual sign
// plane and residual norm -> packed 32-bit words.
//
// Reference: ultra_fused_full_fusion_kernel_v8 (KudaHitamCUDA.cu:13-195) runs
// three FWHT passes per row (forward :58-84, reconstruct :113-139, residual
// :161-187).  Here only the forward transform is computed: the residual
// sign and norm follow from the rotated-domain identity
//     H(d (.) (x - k_mse)) = sqrt(D) ||x|| (y - c[idx]),   y = H(d (.) x)/(sqrt(D)||x||)
// (k_mse = ||x|| d (.) H c[idx] / sqrt(D) and H H = D I), so
//     sign plane = sign(y - c[idx]),  r_norm = ||x|| * ||y - c[idx]||.
//
// Thread mapping: a warp owns a tile of 32 rows (D=128, one row per lane) or
// 16 rows (D=256, two lanes per row, each producing one half of the output
// after the top butterfly stage).  Each warp runs its own STAGES-deep TMA
// ring, so loads of the next tiles overlap the arithmetic of this one.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "kh_common.cuh"
#include "kh_internal.h"
#include "kh_quant.cuh"

namespace kh {
namespace {

template <int MAXSEG>
struct alignas(64) CompressParams {
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
  // fp32 input: per-element sign mask.  16-bit input: per element PAIR
  // (bit 15 -> element 2k, bit 31 -> element 2k+1).
  uint32_t dflip[256];
};

template <typename T, int D, int CK, bool RES, int MAXSEG, int WARPS,
          int STAGES>
struct Cfg {
  static constexpr int kTPR = D / 128;        // lanes per row
  static constexpr int kRows = 32 / kTPR;     // rows per warp tile
  static constexpr int kEB = (int)sizeof(T);  // element bytes
  static constexpr int kBoxInner = 128 / kEB; // elements per 128 B box row
  static constexpr int kNBox = D / kBoxInner;
  static constexpr int kBoxBytes = kRows * 128;
  static constexpr int kTileBytes = kNBox * kBoxBytes;
  static constexpr int kSmem = 1024 + WARPS * STAGES * kTileBytes +
                               WARPS * STAGES * 8;
  static constexpr int kCodeWordsPerRow = (CK == kCbGen4 ? D / 16 : D / 32);
};

template <typename T, int D, int CK, bool RES, int MAXSEG, int WARPS,
          int STAGES>
__global__ void __launch_bounds__(WARPS * 32, 1)
    compress_simt_kernel(const __grid_constant__ CompressParams<MAXSEG> P) {
  using C = Cfg<T, D, CK, RES, MAXSEG, WARPS, STAGES>;
  using Q = Quant<CK, RES>;
  constexpr int kEPC = Chunk<T>::kElems;  // elements per 16-B chunk
  constexpr int kCPB = 8;                 // 16-B chunks per 128-B box row

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t wbuf = base + warp * STAGES * C::kTileBytes;
  uint8_t* wbuf_g = gbase + warp * STAGES * C::kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(
                       gbase + WARPS * STAGES * C::kTileBytes) +
                   warp * STAGES;

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  const int64_t total = P.tile_begin[P.n_seg];
  const int64_t gw = (int64_t)blockIdx.x * WARPS + warp;
  const int64_t nw = (int64_t)gridDim.x * WARPS;
  const uint64_t policy = l2_policy_evict_first();

  // Segment of tile t, resumed from a cursor: the issuer and the consumer
  // each visit their tiles in increasing order (amortised O(1) per tile).
  auto seg_of = [&](int64_t t, int& sg) {
#pragma unroll 1
    while (sg + 1 < P.n_seg && t >= P.tile_begin[sg + 1]) ++sg;
    return sg;
  };
  int sg_issue = 0, sg_use = 0;
  auto issue = [&](int64_t t, int s) {
    const int sg = seg_of(t, sg_issue);
    const int32_t row0 = (int32_t)((t - P.tile_begin[sg]) * C::kRows);
    mbar_arrive_expect_tx(&bars[s], C::kTileBytes);
#pragma unroll
    for (int b = 0; b < C::kNBox; ++b)
      tma_load_2d(wbuf_g + s * C::kTileBytes + b * C::kBoxBytes, &P.tmap[sg],
                  b * C::kBoxInner, row0, &bars[s], policy);
  };

  if (lane == 0) {
    if (gw < total) {
      int sg0 = 0;
      prefetch_tmap(&P.tmap[seg_of(gw, sg0)]);
    }
    // launched as a programmatic dependent: rows are read (and outputs
    // written) only once the previous kernel in the stream has completed
    grid_dependency_wait();
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      const int64_t t = gw + s * nw;
      if (t < total) issue(t, s);
    }
  }

  const int r = lane / C::kTPR;       // row within the tile
  const int part = lane % C::kTPR;    // which half of the output (D=256)
  const uint32_t sw = (uint32_t)(r & 7);  // 128B-swizzle phase of this row

  int k = 0;
  for (int64_t t = gw; t < total; t += nw, ++k) {
    const int s = k % STAGES;
    const uint32_t ph = (uint32_t)((k / STAGES) & 1);
    if (!mbar_wait(&bars[s], ph, P.err)) break;

    const int sg = seg_of(t, sg_use);
    const int64_t row = (t - P.tile_begin[sg]) * C::kRows + r;
    const uint32_t rowbase = wbuf + s * C::kTileBytes + r * 128;

    // ---- load + d-flip + (D=256) top butterfly + sum of squares --------
    float x[128];
    float2 ss2 = make_float2(0.f, 0.f);
    if constexpr (D == 128) {
#pragma unroll
      for (int b = 0; b < C::kNBox; ++b) {
#pragma unroll
        for (int c = 0; c < kCPB; ++c) {
          const uint4 v =
              lds128(rowbase + b * C::kBoxBytes + (((uint32_t)c ^ sw) << 4));
          const int e0 = b * C::kBoxInner + c * kEPC;
          Chunk<T>::load(v, P, e0, &x[e0]);
        }
      }
#pragma unroll
      for (int e = 0; e < 128; e += 2) {
        const float2 p = make_float2(x[e], x[e + 1]);
        ss2 = __ffma2_rn(p, p, ss2);
      }
    } else {
      // D == 256: lane `part` keeps w = x_lo + sgn * x_hi  (sgn = +1 / -1).
      const float sgn = part ? -1.f : 1.f;
      const float2 sg2 = make_float2(sgn, sgn);
      constexpr int kHalfBox = C::kNBox / 2;
#pragma unroll
      for (int b = 0; b < kHalfBox; ++b) {
#pragma unroll
        for (int c = 0; c < kCPB; ++c) {
          const uint32_t off = (((uint32_t)c ^ sw) << 4);
          const uint4 vlo = lds128(rowbase + b * C::kBoxBytes + off);
          const uint4 vhi = lds128(rowbase + (b + kHalfBox) * C::kBoxBytes + off);
          const int e0 = b * C::kBoxInner + c * kEPC;
          float lo[kEPC], hi[kEPC];
          Chunk<T>::load(vlo, P, e0, lo);
          Chunk<T>::load(vhi, P, e0 + 128, hi);
#pragma unroll
          for (int j = 0; j < kEPC; j += 2) {
            const float2 w = __ffma2_rn(make_float2(hi[j], hi[j + 1]), sg2,
                                        make_float2(lo[j], lo[j + 1]));
            x[e0 + j] = w.x;
            x[e0 + j + 1] = w.y;
            ss2 = __ffma2_rn(w, w, ss2);
          }
        }
      }
    }
    float ss = ss2.x + ss2.y;
    if constexpr (D == 256) {
      // sum over both lanes of (lo+hi)^2 + (lo-hi)^2 = 2 ||x||^2
      ss = (ss + __shfl_xor_sync(0xffffffffu, ss, 1)) * 0.5f;
    }
    // Every lane has consumed its shared-memory chunks (ss depends on all of
    // them): the stage can be refilled.
    __syncwarp();
    if (lane == 0) {
      const int64_t tn = t + (int64_t)STAGES * nw;
      if (tn < total) issue(tn, s);
    }

    const float norm = ss > 0.f ? sqrtf(ss) : 1e-8f;  // KudaHitamCUDA.cu:50
    const float rs = 1.0f / (norm * (D == 128 ? 11.313708498984761f : 16.0f));

    fwht_regs<128>(x);

    uint32_t code[4 * Q::kCodeWords];
    uint32_t resw[4];
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      Q::run(&x[32 * g], rs, P, &code[g * Q::kCodeWords], resw[g], acc);
    }

    float rn = 0.f;
    if (RES) {
      float a = acc.x + acc.y;
      if constexpr (D == 256) a += __shfl_xor_sync(0xffffffffu, a, 1);
      rn = a > 0.f ? norm * sqrtf(a) : 1e-8f;  // KudaHitamCUDA.cu:158
    }

    if (row < P.n_rows[sg]) {
      uint32_t* cdst = P.code[sg] + row * C::kCodeWordsPerRow +
                       part * 4 * Q::kCodeWords;
#pragma unroll
      for (int i = 0; i < Q::kCodeWords; ++i) {
        uint4 v;
        v.x = code[4 * i + 0];
        v.y = code[4 * i + 1];
        v.z = code[4 * i + 2];
        v.w = code[4 * i + 3];
        reinterpret_cast<uint4*>(cdst)[i] = v;
      }
      if (RES) {
        uint32_t* rdst = P.res[sg] + row * (D / 32) + part * 4;
        *reinterpret_cast<uint4*>(rdst) = make_uint4(resw[0], resw[1], resw[2], resw[3]);
      }
      if (part == 0) {
        P.norms[sg][row] = norm;
        if (RES) P.rnorms[sg][row] = rn;
      }
    }
  }
  // this warp is done: the next kernel in the stream may be scheduled once
  // every CTA has signalled
  grid_dependents_launch();
}

// ------------------------------------------------------------------ host
template <typename T, int D, int CK, bool RES, int MAXSEG>
kh_status launch_typed(const CompressRequest& req, cudaStream_t stream) {
  constexpr int kWarps = 4;
  constexpr int kStages = (sizeof(T) == 4) ? 1 : 2;
  using C = Cfg<T, D, CK, RES, MAXSEG, kWarps, kStages>;
  auto kern = compress_simt_kernel<T, D, CK, RES, MAXSEG, kWarps, kStages>;

  static std::once_flag attr_once[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KH_ECUDA;
  static int blocks_per_sm[64];
  std::call_once(attr_once[dev & 63], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         C::kSmem);
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kWarps * 32,
                                                  C::kSmem);
    blocks_per_sm[dev & 63] = n > 0 ? n : 1;
  });

  CompressParams<MAXSEG> P;
  memset(&P, 0, sizeof(P));
  CUtensorMapDataType dt = sizeof(T) == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : std::is_same<T, __half>::value
                               ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                               : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  int64_t tiles = 0;
  P.n_seg = req.n_seg;
  for (int i = 0; i < req.n_seg; ++i) {
    const CompressSegHost& s = req.seg[i];
    P.tile_begin[i] = tiles;
    const int64_t nt = (s.n_rows + C::kRows - 1) / C::kRows;
    tiles += nt;
    P.code[i] = s.code;
    P.res[i] = s.res;
    P.norms[i] = s.norms;
    P.rnorms[i] = s.rnorms;
    P.n_rows[i] = s.n_rows;
    if (s.n_rows > 0) {
      CUresult cr = encode_tensor_map_2d(
          &P.tmap[i], dt, const_cast<void*>(s.x), (uint64_t)D,
          (uint64_t)s.n_rows, (uint64_t)(s.row_stride * (int64_t)sizeof(T)),
          (uint32_t)C::kBoxInner, (uint32_t)C::kRows,
          CU_TENSOR_MAP_SWIZZLE_128B);
      if (cr != CUDA_SUCCESS) return KH_ECUDA;
    }
  }
  P.tile_begin[req.n_seg] = tiles;
  if (tiles == 0) return KH_OK;
  P.err = device_error_ptr();
  P.cb = req.cb;
  if (sizeof(T) == 4) {
    for (int e = 0; e < D; ++e) P.dflip[e] = req.dflip[e];
  } else {
    for (int k = 0; k < D / 2; ++k)
      P.dflip[k] = (req.dflip[2 * k] >> 16) | req.dflip[2 * k + 1];
  }
  const int64_t want = (tiles + kWarps - 1) / kWarps;
  const int64_t cap = (int64_t)sm_count() * blocks_per_sm[dev & 63];
  const int grid = (int)std::max<int64_t>(1, std::min(want, cap));
  if (launch_programmatic(kern, dim3((unsigned)grid), dim3(kWarps * 32), C::kSmem, stream, P) !=
      cudaSuccess)
    return KH_ELAUNCH;
  return cudaGetLastError() == cudaSuccess ? KH_OK : KH_ELAUNCH;
}

template <typename T, int D, int MAXSEG>
kh_status dispatch_cb(const CompressRequest& req, cudaStream_t s) {
  const bool res = req.residual != 0;
  switch (req.cb.kind) {
    case kCbSym2:
      return res ? launch_typed<T, D, kCbSym2, true, MAXSEG>(req, s)
                 : launch_typed<T, D, kCbSym2, false, MAXSEG>(req, s);
    case kCbGen2:
      return res ? launch_typed<T, D, kCbGen2, true, MAXSEG>(req, s)
                 : launch_typed<T, D, kCbGen2, false, MAXSEG>(req, s);
    case kCbGen4:
      return res ? launch_typed<T, D, kCbGen4, true, MAXSEG>(req, s)
                 : launch_typed<T, D, kCbGen4, false, MAXSEG>(req, s);
  }
  return KH_EINVAL;
}

template <typename T, int MAXSEG>
kh_status dispatch_d(const CompressRequest& req, cudaStream_t s) {
  return req.head_dim == 128 ? dispatch_cb<T, 128, MAXSEG>(req, s)
                             : dispatch_cb<T, 256, MAXSEG>(req, s);
}

template <int MAXSEG>
kh_status dispatch_t(const CompressRequest& req, cudaStream_t s) {
  switch (req.dtype) {
    case KH_F32: return dispatch_d<float, MAXSEG>(req, s);
    case KH_F16: return dispatch_d<__half, MAXSEG>(req, s);
    case KH_BF16: return dispatch_d<__nv_bfloat16, MAXSEG>(req, s);
  }
  return KH_EINVAL;
}

}  // namespace

kh_status launch_compress_simt(const CompressRequest& req, cudaStream_t stream) {
  if (req.n_seg <= 2) return dispatch_t<2>(req, stream);
  return dispatch_t<kMaxSegments>(req, stream);
}

kh_status launch_compress(const CompressRequest& req, cudaStream_t stream) {
  const bool sixteen = req.dtype == KH_F16 || req.dtype == KH_BF16;
  const char* env = getenv("KUDAHITAM_COMPRESS_PATH");
  const bool force_simt = env && strcmp(env, "simt") == 0;
  if (sixteen && !force_simt) return launch_compress_tc(req, stream);
  return launch_compress_simt(req, stream);
}

}  // namespace kh
