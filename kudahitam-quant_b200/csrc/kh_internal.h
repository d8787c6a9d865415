// kh_internal.h -- host-side interfaces between the C-ABI layer (kh_api.cu)
// and the kernel translation units.  Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kudahitam.h"

namespace kh {

constexpr int kMaxSegments = 64;

// Codebook kinds the compress kernels specialise on.
enum CodebookKind : int {
  kCbSym2 = 0,  // 2 levels, c0 == -c1 exactly (the Lloyd-Max bits=1 codebook)
  kCbGen2 = 1,  // 2 levels, arbitrary sorted values
  kCbGen4 = 2,  // 4 levels (bits=2 codebook), sorted ascending
};

// Per-call constants baked into every launch (passed by value).
struct Codebook {
  int kind;        // CodebookKind
  int n_c;         // 2 or 4
  float c[4];      // centroids, ascending
  float mid[3];    // decision midpoints (c[i] + c[i+1]) / 2, float
  float sel[2];    // kCbGen2: mid[0] - c[0], mid[0] - c[1]
};

struct CompressSegHost {
  const void* x;
  int64_t n_rows;
  int64_t row_stride;  // elements
  uint32_t* code;
  uint32_t* res;
  float* norms;
  float* rnorms;
};

struct CompressRequest {
  int dtype;  // kh_dtype
  int head_dim;
  int residual;
  Codebook cb;
  uint32_t dflip[256];  // per element: 0 or 0x80000000 (sign flip for d=-1)
  int n_seg;
  CompressSegHost seg[kMaxSegments];
};

// Launch the fused compression kernel.  Arguments are already validated.
// Picks the datapath: the tensor-core kernel for fp16 / bf16 rows, the SIMT
// kernel for fp32.  Environment KUDAHITAM_COMPRESS_PATH=simt sends 16-bit
// inputs to the SIMT kernel too (used to test and compare both datapaths).
kh_status launch_compress(const CompressRequest& req, cudaStream_t stream);
kh_status launch_compress_simt(const CompressRequest& req, cudaStream_t stream);
kh_status launch_compress_tc(const CompressRequest& req, cudaStream_t stream);

// Materialise reference-layout tensors from a packed cache.
kh_status launch_materialize(const uint32_t* code, const uint32_t* res,
                             const float* norms, int64_t n_rows, int D,
                             const float* d, const Codebook& cb, uint8_t* idx,
                             float* kmse, int8_t* signs, cudaStream_t stream);

kh_status launch_fwht(float* x, int64_t n_rows, int D, cudaStream_t stream);

kh_status launch_score_packed_compat(const void* q, int64_t n_heads, int D, int64_t seq_len,
                                     const uint8_t* k_packed, const void* signs,
                                     const float* d, const float* k_norms,
                                     const float* r_norms, const float* centroids,
                                     int nibble, float scale, float* out,
                                     cudaStream_t stream);
kh_status launch_score(const float* q, int64_t n_groups, int n_q, int D,
                       const uint32_t* code, const uint32_t* res,
                       const float* norms, const float* rnorms,
                       int64_t seq_len, const float* d, const Codebook& cb,
                       float* out, cudaStream_t stream);

struct DecodeRequest {
  const float* q;
  int64_t n_groups;
  int D;
  const uint32_t *k_code, *k_res, *v_code, *v_res;
  const float *k_norms, *k_rnorms, *v_norms, *v_rnorms;
  int64_t seq_len, seq_begin, seq_end;
  float dk[256];
  Codebook cb;
  float sm_scale;
  int n_splits;
  int n_q = 1;  // queries per cache group; q and partials have n_groups * n_q rows
  float* partials;
  int64_t part_stride, part_offset;
  // peer mode (world > 0): records to every rank's buffer, flags raised
  int world = 0, rank = 0;
  uint32_t epoch = 0;
  uint32_t* counter = nullptr;
  float* const* peer_records = nullptr;
  uint32_t* const* peer_flags = nullptr;
  // peer mode: out != nullptr also merges every rank's records into out
  // [n_groups * n_q][D] (V's diagonal dv) once all flags arrived
  float* out = nullptr;
  float dv[256];
};

kh_status launch_decode_partial(const DecodeRequest& r, cudaStream_t stream);
// Merges n_parts records per query row (record p of row g at
// partials + g * group_stride + p * part_stride floats): records = true writes
// merged records (D + 2 floats per row), else d (.) H(acc) / l into out[g][D].
kh_status launch_decode_combine(const float* partials, int64_t n_groups, int n_parts,
                                int64_t group_stride, int64_t part_stride, int D,
                                const float* dv, bool records, float* out,
                                cudaStream_t stream);

// Fused record exchange of a sequence-sharded decode (world <= 8 ranks).
kh_status launch_decode_merge_to_peers(const float* partials, int64_t n_rows, int n_parts,
                                      int64_t group_stride, int64_t part_stride, int D,
                                      float* const* peer_records, uint32_t* const* peer_flags,
                                      int rank, int world, uint32_t epoch, uint32_t* counter,
                                      cudaStream_t stream);
kh_status launch_decode_combine_from_peers(const float* records, const uint32_t* flags,
                                           uint32_t epoch, int64_t n_rows, int n_parts,
                                           int world, int D, const float* dv, float* out,
                                           cudaStream_t stream);

// HBBA encoder and calibrator (kh_hbba.cu).  d, cent, mask and n_map are
// device arrays, as in the reference binding.
kh_status launch_hbba_compress(const void* x, int dtype, int64_t n_rows, int D,
                               int64_t row_stride, const float* d, const float* cent,
                               const uint32_t* mask, int is_hbba, uint8_t* packed,
                               float* norms, float* rnorms, void* signs, cudaStream_t stream);
kh_status launch_hbba_calibrate(const float* sample, int64_t n, int D, const int* n_map,
                                float* out, cudaStream_t stream);

// Device address of the sticky error word on the current device.
uint32_t* device_error_ptr();

// Number of SMs of the current device (cached per device).
int sm_count();

// Resolve cuTensorMapEncodeTiled through the runtime (no -lcuda needed).
CUresult encode_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dt,
                              void* base, uint64_t inner, uint64_t rows,
                              uint64_t row_stride_bytes, uint32_t box_inner,
                              uint32_t box_rows, CUtensorMapSwizzle swz);

inline int dtype_size(int dtype) { return dtype == KH_F32 ? 4 : 2; }

}  // namespace kh
