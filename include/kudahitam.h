/*
 * kudahitam.h -- C ABI of the B200 (sm_100a) KV-cache compression engine.
 *
 * Everything here is plain C: raw pointers, sizes and an opaque stream handle
 * (a cudaStream_t passed as void*; NULL = the legacy default stream).  No call
 * allocates device memory: the caller owns every buffer.  Calls are
 * asynchronous and stream-ordered; they return a status code and never abort
 * the process or trap the GPU.
 *
 * Packed cache layout (per tensor of n_rows rows of head_dim D, D in {128,256}):
 *   code_bits : uint32[n_rows][D/32]  (bits=1) -- Lloyd-Max index of element i
 *               at bit (i & 31) of word (i >> 5); bit 1 = centroid c[1].
 *               This is the reference's LSB-first 1-bit packing
 *               (KudaHitamCUDA.cu:362-364 write, :756 read) read as 32-bit words.
 *               uint32[n_rows][D/16]  (bits=2) -- 2-bit index of element i at
 *               bits 2*(i & 15) of word (i >> 4) (nibble order of :358-360
 *               extended to 2-bit fields).
 *   res_bits  : uint32[n_rows][D/32] -- QJL sign of the residual after the
 *               Hadamard projection, bit 1 = sign +1 (KudaHitamCUDA.cu:189-194).
 *   norms     : float[n_rows]  -- ||x|| (1e-8 for an all-zero row, :50).
 *   r_norms   : float[n_rows]  -- ||x - k_mse|| (1e-8 when zero, :158).
 *
 * Host pointers vs device pointers: x, code_bits, res_bits, norms, r_norms,
 * q, out and workspace are DEVICE pointers.  d (the +-1 Rademacher diagonal)
 * and centroids are HOST float arrays read during the call and baked into the
 * launch, so they may be freed as soon as the call returns.
 */
#ifndef KUDAHITAM_H_
#define KUDAHITAM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum kh_status {
  KH_OK = 0,
  KH_EINVAL = 1,   /* bad size / mode / pointer combination                 */
  KH_EALIGN = 2,   /* a pointer or row stride is not 16-byte aligned         */
  KH_ELAUNCH = 3,  /* the kernel launch was rejected (cudaGetLastError)      */
  KH_ECUDA = 4,    /* another CUDA runtime / driver call failed              */
  KH_ENOTSUP = 5   /* valid request the engine does not implement            */
} kh_status;

typedef enum kh_dtype { KH_F32 = 0, KH_F16 = 1, KH_BF16 = 2 } kh_dtype;

/* Human readable name of a status code (static storage). */
const char* kh_status_string(int status);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int kh_version(void);

/* Every entry point launches on `stream`, which must belong to the CURRENT
 * device (as with any CUDA runtime launch).
 *
 * Sticky device-side error word of the current device (bounded waits that
 * gave up set a bit).  Synchronous: reads device memory.  0 = no error.
 * Bit 0: an mbarrier wait of a compressor gave up; bit 1: a tile index fell
 * outside every segment; bit 2: kh_decode_combine_from_peers stopped waiting
 * for a peer's flag. */
int kh_device_error(uint32_t* out_flags);
int kh_clear_device_error(void);

/*
 * kh_compress -- fused single-pass KV compression of one tensor.
 * Replaces ultra_fused_full_fusion_cuda (KudaHitamCUDA.cu:197-231, kernel
 * :13-195), the op called by KudahitamCompressorV2.compress
 * (KudaHitamQuant_full.py:334,356).
 *
 *   x          device [n_rows rows] x [head_dim] elements of `dtype`, row r at
 *              x + r*row_stride elements.  16-byte aligned; row_stride*elt
 *              must be a multiple of 16 bytes.
 *   d_host     head_dim floats, each +1 or -1.
 *   centroids  n_centroids floats (2 -> bits=1 codebook, 4 -> bits=2), sorted
 *              ascending.
 *   residual   0: "1-bit mode" (code_bits + norms only; res_bits and r_norms
 *              may be NULL).  1: the reference's full output (code + residual
 *              sign plane + both norms).
 * Outputs are written for rows [0, n_rows).  n_rows == 0 is a no-op.
 */
int kh_compress(const void* x, int dtype, int64_t n_rows, int head_dim,
                int64_t row_stride, const float* d_host,
                const float* centroids_host, int n_centroids, int residual,
                uint32_t* code_bits, uint32_t* res_bits, float* norms,
                float* r_norms, void* stream);

/*
 * kh_compress_batched -- the same compression over n_segments independent
 * tensors (e.g. K and V of every layer) in ONE launch.  Array arguments are
 * HOST arrays of length n_segments holding per-segment device pointers / row
 * counts / row strides.  All segments share dtype, head_dim, d, centroids and
 * mode.  n_segments <= kh_max_segments().
 * No reference counterpart (the reference compresses one tensor per call,
 * KudaHitamQuant_full.py:621-649); it batches the same op.
 */
int kh_max_segments(void);
int kh_compress_batched(int n_segments, const void* const* x,
                        const int64_t* n_rows, const int64_t* row_stride,
                        uint32_t* const* code_bits, uint32_t* const* res_bits,
                        float* const* norms, float* const* r_norms, int dtype,
                        int head_dim, const float* d_host,
                        const float* centroids_host, int n_centroids,
                        int residual, void* stream);

/*
 * kh_fwht_inplace -- orthonormal Walsh-Hadamard transform of float rows
 * (x <- H x / sqrt(D)), in place.  Replaces fwht_cuda_forward
 * (KudaHitamCUDA.cu:233-283), reached from fwht() (KudaHitamQuant_full.py:207-215).
 * head_dim is a power of two in [2, 1024]; rows are contiguous.
 */
int kh_fwht_inplace(float* x, int64_t n_rows, int head_dim, void* stream);

/*
 * kh_materialize -- expand a packed cache back to the reference kernel's
 * output tensors: idx uint8[n,D], k_mse float[n,D], signs int8[n,D]
 * (KudaHitamCUDA.cu:105-111, :141-149, :189-194).  Any output may be NULL;
 * signs needs res_bits.  k_mse = norm * d (.) H(c[idx]) / sqrt(D).
 * out_idx and out_signs must be 8-byte aligned (each lane stores 4 or 8 of
 * a row's bytes at once), out_kmse 4-byte aligned.
 */
int kh_materialize(const uint32_t* code_bits, const uint32_t* res_bits,
                   const float* norms, int64_t n_rows, int head_dim,
                   const float* d_host, const float* centroids_host,
                   int n_centroids, uint8_t* out_idx, float* out_kmse,
                   int8_t* out_signs, void* stream);

/*
 * kh_score -- asymmetric attention scores straight from the packed cache.
 * Replaces KudahitamCompressorV2.asymmetric_attention_scores
 * (KudaHitamQuant_full.py:373-377):
 *   out[g,j,s] = q_gj . k_mse_gs + (1/sqrt(D)) <fwht(q_gj (.) d), sign_gs> r_norm_gs
 * evaluated as norm*<q~, c[idx]> + r_norm/sqrt(D) <q~, sign> with
 * q~ = H(q (.) d)/sqrt(D).
 *   q      device float [n_groups][n_q][D]
 *   cache  rows of group g are rows [g*seq_len, (g+1)*seq_len) of the packed
 *          cache; res_bits / r_norms may be NULL (1-bit mode: no QJL term).
 *   out    device float [n_groups][n_q][seq_len]
 */
int kh_score(const float* q, int64_t n_groups, int n_q, int head_dim,
             const uint32_t* code_bits, const uint32_t* res_bits,
             const float* norms, const float* r_norms, int64_t seq_len,
             const float* d_host, const float* centroids_host, int n_centroids,
             float* out, void* stream);

/*
 * kh_score_packed_compat -- the reference's packed-cache scorer with its own
 * argument layout and arithmetic.  Replaces fused_asymmetric_attention
 * (fused_asymmetric_attention_packed_cuda / _kernel, KudaHitamCUDA.cu:695-797,
 * called from KudaHitamQuant_full-reasoning.py:411 and :563):
 *   q~   = H(q_h (.) d) / sqrt(D)   (unnormalised Hadamard, strides 1,2,4,..)
 *   sum1 = sum_i q~_i * (centroids[i][v_i] * k_norm)
 *   sum2 = sum_i q_i * signs_i      (unrotated q, raw signs values)
 *   out  = sum1 + k_norm * scale * sum2 * r_norm
 * v_i = bit (i & 7) of byte (i >> 3) of the row's 32 packed bytes; when
 * 0 <= layer_id < 8 and bit layer_id of active_mask is set, v_i = nibble
 * (i & 1) of byte (i >> 1) of the row's 128 packed bytes.  Same summation
 * order as the reference kernel (per-lane fused multiply-adds over
 * i = lane, lane + 32, ..., then a butterfly reduction).
 *   q         device fp16 [n_heads][D]
 *   k_packed  device uint8 [n_heads][seq_len][32 or 128], 4-byte aligned
 *   signs     device fp16 [n_heads][seq_len][D]
 *   d         device float [D]
 *   k_norms, r_norms  device float [n_heads][seq_len]
 *   centroids device float [D][16]
 *   out       device float [n_heads][seq_len]
 * Unlike the other entry points, d and centroids are DEVICE arrays here, as
 * in the reference binding.  D is a power of two in [32, 256].
 */
int kh_score_packed_compat(const void* q, int64_t n_heads, int head_dim,
                           int64_t seq_len, const uint8_t* k_packed,
                           const void* signs, const float* d,
                           const float* k_norms, const float* r_norms,
                           const float* centroids, int layer_id,
                           int active_mask, float scale, float* out,
                           void* stream);

/*
 * kh_compress_hbba -- the HBBA mixed-codebook encoder.  Replaces
 * ultra_fused_packed_hbba_fusion_cuda / _kernel (KudaHitamCUDA.cu:285-420),
 * bound as ultra_fused_hbba_fusion (:801) and called by
 * KudahitamCompressorHBBA.compress (KudaHitamQuant_full-reasoning.py:521).
 * Its output is the packed cache kh_score_packed_compat reads.  Per row of
 * x (fp32 / fp16 / bf16, row r at x + r*row_stride elements):
 *   norm   = sqrt(sum x^2 + 1e-8)
 *   y      = H(x / norm (.) d) / sqrt(D)
 *   idx_i  = argmin_c |y_i - fp16(centroids[i][c])| over 16 levels when the
 *            layer is HBBA ((active_mask >> layer_id) & 1, 0 <= layer_id < 8)
 *            and bit (i & 31) of hbba_mask[i >> 5] is set, else over 2
 *   out_packed  uint8 [n_rows][128] (HBBA layer: nibble (i & 1) of byte
 *               i >> 1) or [n_rows][32] (bit (i & 7) of byte i >> 3); bytes
 *               past the row's D indices are zero
 *   out_norms   float [n_rows]; out_rnorms = sqrt(sum (y - c)^2 * D + 1e-8)
 *   out_signs   fp16 [n_rows][D] = H(y - c[idx]) (unnormalised)
 * Both sums of squares run over the whole row (the reference's reduce
 * within one warp of its 256 threads, :312-314 and :377).  d [D],
 * centroids [D][16] and hbba_mask [8] are DEVICE arrays, as in the
 * reference binding.
 */
int kh_compress_hbba(const void* x, int dtype, int64_t n_rows, int head_dim,
                     int64_t row_stride, const float* d, const float* centroids,
                     const uint32_t* hbba_mask, int layer_id, int active_mask,
                     uint8_t* out_packed, float* out_norms, float* out_rnorms,
                     void* out_signs, void* stream);

/*
 * kh_hbba_calibrate -- per-dimension Lloyd-Max levels for the HBBA encoder.
 * Replaces hbba_calibrate_cuda / hbba_calibrate_cuda_kernel
 * (KudaHitamCUDA.cu:423-516, called from
 * KudaHitamQuant_full-reasoning.py:490).  For dimension d with
 * n = n_map[d] levels (clamped to [1, 16]): levels start uniform between
 * the sample's min and max, then 10 rounds of nearest level (strict <,
 * lowest index) and mean update (a level with no samples keeps its value).
 * sample float [n_rows][head_dim] and n_map int [head_dim] are device
 * arrays; writes out_centroids float [head_dim][16], unused entries 0.
 * Sums accumulate in double in a fixed order (deterministic).
 */
int kh_hbba_calibrate(const float* sample, int64_t n_rows, int head_dim, const int* n_map,
                      float* out_centroids, void* stream);

/*
 * kh_decode_partial_gqa -- kh_decode_partial for grouped-query attention:
 * n_q query heads share each cache group (H_q = n_q * H_kv).  q is
 * [n_groups][n_q][D]; partial records (and the combine step's n_groups
 * argument and output) cover n_groups * n_q query rows, query row
 * g * n_q + j reading cache group g.  The cache is not expanded: the n_q
 * CTAs of a group read the same rows (from L2 after the first).  No
 * counterpart in the reference, which expands K and V to the query heads
 * before scoring (KudaHitamQuant_full-reasoning.py:389-403).
 * kh_decode_partial is this call with n_q = 1.
 */
int kh_decode_partial_gqa(const float* q, int64_t n_groups, int n_q, int head_dim,
                          const uint32_t* k_code, const uint32_t* k_res,
                          const float* k_norms, const float* k_rnorms,
                          const uint32_t* v_code, const uint32_t* v_res,
                          const float* v_norms, const float* v_rnorms,
                          int64_t seq_len, int64_t seq_begin, int64_t seq_end,
                          const float* d_k_host, const float* d_v_host,
                          const float* centroids_host, int n_centroids,
                          float sm_scale, int n_splits, float* partials,
                          int64_t part_stride, int64_t part_offset, void* stream);

/*
 * Decode attention over a compressed K/V cache (split-K / flash-decoding).
 * Not present in the reference, which stops at the scores
 * (KudaHitamQuant_full.py:373-386); softmax(score * sm_scale) . V_hat with
 *   V_hat_s = d (.) H( norm_s c[idx_s] / sqrt(D)
 *                      + r_norm_s sqrt(2/pi) / D * sign_s )
 * (the MSE reconstruction of KudaHitamCUDA.cu:141-149 plus the MSE-optimal
 * dequantisation of the 1-bit QJL residual).  Both caches must carry the
 * residual plane (residual=1 at compression).
 *
 * kh_decode_partial: one query per group, cache rows [seq_begin, seq_end) of
 * each group (group stride seq_len rows).  Writes n_splits partial records of
 * (D+2) floats per group -- (running max, running sum-exp, D rotated-domain
 * accumulators) -- at partials + (g*part_stride + part_offset + split)*(D+2).
 * kh_decode_combine merges n_parts records per group and writes
 * out[g][D] = d (.) H(sum acc) / sum l.  kh_decode_combine_strided does the
 * same with record p of group g at partials + g*group_stride + p*part_stride
 * (strides in floats, so a transposed view of gathered records works).
 * kh_decode_merge merges the same way but writes one record of (D+2) floats
 * per group at merged + g*(D+2), still in the rotated domain: a rank of a
 * sequence-sharded decode merges its own splits with it and gathers one
 * record per group from every rank.  Records with l = 0 are skipped.
 * kh_decode_attn = partial + combine using a caller workspace of
 * kh_decode_workspace_bytes(n_groups, n_splits, D) bytes.
 */
int64_t kh_decode_workspace_bytes(int64_t n_groups, int n_splits, int head_dim);

int kh_decode_partial(const float* q, int64_t n_groups, int head_dim,
                      const uint32_t* k_code, const uint32_t* k_res,
                      const float* k_norms, const float* k_rnorms,
                      const uint32_t* v_code, const uint32_t* v_res,
                      const float* v_norms, const float* v_rnorms,
                      int64_t seq_len, int64_t seq_begin, int64_t seq_end,
                      const float* d_k_host, const float* d_v_host,
                      const float* centroids_host, int n_centroids,
                      float sm_scale, int n_splits, float* partials,
                      int64_t part_stride, int64_t part_offset, void* stream);

int kh_decode_combine(const float* partials, int64_t n_groups, int n_parts,
                      int head_dim, const float* d_v_host, float* out,
                      void* stream);

int kh_decode_combine_strided(const float* partials, int64_t n_groups, int n_parts,
                              int64_t group_stride, int64_t part_stride, int head_dim,
                              const float* d_v_host, float* out, void* stream);

int kh_decode_merge(const float* partials, int64_t n_groups, int n_parts,
                    int64_t group_stride, int64_t part_stride, int head_dim,
                    float* merged, void* stream);

/* Sequence-sharded decode with the record exchange fused into the merge, over
 * peer memory (no counterpart in the reference, which has no decode; this
 * replaces kh_decode_merge + an all-gather + kh_decode_combine_strided).
 * Every rank holds a record buffer [world][n_groups][D+2] and a flag array
 * [world] (uint32, zero before the first call) that all ranks can address
 * (peer or symmetric memory), and a local counter word (zero before the
 * first call).
 * kh_decode_merge_to_peers merges this rank's n_parts split records per
 * group (strides as in kh_decode_merge) and stores the merged record into
 * slot [rank] of every rank's record buffer (peer_records[r] = rank r's
 * buffer, a host array of world device pointers); its last CTA then stores
 * epoch into slot [rank] of every rank's flag array (peer_flags[r]).
 * kh_decode_combine_from_peers waits until all world local flags equal
 * epoch, then writes out[g][D] like kh_decode_combine.  Its wait gives up
 * after about a second, sets bit 2 of kh_device_error() and writes zeros.
 * epoch must be non-zero and differ from the flags' current value; callers
 * alternate two buffer/flag sets between consecutive calls (a rank may be one
 * call ahead of a peer) and increase epoch every call.  world <= 8. */
int kh_decode_merge_to_peers(const float* partials, int64_t n_groups, int n_parts,
                             int64_t group_stride, int64_t part_stride, int head_dim,
                             float* const* peer_records, uint32_t* const* peer_flags,
                             int rank, int world, uint32_t epoch, uint32_t* counter,
                             void* stream);

int kh_decode_combine_from_peers(const float* records, const uint32_t* flags, uint32_t epoch,
                                 int64_t n_groups, int world, int head_dim,
                                 const float* d_v_host, float* out, void* stream);

/* Sequence-sharded decode with the record exchange fused into the partial
 * kernel itself (no counterpart in the reference; replaces
 * kh_decode_partial_gqa + kh_decode_merge + an all-gather +
 * kh_decode_combine_strided, or kh_decode_partial + the two calls above).
 * Every rank holds a record buffer [world][n_groups * n_q][n_splits][D+2]
 * and a flag array [world] (uint32, zero before the first call) that all
 * ranks can address, and a local counter word (zero before the first call).
 * kh_decode_partial_to_peers takes the arguments of kh_decode_partial_gqa
 * except the partials view: each CTA stores its split records into slot
 * [rank] of every rank's record buffer (peer_records[r], a host array of
 * world device pointers; slots a group does not use are marked empty), and
 * the last CTA stores epoch into slot [rank] of every rank's flag array.
 * Only the table kernels (2-level codebook at D = 128 or 256, 4-level at
 * D = 128) take this path: other requests return KH_ENOTSUP.
 * With out != NULL the call also completes the step: once all world flags of
 * this rank carry epoch, the world x n_splits records of each query row are
 * merged into out[n_groups * n_q][D] with d_v_host applied (inside the same
 * kernel when all its CTAs fit on the GPU at once, else by a second kernel
 * on the stream).  With out == NULL, call kh_decode_combine_peer_records.
 * kh_decode_combine_peer_records waits until all world local flags equal
 * epoch and merges the world x n_parts records of each of the n_groups query
 * rows into out[g][D] like kh_decode_combine (kh_decode_combine_from_peers is
 * this call with n_parts = 1).  Its wait gives up after about a second, sets
 * bit 2 of kh_device_error() and writes zeros.  epoch rules as above. */
int kh_decode_partial_to_peers(const float* q, int64_t n_groups, int n_q, int head_dim,
                               const uint32_t* k_code, const uint32_t* k_res,
                               const float* k_norms, const float* k_rnorms,
                               const uint32_t* v_code, const uint32_t* v_res,
                               const float* v_norms, const float* v_rnorms,
                               int64_t seq_len, int64_t seq_begin, int64_t seq_end,
                               const float* d_k_host, const float* d_v_host,
                               const float* centroids_host, int n_centroids,
                               float sm_scale, int n_splits, float* const* peer_records,
                               uint32_t* const* peer_flags, int rank, int world,
                               uint32_t epoch, uint32_t* counter, float* out, void* stream);

int kh_decode_combine_peer_records(const float* records, const uint32_t* flags, uint32_t epoch,
                                   int64_t n_groups, int n_parts, int world, int head_dim,
                                   const float* d_v_host, float* out, void* stream);

int kh_decode_attn(const float* q, int64_t n_groups, int head_dim,
                   const uint32_t* k_code, const uint32_t* k_res,
                   const float* k_norms, const float* k_rnorms,
                   const uint32_t* v_code, const uint32_t* v_res,
                   const float* v_norms, const float* v_rnorms,
                   int64_t seq_len, const float* d_k_host,
                   const float* d_v_host, const float* centroids_host,
                   int n_centroids, float sm_scale, int n_splits,
                   void* workspace, int64_t workspace_bytes, float* out,
                   void* stream);

/*
 * kh_decode_attn_static -- kh_decode_attn without a workspace argument, for
 * callers that cannot allocate device memory when they call: for example a
 * server that has reserved all device memory in its own pool and forbids
 * further allocations, or a C/FFI caller that only holds the buffers it was
 * given.  No counterpart in the reference (it has no decode step at all).
 * The split-K scratch comes from one array of KH_DECODE_STATIC_SCRATCH_BYTES
 * compiled into the library, held on every GPU that loads it until exit.
 * Requests needing more than that return KH_EINVAL (see
 * kh_decode_workspace_bytes).  Calls on the same device share the array:
 * calls whose GPU work overlaps race, so order them.  The first call on a
 * device resolves the array's address (cudaGetSymbolAddress) and should come
 * before any stream capture.  The array is the CURRENT device's: the stream
 * must belong to the current device, and a stream of another device is
 * refused with KH_EINVAL.  n_groups == 0 is a no-op (after the size check).
 * Allocates nothing (no cudaMalloc / cudaFree).
 */
#define KH_DECODE_STATIC_SCRATCH_BYTES (4 * 1024 * 1024)

int kh_decode_attn_static(const float* q, int64_t n_groups, int head_dim,
                          const uint32_t* k_code, const uint32_t* k_res,
                          const float* k_norms, const float* k_rnorms,
                          const uint32_t* v_code, const uint32_t* v_res,
                          const float* v_norms, const float* v_rnorms,
                          int64_t seq_len, const float* d_k_host,
                          const float* d_v_host, const float* centroids_host,
                          int n_centroids, float sm_scale, int n_splits,
                          float* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KUDAHITAM_H_ */
