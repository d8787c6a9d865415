/*
 * kh_oracle.c -- CPU restatement of the reference's KV-compression path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker (and the timed CPU
 * baseline): it is never linked into or called by the engine.
 *
 * Sources restated, all in the reference project:
 *   compress : ultra_fused_full_fusion_kernel_v8, KudaHitamCUDA.cu:13-195
 *   fwht     : fwht_cuda_forward_kernel,          KudaHitamCUDA.cu:233-273
 *   score    : KudahitamCompressorV2.asymmetric_attention_scores,
 *              KudaHitamQuant_full.py:373-377 (with fwht() = the GPU
 *              `forward` kernel, i.e. orthonormal)
 *   compat   : fused_asymmetric_attention_packed_kernel,
 *              KudaHitamCUDA.cu:695-772 (packed-byte scorer); pinned bit for
 *              bit against the reference kernel itself on the GPU
 *              (build_ref.py, tests/test_gpu_reference_kernels.py)
 *   hbba     : ultra_fused_packed_hbba_fusion_kernel, KudaHitamCUDA.cu:285-395
 *              (with whole-row reductions; see khx_hbba_compress) and
 *              hbba_calibrate_cuda_kernel, :423-496
 *
 * Arithmetic follows the kernel in fp32 and in its order: the same
 * butterfly stage order, the same segmented shuffle-tree reductions, the
 * same division by the norm and the same 1e-8 guards.  Built with
 * -ffp-contract=off, so no step is fused unless the source fuses it.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define KHX_F32 0
#define KHX_F16 1
#define KHX_BF16 2

static float load_elt(const void* x, int dtype, int64_t i) {
  if (dtype == KHX_F32) return ((const float*)x)[i];
  if (dtype == KHX_F16) return (float)((const _Float16*)x)[i];
  uint32_t u = (uint32_t)((const uint16_t*)x)[i] << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/*
 * Butterfly stages of the v8 kernel for a row of D = 8 * TPR values, where
 * element e lives in lane e/8, register e%8:
 *   stride 1 and 2 inside a register group of 4   (KudaHitamCUDA.cu:59-71)
 *   strides 8, 16, ... across lanes (xor-shuffle)  (:72-79)
 *   stride 4 inside the 8 registers                (:80-84)
 * Each stage maps (a, b) at (e, e + h) to (a + b, a - b).
 */
static void stage(float* r, int D, int h) {
  for (int e = 0; e < D; ++e) {
    if (e & h) continue;
    const float a = r[e], b = r[e + h];
    r[e] = a + b;
    r[e + h] = a - b;
  }
}

void khx_fwht_v8(float* r, int D) {
  /* the reference kernels need D >= 8 (D/8 lanes per row); smaller rows get
   * the natural stage order */
  if (D < 8) {
    for (int h = 1; h < D; h <<= 1) stage(r, D, h);
    return;
  }
  stage(r, D, 1);
  stage(r, D, 2);
  for (int h = 8; h < D; h <<= 1) stage(r, D, h);
  stage(r, D, 4);
}

/* Segmented __shfl_down_sync tree over TPR lanes (:47-50, :155-158): lane 0
 * ends with the value below. */
static float lane_tree(float* part, int tpr) {
  for (int off = tpr >> 1; off > 0; off >>= 1)
    for (int l = 0; l < off; ++l) part[l] = part[l] + part[l + off];
  return part[0];
}

/* One row of the v8 kernel.  out_* may be NULL. */
static void compress_row(const void* x, int dtype, int64_t row, int64_t stride,
                         int D, const float* d, const float* c, int n_c,
                         uint8_t* idx, float* norm_out, float* kmse,
                         float* rnorm_out, int8_t* signs) {
  const int tpr = D / 8;
  float orig[256], r[256], part[32] = {0};
  for (int e = 0; e < D; ++e) orig[e] = load_elt(x, dtype, row * stride + e);

  /* 1-2. per-lane sum of squares in pairs (:38-44), then the tree */
  for (int l = 0; l < tpr; ++l) {
    float s = 0.0f;
    for (int i = 0; i < 4; ++i) {
      const float a = orig[8 * l + 2 * i], b = orig[8 * l + 2 * i + 1];
      s += a * a + b * b;
    }
    part[l] = s;
  }
  const float sum_sq = lane_tree(part, tpr);
  const float norm = sum_sq > 0 ? sqrtf(sum_sq) : 1e-8f; /* :50 */
  if (norm_out) *norm_out = norm;

  /* 3. r = x * d / norm (:55-56) ; 4. forward FWHT */
  for (int e = 0; e < D; ++e) r[e] = (orig[e] * d[e]) / norm;
  khx_fwht_v8(r, D);

  /* 5. quantise: argmin |y - c|, strict <, lowest index on ties (:91-103) */
  const float f_scale = 1.0f / sqrtf((float)D);
  for (int e = 0; e < D; ++e) {
    const float projected = r[e] * f_scale;
    int best = 0;
    float min_dist = 1e18f;
    for (int k = 0; k < n_c; ++k) {
      const float dist = fabsf(projected - c[k]);
      if (dist < min_dist) {
        min_dist = dist;
        best = k;
      }
    }
    if (idx) idx[e] = (uint8_t)best;
    r[e] = c[best];
  }

  /* 6. reconstruct: FWHT of the centroids (:113-139) */
  khx_fwht_v8(r, D);

  /* 7. k_mse, residual, residual norm (:141-159) */
  const float b_scale = 1.0f / sqrtf((float)D);
  const float m_base = b_scale * norm;
  for (int l = 0; l < tpr; ++l) part[l] = 0.0f;
  for (int e = 0; e < D; ++e) {
    const float k = r[e] * m_base * d[e];
    if (kmse) kmse[e] = k;
    const float diff = orig[e] - k;
    r[e] = diff * d[e];
    part[e / 8] += diff * diff;
  }
  const float res_sum_sq = lane_tree(part, tpr);
  const float r_norm = res_sum_sq > 0 ? sqrtf(res_sum_sq) : 1e-8f; /* :158 */
  if (rnorm_out) *rnorm_out = r_norm;

  /* 8-9. FWHT of d * diff and its sign, >= 0 -> +1 (:161-194) */
  khx_fwht_v8(r, D);
  if (signs)
    for (int e = 0; e < D; ++e) signs[e] = (r[e] >= 0) ? (int8_t)1 : (int8_t)-1;
}

/*
 * Compress n rows.  Any output may be NULL; idx / kmse / signs are [n][D].
 * n_threads <= 0 uses every OpenMP thread.
 */
void khx_compress_v8(const void* x, int dtype, int64_t n, int D, int64_t stride,
                     const float* d, const float* c, int n_c, uint8_t* idx,
                     float* norms, float* kmse, float* rnorms, int8_t* signs,
                     int n_threads) {
#ifdef _OPENMP
  if (n_threads <= 0) n_threads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(n_threads)
#endif
  for (int64_t i = 0; i < n; ++i) {
    compress_row(x, dtype, i, stride, D, d, c, n_c, idx ? idx + i * D : NULL,
                 norms ? norms + i : NULL, kmse ? kmse + i * D : NULL,
                 rnorms ? rnorms + i : NULL, signs ? signs + i * D : NULL);
  }
  (void)n_threads;
}

/* The GPU `forward` op: x <- H x / sqrt(D) (KudaHitamCUDA.cu:233-273). */
void khx_fwht_forward(float* x, int64_t n, int D) {
  const float scale = 1.0f / sqrtf((float)D);
  for (int64_t i = 0; i < n; ++i) {
    float* r = x + i * D;
    khx_fwht_v8(r, D);
    for (int e = 0; e < D; ++e) r[e] = r[e] * scale;
  }
}

/*
 * Reference scores (KudaHitamQuant_full.py:373-377):
 *   term1  = q . k_mse
 *   q_proj = fwht(q * d)          (orthonormal GPU semantics)
 *   out    = term1 + (1/sqrt(D)) (q_proj . signs) r_norm
 * Dot products accumulate in double (the reference runs them through
 * cuBLAS with TF32 allowed, KudaHitamQuant_full.py:26, which is less
 * precise than either).  signs may be NULL (no QJL term).
 * q [G][nq][D], kmse [G][S][D], signs [G][S][D], rnorms [G][S],
 * out [G][nq][S].
 */
void khx_score(const float* q, int64_t G, int nq, int D, const float* kmse,
               const int8_t* signs, const float* rnorms, int64_t S,
               const float* d, float* out) {
  const float scale = (float)(1.0 / sqrt((double)D));
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t g = 0; g < G; ++g) {
    float qp[256];
    for (int j = 0; j < nq; ++j) {
      const float* qv = q + (g * nq + j) * D;
      for (int e = 0; e < D; ++e) qp[e] = qv[e] * d[e];
      khx_fwht_forward(qp, 1, D);
      for (int64_t s = 0; s < S; ++s) {
        const float* k = kmse + (g * S + s) * D;
        double t1 = 0.0, ip = 0.0;
        for (int e = 0; e < D; ++e) t1 += (double)qv[e] * (double)k[e];
        if (signs) {
          const int8_t* sg = signs + (g * S + s) * D;
          for (int e = 0; e < D; ++e) ip += (double)qp[e] * (double)sg[e];
        }
        const double t2 = signs ? (double)scale * ip * (double)rnorms[g * S + s] : 0.0;
        out[(g * nq + j) * S + s] = (float)(t1 + t2);
      }
    }
  }
}

/*
 * Decode attention (no reference counterpart; definition documented in the
 * engine's kh_decode.cu), in double:
 *   p   = softmax(score * sm_scale)
 *   out = sum_s p_s ( v_kmse_s + r_norm_s sqrt(2/pi)/D d (.) H sign_s )
 * q [G][D]; k_* / v_* as for khx_score with one query; out [G][D].
 */
void khx_decode(const float* q, int64_t G, int D, const float* k_kmse,
                const int8_t* k_signs, const float* k_rnorms,
                const float* v_kmse, const int8_t* v_signs,
                const float* v_rnorms, int64_t S, const float* dk,
                const float* dv, float sm_scale, float* out) {
  const double qjl = sqrt(2.0 / M_PI) / (double)D;
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t g = 0; g < G; ++g) {
    float* logits = (float*)malloc(sizeof(float) * (size_t)(S > 0 ? S : 1));
    khx_score(q + g * D, 1, 1, D, k_kmse + g * S * D, k_signs + g * S * D,
              k_rnorms + g * S, S, dk, logits);
    double m = -INFINITY;
    for (int64_t s = 0; s < S; ++s) {
      const double l = (double)logits[s] * (double)sm_scale;
      if (l > m) m = l;
    }
    double acc[256], h[256], L = 0.0;
    for (int e = 0; e < D; ++e) acc[e] = 0.0;
    for (int64_t s = 0; s < S; ++s) {
      const double p = exp((double)logits[s] * (double)sm_scale - m);
      L += p;
      const float* vk = v_kmse + (g * S + s) * D;
      const int8_t* vs = v_signs + (g * S + s) * D;
      /* residual estimate d (.) H sign / D * r_norm sqrt(2/pi) */
      for (int e = 0; e < D; ++e) h[e] = (double)vs[e];
      for (int hh = 1; hh < D; hh <<= 1)
        for (int e = 0; e < D; ++e)
          if (!(e & hh)) {
            const double a = h[e], b = h[e + hh];
            h[e] = a + b;
            h[e + hh] = a - b;
          }
      const double w = qjl * (double)v_rnorms[g * S + s];
      for (int e = 0; e < D; ++e)
        acc[e] += p * ((double)vk[e] + w * (double)dv[e] * h[e]);
    }
    for (int e = 0; e < D; ++e) out[g * D + e] = L > 0 ? (float)(acc[e] / L) : 0.0f;
    free(logits);
  }
}

/*
 * Packed-byte scorer of the reference, KudaHitamCUDA.cu:695-772, in its
 * order: q~ = H(q (.) d) with butterfly strides 1, 2, 4, ... (:723-733),
 * times 1/sqrtf(D) (:734); lane l of the row's warp accumulates elements
 * l, l+32, ... with one fused multiply-add each (k_recon = c[i][v] * k_norm
 * rounded first, :758-761); a butterfly xor reduction over the 32 lanes
 * (:765-768); out = fma(k_norm * scale * sum2, r_norm, sum1) (:771).
 * v = bit (i & 7) of byte (i >> 3) (nibble = 0), or nibble (i & 1) of byte
 * (i >> 1) (nibble = 1).  q fp16 [H][D]; k_packed [H][S][bpt]; signs fp16
 * [H][S][D]; k_norms, r_norms [H][S]; centroids [D][16]; out [H][S].
 */
void khx_compat_score(const _Float16* q, int64_t H, int D, int64_t S,
                      const uint8_t* k_packed, int nibble, const _Float16* signs,
                      const float* d, const float* k_norms, const float* r_norms,
                      const float* centroids, float scale, float* out) {
  const int bpt = nibble ? 128 : 32;
  const float inv = 1.0f / sqrtf((float)D);
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t h = 0; h < H; ++h) {
    float sq[256], qp[256];
    for (int i = 0; i < D; ++i) {
      sq[i] = (float)q[h * D + i];
      qp[i] = sq[i] * d[i];
    }
    for (int len = 1; len < D; len <<= 1) stage(qp, D, len);
    for (int i = 0; i < D; ++i) qp[i] *= inv;
    for (int64_t s = 0; s < S; ++s) {
      const int64_t row = h * S + s;
      const uint8_t* kp = k_packed + row * bpt;
      const _Float16* sg = signs + row * D;
      const float kn = k_norms[row];
      float l1[32], l2[32];
      for (int lane = 0; lane < 32; ++lane) {
        float s1 = 0.f, s2 = 0.f;
        for (int i = lane; i < D; i += 32) {
          const int v = nibble ? (kp[i >> 1] >> ((i & 1) ? 4 : 0)) & 15 : (kp[i >> 3] >> (i & 7)) & 1;
          const float k_recon = centroids[i * 16 + v] * kn;
          s1 = fmaf(qp[i], k_recon, s1);
          s2 = fmaf(sq[i], (float)sg[i], s2);
        }
        l1[lane] = s1;
        l2[lane] = s2;
      }
      for (int o = 16; o > 0; o >>= 1) {
        float n1[32], n2[32];
        for (int lane = 0; lane < 32; ++lane) {
          n1[lane] = l1[lane] + l1[lane ^ o];
          n2[lane] = l2[lane] + l2[lane ^ o];
        }
        memcpy(l1, n1, sizeof(l1));
        memcpy(l2, n2, sizeof(l2));
      }
      const float t2 = kn * scale * l2[0];
      out[row] = fmaf(t2, r_norms[row], l1[0]);
    }
  }
}

/*
 * HBBA mixed-codebook encoder, ultra_fused_packed_hbba_fusion_kernel
 * (KudaHitamCUDA.cu:285-395), with the reductions it intends.  The
 * reference sums ||x||^2 and the residual's squares with a warp shuffle
 * only (:312-314, :377) while 256 threads hold the row, so for D > 32 each
 * warp divides its 32 elements by its own partial norm and the stored norms
 * cover elements 0..31; its thread 0 also copies the packed bytes out
 * (:378-381) with no barrier after the other warps' atomicOr.  Here both
 * sums run over the whole row.  Per row:
 *   norm   = sqrtf(sum x^2 + 1e-8)                                 (:313-315)
 *   y      = H(x / norm (.) d) / sqrt(D), Sylvester order          (:323-341)
 *   n_c    = 16 if the layer is HBBA and bit i of mask is set, else 2 (:345-347)
 *   idx_i  = argmin_c |y_i - half(c[i][c])|, strict <, lowest index (:349-353)
 *   packed = nibble (i & 1) of byte i >> 1 (HBBA layer, 128 bytes per row)
 *            or bit (i & 7) of byte i >> 3 (32 bytes per row)        (:356-366)
 *   diff_i = y_i - half(c[i][idx_i]); r_norm = sqrtf(sum diff^2 * D + 1e-8)
 *   signs  = half(H diff), unnormalised                            (:368-395)
 * Sums of squares accumulate in double.  x [n][D]; cent [D][16];
 * mask [8]; packed [n][32 or 128] (zero-filled); signs [n][D].
 */
void khx_hbba_compress(const void* x, int dtype, int64_t n, int D, const float* d,
                       const float* cent, const uint32_t* mask, int is_hbba,
                       uint8_t* packed, float* norms, float* rnorms, _Float16* signs) {
  const int bpt = is_hbba ? 128 : 32;
  const float f_scale = 1.0f / sqrtf((float)D);
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int64_t r = 0; r < n; ++r) {
    float v[256], c16[256][16];
    for (int i = 0; i < D; ++i)
      for (int c = 0; c < 16; ++c) c16[i][c] = (float)(_Float16)cent[i * 16 + c];
    double ss = 0.0;
    for (int i = 0; i < D; ++i) {
      v[i] = load_elt(x, dtype, r * D + i);
      ss += (double)v[i] * (double)v[i];
    }
    const float norm = sqrtf((float)ss + 1e-8f);
    norms[r] = norm;
    const float inv = 1.0f / norm;
    for (int i = 0; i < D; ++i) v[i] = (v[i] * inv) * d[i];
    for (int h = 1; h < D; h <<= 1) stage(v, D, h);
    uint8_t* pk = packed + r * bpt;
    memset(pk, 0, bpt);
    double rs = 0.0;
    for (int i = 0; i < D; ++i) {
      const float y = v[i] * f_scale;
      const int n_c = (is_hbba && ((mask[i >> 5] >> (i & 31)) & 1u)) ? 16 : 2;
      int best = 0;
      float md = 1e18f;
      for (int c = 0; c < n_c; ++c) {
        const float dist = fabsf(y - c16[i][c]);
        if (dist < md) {
          md = dist;
          best = c;
        }
      }
      if (is_hbba) pk[i >> 1] |= (uint8_t)((best & 15) << ((i & 1) ? 4 : 0));
      else pk[i >> 3] |= (uint8_t)((best & 1) << (i & 7));
      const float diff = y - c16[i][best];
      rs += (double)diff * (double)diff;
      v[i] = diff;
    }
    rnorms[r] = sqrtf((float)rs * (float)D + 1e-8f);
    for (int h = 1; h < D; h <<= 1) stage(v, D, h);
    for (int i = 0; i < D; ++i) signs[r * D + i] = (_Float16)v[i];
  }
}

/*
 * HBBA calibrator, hbba_calibrate_cuda_kernel (KudaHitamCUDA.cu:423-496):
 * per dimension d with n_c = n_map[d] levels (<= 16), centroids start
 * uniform between the sample's min and max, c_k = min + k (max - min) /
 * max(1, n_c - 1) (:458-462), then 10 rounds of nearest-centroid assignment
 * (strict <, lowest index) and mean update, a centroid with no samples
 * keeping its value (:466-488).  Sums accumulate in double (the reference
 * adds with float atomics in unspecified order).  sample [n][D]; out
 * [D][16], unused entries 0.
 */
void khx_hbba_calibrate(const float* sample, int64_t n, int D, const int* n_map, float* out) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
  for (int d = 0; d < D; ++d) {
    const int n_c = n_map[d] < 1 ? 1 : (n_map[d] > 16 ? 16 : n_map[d]);
    float mn = 1e18f, mx = -1e18f;
    for (int64_t i = 0; i < n; ++i) {
      const float v = sample[i * D + d];
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    float c[16];
    for (int k = 0; k < n_c; ++k)
      c[k] = mn + (float)k * (mx - mn) / fmaxf(1.0f, (float)(n_c - 1));
    for (int it = 0; it < 10; ++it) {
      double sum[16] = {0};
      int64_t cnt[16] = {0};
      for (int64_t i = 0; i < n; ++i) {
        const float v = sample[i * D + d];
        int best = 0;
        float md = 1e18f;
        for (int k = 0; k < n_c; ++k) {
          const float dist = fabsf(v - c[k]);
          if (dist < md) {
            md = dist;
            best = k;
          }
        }
        sum[best] += v;
        cnt[best] += 1;
      }
      for (int k = 0; k < n_c; ++k)
        if (cnt[k] > 0) c[k] = (float)(sum[k] / (double)cnt[k]);
    }
    for (int k = 0; k < 16; ++k) out[d * 16 + k] = k < n_c ? c[k] : 0.0f;
  }
}

int khx_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
