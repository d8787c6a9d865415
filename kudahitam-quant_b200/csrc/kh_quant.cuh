// kh_quant.cuh -- element conversion and the Lloyd-Max quantiser shared by
// the SIMT and tensor-core compressors, so both produce identical bits from
// identical transformed values.
#pragma once

#include <cstring>

#include "kh_common.cuh"
#include "kh_internal.h"

namespace kh {

// ---- conversion of one 16-byte chunk (already sign-flipped by d) --------
template <typename T>
struct Chunk;

template <>
struct Chunk<__nv_bfloat16> {
  static constexpr int kElems = 8;
  template <class P>
  __device__ __forceinline__ static void load(const uint4 v, const P& prm,
                                              int e0, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t m = prm.dflip[(e0 >> 1) + j];
      const uint32_t u = w[j] ^ m;
      f[2 * j] = __uint_as_float(u << 16);
      f[2 * j + 1] = __uint_as_float(u & 0xffff0000u);
    }
  }
};

template <>
struct Chunk<__half> {
  static constexpr int kElems = 8;
  template <class P>
  __device__ __forceinline__ static void load(const uint4 v, const P& prm,
                                              int e0, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t u = w[j] ^ prm.dflip[(e0 >> 1) + j];
      __half2 h;
      memcpy(&h, &u, 4);
      const float2 t = __half22float2(h);
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
};

template <>
struct Chunk<float> {
  static constexpr int kElems = 4;
  template <class P>
  __device__ __forceinline__ static void load(const uint4 v, const P& prm,
                                              int e0, float* f) {
    f[0] = __uint_as_float(v.x ^ prm.dflip[e0 + 0]);
    f[1] = __uint_as_float(v.y ^ prm.dflip[e0 + 1]);
    f[2] = __uint_as_float(v.z ^ prm.dflip[e0 + 2]);
    f[3] = __uint_as_float(v.w ^ prm.dflip[e0 + 3]);
  }
};

// Quantise 32 consecutive transformed values u[e0 .. e0+31] of one row.
// rs = 1 / (||x|| sqrt(D)) turns u into the orthonormal projection y.
// Returns the code word(s) and the residual sign word; accumulates
// sum (y - c[idx])^2 into acc.
template <int CK, bool RES>
struct Quant;

// c0 == -c1: idx = [y > 0] read from the sign bit of q = 0 - y (computed as
// fma(-u, rs, +0) so that y = +-0 gives q = +0 and idx 0, the reference's
// lowest-index tie rule, KudaHitamCUDA.cu:96-99).
// y - c[idx] = copysign(c1, q) - q.
template <bool RES>
struct Quant<kCbSym2, RES> {
  static constexpr int kCodeWords = 1;
  template <class P>
  __device__ __forceinline__ static void run(const float* u, float rs,
                                             const P& prm, uint32_t* code,
                                             uint32_t& resw, float2& acc) {
    const uint32_t c1b = __float_as_uint(prm.cb.c[1]);
    const float2 nrs = make_float2(-rs, -rs);
    const float2 zero = make_float2(0.f, 0.f);
    const float2 neg1 = make_float2(-1.f, -1.f);
    uint32_t cw = 0, rw = 0;
#pragma unroll
    for (int k = 30; k >= 0; k -= 2) {
      const float2 q = __ffma2_rn(make_float2(u[k], u[k + 1]), nrs, zero);
      cw = push_sign(cw, q.y);
      cw = push_sign(cw, q.x);
      if (RES) {
        const float2 cs =
            make_float2(__uint_as_float((__float_as_uint(q.x) & 0x80000000u) | c1b),
                        __uint_as_float((__float_as_uint(q.y) & 0x80000000u) | c1b));
        const float2 v = __ffma2_rn(q, neg1, cs);  // cs - q
        rw = push_sign(rw, v.y);
        rw = push_sign(rw, v.x);
        acc = __ffma2_rn(v, v, acc);
      }
    }
    code[0] = cw;
    resw = ~rw;  // residual bit = [v >= 0]; v is never -0 here
  }
};

// Two arbitrary levels: idx = [y > mid], q = mid - y.
template <bool RES>
struct Quant<kCbGen2, RES> {
  static constexpr int kCodeWords = 1;
  template <class P>
  __device__ __forceinline__ static void run(const float* u, float rs,
                                             const P& prm, uint32_t* code,
                                             uint32_t& resw, float2& acc) {
    const float mid = prm.cb.mid[0];
    const float a0 = prm.cb.sel[0], a1 = prm.cb.sel[1];
    uint32_t cw = 0, rw = 0;
    float s = 0.f;
#pragma unroll
    for (int k = 31; k >= 0; --k) {
      const float q = __fmaf_rn(-u[k], rs, mid);
      cw = push_sign(cw, q);
      if (RES) {
        const float v = (__float_as_int(q) < 0 ? a1 : a0) - q;
        rw = push_sign(rw, v);
        s = __fmaf_rn(v, v, s);
      }
    }
    acc.x += s;
    code[0] = cw;
    resw = ~rw;
  }
};

// Four levels (bits=2): idx = [y>m01] + [y>m12] + [y>m23], packed 2 bits per
// element, element i at bits 2*(i&15) of word i>>4.
template <bool RES>
struct Quant<kCbGen4, RES> {
  static constexpr int kCodeWords = 2;
  template <class P>
  __device__ __forceinline__ static void run(const float* u, float rs,
                                             const P& prm, uint32_t* code,
                                             uint32_t& resw, float2& acc) {
    const float m0 = prm.cb.mid[0], m1 = prm.cb.mid[1], m2 = prm.cb.mid[2];
    const float c0 = prm.cb.c[0], c1 = prm.cb.c[1], c2 = prm.cb.c[2],
                c3 = prm.cb.c[3];
    uint32_t cw[2] = {0u, 0u}, rw = 0;
    float s = 0.f;
#pragma unroll
    for (int k = 31; k >= 0; --k) {
      const float y = u[k] * rs;
      const bool b1 = y > m1;
      const bool b2 = b1 ? (y > m2) : (y > m0);
      const uint32_t idx = (b1 ? 2u : 0u) | (b2 ? 1u : 0u);
      cw[k >> 4] = (cw[k >> 4] << 2) | idx;
      if (RES) {
        const float c = b1 ? (b2 ? c3 : c2) : (b2 ? c1 : c0);
        const float v = y - c;
        rw = push_sign(rw, v);
        s = __fmaf_rn(v, v, s);
      }
    }
    acc.x += s;
    code[0] = cw[0];
    code[1] = cw[1];
    resw = ~rw;
  }
};

// NG groups of 32 transformed values, symmetric 2-level codebook, with the
// 2*NG bit-packing chains interleaved (a single chain of 32 dependent funnel
// shifts per word stalls on latency).  Residual bit via
//   v = y - c[idx] >= 0  <=>  idx XOR [|y| < c1]     (except |y| == c1 exactly)
// and sum (y - c[idx])^2 = sum (|y| - c1)^2.
template <int NG, bool RES>
__device__ __forceinline__ void quant_sym2_groups(const float (&u)[NG][32], float rs,
                                                  float c1, uint32_t* code,
                                                  uint32_t* resw, float2& acc,
                                                  uint32_t row_mask = 0xffffffffu) {
  // The code bit is 1 for y > 0: push the sign bits of u itself (rs > 0)
  // and invert the finished word.  An exact +0 then reads as 1 where the
  // reference's strict argmin picks index 0; such elements are ties inside
  // the 1e-6 band and either index is correct.  An all-zero row (row_mask
  // 0) keeps index 0 throughout, as in the reference.
  uint32_t cw[NG], sw[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) cw[g] = sw[g] = 0u;
  float2 a2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int k = 30; k >= 0; k -= 2) {
#pragma unroll
    for (int g = 0; g < NG; ++g) {
      cw[g] = push_sign(cw[g], u[g][k + 1]);
      cw[g] = push_sign(cw[g], u[g][k]);
      if (RES) {
        const float t0 = __fmaf_rn(fabsf(u[g][k]), rs, -c1);
        const float t1 = __fmaf_rn(fabsf(u[g][k + 1]), rs, -c1);
        sw[g] = push_sign(sw[g], t1);
        sw[g] = push_sign(sw[g], t0);
        const float2 t = make_float2(t0, t1);
        a2[g & 1] = __ffma2_rn(t, t, a2[g & 1]);
      }
    }
  }
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    const uint32_t c = ~cw[g] & row_mask;
    code[g] = c;
    if (RES) resw[g] = c ^ sw[g];
  }
  acc = __fadd2_rn(acc, __fadd2_rn(a2[0], a2[1]));
}

}  // namespace kh
