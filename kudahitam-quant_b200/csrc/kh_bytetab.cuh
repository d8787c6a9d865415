// kh_bytetab.cuh -- helpers shared by the kernels that read packed planes a
// byte at a time through shared-memory tables (decode attention, scores).
//
// Bank-conflict-free addressing: a table entry (slot j, byte value v) lives
// in bank j.  Lane l of a warp visits a lane-dependent byte position p at
// step k (P = D/8 byte positions per plane), in copy c = l / P of the table
// (32 / P copies), slot j = p + P c, such that the 32 lanes of a warp always
// touch 32 distinct banks.  Two orders are used:
// * rotated, p = (k + l) mod P: the plane's words are rotated by
//   (l mod P) / 4 and funnel-shifted by 8 (l mod 4) bits;
// * XOR, p = k ^ (l mod P): the words are permuted by (l mod P) / 4 and a
//   per-lane byte-permute selector picks byte (k mod 4) ^ (l mod 4), so no
//   shift is needed (two to four fewer instructions per plane word; measured
//   2-4 % faster in the decode and score kernels).
#pragma once

#include <cstdint>
#include <type_traits>
#include <utility>

#include <cuda_runtime.h>

#include "kh_common.cuh"

namespace kh {

// Calls f(std::integral_constant<int, I>) for I = 0 .. N-1, fully unrolled.
template <class F, int... I>
__device__ __forceinline__ void static_for_impl(F&& f, std::integer_sequence<int, I...>) {
  (f(std::integral_constant<int, I>{}), ...);
}
template <int N, class F>
__device__ __forceinline__ void static_for(F&& f) {
  static_for_impl(f, std::make_integer_sequence<int, N>{});
}

// Rotated view of one row plane: byte k of the result = plane byte
// (k + r) mod P, r = lane mod P.
template <int D>
__device__ __forceinline__ void load_rotated(const uint32_t* __restrict__ plane, int wr,
                                             int bs, uint32_t (&rot)[D / 32]) {
  constexpr int kW = D / 32;
  uint32_t w[kW];
  static_for<kW>([&](auto ic) {
    constexpr int i = decltype(ic)::value;
    w[i] = __ldg(plane + ((i + wr) & (kW - 1)));
  });
  static_for<kW>([&](auto ic) {
    constexpr int i = decltype(ic)::value;
    rot[i] = __funnelshift_r(w[i], w[(i + 1) % kW], bs);
  });
}

// byte k of a rotated plane, zero-extended
template <int K>
__device__ __forceinline__ uint32_t byte_of(const uint32_t* rot) {
  return __byte_perm(rot[K >> 2], 0u, 0x4440u + (K & 3));
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += red[i];
  return r;
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}


// Fills entries 0..31 of the 256 table rows (row stride 64 floats):
// T[v][slot] = sum of q~ over the set bits of byte value v at the slot's
// byte position slot mod (D / 8).  Thread t of a 256-thread block fills slot
// t mod 32 for the byte values v = t / 32 + 8 k (k < 32): the low nibble of
// v is t / 32 + 8 (k mod 2), the high nibble k / 2; the eight q~ elements of
// the byte position stay in registers.
template <int D>
__device__ __forceinline__ void build_byte_table(float* tab, const float* qt, int t) {
  const int slot = t & 31, pos = slot % (D / 8), w = t >> 5;
  float qb[8];
#pragma unroll
  for (int b = 0; b < 8; ++b) qb[b] = qt[8 * pos + b];
  float lo[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int nv = w + 8 * h;
    lo[h] = ((nv & 1) ? qb[0] : 0.f) + ((nv & 2) ? qb[1] : 0.f) +
            ((nv & 4) ? qb[2] : 0.f) + ((nv & 8) ? qb[3] : 0.f);
  }
  float* tf = tab + slot;
  static_for<32>([&](auto kc) {
    constexpr int k = decltype(kc)::value, hv = k >> 1;
    float hi = 0.f;
    if constexpr ((hv & 1) != 0) hi += qb[4];
    if constexpr ((hv & 2) != 0) hi += qb[5];
    if constexpr ((hv & 4) != 0) hi += qb[6];
    if constexpr ((hv & 8) != 0) hi += qb[7];
    tf[(w + 8 * k) * 64] = lo[k & 1] + hi;
  });
}

// Byte address 256 * (byte B of x) + (byte B of slots): one byte-permute.
// slots packs four lane slot offsets (each 4 * slot < 128) one per byte;
// result bytes 2 and 3 replicate the (zero) sign bit of the slot byte.
// (prmt.b32 generic mode: a selector nibble with its msb set replicates the
// sign bit of the selected byte.)
template <int B>
__device__ __forceinline__ uint32_t tab_addr(uint32_t x, uint32_t slots) {
  constexpr uint32_t ys = 4u + B;  // selector of byte B of `slots`
  constexpr uint32_t sel = ((8u | ys) << 12) | ((8u | ys) << 8) | (B << 4) | ys;
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(slots), "n"(sel));
  return r;
}

// 2^x by the SFU's approximate base-2 exponential (ex2.approx.ftz: relative
// error about 2^-22, -inf -> +0, results below 2^-126 flushed to zero).  The
// softmax weights here are 2^(logit - running max) <= 1, where a flushed
// weight is negligible against the row that set the max.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// L2 eviction-priority policies (createpolicy) and loads that carry one.
// Streams read once are loaded evict-first; values read again by the same
// CTA later (decode's V norms, phase 1 then phase 2) evict-last, so the
// rows streaming past in between do not push them out of L2.
// (l2_policy_evict_first is in kh_common.cuh, with the TMA helpers.)
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ float ldg_policy(const float* p, uint64_t pol) {
  float v;
  asm("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ uint32_t ldg_policy(const uint32_t* p, uint64_t pol) {
  uint32_t v;
  asm("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ uint4 ldg_policy(const uint4* p, uint64_t pol) {
  uint4 v;
  asm("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(pol));
  return v;
}

// load_plane with an L2 policy (see load_plane below for the layouts).
template <int D>
__device__ __forceinline__ void load_plane_policy(const uint32_t* __restrict__ plane, int wr,
                                                  uint64_t pol, uint32_t (&w)[D / 32]) {
  if constexpr (D == 128) {
    const uint4 v = ldg_policy(reinterpret_cast<const uint4*>(plane), pol);
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  } else {
    constexpr int kW = D / 32;
    static_for<kW>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      w[i] = ldg_policy(plane + ((i + wr) & (kW - 1)), pol);
    });
  }
}

// Row-per-thread table lookups read a plane in two steps, so that the
// rotation's data-dependent instructions run where the bytes are used, one
// batch after the load was issued, and never stall the loads behind them.
// load_plane: D = 128, one 16-byte load per row (4 L1 wavefronts per warp
// instead of 16 for four 4-byte loads); D = 256, eight 4-byte loads whose
// word order is already rotated by wr through the addresses.
template <int D>
__device__ __forceinline__ void load_plane(const uint32_t* __restrict__ plane, int wr,
                                           uint32_t (&w)[D / 32]) {
  if constexpr (D == 128) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(plane));
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  } else {
    constexpr int kW = D / 32;
    static_for<kW>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      w[i] = __ldg(plane + ((i + wr) & (kW - 1)));
    });
  }
}

// rotate_plane: the rotated view of a plane read by load_plane (byte k =
// plane byte (k + r) mod P, r = 4 wr + bs / 8).  D = 128 rotates the words
// by wr here (two select stages); both then shift by bs bits.
template <int D>
__device__ __forceinline__ void rotate_plane(const uint32_t (&w)[D / 32], int wr, int bs,
                                             uint32_t (&rot)[D / 32]) {
  if constexpr (D == 128) {
    const bool h = wr & 2, o = wr & 1;
    const uint32_t y0 = h ? w[2] : w[0], y1 = h ? w[3] : w[1];
    const uint32_t y2 = h ? w[0] : w[2], y3 = h ? w[1] : w[3];
    const uint32_t z0 = o ? y1 : y0, z1 = o ? y2 : y1;
    const uint32_t z2 = o ? y3 : y2, z3 = o ? y0 : y3;
    rot[0] = __funnelshift_r(z0, z1, bs);
    rot[1] = __funnelshift_r(z1, z2, bs);
    rot[2] = __funnelshift_r(z2, z3, bs);
    rot[3] = __funnelshift_r(z3, z0, bs);
  } else {
    constexpr int kW = D / 32;
    static_for<kW>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      rot[i] = __funnelshift_r(w[i], w[(i + 1) % kW], bs);
    });
  }
}

// ---------------------------------------------------------------------------
// XOR byte order.  Lane l visits byte position p = k ^ r at step k, r = l mod
// P (P = D / 8 positions, a power of two), in table copy l / P: slot
// j = p + P (l / P).  For a fixed k the P lanes of one copy cover all P
// positions, so a warp's 32 lookups still hit 32 distinct banks.  Position p
// sits in word p >> 2 at byte p & 3; with the words permuted per lane to
// z[i] = w[i ^ (r >> 2)], step k reads word z[k >> 2] (a fixed register) at
// byte (k & 3) ^ (r & 3), which a per-lane prmt selector picks out, so no
// funnel shift is needed.

// prmt selectors of the four byte steps within a word: result byte 0 = byte
// b of the slot word, byte 1 = byte b ^ (r & 3) of the plane word, bytes 2
// and 3 replicate the (zero) sign bit of the slot byte.
struct XorSel {
  uint32_t s[4];
};
__device__ __forceinline__ XorSel xor_selectors(int r) {
  XorSel x;
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t ys = 4u + b;
    x.s[b] = ((8u | ys) << 12) | ((8u | ys) << 8) | ((uint32_t)(b ^ (r & 3)) << 4) | ys;
  }
  return x;
}

// Byte address 256 * (selected byte of x) + (byte b of slots), the selector
// from xor_selectors (one byte-permute with a register selector).
__device__ __forceinline__ uint32_t tab_addr_x(uint32_t x, uint32_t slots, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(slots), "r"(sel));
  return r;
}

// Packed slot offsets of the XOR order: byte j of the result = 4 * slot of
// step k = 4 m + j, for a lane with XOR mask r in table copy cp (P positions
// per copy).
template <int P>
__device__ __forceinline__ uint32_t xor_slots(int m, int r, int cp) {
  uint32_t w = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) w |= (4u * (uint32_t)(((4 * m + j) ^ r) + P * cp)) << (8 * j);
  return w;
}

// load_plane_policy in the XOR order: D = 128 one 16-byte load (permuted by
// xor_plane afterwards); D = 256 eight 4-byte loads whose word order is
// already permuted (word i ^ wx at register i) through the addresses.
template <int D>
__device__ __forceinline__ void load_plane_x(const uint32_t* __restrict__ plane, int wx,
                                             uint64_t pol, uint32_t (&w)[D / 32]) {
  if constexpr (D == 128) {
    const uint4 v = ldg_policy(reinterpret_cast<const uint4*>(plane), pol);
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  } else {
    static_for<D / 32>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      w[i] = ldg_policy(plane + (i ^ wx), pol);
    });
  }
}

// load_plane_x without an L2 policy.
template <int D>
__device__ __forceinline__ void load_plane_xg(const uint32_t* __restrict__ plane, int wx,
                                              uint32_t (&w)[D / 32]) {
  if constexpr (D == 128) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(plane));
    w[0] = v.x;
    w[1] = v.y;
    w[2] = v.z;
    w[3] = v.w;
  } else {
    static_for<D / 32>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      w[i] = __ldg(plane + (i ^ wx));
    });
  }
}

// The XOR view of a plane read by load_plane_x: z[i] = plane word i ^ wx.
// D = 128 permutes the words here (two select stages); D = 256 got them
// permuted by its load addresses.
template <int D>
__device__ __forceinline__ void xor_plane(const uint32_t (&w)[D / 32], int wx,
                                          uint32_t (&z)[D / 32]) {
  if constexpr (D == 128) {
    const bool h = wx & 2, o = wx & 1;
    const uint32_t y0 = h ? w[2] : w[0], y1 = h ? w[3] : w[1];
    const uint32_t y2 = h ? w[0] : w[2], y3 = h ? w[1] : w[3];
    z[0] = o ? y1 : y0;
    z[1] = o ? y0 : y1;
    z[2] = o ? y3 : y2;
    z[3] = o ? y2 : y3;
  } else {
    static_for<D / 32>([&](auto ic) {
      constexpr int i = decltype(ic)::value;
      z[i] = w[i];
    });
  }
}

// A 32-byte plane (8 words) in the XOR order, as two 16-byte loads: bit 2
// of wx swaps the two halves through the addresses, and xor_plane32 then
// permutes the words within each half by wx mod 4, so that z[i] = plane word
// i ^ wx.  (Eight 4-byte loads at permuted addresses touch four times as
// many L1 wavefronts per warp.)
__device__ __forceinline__ void load_plane32_x(const uint32_t* __restrict__ plane, int wx,
                                               uint64_t pol, uint32_t (&w)[8]) {
  const int hs = (wx >> 2) & 1;
  const uint4 a = ldg_policy(reinterpret_cast<const uint4*>(plane) + hs, pol);
  const uint4 b = ldg_policy(reinterpret_cast<const uint4*>(plane) + (hs ^ 1), pol);
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}
__device__ __forceinline__ void load_plane32_xg(const uint32_t* __restrict__ plane, int wx,
                                                uint32_t (&w)[8]) {
  const int hs = (wx >> 2) & 1;
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(plane) + hs);
  const uint4 b = __ldg(reinterpret_cast<const uint4*>(plane) + (hs ^ 1));
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}
__device__ __forceinline__ void xor_plane32(const uint32_t (&w)[8], int wx, uint32_t (&z)[8]) {
  const uint32_t lo[4] = {w[0], w[1], w[2], w[3]}, hi[4] = {w[4], w[5], w[6], w[7]};
  uint32_t zl[4], zh[4];
  xor_plane<128>(lo, wx, zl);
  xor_plane<128>(hi, wx, zh);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    z[i] = zl[i];
    z[4 + i] = zh[i];
  }
}

}  // namespace kh
