// kh_common.cuh -- shared device helpers for the sm_100a kernels.
//
// Inline-PTX wrappers for mbarriers and TMA (cp.async.bulk.tensor), written
// from the PTX ISA.  Every TMA load here is a plain per-CTA load.
#pragma once

#include <utility>

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "kudahitam.h"

namespace kh {

// Bits of the sticky device error word (kh_device_error()).
enum : uint32_t {
  kErrWaitTimeout = 1u << 0,   // an mbarrier wait gave up
  kErrBadSegment = 1u << 1,    // tile index fell outside every segment
  kErrPeerTimeout = 1u << 2,   // a peer's record flag did not arrive in time
};

// The error word lives in kh_api.cu; kernels receive its address.
__device__ __forceinline__ void flag_error(uint32_t* err, uint32_t bits) {
  if (err) atomicOr(err, bits);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up after
// ~2^31 clock cycles (about a second at B200 clocks), records
// kErrWaitTimeout and returns false; the caller must then stop issuing work.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > (1ll << 31)) {
      flag_error(err, kErrWaitTimeout);
      return false;
    }
  }
  return true;
}

// ------------------------------------------- programmatic dependent launch
// Wait until the previous grid in the stream has completed and its memory
// operations are visible (returns at once when this grid was not launched
// as a programmatic dependent).
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Allow the next grid in the stream (if launched as a programmatic
// dependent) to be scheduled once every CTA of this grid has signalled.
__device__ __forceinline__ void grid_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Host: launch with programmatic stream serialisation, so that the kernel's
// CTAs may start (and run their parameter-only set-up) while the previous
// kernel in the stream finishes.  The kernel must call grid_dependency_wait()
// before it touches global memory that earlier work may write or read.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_programmatic(void (*kern)(KArgs...), dim3 grid, dim3 block,
                                       size_t smem, cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m))
               : "memory");
}

// 2-D tiled bulk tensor load global -> shared, completion on an mbarrier.
// x = innermost coordinate (elements), y = row.  The caller guarantees
// x * element_size is a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* m,
                                            int32_t x, int32_t y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
               : "=l"(p));
  return p;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// Streaming (evict-first) 16-byte global store.
__device__ __forceinline__ void stg128_cs(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void stg32_cs(void* p, uint32_t v) {
  asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---------------------------------------------------------------- bits
// (hi:lo) << 1, upper word: shifts the sign bit of `f` into the low end of w.
__device__ __forceinline__ uint32_t push_sign(uint32_t w, float f) {
  return __funnelshift_l(__float_as_uint(f), w, 1);
}

// ---------------------------------------------------------------- FWHT
// One packed butterfly stage of stride H >= 2 over N register values: pairs
// adjacent registers and runs on the sm_100 f32x2 datapath (one instruction
// per two butterfly halves).  H is a template parameter so every loop has
// compile-time bounds and r[] stays in registers.
template <int N, int H>
__device__ __forceinline__ void fwht_stage_x2(float (&r)[N]) {
  const float2 neg1 = make_float2(-1.f, -1.f);
#pragma unroll
  for (int i = 0; i < N; i += 2 * H) {
#pragma unroll
    for (int j = i; j < i + H; j += 2) {
      const float2 a = make_float2(r[j], r[j + 1]);
      const float2 b = make_float2(r[j + H], r[j + H + 1]);
      const float2 s = __fadd2_rn(a, b);
      const float2 t = __ffma2_rn(b, neg1, a);  // a - b, exact
      r[j] = s.x;
      r[j + 1] = s.y;
      r[j + H] = t.x;
      r[j + H + 1] = t.y;
    }
  }
}

template <int N, int H>
__device__ __forceinline__ void fwht_stages_x2(float (&r)[N]) {
  if constexpr (H < N) {
    fwht_stage_x2<N, H>(r);
    fwht_stages_x2<N, 2 * H>(r);
  }
}

// Unnormalised Sylvester Walsh-Hadamard transform of N register values
// (H_N x with H_{2n} = [[H_n, H_n], [H_n, -H_n]]).  Stage 1 runs as scalar
// FADDs, stages 2..N/2 packed.
template <int N>
__device__ __forceinline__ void fwht_regs(float (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; i += 2) {
    const float a = r[i], b = r[i + 1];
    r[i] = a + b;
    r[i + 1] = a - b;
  }
  fwht_stages_x2<N, 2>(r);
}

}  // namespace kh
