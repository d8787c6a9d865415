// kh_decode_static.cu -- decode attention that allocates nothing, not even
// its split-K scratch.
//
// kh_decode_attn needs a workspace of (D+2) floats per (group, split): the
// split-K partial records.  Some callers cannot allocate device memory at the
// point of the call.  Examples: an inference server that reserves all device
// memory in its own pool up front and forbids later cudaMalloc calls; a C or
// FFI caller that only holds the device buffers it was handed and has no
// device allocator of its own; a latency-critical decode loop where the
// implicit synchronisation of cudaMalloc/cudaFree is not acceptable.  For
// them, kh_decode_attn_static takes the records from a fixed array compiled
// into this library (g_decode_scratch below).  The caller still passes the
// query, the caches and the output.
//
// Properties of the shared array:
// * KH_DECODE_STATIC_SCRATCH_BYTES (4 MiB) on every GPU that loads the
//   library, held until the process exits;
// * requests needing more are rejected with KH_EINVAL before any GPU work;
// * one array per device, shared by every call on that device: calls whose
//   GPU work overlaps (different streams, threads or processes sharing a
//   context) race on it, so callers must order them;
// * nothing needs clearing between calls: every call rewrites each record
//   it reads.
//
// The first call on a device resolves the array's device address with
// cudaGetSymbolAddress, with that device current.  Make that first call
// before any stream capture.  The stream must belong to the current device
// (checked: a stream of another device is refused with KH_EINVAL).
#include <cuda_runtime.h>

#include <mutex>

#include "kh_internal.h"
#include "kudahitam.h"

namespace kh {
namespace {

constexpr int64_t kScratchFloats = KH_DECODE_STATIC_SCRATCH_BYTES / 4;

// The scratch itself.  In host code this name is only a stand-in for the
// symbol, never a device address: host code must use the pointer obtained
// from cudaGetSymbolAddress below.
static __device__ __align__(256) float g_decode_scratch[kScratchFloats];

constexpr int kMaxDev = 64;
std::mutex g_mu;
float* g_ptr[kMaxDev] = {};

// Device address of the scratch on the current device (set up once per
// device); nullptr if the runtime call fails.  The address belongs to the
// current device, so the caller first checks that the stream runs there.
float* scratch_ptr(int dev) {
  if (dev < 0 || dev >= kMaxDev) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess) return nullptr;
    g_ptr[dev] = static_cast<float*>(p);
  }
  return g_ptr[dev];
}

}  // namespace
}  // namespace kh

extern "C" int kh_decode_attn_static(
    const float* q, int64_t n_groups, int head_dim, const uint32_t* k_code,
    const uint32_t* k_res, const float* k_norms, const float* k_rnorms,
    const uint32_t* v_code, const uint32_t* v_res, const float* v_norms,
    const float* v_rnorms, int64_t seq_len, const float* d_k_host,
    const float* d_v_host, const float* centroids_host, int n_centroids,
    float sm_scale, int n_splits, float* out, void* stream) {
  const int64_t need = kh_decode_workspace_bytes(n_groups, n_splits, head_dim);
  if (need < 0) return KH_EINVAL;
  if (need > KH_DECODE_STATIC_SCRATCH_BYTES) return KH_EINVAL;  // too big for the array
  if (n_groups == 0) return KH_OK;
  // The array's address is per device: resolving it for the current device
  // while the stream belongs to another GPU would hand that GPU's kernels
  // an address of the wrong device.  Such a call is refused.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return KH_ECUDA;
  if (stream) {
    int sdev = -1;
    if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev) != cudaSuccess)
      return KH_ECUDA;
    if (sdev != dev) return KH_EINVAL;
  }
  float* scratch = kh::scratch_ptr(dev);
  if (!scratch) return KH_ECUDA;
  const int st = kh_decode_partial(q, n_groups, head_dim, k_code, k_res, k_norms, k_rnorms,
                                   v_code, v_res, v_norms, v_rnorms, seq_len, 0, seq_len,
                                   d_k_host, d_v_host, centroids_host, n_centroids,
                                   sm_scale, n_splits, scratch, n_splits, 0, stream);
  if (st != KH_OK) return st;
  return kh_decode_combine(scratch, n_groups, n_splits, head_dim, d_v_host, out, stream);
}
