// Decode attention for callers that cannot allocate device memory.
//
// helm_paged_decode_attention needs a scratch workspace (split-KV partial
// softmax states) that its caller allocates.  Some
// callers cannot do that: a serving process that hands all of HBM to its own
// page pool at start-up, so any later cudaMalloc fails or fragments that pool;
// or a decode loop that must not stall on the device-wide synchronisation that
// cudaFree (and, on some paths, cudaMalloc) performs.  This entry point takes
// the same inputs and outputs but uses a fixed scratch array that lives in the
// library itself, so it allocates nothing.
//
// Limits and rules for users:
//  * The scratch is kNoAllocScratchBytes (8 MiB) per GPU, held by every GPU
//    that loads this library until the process exits.  A shape whose workspace
//    (helm_paged_decode_workspace_bytes) is larger is rejected with
//    HELM_ERR_WORKSPACE before anything is launched.
//  * The first call on a device looks up the array's device address (one-time
//    set-up on the device that is current); make that first call before any
//    stream capture.
//  * Every call uses the same array.  Calls that overlap on the GPU (different
//    streams, or different host threads without ordering) race on it and give
//    wrong results; order them on one stream.
//  * Nothing in the array has to start at zero: every value a call reads was
//    written earlier in the same call, so a call never depends on what an
//    earlier (or an abandoned) call left behind.
#include <atomic>

#include "common.cuh"

namespace helm {
namespace {

constexpr int64_t kNoAllocScratchBytes = int64_t(8) << 20;

// The scratch itself.  In host code this name is only a stand-in for the
// device array: the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Per device, filled on first use.  Two host threads making the first call on
// one device at the same time both look the address up and store the same
// value; the atomics make that well defined.
std::atomic<void*> g_noalloc_scratch_addr[64];

}  // namespace
}  // namespace helm

extern "C" int helm_paged_decode_attention_noalloc(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* kv_pool, int64_t pool_pages,
    const int32_t* page_table, int64_t pt_stride_b, int max_pages, const int32_t* kv_lens,
    const int32_t* num_pages, const int32_t* page_used, const int32_t* page_start,
    const void* mask, int mask_dtype, int64_t mask_stride_b, void* out, int64_t out_stride_b,
    int64_t out_stride_h, float* lse, int batch, int num_q_heads, int num_kv_heads, int head_dim,
    int page_size, int dtype, float scale, float softcap, int max_kv_len_hint, void* stream) {
  using namespace helm;
  if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return HELM_ERR_INVALID_ARGUMENT;
  const int64_t need =
      helm_paged_decode_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim);
  if (need <= 0) return HELM_ERR_INVALID_ARGUMENT;
  if (need > kNoAllocScratchBytes) return HELM_ERR_WORKSPACE;

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) return HELM_ERR_UNSUPPORTED;
  void* scratch = g_noalloc_scratch_addr[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) {  // one-time set-up for this device
    e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return HELM_ERR_CUDA;
    }
    g_noalloc_scratch_addr[dev].store(scratch, std::memory_order_release);
  }
  return helm_paged_decode_attention(
      q, q_stride_b, q_stride_h, kv_pool, pool_pages, page_table, pt_stride_b, max_pages, kv_lens,
      num_pages, page_used, page_start, mask, mask_dtype, mask_stride_b, out, out_stride_b,
      out_stride_h, lse, scratch, kNoAllocScratchBytes, batch, num_q_heads, num_kv_heads,
      head_dim, page_size, dtype, dtype, scale, softcap, max_kv_len_hint, stream);
}
