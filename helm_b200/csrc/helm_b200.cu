// Single translation unit of libhelm_b200.so: the kernels' sources are
// included here so that device-side globals (the status word) exist once.
#include "common.cuh"

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "kv_append.cu"
#include "kv_ops.cu"
#include "paged_attention.cu"
#include "paged_attention_noalloc.cu"
#include "paged_prefill.cu"
#include "paged_prefill_tc.cu"
#include "peer_exchange.cu"
#include "decode_gemv.cu"

namespace helm {

namespace {
thread_local char t_last_error[256] = "";
thread_local int t_decode_overlap = 0;
}

bool decode_overlap_enabled() { return t_decode_overlap != 0; }

void set_last_cuda_error(cudaError_t e) {
  std::snprintf(t_last_error, sizeof(t_last_error), "%s: %s", cudaGetErrorName(e),
                cudaGetErrorString(e));
}

int num_sms_current_device() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace helm

extern "C" int helm_version(void) { return 100; }

extern "C" int helm_set_decode_overlap(int enable) {
  const int prev = helm::t_decode_overlap;
  helm::t_decode_overlap = enable != 0 ? 1 : 0;
  return prev;
}

extern "C" const char* helm_status_string(int status) {
  switch (status) {
    case HELM_OK:
      return "ok";
    case HELM_ERR_INVALID_ARGUMENT:
      return "invalid argument";
    case HELM_ERR_UNSUPPORTED:
      return "unsupported shape or dtype";
    case HELM_ERR_CUDA:
      return "CUDA error";
    case HELM_ERR_WORKSPACE:
      return "workspace too small";
    case HELM_ERR_ALIGNMENT:
      return "misaligned pointer or stride";
    default:
      return "unknown status";
  }
}

extern "C" const char* helm_last_cuda_error(void) { return helm::t_last_error; }

extern "C" int helm_get_device_status(unsigned int* out, int reset, void* stream) {
  if (out == nullptr) return HELM_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e == cudaSuccess)
    e = cudaMemcpyFromSymbol(out, helm::g_device_status, sizeof(unsigned int), 0,
                             cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && reset) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(helm::g_device_status, &zero, sizeof(unsigned int), 0,
                           cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) {
    helm::set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  return HELM_OK;
}
