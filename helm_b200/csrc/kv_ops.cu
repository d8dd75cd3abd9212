// Page movement and attention-state merging for sm_100a.
//
//  helm_copy_pages            page-slot copies between tiers (copy engine)
//  helm_gather_kv             paged K/V -> dense [B, Hkv, T, D] (zero padded)
//  helm_merge_attention_states  merge of partial (O, LSE) over disjoint key ranges
#include "common.cuh"

#include <vector>

namespace helm {
namespace {

// One thread moves 16 bytes; grid-stride over B*Hkv*T_max*D/8 vectors of K and V.
template <typename T>
__global__ void gather_kv_kernel(const T* __restrict__ pool, int64_t pool_pages,
                                 const int32_t* __restrict__ page_table, int64_t pt_sb,
                                 int max_pages, const int32_t* __restrict__ kv_lens,
                                 T* __restrict__ k_out, T* __restrict__ v_out, int batch, int hkv,
                                 int head_dim, int page_size, int t_max) {
  const int vecs_per_row = head_dim / 8;
  const int64_t total = static_cast<int64_t>(batch) * hkv * t_max * vecs_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int dv = static_cast<int>(i % vecs_per_row);
    int64_t r = i / vecs_per_row;
    const int t = static_cast<int>(r % t_max);
    r /= t_max;
    const int h = static_cast<int>(r % hkv);
    const int b = static_cast<int>(r / hkv);
    uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    const int page = t / page_size;
    if (t < kv_lens[b] && page < max_pages) {
      int64_t slot = page_table[b * pt_sb + page];
      if (slot >= 0 && slot < pool_pages) {
        const int64_t head_elems = static_cast<int64_t>(page_size) * head_dim;
        const int64_t off = (slot * 2 * hkv + h) * head_elems +
                            static_cast<int64_t>(t - page * page_size) * head_dim + dv * 8;
        kv = *reinterpret_cast<const uint4*>(pool + off);
        vv = *reinterpret_cast<const uint4*>(pool + off + hkv * head_elems);
      } else {
        report_status(HELM_DEV_BAD_PAGE);
      }
    }
    const int64_t o = ((static_cast<int64_t>(b) * hkv + h) * t_max + t) * head_dim + dv * 8;
    *reinterpret_cast<uint4*>(k_out + o) = kv;
    *reinterpret_cast<uint4*>(v_out + o) = vv;
  }
}

template <typename TI>
__device__ __forceinline__ float load_any(const void* p, int64_t i) {
  return to_float<TI>(static_cast<const TI*>(p)[i]);
}

__device__ __forceinline__ float load_dt(const void* p, int dt, int64_t i) {
  if (dt == HELM_DTYPE_FP32) return static_cast<const float*>(p)[i];
  if (dt == HELM_DTYPE_BF16) return load_any<__nv_bfloat16>(p, i);
  return load_any<__half>(p, i);
}

__device__ __forceinline__ void store_dt(void* p, int dt, int64_t i, float x) {
  if (dt == HELM_DTYPE_FP32)
    static_cast<float*>(p)[i] = x;
  else if (dt == HELM_DTYPE_BF16)
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else
    static_cast<__half*>(p)[i] = __float2half_rn(x);
}

// One CTA per row (sequence, query head); threads stride over the head dim.
// Part r's O row starts at o_parts + r*o_stride + row*D, its LSE at
// lse_parts[r*lse_stride + row].
__global__ void merge_states_kernel(const void* __restrict__ o_parts, int o_dtype,
                                    int64_t o_stride, const float* __restrict__ lse_parts,
                                    int64_t lse_stride, int parts, int64_t rows, int head_dim,
                                    void* __restrict__ out, int out_dtype,
                                    float* __restrict__ lse_out) {
  const int64_t row = blockIdx.x;
  float M = -INFINITY;
  for (int r = 0; r < parts; ++r) M = fmaxf(M, lse_parts[r * lse_stride + row]);
  const float m_use = M == -INFINITY ? 0.f : M;
  float L = 0.f;
  for (int r = 0; r < parts; ++r) L += expf(lse_parts[r * lse_stride + row] - m_use);
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < parts; ++r) {
      const float w = expf(lse_parts[r * lse_stride + row] - m_use);
      if (w > 0.f) acc += w * load_dt(o_parts, o_dtype, r * o_stride + row * head_dim + d);
    }
    store_dt(out, out_dtype, row * head_dim + d, acc * inv);
  }
  if (threadIdx.x == 0 && lse_out != nullptr)
    lse_out[row] = (M == -INFINITY || L <= 0.f) ? -INFINITY : M + logf(L);
}

}  // namespace
}  // namespace helm

extern "C" int helm_copy_pages(void* dst_pool, const void* src_pool, int64_t page_bytes,
                               const int64_t* dst_slots, const int64_t* src_slots, int64_t n,
                               void* stream) {
  using namespace helm;
  if (n < 0 || page_bytes <= 0) return HELM_ERR_INVALID_ARGUMENT;
  if (n == 0) return HELM_OK;
  if (dst_pool == nullptr || src_pool == nullptr || dst_slots == nullptr || src_slots == nullptr)
    return HELM_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t i = 0;
  while (i < n) {
    if (dst_slots[i] < 0 || src_slots[i] < 0) return HELM_ERR_INVALID_ARGUMENT;
    int64_t run = 1;  // merge runs of consecutive slots on both sides into one copy
    while (i + run < n && dst_slots[i + run] == dst_slots[i] + run &&
           src_slots[i + run] == src_slots[i] + run)
      ++run;
    cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(dst_pool) + dst_slots[i] * page_bytes,
                                    static_cast<const uint8_t*>(src_pool) + src_slots[i] * page_bytes,
                                    static_cast<size_t>(run * page_bytes), cudaMemcpyDefault, s);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return HELM_ERR_CUDA;
    }
    i += run;
  }
  return HELM_OK;
}

extern "C" int helm_gather_kv(const void* kv_pool, int64_t pool_pages, const int32_t* page_table,
                              int64_t pt_stride_b, int max_pages, const int32_t* kv_lens,
                              void* k_out, void* v_out, int batch, int num_kv_heads, int head_dim,
                              int page_size, int t_max, int dtype, void* stream) {
  using namespace helm;
  if (kv_pool == nullptr || page_table == nullptr || kv_lens == nullptr || k_out == nullptr ||
      v_out == nullptr)
    return HELM_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || num_kv_heads <= 0 || page_size <= 0 || t_max < 0 || head_dim % 8)
    return HELM_ERR_INVALID_ARGUMENT;
  if (dtype != HELM_DTYPE_BF16 && dtype != HELM_DTYPE_FP16) return HELM_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(kv_pool) | reinterpret_cast<uintptr_t>(k_out) |
       reinterpret_cast<uintptr_t>(v_out)) &
      15)
    return HELM_ERR_ALIGNMENT;
  if (t_max == 0) return HELM_OK;
  const int64_t vecs = static_cast<int64_t>(batch) * num_kv_heads * t_max * (head_dim / 8);
  const int threads = 256;
  const int blocks = static_cast<int>(std::min<int64_t>((vecs + threads - 1) / threads,
                                                        static_cast<int64_t>(num_sms_current_device()) * 16));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // K/V are moved as raw 16-bit words, so one instantiation serves bf16 and fp16.
  gather_kv_kernel<uint16_t><<<blocks, threads, 0, s>>>(
      static_cast<const uint16_t*>(kv_pool), pool_pages, page_table, pt_stride_b, max_pages, kv_lens,
      static_cast<uint16_t*>(k_out), static_cast<uint16_t*>(v_out), batch, num_kv_heads, head_dim,
      page_size, t_max);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  return HELM_OK;
}

extern "C" int helm_merge_attention_states(const void* o_parts, int o_dtype, int64_t o_part_stride,
                                           const float* lse_parts, int64_t lse_part_stride,
                                           int num_parts, int64_t rows, int head_dim, void* out,
                                           int out_dtype, float* lse_out, void* stream) {
  using namespace helm;
  if (o_parts == nullptr || lse_parts == nullptr || out == nullptr || num_parts <= 0 ||
      rows < 0 || head_dim <= 0)
    return HELM_ERR_INVALID_ARGUMENT;
  if (o_part_stride < rows * head_dim || lse_part_stride < rows) return HELM_ERR_INVALID_ARGUMENT;
  auto dt_ok = [](int d) {
    return d == HELM_DTYPE_FP32 || d == HELM_DTYPE_BF16 || d == HELM_DTYPE_FP16;
  };
  if (!dt_ok(o_dtype) || !dt_ok(out_dtype)) return HELM_ERR_UNSUPPORTED;
  if (rows == 0) return HELM_OK;
  if (rows > 0x7fffffff) return HELM_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  merge_states_kernel<<<static_cast<unsigned>(rows), 128, 0, s>>>(
      o_parts, o_dtype, o_part_stride, lse_parts, lse_part_stride, num_parts, rows, head_dim, out,
      out_dtype, lse_out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  return HELM_OK;
}
