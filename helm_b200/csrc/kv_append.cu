// Fused KV append for sm_100a: per-head RMSNorm of q and k, rotary embedding,
// and the scatter of the token's K and V rows into their page slots.
//
// Replaces, in one launch per layer, the eager sequence of the patched HF
// attention forwards (helm/runtime/kv_offload.py:368-373: q_norm, k_norm,
// apply_rotary_pos_emb) and the page writes of KVCacheManager.append_decode /
// append_prefill (helm/runtime/kv_cache.py:113-171).
//
// Rounding follows the eager reference op by op, so results match it bit for
// bit except where the fp32 variance sum lands on the other side of a bf16
// rounding boundary:
//   RMSNorm:  y = dtype(x_f32 * rsqrt(mean(x_f32^2) + eps));  z = dtype(w * y)
//   RoPE:     out = dtype( dtype(z * cos) + dtype(rotate_half(z) * sin) )
// (HF Qwen3RMSNorm / apply_rotary_pos_emb, transformers modeling_qwen3.py.)
#include "common.cuh"

namespace helm {
namespace {

constexpr int kAppendWarps = 4;

template <typename T, int EPL>
struct __align__(sizeof(T) * EPL) RowVec {
  T v[EPL];
};

template <typename T, int EPL>
__device__ __forceinline__ void load_row(const T* p, float (&x)[EPL]) {
  const RowVec<T, EPL> r = *reinterpret_cast<const RowVec<T, EPL>*>(p);
#pragma unroll
  for (int e = 0; e < EPL; ++e) x[e] = to_float<T>(r.v[e]);
}

template <typename T, int EPL>
__device__ __forceinline__ void store_row(T* p, const float (&x)[EPL]) {
  RowVec<T, EPL> r;
#pragma unroll
  for (int e = 0; e < EPL; ++e) r.v[e] = from_float<T>(x[e]);
  *reinterpret_cast<RowVec<T, EPL>*>(p) = r;
}

// Rounds through the storage dtype, as an eager elementwise op would.
template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return to_float<T>(from_float<T>(x));
}

template <typename T, int D>
__device__ __forceinline__ void norm_rope(float (&x)[D / 32], const T* w, float eps,
                                          const T* cos, const T* sin, int lane) {
  constexpr int EPL = D / 32;
  const int d0 = lane * EPL;
  if (w != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) ss += x[e] * x[e];
    ss = warp_sum_xor(ss, 1, 16);
    const float r = rsqrtf(ss / static_cast<float>(D) + eps);
    float wv[EPL];
    load_row<T, EPL>(w + d0, wv);
#pragma unroll
    for (int e = 0; e < EPL; ++e) x[e] = rnd<T>(wv[e] * rnd<T>(x[e] * r));
  }
  if (cos != nullptr) {
    float c[EPL], s[EPL], partner[EPL];
    load_row<T, EPL>(cos + d0, c);
    load_row<T, EPL>(sin + d0, s);
#pragma unroll
    for (int e = 0; e < EPL; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const bool low = lane < 16;  // dims [0, D/2)
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const float rot = low ? -partner[e] : partner[e];
      x[e] = rnd<T>(rnd<T>(x[e] * c[e]) + rnd<T>(rot * s[e]));
    }
  }
}

struct AppendArgs {
  const void* q;
  int64_t q_st, q_sh;
  const void* k;
  int64_t k_st, k_sh;
  const void* v;
  int64_t v_st, v_sh;
  const void* qw;
  const void* kw;
  float eps;
  const void* cos;
  const void* sin;
  int64_t rope_st;
  void* q_out;
  int64_t qo_st, qo_sh;
  void* k_out;
  void* v_out;
  void* pool;
  int64_t pool_pages;
  const int64_t* slot_rows;
  int hq, hkv, page_size;
};

template <typename T, int D>
__global__ void __launch_bounds__(kAppendWarps * 32) kv_append_kernel(const AppendArgs a) {
  // Programmatic dependent launch both ways: a decode kernel launched with
  // overlap may be placed now (it waits for this grid before reading the rows
  // written here), and this grid waits for the kernel before it (which
  // writes q / k / v) before reading anything.
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  constexpr int EPL = D / 32;
  const int tok = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* cosp = a.cos ? static_cast<const T*>(a.cos) + tok * a.rope_st : nullptr;
  const T* sinp = a.sin ? static_cast<const T*>(a.sin) + tok * a.rope_st : nullptr;
  int64_t row = a.slot_rows ? a.slot_rows[tok] : -1;
  int64_t slot = -1, r_in = 0;
  if (row >= 0) {
    slot = row / a.page_size;
    r_in = row - slot * a.page_size;
    if (slot >= a.pool_pages) {
      report_status(HELM_DEV_BAD_PAGE);
      slot = -1;
    }
  }
  const int64_t head_elems = static_cast<int64_t>(a.page_size) * D;
  T* pool = static_cast<T*>(a.pool);
  const int rows_total = a.hq + 2 * a.hkv;
  // one head row per warp: grid.y covers the token's q, k and v rows
  const int hr = blockIdx.y * kAppendWarps + warp;
  if (hr < rows_total) {
    float x[EPL];
    if (hr < a.hq) {
      if (a.q_out == nullptr) return;
      load_row<T, EPL>(static_cast<const T*>(a.q) + tok * a.q_st + hr * a.q_sh + lane * EPL, x);
      norm_rope<T, D>(x, static_cast<const T*>(a.qw), a.eps, cosp, sinp, lane);
      store_row<T, EPL>(static_cast<T*>(a.q_out) + tok * a.qo_st + hr * a.qo_sh + lane * EPL, x);
    } else if (hr < a.hq + a.hkv) {
      const int h = hr - a.hq;
      load_row<T, EPL>(static_cast<const T*>(a.k) + tok * a.k_st + h * a.k_sh + lane * EPL, x);
      norm_rope<T, D>(x, static_cast<const T*>(a.kw), a.eps, cosp, sinp, lane);
      if (slot >= 0)
        store_row<T, EPL>(pool + (slot * 2 * a.hkv + h) * head_elems + r_in * D + lane * EPL, x);
      if (a.k_out)
        store_row<T, EPL>(static_cast<T*>(a.k_out) + (static_cast<int64_t>(tok) * a.hkv + h) * D +
                              lane * EPL,
                          x);
    } else {
      const int h = hr - a.hq - a.hkv;
      load_row<T, EPL>(static_cast<const T*>(a.v) + tok * a.v_st + h * a.v_sh + lane * EPL, x);
      if (slot >= 0)
        store_row<T, EPL>(
            pool + ((slot * 2 + 1) * a.hkv + h) * head_elems + r_in * D + lane * EPL, x);
      if (a.v_out)
        store_row<T, EPL>(static_cast<T*>(a.v_out) + (static_cast<int64_t>(tok) * a.hkv + h) * D +
                              lane * EPL,
                          x);
    }
  }
}

// Plain row write for shapes the fused kernel does not cover (fp32 pages, any
// head_dim): element-wise copy of each token's K and V rows into the pool.
template <typename E>
__global__ void kv_scatter_rows_kernel(const AppendArgs a, int head_dim) {
  const int tok = blockIdx.x;
  const int64_t row = a.slot_rows[tok];
  if (row < 0) return;
  const int64_t slot = row / a.page_size, r_in = row - (row / a.page_size) * a.page_size;
  if (slot >= a.pool_pages) {
    if (threadIdx.x == 0) report_status(HELM_DEV_BAD_PAGE);
    return;
  }
  const int64_t head_elems = static_cast<int64_t>(a.page_size) * head_dim;
  E* pool = static_cast<E*>(a.pool);
  for (int e = threadIdx.x; e < 2 * a.hkv * head_dim; e += blockDim.x) {
    const int kv = e / (a.hkv * head_dim), rem = e - kv * a.hkv * head_dim;
    const int h = rem / head_dim, d = rem - h * head_dim;
    const E* src = kv == 0 ? static_cast<const E*>(a.k) + tok * a.k_st + h * a.k_sh
                           : static_cast<const E*>(a.v) + tok * a.v_st + h * a.v_sh;
    pool[((slot * 2 + kv) * a.hkv + h) * head_elems + r_in * head_dim + d] = src[d];
  }
}

template <typename T>
int launch_append(int head_dim, const AppendArgs& a, int n, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n, (a.hq + 2 * a.hkv + kAppendWarps - 1) / kAppendWarps);
  cfg.blockDim = dim3(kAppendWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (head_dim) {
    case 64:
      e = cudaLaunchKernelEx(&cfg, kv_append_kernel<T, 64>, a);
      break;
    case 128:
      e = cudaLaunchKernelEx(&cfg, kv_append_kernel<T, 128>, a);
      break;
    case 256:
      e = cudaLaunchKernelEx(&cfg, kv_append_kernel<T, 256>, a);
      break;
    default:
      return HELM_ERR_UNSUPPORTED;
  }
  return e == cudaSuccess ? HELM_OK : HELM_ERR_CUDA;
}

}  // namespace
}  // namespace helm

extern "C" int helm_kv_append(const void* q, int64_t q_stride_t, int64_t q_stride_h, const void* k,
                              int64_t k_stride_t, int64_t k_stride_h, const void* v,
                              int64_t v_stride_t, int64_t v_stride_h, const void* q_norm_w,
                              const void* k_norm_w, float eps, const void* cos, const void* sin,
                              int64_t rope_stride_t, void* q_out, int64_t q_out_stride_t,
                              int64_t q_out_stride_h, void* k_out, void* v_out, void* kv_pool,
                              int64_t pool_pages, const int64_t* slot_rows, int num_tokens,
                              int num_q_heads, int num_kv_heads, int head_dim, int page_size,
                              int dtype, void* stream) {
  using namespace helm;
  if (num_tokens < 0 || num_q_heads < 0 || num_kv_heads <= 0 || page_size <= 0)
    return HELM_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return HELM_OK;
  if (k == nullptr || v == nullptr) return HELM_ERR_INVALID_ARGUMENT;
  if (q_out != nullptr && q == nullptr) return HELM_ERR_INVALID_ARGUMENT;
  if ((cos == nullptr) != (sin == nullptr)) return HELM_ERR_INVALID_ARGUMENT;
  if (slot_rows != nullptr && kv_pool == nullptr) return HELM_ERR_INVALID_ARGUMENT;
  const bool processing = q_out != nullptr || q_norm_w != nullptr || k_norm_w != nullptr ||
                          cos != nullptr || k_out != nullptr || v_out != nullptr;
  const bool fused_shape = (dtype == HELM_DTYPE_BF16 || dtype == HELM_DTYPE_FP16) &&
                           (head_dim == 64 || head_dim == 128 || head_dim == 256);
  if (!fused_shape) {
    // plain page write of any dtype / head_dim; norm and RoPE need the fused shape
    if (processing || slot_rows == nullptr || head_dim <= 0) return HELM_ERR_UNSUPPORTED;
    if (dtype != HELM_DTYPE_FP32 && dtype != HELM_DTYPE_BF16 && dtype != HELM_DTYPE_FP16)
      return HELM_ERR_UNSUPPORTED;
    AppendArgs a{};
    a.k = k;
    a.k_st = k_stride_t;
    a.k_sh = k_stride_h;
    a.v = v;
    a.v_st = v_stride_t;
    a.v_sh = v_stride_h;
    a.pool = kv_pool;
    a.pool_pages = pool_pages;
    a.slot_rows = slot_rows;
    a.hkv = num_kv_heads;
    a.page_size = page_size;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dtype == HELM_DTYPE_FP32)
      kv_scatter_rows_kernel<float><<<num_tokens, 128, 0, s>>>(a, head_dim);
    else
      kv_scatter_rows_kernel<uint16_t><<<num_tokens, 128, 0, s>>>(a, head_dim);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return HELM_ERR_CUDA;
    }
    return HELM_OK;
  }
  // Each lane moves D/32 contiguous elements: rows must be aligned to that.
  const int64_t vec = head_dim / 32;  // elements per lane
  auto bad = [&](const void* p, std::initializer_list<int64_t> strides) {
    if (p == nullptr) return false;
    if (reinterpret_cast<uintptr_t>(p) % (vec * 2)) return true;
    for (int64_t st : strides)
      if (st % vec) return true;
    return false;
  };
  if (bad(q, {q_stride_t, q_stride_h}) || bad(k, {k_stride_t, k_stride_h}) ||
      bad(v, {v_stride_t, v_stride_h}) || bad(q_out, {q_out_stride_t, q_out_stride_h}) ||
      bad(cos, {rope_stride_t}) || bad(sin, {rope_stride_t}) || bad(q_norm_w, {}) ||
      bad(k_norm_w, {}) || bad(k_out, {}) || bad(v_out, {}) || bad(kv_pool, {}))
    return HELM_ERR_ALIGNMENT;
  AppendArgs a;
  a.q = q;
  a.q_st = q_stride_t;
  a.q_sh = q_stride_h;
  a.k = k;
  a.k_st = k_stride_t;
  a.k_sh = k_stride_h;
  a.v = v;
  a.v_st = v_stride_t;
  a.v_sh = v_stride_h;
  a.qw = q_norm_w;
  a.kw = k_norm_w;
  a.eps = eps;
  a.cos = cos;
  a.sin = sin;
  a.rope_st = rope_stride_t;
  a.q_out = q_out;
  a.qo_st = q_out_stride_t;
  a.qo_sh = q_out_stride_h;
  a.k_out = k_out;
  a.v_out = v_out;
  a.pool = kv_pool;
  a.pool_pages = pool_pages;
  a.slot_rows = slot_rows;
  a.hq = q_out != nullptr ? num_q_heads : 0;
  a.hkv = num_kv_heads;
  a.page_size = page_size;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rc = dtype == HELM_DTYPE_BF16 ? launch_append<__nv_bfloat16>(head_dim, a, num_tokens, s)
                                          : launch_append<__half>(head_dim, a, num_tokens, s);
  if (rc == HELM_ERR_CUDA) set_last_cuda_error(cudaGetLastError());
  return rc;
}
