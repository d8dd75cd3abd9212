// Matrix-vector products of a decode step (batch of B <= 16 token rows), with
// the element-wise work around them fused in.
//
// A decoder layer at decode time is a chain of GEMVs -- y[b] = W x[b] with W
// [N, K] row-major -- separated by RMSNorm, SwiGLU and residual adds.  Run as
// library GEMMs plus eager element-wise ops that is ~25 launches per layer,
// and at batch 1 the launches, not the weight bytes, set the step time.  Here
// one launch does:
//
//   y = W . rmsnorm(x)              (norm_w given: input_layernorm + q/k/v proj,
//                                    final norm + lm_head)
//   y = silu(W x) * (W2 x)          (W2 given: gate/up proj + act, SwiGLU)
//   y = residual + W x              (residual given: o_proj / down_proj + add)
//   y = residual + sum_r W_r x_r    (peer buffers given: the row-parallel
//                                    projection of tensor parallelism, its
//                                    all-reduce done in the same kernel)
//
// with the rounding of HF's eager modules: the RMSNorm output is rounded to the
// model dtype before the weight multiply (Qwen3RMSNorm / LlamaRMSNorm), each
// projection output is rounded before the next op, and SiLU, the product and
// the residual add each round once.  Dot products accumulate in fp32.
//
// Layout: the CTA stages x (normalised) for all B rows in shared memory; each
// warp owns one output row at a time and streams that row of W with 16-byte
// non-allocating loads, four chunks in flight per lane, FMA-ing against every
// batch row.  The op is HBM-bound on W (N x K x 2 bytes per launch).
#include "common.cuh"

namespace helm {
namespace {

constexpr int kGemvUnroll = 4;
// threads per CTA: fewer for wide batches so that the accumulators fit
template <int NB>
struct GemvShape {
  static constexpr int kThreads = NB == 1 ? 512 : 256;
  static constexpr int kWarps = kThreads / 32;
  static constexpr int kMinBlocks = NB <= 4 ? 2 : 1;  // at least two CTAs per SM when narrow
};

constexpr int kArMaxRanks = 8;
constexpr int64_t kArHeaderBytes = 8192;  // uint32 epoch per CTA (<= 2048 CTAs)

struct GemvArgs {
  unsigned char* bufs[kArMaxRanks];  // all-reduce exchange buffers of every rank
  int rank, world;
  uint64_t timeout_ns;
  const void* x;
  int64_t x_stride;
  const void* norm_w;
  float eps;
  const void* w;
  const void* w2;
  int64_t n, k;
  const void* residual;
  int64_t res_stride;
  void* y;
  int64_t y_stride;
  int y_fp32;
  int batch;
};

__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t v);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return to_float<T>(from_float<T>(x));
}

template <typename T>
__device__ __forceinline__ float dot8(const uint4& w, const uint4& x) {
  const float2 w0 = unpack2<T>(w.x), w1 = unpack2<T>(w.y), w2 = unpack2<T>(w.z),
               w3 = unpack2<T>(w.w);
  const float2 x0 = unpack2<T>(x.x), x1 = unpack2<T>(x.y), x2 = unpack2<T>(x.z),
               x3 = unpack2<T>(x.w);
  float s = w0.x * x0.x;
  s = fmaf(w0.y, x0.y, s);
  s = fmaf(w1.x, x1.x, s);
  s = fmaf(w1.y, x1.y, s);
  s = fmaf(w2.x, x2.x, s);
  s = fmaf(w2.y, x2.y, s);
  s = fmaf(w3.x, x3.x, s);
  s = fmaf(w3.y, x3.y, s);
  return s;
}

__device__ __forceinline__ void st_volatile_u2(uint2* p, uint32_t a, uint32_t b) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

__device__ __forceinline__ uint2 ld_volatile_u2(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t gemv_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// All-reduce of one output value over the ranks (tensor-parallel row-parallel
// projection).  Words {fp32 value, epoch} [2 parities][world][n][batch] in
// every rank's buffer; this lane stores its partial for (row, b) into slot
// `rank` of every buffer, then polls its own buffer for all ranks' partials of
// (row, b) and returns their sum in rank order (the same on every rank).
// Returns false when the poll ran out of time (status word set).
__device__ __forceinline__ bool allreduce_value(const GemvArgs& a, uint32_t e, int64_t row, int b,
                                                float part, float& sum) {
  const int par = static_cast<int>(e & 1u);
  const int64_t slot_words = a.n * a.batch;
  const int64_t off = row * a.batch + b;
  for (int p = 0; p < a.world; ++p) {
    uint2* dst = reinterpret_cast<uint2*>(a.bufs[p] + kArHeaderBytes) +
                 (static_cast<int64_t>(par) * a.world + a.rank) * slot_words + off;
    st_volatile_u2(dst, __float_as_uint(part), e);
  }
  const uint2* own = reinterpret_cast<const uint2*>(a.bufs[a.rank] + kArHeaderBytes) +
                     static_cast<int64_t>(par) * a.world * slot_words + off;
  uint2 w[kArMaxRanks];
  const uint64_t t0 = gemv_timer_ns();
  for (int spin = 0;; ++spin) {
    bool ready = true;
#pragma unroll
    for (int p = 0; p < kArMaxRanks; ++p) {
      if (p >= a.world) break;
      if (spin == 0 || w[p].y != e) w[p] = ld_volatile_u2(own + p * slot_words);
      ready = ready && w[p].y == e;
    }
    if (ready) break;
    if ((spin & 15) == 15 && gemv_timer_ns() - t0 > a.timeout_ns) {
      report_status(HELM_DEV_TIMEOUT);
      return false;
    }
  }
  sum = 0.f;
#pragma unroll
  for (int p = 0; p < kArMaxRanks; ++p)
    if (p < a.world) sum += __uint_as_float(w[p].x);
  return true;
}

template <typename T, int NB, bool AR>
__global__ void __launch_bounds__(GemvShape<NB>::kThreads, AR ? 1 : GemvShape<NB>::kMinBlocks) decode_gemv_kernel(const GemvArgs a) {
  constexpr int kGemvThreads = GemvShape<NB>::kThreads;
  constexpr int kGemvWarps = GemvShape<NB>::kWarps;
  extern __shared__ __align__(16) uint8_t gemv_smem[];
  T* xs = reinterpret_cast<T*>(gemv_smem);  // [NB][K]
  __shared__ float s_red[kGemvWarps];
  __shared__ float s_scale;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t K = a.k;
  const T* x = static_cast<const T*>(a.x);
  const T* nw = static_cast<const T*>(a.norm_w);
  const T* W = static_cast<const T*>(a.w);
  const T* W2 = static_cast<const T*>(a.w2);
  const bool glu = W2 != nullptr;
  const int64_t chunks = K / 8;  // 16-byte chunks per row (K % 8 == 0)
  // Launched as a programmatic dependent of the kernel before it.  The weights
  // are static: the first chunks of this warp's first row are loaded into
  // registers before waiting for that kernel (which writes x / the residual)
  // and while x is staged.
  // (with the all-reduce, later kernels are not placed early: they could take
  // the space of CTAs that other ranks' CTAs are waiting for)
  if (!AR) asm volatile("griddepcontrol.launch_dependents;");
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kGemvWarps + warp;
  uint4 wv[kGemvUnroll], wv2[kGemvUnroll];  // weight chunks in flight
#pragma unroll
  for (int u = 0; u < kGemvUnroll; ++u) {
    const int64_t c = lane + u * 32;
    if (row0 < a.n && c < chunks) {
      wv[u] = ld_stream_v4(W + row0 * K + c * 8);
      if (glu) wv2[u] = ld_stream_v4(W2 + row0 * K + c * 8);
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // all-reduce: this CTA's epoch (one counter per CTA index, same rows on
  // every rank), advanced at the end of the call
  __shared__ uint32_t s_epoch;
  __shared__ int s_ar_ok;
  if (AR && threadIdx.x == 0) {
    s_epoch = reinterpret_cast<uint32_t*>(a.bufs[a.rank])[blockIdx.x] + 1u;
    s_ar_ok = 1;
  }

  // ---- stage x (rows >= batch are zero), RMSNorm'd when norm_w is given ----
  for (int b = 0; b < NB; ++b) {
    if (b >= a.batch) {
      for (int64_t i = threadIdx.x; i < K; i += kGemvThreads) xs[b * K + i] = from_float<T>(0.f);
      continue;
    }
    const T* xb = x + b * a.x_stride;
    if (nw == nullptr) {
      for (int64_t i = threadIdx.x; i < K; i += kGemvThreads) xs[b * K + i] = xb[i];
      continue;
    }
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < K; i += kGemvThreads) {
      const float v = to_float<T>(xb[i]);
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int w = 0; w < kGemvWarps; ++w) t += s_red[w];
      s_scale = rsqrtf(t / static_cast<float>(K) + a.eps);
    }
    __syncthreads();
    const float sc = s_scale;
    for (int64_t i = threadIdx.x; i < K; i += kGemvThreads) {
      const float xn = round_to<T>(to_float<T>(xb[i]) * sc);        // x.to(dtype)
      xs[b * K + i] = from_float<T>(to_float<T>(nw[i]) * xn);      // weight * x
    }
    __syncthreads();
  }
  __syncthreads();

  // ---- one output row per warp at a time ----
  bool preloaded = true;
  for (int64_t row = row0; row < a.n; row += static_cast<int64_t>(gridDim.x) * kGemvWarps) {
    float acc[NB], acc2[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = acc2[b] = 0.f;
    const T* wr = W + row * K;
    const T* wr2 = glu ? W2 + row * K : nullptr;
    for (int64_t c0 = lane; c0 < chunks; c0 += 32 * kGemvUnroll) {
      if (preloaded) {  // the first chunk group of the first row is in flight already
        preloaded = false;
      } else {
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
          const int64_t c = c0 + u * 32;
          if (c < chunks) {
            wv[u] = ld_stream_v4(wr + c * 8);
            if (glu) wv2[u] = ld_stream_v4(wr2 + c * 8);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kGemvUnroll; ++u) {
        const int64_t c = c0 + u * 32;
        if (c < chunks) {
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + b * K + c * 8);
            acc[b] += dot8<T>(wv[u], xv);
            if (glu) acc2[b] += dot8<T>(wv2[u], xv);
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
        if (glu) acc2[b] += __shfl_xor_sync(0xffffffffu, acc2[b], o);
      }
    }
    // lane b writes batch row b
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      if (lane != b || b >= a.batch) continue;
      if (AR) {  // sum the ranks' partial dot products before rounding
        float sum = 0.f;
        if (!allreduce_value(a, s_epoch, row, b, acc[b], sum)) {
          atomicExch(&s_ar_ok, 0);
          continue;
        }
        acc[b] = sum;
      }
      float v = round_to<T>(acc[b]);  // projection output in the model dtype
      if (glu) {
        const float u = round_to<T>(acc2[b]);
        const float s = round_to<T>(v / (1.f + expf(-v)));  // act_fn(gate)
        v = round_to<T>(s * u);
      }
      if (a.residual != nullptr)
        v = round_to<T>(to_float<T>(static_cast<const T*>(a.residual)[b * a.res_stride + row]) + v);
      if (a.y_fp32)
        static_cast<float*>(a.y)[b * a.y_stride + row] = v;
      else
        static_cast<T*>(a.y)[b * a.y_stride + row] = from_float<T>(v);
    }
  }
  if (AR) {
    __syncthreads();
    if (threadIdx.x == 0 && s_ar_ok) reinterpret_cast<uint32_t*>(a.bufs[a.rank])[blockIdx.x] = s_epoch;
  }
}

template <typename T, int NB, bool AR>
int launch_gemv(const GemvArgs& a, cudaStream_t stream) {
  static unsigned long long configured = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return HELM_ERR_CUDA;
  const size_t smem = static_cast<size_t>(NB) * a.k * sizeof(T);
  if (smem > 200 * 1024) return HELM_ERR_UNSUPPORTED;
  if (!(configured & (1ull << dev))) {
    if (cudaFuncSetAttribute(decode_gemv_kernel<T, NB, AR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             200 * 1024) != cudaSuccess)
      return HELM_ERR_CUDA;
    configured |= 1ull << dev;
  }
  int per_sm = smem <= 48 * 1024 ? 4 : (smem <= 100 * 1024 ? 2 : 1);
  if (AR) {
    // every CTA must be resident at once: CTA c waits for CTA c of the other
    // ranks, whose own CTAs may wait for ours
    int fit = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&fit, decode_gemv_kernel<T, NB, AR>,
                                                      GemvShape<NB>::kThreads, smem) != cudaSuccess ||
        fit <= 0)
      return HELM_ERR_CUDA;
    per_sm = std::min(per_sm, fit);
  }
  constexpr int kWarps = GemvShape<NB>::kWarps;
  const int64_t want = (a.n + kWarps - 1) / kWarps;
  const int grid = static_cast<int>(std::min<int64_t>(want, int64_t(num_sms_current_device()) * per_sm));
  if (AR && grid * 4 > kArHeaderBytes) return HELM_ERR_UNSUPPORTED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GemvShape<NB>::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_gemv_kernel<T, NB, AR>, a) == cudaSuccess ? HELM_OK
                                                                                : HELM_ERR_CUDA;
}

template <typename T, bool AR>
int dispatch_gemv(const GemvArgs& a, cudaStream_t s) {
  if (a.batch <= 1) return launch_gemv<T, 1, AR>(a, s);
  if (a.batch <= 2) return launch_gemv<T, 2, AR>(a, s);
  if (a.batch <= 4) return launch_gemv<T, 4, AR>(a, s);
  if (a.batch <= 8) return launch_gemv<T, 8, AR>(a, s);
  return launch_gemv<T, 16, AR>(a, s);
}



}  // namespace
}  // namespace helm

namespace helm {
namespace {
int gemv_entry(const void* x, int64_t x_stride, const void* norm_w, float eps, const void* w,
               const void* w2, int64_t n, int64_t k, const void* residual, int64_t res_stride,
               void* y, int64_t y_stride, int y_fp32, int batch, int dtype, void* const* bufs,
               int rank, int world, uint64_t timeout_ns, void* stream);
}
}  // namespace helm

extern "C" int helm_decode_gemv_allreduce(void* const* bufs, int rank, int world,
                                          const void* x, int64_t x_stride, const void* w,
                                          int64_t n, int64_t k, const void* residual,
                                          int64_t res_stride, void* y, int64_t y_stride,
                                          int batch, int dtype, uint64_t timeout_ns,
                                          void* stream) {
  using namespace helm;
  if (bufs == nullptr || world < 1 || world > kArMaxRanks || rank < 0 || rank >= world ||
      timeout_ns == 0)
    return HELM_ERR_INVALID_ARGUMENT;
  for (int r = 0; r < world; ++r)
    if (bufs[r] == nullptr || (reinterpret_cast<uintptr_t>(bufs[r]) & 255u) != 0)
      return HELM_ERR_ALIGNMENT;
  return gemv_entry(x, x_stride, nullptr, 0.f, w, nullptr, n, k, residual, res_stride, y,
                    y_stride, 0, batch, dtype, bufs, rank, world, timeout_ns, stream);
}

extern "C" int64_t helm_decode_gemv_allreduce_bytes(int64_t n, int batch, int world) {
  if (n <= 0 || batch <= 0 || world < 1 || world > helm::kArMaxRanks) return -1;
  return helm::kArHeaderBytes + 2 * static_cast<int64_t>(world) * n * batch * 8;
}

extern "C" int helm_decode_gemv(const void* x, int64_t x_stride, const void* norm_w, float eps,
                                const void* w, const void* w2, int64_t n, int64_t k,
                                const void* residual, int64_t res_stride, void* y,
                                int64_t y_stride, int y_fp32, int batch, int dtype,
                                void* stream) {
  return helm::gemv_entry(x, x_stride, norm_w, eps, w, w2, n, k, residual, res_stride, y, y_stride,
                          y_fp32, batch, dtype, nullptr, 0, 1, 0, stream);
}

namespace helm {
namespace {
int gemv_entry(const void* x, int64_t x_stride, const void* norm_w, float eps, const void* w,
               const void* w2, int64_t n, int64_t k, const void* residual, int64_t res_stride,
               void* y, int64_t y_stride, int y_fp32, int batch, int dtype, void* const* bufs,
               int rank, int world, uint64_t timeout_ns, void* stream) {
  if (x == nullptr || w == nullptr || y == nullptr) return HELM_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || n <= 0 || k <= 0) return HELM_ERR_INVALID_ARGUMENT;
  if (batch > 16) return HELM_ERR_UNSUPPORTED;
  if (dtype != HELM_DTYPE_BF16 && dtype != HELM_DTYPE_FP16) return HELM_ERR_UNSUPPORTED;
  if (k % 8 != 0) return HELM_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (w2 != nullptr && (reinterpret_cast<uintptr_t>(w2) & 15)))
    return HELM_ERR_ALIGNMENT;
  GemvArgs a;
  a.x = x;
  a.x_stride = x_stride;
  a.norm_w = norm_w;
  a.eps = eps;
  a.w = w;
  a.w2 = w2;
  a.n = n;
  a.k = k;
  a.residual = residual;
  a.res_stride = res_stride;
  a.y = y;
  a.y_stride = y_stride;
  a.y_fp32 = y_fp32;
  a.batch = batch;
  for (int r = 0; r < kArMaxRanks; ++r)
    a.bufs[r] = (bufs != nullptr && r < world) ? static_cast<unsigned char*>(bufs[r]) : nullptr;
  a.rank = rank;
  a.world = world;
  a.timeout_ns = timeout_ns;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  if (bufs != nullptr)
    rc = dtype == HELM_DTYPE_BF16 ? dispatch_gemv<__nv_bfloat16, true>(a, s)
                                  : dispatch_gemv<__half, true>(a, s);
  else
    rc = dtype == HELM_DTYPE_BF16 ? dispatch_gemv<__nv_bfloat16, false>(a, s)
                                  : dispatch_gemv<__half, false>(a, s);
  if (rc == HELM_ERR_CUDA) set_last_cuda_error(cudaGetLastError());
  return rc;
}
}  // namespace
}  // namespace helm
