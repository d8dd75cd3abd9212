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

constexpr int kGemvMaxSmem = 224 * 1024;  // x of all batch rows, staged per CTA
// threads per CTA: fewer for wide batches so that the accumulators fit
template <int NB>
struct GemvShape {
  static constexpr int kThreads = NB == 1 ? 512 : 256;
  static constexpr int kWarps = kThreads / 32;
  // bytes of weight stream in flight per lane (cp.async ring): 64 KB per CTA
  // for one batch row (512 threads), 64 KB for 2-4 rows, 32 KB where x of 8-16
  // rows takes the shared memory
  static constexpr int kRingPerLane = (NB >= 8 || NB == 1) ? 128 : 256;
  // One batch row: two CTAs per SM (registers capped at 64 per thread), so the
  // grid holds 128 KB in flight per SM as before, and the next launch of a
  // decode step (a programmatic dependent) finds room on every SM while this
  // one streams: its ring fill and norm-weight prefetch run under it.
  static constexpr int kMinBlocks = NB == 1 ? 2 : 1;
  static constexpr int kStageV = NB == 1 ? 4 : 8;  // x chunks in flight per thread
  static constexpr int kCcItemGlu = 2;     // 16-byte chunks per lane per ring item
  static constexpr int kCcItemPlain = 4;
};

template <int NB>
__host__ __device__ __forceinline__ int64_t gemv_x_stride(int64_t k) {
  return NB == 1 ? k : k + 8;  // rows of x in smem start 4 banks apart
}

// Dynamic shared memory: x of NB rows, [the norm weight (one batch row with
// RMSNorm: prefetched before the dependency wait)], the weight-stream ring.
template <typename T, int NB>
__host__ __device__ __forceinline__ size_t gemv_x_bytes(int64_t k) {
  return (static_cast<size_t>(NB) * gemv_x_stride<NB>(k) * sizeof(T) + 127) / 128 * 128;
}

template <typename T, int NB>
__host__ __device__ __forceinline__ size_t gemv_nw_bytes(int64_t k, bool norm) {
  return (NB == 1 && norm) ? (static_cast<size_t>(k) * sizeof(T) + 127) / 128 * 128 : 0;
}

template <typename T, int NB>
size_t gemv_smem_bytes(int64_t k, bool norm) {
  return gemv_x_bytes<T, NB>(k) + gemv_nw_bytes<T, NB>(k, norm) +
         static_cast<size_t>(GemvShape<NB>::kThreads) * GemvShape<NB>::kRingPerLane;
}

constexpr int kArMaxRanks = 8;
// Exchange buffer: header {uint32 call epoch, uint32 CTAs done} (padded to
// 256 bytes), then words {fp32 value, epoch} [2 parities][world][kArBatch][n].
// The epoch belongs to the call, not to a CTA, and the batch stride is fixed:
// consecutive calls with different grids or batch slices then use disjoint
// parity halves for every (row, batch row) word, so a rank one call ahead
// never overwrites a word a slower rank has still to read.  Every call on one
// buffer has the same n (the buffer is sized for it; the tensor-parallel
// projections that all-reduce all produce the hidden size).
constexpr int64_t kArHeaderBytes = 256;
constexpr int kArBatch = 16;  // the widest batch one call takes
// rows one CTA of the CUDA-core form owns in an all-reduce call (a contiguous
// range; their partials are staged in shared memory, pushed group by group as
// coalesced writes, and summed after the loop)
constexpr int kArCtaRows = 256;

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
  int ksplit;
};

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

// Epoch of this call: one more than the previous call's, read after
// griddepcontrol.wait (every earlier kernel of the stream has completed).
__device__ __forceinline__ uint32_t ar_read_epoch(const GemvArgs& a) {
  const volatile uint32_t* hdr = reinterpret_cast<const volatile uint32_t*>(a.bufs[a.rank]);
  return hdr[0] + 1u;
}

// The last CTA of the call to get here stores the call's epoch (and re-arms
// the done counter) for the next call; a timed-out call advances it too, and
// the buffers of all ranks are then re-zeroed before the next use.
__device__ __forceinline__ void ar_finish_call(const GemvArgs& a, uint32_t e) {
  uint32_t* hdr = reinterpret_cast<uint32_t*>(a.bufs[a.rank]);
  __threadfence();
  if (atomicAdd(hdr + 1, 1u) == gridDim.x - 1) {
    hdr[1] = 0u;
    hdr[0] = e;
    __threadfence();
  }
}

__device__ __forceinline__ uint64_t gemv_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// All-reduce of the output values over the ranks (tensor-parallel
// row-parallel projection).  Words {fp32 value, epoch} in every rank's buffer,
// laid out [2 parities][world][kArBatch][n]: the words of consecutive rows of
// one batch row are consecutive, so the rows a CTA owns go to a peer as a few
// coalesced NVLink writes instead of one 8-byte write each (at 8 ranks the
// per-word form spent most of its time on the links' small-write rate).
// ar_word: the word of (source rank slot, batch row b, row) in buffer buf.
__device__ __forceinline__ uint2* ar_word(const GemvArgs& a, unsigned char* buf, int par,
                                          int slot, int b, int64_t row) {
  return reinterpret_cast<uint2*>(buf + kArHeaderBytes) +
         ((static_cast<int64_t>(par) * a.world + slot) * kArBatch + b) * a.n + row;
}

// ar_push stores this rank's partial for (row, b) into slot `rank` of every
// buffer (NVLink stores, no wait); ar_poll later reads all ranks' partials of
// (row, b) from this rank's buffer and returns their sum in rank order (the
// same on every rank), or false when the poll ran out of time (status word
// set).  Pushing every row first and polling afterwards costs one NVLink round
// trip per call instead of one per row group.
__device__ __forceinline__ void ar_push(const GemvArgs& a, uint32_t e, int64_t row, int b,
                                        float part) {
  const int par = static_cast<int>(e & 1u);
  for (int p = 0; p < a.world; ++p)
    st_volatile_u2(ar_word(a, a.bufs[p], par, a.rank, b, row), __float_as_uint(part), e);
}

__device__ __forceinline__ bool ar_poll(const GemvArgs& a, uint32_t e, int64_t row, int b,
                                        uint64_t t0, float& sum) {
  const int par = static_cast<int>(e & 1u);
  const int64_t slot_words = static_cast<int64_t>(kArBatch) * a.n;
  const uint2* own = ar_word(a, a.bufs[a.rank], par, 0, b, row);
  uint2 w[kArMaxRanks];
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

// Epilogue of one output value: projection rounding, SwiGLU, residual, store.
template <typename T, bool GLU>
__device__ __forceinline__ void emit_value(const GemvArgs& a, int64_t row, int b, float dot,
                                           float dot2) {
  float v = round_to<T>(dot);  // projection output in the model dtype
  if (GLU) {
    const float up = round_to<T>(dot2);
    const float sg = round_to<T>(v / (1.f + expf(-v)));  // act_fn(gate)
    v = round_to<T>(sg * up);
  }
  if (a.residual != nullptr)
    v = round_to<T>(to_float<T>(static_cast<const T*>(a.residual)[b * a.res_stride + row]) + v);
  if (a.y_fp32)
    static_cast<float*>(a.y)[b * a.y_stride + row] = v;
  else
    static_cast<T*>(a.y)[b * a.y_stride + row] = from_float<T>(v);
}

template <typename T>
__device__ __forceinline__ float sumsq8(const uint4& v) {
  const float2 a = unpack2<T>(v.x), b = unpack2<T>(v.y), c = unpack2<T>(v.z), d = unpack2<T>(v.w);
  float s = a.x * a.x;
  s = fmaf(a.y, a.y, s);
  s = fmaf(b.x, b.x, s);
  s = fmaf(b.y, b.y, s);
  s = fmaf(c.x, c.x, s);
  s = fmaf(c.y, c.y, s);
  s = fmaf(d.x, d.x, s);
  s = fmaf(d.y, d.y, s);
  return s;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// RMSNorm of 8 elements, rounding as HF's module does: xn = dtype(x * scale),
// y = dtype(w * xn).
template <typename T>
__device__ __forceinline__ uint4 norm8(const uint4& x, const uint4& w, float sc) {
  const uint32_t xi[4] = {x.x, x.y, x.z, x.w}, wi[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 xv = unpack2<T>(xi[i]), wv = unpack2<T>(wi[i]);
    o[i] = pack2<T>(wv.x * round_to<T>(xv.x * sc), wv.y * round_to<T>(xv.y * sc));
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Stages the NB rows of x into shared memory xs[NB][XS] (rows >= batch are
// zero), RMSNorm'd when norm_w is given.  Rows move as 16-byte chunks with
// kStageV loads in flight per thread, so staging costs about one memory round
// trip per pass: the first pass copies the raw row to shared memory and sums
// its squares, the second reads it back, normalises it with the (vector-
// loaded) norm weight and overwrites it.  Unaligned inputs take an element
// loop.
template <typename T, int NB, int kThreads, int kStageV>
__device__ __forceinline__ void stage_x(const GemvArgs& a, T* xs, int64_t XS, float* s_red,
                                        float* s_scale, const T* nw_smem = nullptr) {
  const int64_t K = a.k;
  const int64_t chunks = K / 8;
  const T* x = static_cast<const T*>(a.x);
  const T* nw = static_cast<const T*>(a.norm_w);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(nw) |
                     static_cast<uintptr_t>(a.x_stride * sizeof(T))) & 15u) == 0;
  for (int b = 0; b < NB; ++b) {
    T* row = xs + b * XS;
    uint4* row4 = reinterpret_cast<uint4*>(row);
    if (b >= a.batch) {
      for (int64_t c = tid; c < chunks; c += kThreads) row4[c] = make_uint4(0u, 0u, 0u, 0u);
      continue;
    }
    const T* xb = x + b * a.x_stride;
    float ss = 0.f;
    if (vec) {
      const uint4* src = reinterpret_cast<const uint4*>(xb);
      for (int64_t c0 = 0; c0 < chunks; c0 += static_cast<int64_t>(kStageV) * kThreads) {
        uint4 v[kStageV];
#pragma unroll
        for (int u = 0; u < kStageV; ++u) {
          const int64_t c = c0 + u * kThreads + tid;
          if (c < chunks) v[u] = src[c];
        }
#pragma unroll
        for (int u = 0; u < kStageV; ++u) {
          const int64_t c = c0 + u * kThreads + tid;
          if (c < chunks) {
            row4[c] = v[u];
            if (nw != nullptr) ss += sumsq8<T>(v[u]);
          }
        }
      }
    } else {
      for (int64_t i = tid; i < K; i += kThreads) {
        const T v = xb[i];
        row[i] = v;
        const float f = to_float<T>(v);
        ss = fmaf(f, f, ss);
      }
    }
    if (nw == nullptr) continue;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    if (tid == 0) {
      float t = 0.f;
      for (int w = 0; w < kThreads / 32; ++w) t += s_red[w];
      *s_scale = rsqrtf(t / static_cast<float>(K) + a.eps);
    }
    __syncthreads();
    const float sc = *s_scale;
    if (nw_smem != nullptr) {   // the norm weight is in shared memory already
      const uint4* wsrc = reinterpret_cast<const uint4*>(nw_smem);
      for (int64_t c = tid; c < chunks; c += kThreads) row4[c] = norm8<T>(row4[c], wsrc[c], sc);
    } else if (vec) {
      const uint4* wsrc = reinterpret_cast<const uint4*>(nw);
      for (int64_t c0 = 0; c0 < chunks; c0 += static_cast<int64_t>(kStageV) * kThreads) {
        uint4 wv[kStageV];
#pragma unroll
        for (int u = 0; u < kStageV; ++u) {
          const int64_t c = c0 + u * kThreads + tid;
          if (c < chunks) wv[u] = wsrc[c];
        }
#pragma unroll
        for (int u = 0; u < kStageV; ++u) {
          const int64_t c = c0 + u * kThreads + tid;
          if (c < chunks) row4[c] = norm8<T>(row4[c], wv[u], sc);
        }
      }
    } else {
      for (int64_t i = tid; i < K; i += kThreads) {
        const float xn = round_to<T>(to_float<T>(row[i]) * sc);   // x.to(dtype)
        row[i] = from_float<T>(to_float<T>(nw[i]) * xn);          // weight * x
      }
    }
    __syncthreads();
  }
  __syncthreads();
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Weight stream and math.  A warp owns a block of 16 weight rows and a slice
// of K.  Per 16-wide k-step, lane l copies (cp.async, 16 bytes) row l % 16,
// k-half l / 16 of the block into its own slot of a shared-memory ring; that
// slot is exactly the row address ldmatrix.x4 wants from lane l for the A
// fragment of mma.m16n8k16 (weight rows = M, k = K, batch rows = N, x read
// from shared memory as the B fragment).  Each lane waits only for its own
// copies (cp.async.wait_group) before the warp-wide ldmatrix, after a
// __syncwarp.  kDepth ring items per lane stay in flight without registers.
template <typename T, int NB, bool AR, bool GLU>
__global__ void __launch_bounds__(GemvShape<NB>::kThreads, 1) decode_gemv_kernel(const GemvArgs a) {
  constexpr int kGemvThreads = GemvShape<NB>::kThreads;
  constexpr int kGemvWarps = GemvShape<NB>::kWarps;
  constexpr int kStreams = GLU ? 2 : 1;
  constexpr int kU = GLU ? 2 : 4;  // k-steps per ring item
  constexpr int kDepth = GemvShape<NB>::kRingPerLane / (16 * kU * kStreams);
  static_assert(kDepth >= 2, "ring needs two items");
  constexpr int NT = NB <= 8 ? 1 : 2;  // n-tiles of 8 batch columns
  extern __shared__ __align__(128) uint8_t gemv_smem[];
  const int64_t K = a.k;
  const int64_t XS = gemv_x_stride<NB>(K);  // padded: B-fragment reads avoid bank conflicts
  T* xs = reinterpret_cast<T*>(gemv_smem);  // [NB][XS]
  const uint32_t ring = smem_addr(gemv_smem) +
                        static_cast<uint32_t>((NB * XS * sizeof(T) + 127) / 128 * 128);
  __shared__ float s_red[kGemvWarps];
  __shared__ float s_scale;
  __shared__ float s_part[kGemvWarps][16][NB][kStreams];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const T* W = static_cast<const T*>(a.w);
  const T* W2 = static_cast<const T*>(a.w2);
  const int64_t ksteps = K / 16;
  // Later kernels may be placed now, except after the all-reduce form: an
  // early trigger there made 16-row, batch-sliced all-reduce calls on two
  // GPUs time out in their poll, so its dependents start only when it ends.
  if (!AR) asm volatile("griddepcontrol.launch_dependents;");

  // ---- work: a CTA iteration covers (kGemvWarps / ksplit) row blocks of 16
  //      rows; a block's K is split over ksplit warps ----
  const int ksplit = a.ksplit;
  const int rpi = (kGemvWarps / ksplit) * 16;
  const int wrow = warp / ksplit, ws = warp - (warp / ksplit) * ksplit;
  const int64_t kss = (ksteps + ksplit - 1) / ksplit;
  const int64_t ks_begin = ws * kss, ks_end = min(ksteps, ks_begin + kss);
  const int nj = static_cast<int>((kss + kU - 1) / kU);  // items per row block
  const int64_t first = static_cast<int64_t>(blockIdx.x) * rpi;
  const int64_t gstride = static_cast<int64_t>(gridDim.x) * rpi;
  const int n_groups = first < a.n ? static_cast<int>((a.n - first + gstride - 1) / gstride) : 0;
  const int total = n_groups * nj;

  auto slot_addr = [&](int r, int stream, int u) -> uint32_t {
    return ring + static_cast<uint32_t>((((r * kStreams + stream) * kU + u) * kGemvThreads +
                                         threadIdx.x) * 16);
  };
  int issued = 0, ig = 0, jg = 0, ir = 0;
  auto issue_next = [&]() {
    if (issued < total) {
      const int64_t rowc = first + ig * gstride + wrow * 16 + (lane & 15);
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t kst = ks_begin + jg * kU + u;
        const bool ok = rowc < a.n && kst < ks_end;
        const int64_t off = ok ? rowc * K + kst * 16 + (lane >> 4) * 8 : 0;
        cp_async_16(slot_addr(ir, 0, u), W + off, ok ? 16u : 0u);
        if (GLU) cp_async_16(slot_addr(ir, 1, u), W2 + off, ok ? 16u : 0u);
      }
      ++issued;
      if (++jg == nj) {
        jg = 0;
        ++ig;
      }
      if (++ir == kDepth) ir = 0;
    }
    cp_async_commit();  // one group per item (empty past the end): uniform wait counts
  };
  // the weights are static: fill the ring before waiting for the kernel before
  // this one (which writes x / the residual) and while x is staged
#pragma unroll 1
  for (int i = 0; i < kDepth - 1; ++i) issue_next();
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // all-reduce: the call's epoch (the previous call on this stream has
  // completed and advanced it), advanced by the last CTA to finish
  __shared__ uint32_t s_epoch;
  __shared__ int s_ar_ok;
  if (AR && threadIdx.x == 0) {
    s_epoch = ar_read_epoch(a);
    s_ar_ok = 1;
  }

  // ---- stage x (rows >= batch are zero), RMSNorm'd when norm_w is given ----
  stage_x<T, NB, kGemvThreads, GemvShape<NB>::kStageV>(a, xs, XS, s_red, &s_scale);

  float acc[NT][4], acc2[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[nt][e] = acc2[nt][e] = 0.f;
  int g = 0, j = 0, cr = 0;  // consume pointer: row group, item in the block, ring slot
#pragma unroll 1
  for (int i = 0; i < total; ++i) {
    issue_next();
    cp_async_wait<kDepth - 1>();  // this lane's copies of item i have landed
    __syncwarp();                 // ... and every lane's, before ldmatrix reads them
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t kst = ks_begin + j * kU + u;
      if (kst < ks_end) {  // uniform over the warp
        uint32_t af[4];
        ldsm_x4(slot_addr(cr, 0, u), af[0], af[1], af[2], af[3]);
        uint32_t af2[4];
        if (GLU) ldsm_x4(slot_addr(cr, 1, u), af2[0], af2[1], af2[2], af2[3]);
        const int64_t kk = kst * 16 + 2 * tq;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int col = nt * 8 + gq;
          uint32_t b0 = 0u, b1 = 0u;
          if (col < NB) {
            b0 = *reinterpret_cast<const uint32_t*>(xs + col * XS + kk);
            b1 = *reinterpret_cast<const uint32_t*>(xs + col * XS + kk + 8);
          }
          MmaOp<T>::run(acc[nt], af, b0, b1);
          if (GLU) MmaOp<T>::run(acc2[nt], af2, b0, b1);
        }
      }
    }
    __syncwarp();  // all lanes have read item i's slots before they are refilled
    if (++cr == kDepth) cr = 0;
    const bool block_done = ++j == nj;
    if (block_done) {
      j = 0;
      ++g;
    }
    if (!block_done) continue;
    // ---- end of row group: combine the K slices, epilogue ----
    // thread (gq, tq) holds rows gq / gq + 8, columns nt*8 + 2tq (+1)
    const int64_t rb = first + (g - 1) * gstride + wrow * 16;
    if (ksplit > 1) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = gq + (e >> 1) * 8, c = nt * 8 + 2 * tq + (e & 1);
          if (c < NB) {
            s_part[warp][r][c][0] = acc[nt][e];
            if (GLU) s_part[warp][r][c][kStreams - 1] = acc2[nt][e];
          }
        }
      __syncthreads();
      if (ws == 0) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int r = gq + (e >> 1) * 8, c = nt * 8 + 2 * tq + (e & 1);
            if (c < NB) {
              float t = 0.f, t2 = 0.f;
              for (int q = 0; q < ksplit; ++q) {
                t += s_part[warp + q][r][c][0];
                if (GLU) t2 += s_part[warp + q][r][c][kStreams - 1];
              }
              acc[nt][e] = t;
              acc2[nt][e] = t2;
            }
          }
      }
      __syncthreads();
    }
    if (ws == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t row = rb + gq + (e >> 1) * 8;
          const int b = nt * 8 + 2 * tq + (e & 1);
          if (b >= a.batch || row >= a.n) continue;
          if (AR)
            ar_push(a, s_epoch, row, b, acc[nt][e]);  // summed and emitted after the loop
          else
            emit_value<T, GLU>(a, row, b, acc[nt][e], acc2[nt][e]);
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nt][e] = acc2[nt][e] = 0.f;
  }
  cp_async_wait<0>();
  if (AR && ws == 0) {  // every partial of this CTA is out: sum the ranks', emit
    const uint64_t t0 = gemv_timer_ns();
    for (int g2 = 0; g2 < n_groups; ++g2) {
      const int64_t rb2 = first + g2 * gstride + wrow * 16;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int64_t row = rb2 + gq + (e >> 1) * 8;
          const int b = nt * 8 + 2 * tq + (e & 1);
          if (b >= a.batch || row >= a.n) continue;
          float sum = 0.f;
          if (!ar_poll(a, s_epoch, row, b, t0, sum)) {
            atomicExch(&s_ar_ok, 0);
            continue;
          }
          emit_value<T, GLU>(a, row, b, sum, 0.f);
        }
    }
  }
  if (AR) {
    __syncthreads();
    if (threadIdx.x == 0) ar_finish_call(a, s_epoch);
  }
}

// Narrow batches (1-2 rows): one weight row per warp (split along K over
// ksplit warps for long rows), CUDA-core FMAs on 16-byte chunks; the same
// cp.async ring, each lane reading back only the chunks it copied.  Finer
// work units than the 16-row blocks of the tensor-core form, which matters
// when one row of x leaves the tensor cores idle anyway.
template <typename T, int NB, bool AR, bool GLU>
__global__ void __launch_bounds__(GemvShape<NB>::kThreads, GemvShape<NB>::kMinBlocks)
    decode_gemv_cc_kernel(const GemvArgs a) {
  constexpr int kGemvThreads = GemvShape<NB>::kThreads;
  constexpr int kGemvWarps = GemvShape<NB>::kWarps;
  constexpr int kStreams = GLU ? 2 : 1;
  // 16-byte chunks per lane (and stream) per ring item
  constexpr int kU = GLU ? GemvShape<NB>::kCcItemGlu : GemvShape<NB>::kCcItemPlain;
  constexpr int kDepth = GemvShape<NB>::kRingPerLane / (16 * kU * kStreams);
  static_assert(kDepth >= 2, "ring needs two items");
  extern __shared__ __align__(128) uint8_t gemv_smem[];
  const int64_t K = a.k;
  const int64_t XS = gemv_x_stride<NB>(K);
  T* xs = reinterpret_cast<T*>(gemv_smem);  // [NB][XS]
  const bool nw_pre = NB == 1 && a.norm_w != nullptr &&
                      (reinterpret_cast<uintptr_t>(a.norm_w) & 15u) == 0;
  T* nws = reinterpret_cast<T*>(gemv_smem + gemv_x_bytes<T, NB>(K));  // [K] when nw_pre
  const uint32_t ring = smem_addr(gemv_smem) +
                        static_cast<uint32_t>(gemv_x_bytes<T, NB>(K) +
                                              gemv_nw_bytes<T, NB>(K, a.norm_w != nullptr));
  __shared__ float s_red[kGemvWarps];
  __shared__ float s_scale;
  __shared__ float s_part[kGemvWarps][NB][2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* W = static_cast<const T*>(a.w);
  const T* W2 = static_cast<const T*>(a.w2);
  const int64_t chunks = K / 8;  // 16-byte chunks per row
  if (!AR) asm volatile("griddepcontrol.launch_dependents;");  // (see decode_gemv_kernel)
  const int ksplit = a.ksplit;              // warps per row (divides kGemvWarps)
  const int rpi = kGemvWarps / ksplit;      // rows per CTA iteration
  const int wrow = warp / ksplit, ws = warp - (warp / ksplit) * ksplit;
  const int64_t cs = (chunks + ksplit - 1) / ksplit;
  const int64_t c_begin = ws * cs, c_end = min(chunks, c_begin + cs);
  const int nj = static_cast<int>((cs + 32 * kU - 1) / (32 * kU));  // items per row
  // row groups of this CTA: strided over the grid, or (all-reduce) one
  // contiguous range, so that its rows' words are contiguous in the exchange
  // buffers (groups shared out evenly, one more or less per CTA)
  int64_t first, gstride;
  int n_groups;
  if (AR) {
    const int64_t groups = (a.n + rpi - 1) / rpi;
    const int64_t g0 = groups * blockIdx.x / gridDim.x;
    const int64_t g1 = groups * (blockIdx.x + 1) / gridDim.x;
    first = g0 * rpi;
    gstride = rpi;
    n_groups = static_cast<int>(g1 - g0);
  } else {
    first = static_cast<int64_t>(blockIdx.x) * rpi;
    gstride = static_cast<int64_t>(gridDim.x) * rpi;
    n_groups = first < a.n ? static_cast<int>((a.n - first + gstride - 1) / gstride) : 0;
  }
  const int total = n_groups * nj;
  // all-reduce: this CTA's partials, [row - first][batch row], pushed together
  __shared__ float s_ar[AR ? kArCtaRows : 1][NB];
  auto slot_addr = [&](int r, int stream, int u) -> uint32_t {
    return ring + static_cast<uint32_t>((((r * kStreams + stream) * kU + u) * kGemvThreads +
                                         threadIdx.x) * 16);
  };
  int issued = 0, ig = 0, jg = 0, ir = 0;
  auto issue_next = [&]() {
    if (issued < total) {
      const int64_t row = first + ig * gstride + wrow;
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t c = c_begin + lane + 32 * (jg * kU + u);
        const bool ok = row < a.n && c < c_end;
        const int64_t off = ok ? row * K + c * 8 : 0;
        cp_async_16(slot_addr(ir, 0, u), W + off, ok ? 16u : 0u);
        if (GLU) cp_async_16(slot_addr(ir, 1, u), W2 + off, ok ? 16u : 0u);
      }
      ++issued;
      if (++jg == nj) {
        jg = 0;
        ++ig;
      }
      if (++ir == kDepth) ir = 0;
    }
    cp_async_commit();
  };
  // the norm weight and the first ring items are static: fetch them before
  // waiting for the kernel before this one (which writes x)
  if (nw_pre) {
    const T* nwg = static_cast<const T*>(a.norm_w);
    for (int64_t c = threadIdx.x; c < chunks; c += kGemvThreads)
      cp_async_16(smem_addr(nws + c * 8), nwg + c * 8, 16u);
  }
  cp_async_commit();   // the oldest group: complete once the ring's first wait passes
#pragma unroll 1
  for (int i = 0; i < kDepth - 1; ++i) issue_next();
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ uint32_t s_epoch;
  __shared__ int s_ar_ok;
  if (AR && threadIdx.x == 0) {
    s_epoch = ar_read_epoch(a);
    s_ar_ok = 1;
  }
  cp_async_wait<kDepth - 1>();   // this thread's norm-weight chunks have landed
  stage_x<T, NB, kGemvThreads, GemvShape<NB>::kStageV>(a, xs, XS, s_red, &s_scale,
                                                        nw_pre ? nws : nullptr);
  float acc[NB], acc2[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) acc[b] = acc2[b] = 0.f;
  int g = 0, j = 0, cr = 0;
#pragma unroll 1
  for (int i = 0; i < total; ++i) {
    issue_next();
    cp_async_wait<kDepth - 1>();
    const int64_t row = first + g * gstride + wrow;
    if (row < a.n) {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t c = c_begin + lane + 32 * (j * kU + u);
        if (c < c_end) {
          uint4 wv, wv2;
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(wv.x), "=r"(wv.y), "=r"(wv.z), "=r"(wv.w)
                       : "r"(slot_addr(cr, 0, u)));
          if (GLU)
            asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(wv2.x), "=r"(wv2.y), "=r"(wv2.z), "=r"(wv2.w)
                         : "r"(slot_addr(cr, 1, u)));
#pragma unroll
          for (int b = 0; b < NB; ++b) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + b * XS + c * 8);
            acc[b] += dot8<T>(wv, xv);
            if (GLU) acc2[b] += dot8<T>(wv2, xv);
          }
        }
      }
    }
    if (++cr == kDepth) cr = 0;
    const bool row_done = ++j == nj;
    if (row_done) {
      j = 0;
      ++g;
    }
    if (!row_done) continue;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], o);
        if (GLU) acc2[b] += __shfl_xor_sync(0xffffffffu, acc2[b], o);
      }
    }
    if (ksplit > 1) {
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (lane == b) {
          s_part[warp][b][0] = acc[b];
          s_part[warp][b][1] = acc2[b];
        }
      __syncthreads();
      if (ws == 0) {
#pragma unroll
        for (int b = 0; b < NB; ++b)
          if (lane == b) {
            float t = 0.f, t2 = 0.f;
            for (int q = 0; q < ksplit; ++q) {
              t += s_part[warp + q][b][0];
              t2 += s_part[warp + q][b][1];
            }
            acc[b] = t;
            acc2[b] = t2;
          }
      }
      __syncthreads();
    }
    if (ws == 0 && row < a.n) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (lane != b || b >= a.batch) continue;
        if (AR)
          s_ar[row - first][b] = acc[b];  // pushed below, summed and emitted after the loop
        else
          emit_value<T, GLU>(a, row, b, acc[b], acc2[b]);
      }
    }
    if (AR) {
      // push the group's rows to every rank now, while the next group streams:
      // word (this rank, b, row), consecutive threads on consecutive rows, so
      // the group's rows of one batch row leave as one contiguous write
      __syncthreads();
      const int64_t g0 = first + static_cast<int64_t>(g - 1) * gstride;
      const int grows = static_cast<int>(min(a.n, g0 + rpi) - g0);
      const int items = a.world * a.batch * grows;
      for (int it = threadIdx.x; it < items; it += kGemvThreads) {
        const int r = it % grows, pb = it / grows;
        const int b = pb % a.batch, p = pb / a.batch;
        st_volatile_u2(ar_word(a, a.bufs[p], static_cast<int>(s_epoch & 1u), a.rank, b, g0 + r),
                       __float_as_uint(s_ar[g0 + r - first][b]), s_epoch);
      }
    }
#pragma unroll
    for (int b = 0; b < NB; ++b) acc[b] = acc2[b] = 0.f;
  }
  cp_async_wait<0>();
  if (AR) {
    const int rows = static_cast<int>(min(a.n, first + static_cast<int64_t>(n_groups) * rpi) - first);
    // every row of this CTA is pushed: poll this rank's buffer for every
    // rank's words of our rows, sum in rank order, emit (consecutive threads,
    // consecutive rows)
    const uint64_t t0 = gemv_timer_ns();
    for (int it = threadIdx.x; it < a.batch * max(rows, 0); it += kGemvThreads) {
      const int r = it % rows, b = it / rows;
      float sum = 0.f;
      if (!ar_poll(a, s_epoch, first + r, b, t0, sum)) {
        atomicExch(&s_ar_ok, 0);
        break;
      }
      emit_value<T, GLU>(a, first + r, b, sum, 0.f);
    }
    __syncthreads();
    if (threadIdx.x == 0) ar_finish_call(a, s_epoch);
  }
}

template <typename T, int NB, bool AR, bool GLU>
int launch_gemv(const GemvArgs& a, cudaStream_t stream) {
  // narrow batches: CUDA-core form with one row per warp; wider: tensor cores
  constexpr bool kMma = NB >= 4;
  auto kernel = kMma ? decode_gemv_kernel<T, NB, AR, GLU> : decode_gemv_cc_kernel<T, NB, AR, GLU>;
  static size_t configured[64] = {0};  // dynamic smem allowed so far, per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return HELM_ERR_CUDA;
  const size_t smem = gemv_smem_bytes<T, NB>(a.k, a.norm_w != nullptr);
  // dynamic + static (the K-slice partials) shared memory of one CTA
  if (smem + sizeof(float) * GemvShape<NB>::kWarps * 16 * NB * 2 + 1024 > kGemvMaxSmem)
    return HELM_ERR_UNSUPPORTED;
  if (smem > configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return HELM_ERR_CUDA;
    configured[dev] = smem;
  }
  // one wave of resident CTAs looping over row groups (with the all-reduce,
  // every CTA must be resident at once: CTA c waits for CTA c of the other
  // ranks, whose own CTAs may wait for ours)
  int fit = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&fit, kernel, GemvShape<NB>::kThreads, smem) !=
          cudaSuccess ||
      fit <= 0)
    return HELM_ERR_CUDA;
  constexpr int kWarps = GemvShape<NB>::kWarps;
  GemvArgs args = a;
  // K split over ksplit warps of a CTA, chosen to minimise the busiest warp's
  // ring items: ceil(row groups / CTAs) x ceil(K slice / item width), where an
  // item is 32 lanes x kU chunks (CUDA-core form) or kU k-steps of a 16-row
  // block (tensor cores); each extra split adds a barrier per row group
  const int grid_max = num_sms_current_device() * fit;
  const int unit = kMma ? 16 : 1;  // rows of one warp task
  const int64_t k_units = kMma ? a.k / 16 : a.k / 8;
  const int64_t item_units =
      kMma ? (GLU ? 2 : 4)
           : 32 * (GLU ? GemvShape<NB>::kCcItemGlu : GemvShape<NB>::kCcItemPlain);
  int ks = 1;
  double best = 1e30;
  for (int c = 1; c <= kWarps; c *= 2) {
    const int64_t slice = (k_units + c - 1) / c;
    if (c > 1 && slice < item_units) break;
    const int64_t rows_per_group = static_cast<int64_t>(kWarps / c) * unit;
    const int64_t groups = (a.n + rows_per_group - 1) / rows_per_group;
    const int64_t iters = (groups + grid_max - 1) / grid_max;
    const double cost = static_cast<double>(iters) *
                        (static_cast<double>((slice + item_units - 1) / item_units) +
                         (c > 1 ? 0.5 : 0.0));
    if (cost < best) {
      best = cost;
      ks = c;
    }
  }
  args.ksplit = ks;
  const int rpi = (kWarps / ks) * unit;
  const int64_t want = (a.n + rpi - 1) / rpi;
  const int grid = static_cast<int>(std::min<int64_t>(want, int64_t(num_sms_current_device()) * fit));
  if (AR && a.batch > kArBatch) return HELM_ERR_UNSUPPORTED;
  // CUDA-core all-reduce: a CTA's contiguous rows are staged in shared memory
  if (AR && !kMma && (want + grid - 1) / grid * rpi > kArCtaRows) return HELM_ERR_UNSUPPORTED;
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
  return cudaLaunchKernelEx(&cfg, kernel, args) == cudaSuccess
             ? HELM_OK
             : HELM_ERR_CUDA;
}

template <typename T, int NB, bool AR>
int launch_gemv_glu(const GemvArgs& a, cudaStream_t s) {
  return a.w2 != nullptr ? launch_gemv<T, NB, AR, true>(a, s) : launch_gemv<T, NB, AR, false>(a, s);
}

template <typename T, bool AR>
int dispatch_gemv(const GemvArgs& a, cudaStream_t s) {
  if (a.batch <= 1) return launch_gemv_glu<T, 1, AR>(a, s);
  if (a.batch <= 2) return launch_gemv_glu<T, 2, AR>(a, s);
  if (a.batch <= 4) return launch_gemv_glu<T, 4, AR>(a, s);
  if (a.batch <= 8) return launch_gemv_glu<T, 8, AR>(a, s);
  return launch_gemv_glu<T, 16, AR>(a, s);
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
  if (batch > helm::kArBatch) return -1;
  return helm::kArHeaderBytes + 2 * static_cast<int64_t>(world) * n * helm::kArBatch * 8;
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
  if (k % 16 != 0) return HELM_ERR_UNSUPPORTED;
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
