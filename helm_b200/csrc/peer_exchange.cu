// Exchange + merge of sequence-split partial attention states over peer memory.
//
// Each rank of a sequence split holds a token range of every sequence and
// computes the partial state (O fp32 [rows, D], LSE fp32 [rows]) of its range.
// Every rank then needs the merge of all ranks' states.  Instead of an NCCL
// all-gather followed by a merge kernel, one kernel does both over NVLink, in
// a flag-in-data format: every 8-byte word of the exchange buffer holds one
// fp32 value and the epoch (step number) it belongs to, written together by a
// single store, so a reader that sees the epoch in a word sees its value --
// no fences and no separate flags.
//
//   1. CTA c stores rows [c*chunk, (c+1)*chunk) of this rank's state, tagged
//      with the epoch, into slot `rank` of every rank's exchange buffer
//      (NVLink stores through CUDA IPC mappings);
//   2. each thread polls (bounded) the words it needs from every rank's slot
//      in its own buffer until all carry the epoch, then merges:
//      M = max_r LSE_r, O = sum_r e^(LSE_r - M) O_r / sum_r e^(LSE_r - M),
//      LSE = M + log(sum).
//
// Epochs live in device memory (one counter per CTA, advanced by that CTA at
// its end), so the kernel needs no host-side step number and replays inside
// CUDA graphs.  Data slots alternate by epoch parity.  A rank finishes step e
// only after reading every rank's step-e words, which each rank stores at the
// start of its step-e kernel, after its step e-1 kernel ended; so no rank
// can store step e+1 data before every rank has finished reading step e-1,
// the last user of that parity.  A poll that exceeds timeout_ns sets
// HELM_DEV_TIMEOUT in the device status word and the CTA returns without
// merging or advancing its epoch; the exchange buffers must then be
// re-zeroed by all ranks before the next call.
//
// Exchange buffer layout (identical on every rank, zeroed at allocation):
//   [0, 512)       uint32 epoch per CTA (kMaxChunks), local only
//   [8192, ...)    words {fp32 value, uint32 epoch} [2 parities][world][stride],
//                  stride = rows*D + rows rounded up to an even count; a slot
//                  holds O (rows*D values) then LSE (rows values).

namespace helm {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxChunks = 128;
constexpr int64_t kHeaderBytes = 8192;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void st_volatile_v4(uint2* p, uint32_t a, uint32_t b, uint32_t c,
                                               uint32_t d) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b),
               "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ void st_volatile_v2(uint2* p, uint32_t a, uint32_t b) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}

__device__ __forceinline__ uint4 ld_volatile_v4(const uint2* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ uint2 ld_volatile_v2(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

struct PeerExchangeArgs {
  unsigned char* bufs[kMaxRanks];  // every rank's exchange buffer, mapped here
  const float* o_part;             // this rank's O [rows, D]
  const float* lse_part;           // this rank's LSE [rows]
  void* out;                       // merged O [rows, D] in out_dtype
  float* lse_out;                  // merged LSE [rows] (optional)
  int64_t rows;
  int64_t stride;                  // words per data slot
  uint64_t timeout_ns;
  int rank, world, head_dim, chunk_rows, out_dtype;
};

__device__ __forceinline__ uint2* slot_ptr(unsigned char* buf, int64_t stride, int world, int par,
                                           int r) {
  return reinterpret_cast<uint2*>(buf + kHeaderBytes) + ((int64_t)par * world + r) * stride;
}

__global__ void __launch_bounds__(128) seq_exchange_merge_kernel(PeerExchangeArgs a) {
  // Launched as a programmatic dependent: placed while the kernel before it
  // (the decode kernel and its merge, which write o_part / lse_part) finishes;
  // everything below waits for it.  The next call's decode kernel may be
  // placed now (it reads no exchange state and writes only after waiting).
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int c = blockIdx.x;
  const int D = a.head_dim;
  const int64_t r0 = (int64_t)c * a.chunk_rows;
  const int64_t r1 = min(a.rows, r0 + a.chunk_rows);
  uint32_t* my_epochs = reinterpret_cast<uint32_t*>(a.bufs[a.rank]);
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_epoch = my_epochs[c] + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int par = static_cast<int>(e & 1u);

  // 1. push this CTA's rows, tagged with the epoch, into slot `rank` of every rank
  const int64_t n2 = (r1 - r0) * D / 2;  // pairs of O values
  const float2* src2 = reinterpret_cast<const float2*>(a.o_part + r0 * D);
  for (int p = 0; p < a.world; ++p) {
    uint2* dst = slot_ptr(a.bufs[p], a.stride, a.world, par, a.rank);
    for (int64_t i = threadIdx.x; i < n2; i += blockDim.x) {
      const float2 v = src2[i];
      st_volatile_v4(dst + r0 * D + 2 * i, __float_as_uint(v.x), e, __float_as_uint(v.y), e);
    }
    for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x)
      st_volatile_v2(dst + a.rows * D + r, __float_as_uint(a.lse_part[r]), e);
  }

  // 2. poll and merge: thread owns (row, 2 dims); all ranks' words are loaded
  //    together and only missing ones re-polled
  const int halfD = D / 2;
  const uint64_t t0 = global_timer_ns();
  bool ok = true;
  for (int64_t i = threadIdx.x; ok && i < n2; i += blockDim.x) {
    const int64_t row = r0 + i / halfD;
    const int d = static_cast<int>(i - (i / halfD) * halfD) * 2;
    uint4 ow[kMaxRanks];
    uint2 lw[kMaxRanks];
    bool ready = false;
    for (int spin = 0; !ready; ++spin) {
      ready = true;
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r >= a.world) break;
        if (spin == 0 || lw[r].y != e || ow[r].y != e || ow[r].w != e) {
          const uint2* slot = slot_ptr(a.bufs[a.rank], a.stride, a.world, par, r);
          lw[r] = ld_volatile_v2(slot + a.rows * D + row);
          ow[r] = ld_volatile_v4(slot + row * D + d);
        }
      }
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r >= a.world) break;
        ready = ready && lw[r].y == e && ow[r].y == e && ow[r].w == e;
      }
      if (!ready && (spin & 15) == 15 && global_timer_ns() - t0 > a.timeout_ns) {
        report_status(HELM_DEV_TIMEOUT);
        ok = false;
        break;
      }
    }
    if (!ok) break;
    float M = -INFINITY;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < a.world) M = fmaxf(M, __uint_as_float(lw[r].x));
    const float m_use = M == -INFINITY ? 0.f : M;
    float L = 0.f, acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r >= a.world) break;
      const float w = expf(__uint_as_float(lw[r].x) - m_use);
      L += w;
      if (w > 0.f) {
        acc0 += w * __uint_as_float(ow[r].x);
        acc1 += w * __uint_as_float(ow[r].z);
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    store_dt(a.out, a.out_dtype, row * D + d, acc0 * inv);
    store_dt(a.out, a.out_dtype, row * D + d + 1, acc1 * inv);
    if (d == 0 && a.lse_out != nullptr)
      a.lse_out[row] = (M == -INFINITY || L <= 0.f) ? -INFINITY : M + logf(L);
  }
  if (!ok) atomicExch(&s_ok, 0);
  __syncthreads();
  if (threadIdx.x == 0 && s_ok) my_epochs[c] = e;
}

struct ExchangeGeometry {
  int64_t stride;
  int chunk_rows;
  int chunks;
};

ExchangeGeometry exchange_geometry(int64_t rows, int head_dim) {
  ExchangeGeometry g;
  g.stride = (rows * head_dim + rows + 1) / 2 * 2;
  g.chunk_rows = static_cast<int>((rows + kMaxChunks - 1) / kMaxChunks);
  g.chunks = static_cast<int>((rows + g.chunk_rows - 1) / g.chunk_rows);
  return g;
}

}  // namespace
}  // namespace helm

extern "C" int64_t helm_peer_exchange_bytes(int64_t rows, int head_dim, int world) {
  using namespace helm;
  if (rows <= 0 || head_dim <= 0 || head_dim % 4 != 0 || world < 1 || world > kMaxRanks) return -1;
  const ExchangeGeometry g = exchange_geometry(rows, head_dim);
  return kHeaderBytes + 2 * static_cast<int64_t>(world) * g.stride * 8;
}

extern "C" int helm_ipc_alloc(int64_t bytes, void** ptr_out) {
  using namespace helm;
  if (bytes <= 0 || ptr_out == nullptr) return HELM_ERR_INVALID_ARGUMENT;
  *ptr_out = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  *ptr_out = p;
  return HELM_OK;
}

extern "C" int helm_ipc_free(void* ptr) {
  using namespace helm;
  if (ptr == nullptr) return HELM_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  return HELM_OK;
}

extern "C" int helm_ipc_zero(void* ptr, int64_t bytes, void* stream) {
  using namespace helm;
  if (ptr == nullptr || bytes <= 0) return HELM_ERR_INVALID_ARGUMENT;
  const cudaError_t e =
      cudaMemsetAsync(ptr, 0, static_cast<size_t>(bytes), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  return HELM_OK;
}

extern "C" int helm_ipc_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }

extern "C" int helm_ipc_get_handle(const void* ptr, void* handle_out) {
  using namespace helm;
  if (ptr == nullptr || handle_out == nullptr) return HELM_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  std::memcpy(handle_out, &h, sizeof(h));
  return HELM_OK;
}

extern "C" int helm_ipc_open(const void* handle, void** ptr_out) {
  using namespace helm;
  if (handle == nullptr || ptr_out == nullptr) return HELM_ERR_INVALID_ARGUMENT;
  *ptr_out = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  return HELM_OK;
}

extern "C" int helm_ipc_close(void* ptr) {
  using namespace helm;
  if (ptr == nullptr) return HELM_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  return HELM_OK;
}

extern "C" int helm_seq_exchange_merge(void* const* bufs, int rank, int world, const float* o_part,
                                       const float* lse_part, int64_t rows, int head_dim,
                                       void* out, int out_dtype, float* lse_out,
                                       uint64_t timeout_ns, void* stream) {
  using namespace helm;
  if (bufs == nullptr || o_part == nullptr || lse_part == nullptr || out == nullptr)
    return HELM_ERR_INVALID_ARGUMENT;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || rows <= 0 || head_dim <= 0 ||
      timeout_ns == 0)
    return HELM_ERR_INVALID_ARGUMENT;
  if (head_dim % 4 != 0 || head_dim > 1024) return HELM_ERR_UNSUPPORTED;
  if (out_dtype != HELM_DTYPE_FP32 && out_dtype != HELM_DTYPE_FP16 && out_dtype != HELM_DTYPE_BF16)
    return HELM_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(o_part) & 7u) != 0) return HELM_ERR_ALIGNMENT;
  PeerExchangeArgs a;
  for (int r = 0; r < kMaxRanks; ++r) a.bufs[r] = nullptr;
  for (int r = 0; r < world; ++r) {
    if (bufs[r] == nullptr || (reinterpret_cast<uintptr_t>(bufs[r]) & 255u) != 0)
      return HELM_ERR_ALIGNMENT;
    a.bufs[r] = static_cast<unsigned char*>(bufs[r]);
  }
  const ExchangeGeometry g = exchange_geometry(rows, head_dim);
  a.o_part = o_part;
  a.lse_part = lse_part;
  a.out = out;
  a.lse_out = lse_out;
  a.rows = rows;
  a.stride = g.stride;
  a.timeout_ns = timeout_ns;
  a.rank = rank;
  a.world = world;
  a.head_dim = head_dim;
  a.chunk_rows = g.chunk_rows;
  a.out_dtype = out_dtype;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.chunks);
  cfg.blockDim = dim3(128);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, seq_exchange_merge_kernel, a);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return HELM_ERR_CUDA;
  }
  return HELM_OK;
}
