// Paged chunk-prefill attention on the 5th-generation tensor cores (tcgen05).
//
// Same computation, arguments and results as paged_prefill_kernel (HELM's
// q_len > 1 streaming attention, helm/runtime/kv_cache.py:469-555), with both
// products on tcgen05.mma and the score, probability and output tiles held in
// tensor memory:
//
//   CTA = 128 query rows of one (sequence, kv head) x one split of its keys;
//   rows as in paged_prefill_kernel ((position, query head of the GQA group),
//   head fastest).  Five warps:
//     warp 4      TMA loads of the K/V tiles (64 keys: four 16-row boxes per K
//                 and per V, each inside one page, x D/64 column boxes, 128-byte
//                 swizzle) into a 2-stage ring; one elected lane issues
//                   S[128 x 64]  = Q[128 x D] . K^T    (A, B in shared memory, K-major)
//                   O[128 x D]  += P[128 x 64] . V     (A = P in tensor memory,
//                                                       B = V in shared memory, N-major)
//                 and signals completion with tcgen05.commit on mbarriers
//     warps 0-3   one query row per thread (tensor-memory lane = row): read the
//                 row of S, scale or softcap, additive mask, causal limit, row
//                 max, P = exp2(x - m) written back to tensor memory in the
//                 input type.  The reference max m of a row moves only when the
//                 row's max grows by more than 8 (P <= 2^8 otherwise); when it
//                 moves, the warp rescales its rows of O in tensor memory after
//                 the previous P.V has completed.
//   Tensor memory (256 columns per CTA, two CTAs per SM): S [0, 64), P double
//   buffer [64, 96) and [96, 128), O [128, 128 + D).
//   Q is staged once into shared memory in the 128-byte-swizzled K-major
//   layout, the same layout the TMA boxes give K and V.
//
// Shared-memory descriptors follow the canonical tcgen05 layouts: K-major
// 128-byte swizzle (8-row groups 1024 B apart, a 16-element K step = +32 B of
// the start address) for Q and K; N-major 128-byte swizzle for V (64-column
// blocks kKVHalf apart, 8-key groups 1024 B apart, a 16-key step = +2048 B).
//
// This file is part of the single translation unit helm_b200.cu, after
// paged_prefill.cu (PrefillArgs, unit_keys, pf_mask, plan_prefill, the split
// merge kernel, the pool tensor map), and ends with the C entry points.

namespace helm {

namespace {

constexpr int kTcRows = 128;   // query rows per CTA = MMA M = tensor-memory lanes
constexpr int kTcTile = 64;    // keys per tile
constexpr int kTcSoftWarps = 4;
constexpr int kTcThreads = (kTcSoftWarps + 1) * 32;
constexpr int kTcNS = 2;       // K/V ring stages
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColP = 64, kColO = 128;
constexpr float kRescaleLog2 = 8.f;

template <int D>
struct TcLayout {
  static constexpr int KS = D / 16;                  // K steps of Q.K^T
  static constexpr int kQHalf = kTcRows * 128;       // one 64-column slab of Q
  static constexpr int kQBytes = kTcRows * D * 2;
  static constexpr int kKVHalf = kTcTile * 128;      // one 64-column slab of K or V
  static constexpr int kTileBytes = kTcTile * D * 2;
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kBoxes = D / 64;
  // at least 80 KB, so that no more than two CTAs (2 x 256 tensor-memory
  // columns) are resident on an SM
  static constexpr size_t smem_bytes() {
    return std::max<size_t>(80 * 1024, 1024 + kQBytes + kTcNS * kStageBytes + 16 * sizeof(uint64_t));
  }
};

// ----------------------------------------------------------- tcgen05 wrappers --
// Shared-memory matrix descriptor, 128-byte swizzle (layout code 2), Blackwell
// descriptor version 1 (bits 46-47), base offset 0 (1024-aligned atoms).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo_bytes,
                                              uint32_t sbo_bytes) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor of kind::f16: fp32 accumulate (bits 4-5 = 1), A/B
// type (bits 7-9 / 10-12: 0 f16, 1 bf16), B major (bit 16: 1 = N-major),
// N >> 3 (bits 17-22), M >> 4 (bits 24-28); A K-major, no negation.
__host__ __device__ constexpr uint32_t umma_idesc(bool bf16, int m, int n, bool b_n_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((b_n_major ? 1u : 0u) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma this thread issued before it
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive columns of this warp's 32 lanes (lane field of taddr = 32 x
// warp quarter): thread t gets lane t's columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

// Waits for this thread's tensor-memory loads; the registers are operands so
// that no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
        "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]),
        "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]),
        "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]),
        "+r"(r[31])
      :
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Every lane of the warp waits (bounded) for the phase; true when it completed.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  const bool ok = mbar_wait(bar, parity);
  return __all_sync(0xffffffffu, ok);
}

// Adds the additive mask (log2 units) of keys j0 .. j0+nvalid-1 of query
// position s to x[0 .. nvalid-1].  The dtype is chosen once per tile; a row
// chunk that is 16-byte aligned and complete is read with 16-byte loads, all
// issued before the first use.
template <int N>
__device__ __forceinline__ void add_mask_row(const PrefillArgs& a, int b, int s, int j0,
                                             int nvalid, float (&x)[N]) {
  const int64_t off = static_cast<int64_t>(b) * a.mask_sb + static_cast<int64_t>(s) * a.mask_sq + j0;
  if (a.mask_dtype == HELM_DTYPE_FP32) {
    const float* mp = static_cast<const float*>(a.mask) + off;
    if (nvalid == N && (reinterpret_cast<uintptr_t>(mp) & 15) == 0) {
      float4 v[N / 4];
#pragma unroll
      for (int i = 0; i < N / 4; ++i) v[i] = __ldg(reinterpret_cast<const float4*>(mp) + i);
#pragma unroll
      for (int i = 0; i < N / 4; ++i) {
        x[4 * i] += mask_log2(v[i].x);
        x[4 * i + 1] += mask_log2(v[i].y);
        x[4 * i + 2] += mask_log2(v[i].z);
        x[4 * i + 3] += mask_log2(v[i].w);
      }
    } else {
#pragma unroll
      for (int c = 0; c < N; ++c)
        if (c < nvalid) x[c] += mask_log2(__ldg(mp + c));
    }
    return;
  }
  const bool bf = a.mask_dtype == HELM_DTYPE_BF16;
  const uint16_t* mp = static_cast<const uint16_t*>(a.mask) + off;
  auto cvt = [bf](uint32_t h) -> float {
    return bf ? __uint_as_float(h << 16) : __half2float(__ushort_as_half(static_cast<unsigned short>(h)));
  };
  if (nvalid == N && (reinterpret_cast<uintptr_t>(mp) & 15) == 0) {
    uint4 v[N / 8];
#pragma unroll
    for (int i = 0; i < N / 8; ++i) v[i] = __ldg(reinterpret_cast<const uint4*>(mp) + i);
#pragma unroll
    for (int i = 0; i < N / 8; ++i) {
      const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        x[8 * i + 2 * e] += mask_log2(cvt(w[e] & 0xffffu));
        x[8 * i + 2 * e + 1] += mask_log2(cvt(w[e] >> 16));
      }
    }
  } else {
#pragma unroll
    for (int c = 0; c < N; ++c)
      if (c < nvalid) x[c] += mask_log2(cvt(__ldg(mp + c)));
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kTcThreads, 2)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap tmap, const PrefillArgs a) {
  using L = TcLayout<D>;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescQK = umma_idesc(kBf16, kTcRows, kTcTile, false);
  constexpr uint32_t kIdescPV = umma_idesc(kBf16, kTcRows, D, true);

  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t s_tmem;
  uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint8_t* sq = smem;
  uint8_t* skv = smem + L::kQBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(skv + kTcNS * L::kStageBytes);
  uint64_t* full = bars;                 // [kTcNS] K/V tile landed (TMA bytes)
  uint64_t* empty = bars + kTcNS;        // [kTcNS] P.V of the stage's tile completed
  uint64_t* bar_s = bars + 2 * kTcNS;    // S = Q.K^T completed
  uint64_t* bar_sfree = bar_s + 1;       // the 4 row warps have read S
  uint64_t* bar_p = bar_s + 2;           // [2] P buffer written (4 row warps)
  uint64_t* bar_o = bar_s + 4;           // [2] P.V of tiles with that parity completed
  uint64_t* bar_fin = bar_s + 6;         // drain after an abandoned wait: all MMAs done

  // blockIdx.x = ((b * hkv + h) * splits + split) * row_blocks + rb
  const int rb = blockIdx.x % a.row_blocks;
  const int rest = blockIdx.x / a.row_blocks;
  const int split = rest % a.splits;
  const int pair = rest / a.splits;
  const int b = pair / a.hkv, h = pair - (pair / a.hkv) * a.hkv;
  const int kv_u = unit_keys(a, b, rb, kTcRows);
  const int k_lo = unit_first_key(a, b, kv_u);
  const int t_lo = k_lo / kTcTile;
  const int n_tiles = (kv_u + kTcTile - 1) / kTcTile - t_lo;
  const int t_begin = t_lo + static_cast<int>(static_cast<int64_t>(n_tiles) * split / a.splits);
  const int t_end = t_lo + static_cast<int>(static_cast<int64_t>(n_tiles) * (split + 1) / a.splits);
  const int n = t_end - t_begin;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcNS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(bar_s, 1);
    mbar_init(bar_sfree, kTcSoftWarps);
    mbar_init(&bar_p[0], kTcSoftWarps);
    mbar_init(&bar_p[1], kTcSoftWarps);
    mbar_init(&bar_o[0], 1);
    mbar_init(&bar_o[1], 1);
    mbar_init(bar_fin, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&s_tmem)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // row of this thread (warps 0-3): tensor-memory lane threadIdx.x
  const int r = rb * kTcRows + threadIdx.x;
  const bool okr = warp < kTcSoftWarps && r < a.rows;
  const int s_pos = okr ? r / a.group : 0;
  const int qh = h * a.group + (okr ? r - s_pos * a.group : 0);
  if (warp < kTcSoftWarps) {
    // Q row -> shared memory, K-major 128-byte swizzle: 16-byte chunk c of row
    // t at slab c/8, row t * 128 B, chunk (c % 8) ^ (t % 8)
    const T* qrow = static_cast<const T*>(a.q) + static_cast<int64_t>(b) * a.q_sb +
                    static_cast<int64_t>(qh) * a.q_sh + static_cast<int64_t>(s_pos) * a.q_ss;
    const int t = threadIdx.x;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (okr) v = *reinterpret_cast<const uint4*>(qrow + c * 8);
      *reinterpret_cast<uint4*>(sq + (c >> 3) * L::kQHalf + t * 128 + (((c & 7) ^ (t & 7)) << 4)) = v;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  asm volatile("griddepcontrol.launch_dependents;");

  bool ok = true;
  if (warp == kTcSoftWarps) {
    // ============================== loads + MMAs ==============================
    int loads_issued = 0, loads_seen = 0;  // tiles whose TMA was issued / observed complete
    bool mma_issued = false;
    const int64_t kv_rows = static_cast<int64_t>(a.hkv) * a.page_size;
    const uint32_t sq_addr = smem_addr(sq), skv_addr = smem_addr(skv);
    auto fetch = [&](int i, int& slot, bool& okg) {
      const int j = (t_begin + i) * kTcTile + lane * 16;
      okg = lane < 4 && i < n && j < kv_u;
      slot = okg ? a.page_table[static_cast<int64_t>(b) * a.pt_sb + j / a.page_size] : 0;
    };
    auto issue = [&](int i, int slot, bool okg) {
      const int st = i % kTcNS;
      const unsigned issuing = __ballot_sync(0xffffffffu, okg);
      if (lane == 0) mbar_arrive_expect_tx(&full[st], __popc(issuing) * 2 * L::kBoxes * 2048);
      __syncwarp();
      if (okg) {
        if (slot < 0 || slot >= a.pool_pages) {
          report_status(HELM_DEV_BAD_PAGE);
          slot = 0;
        }
        const int j = (t_begin + i) * kTcTile + lane * 16;
        const int row_off = j - (j / a.page_size) * a.page_size;
        const int row_k = static_cast<int>(
            (static_cast<int64_t>(slot) * 2 * a.hkv + h) * a.page_size + row_off);
        const int row_v = static_cast<int>(row_k + kv_rows);
        uint8_t* kdst = skv + st * L::kStageBytes + lane * 2048;
#pragma unroll
        for (int hb = 0; hb < L::kBoxes; ++hb) {
          tma_load_2d(kdst + hb * L::kKVHalf, &tmap, hb * 64, row_k, &full[st]);
          tma_load_2d(kdst + L::kTileBytes + hb * L::kKVHalf, &tmap, hb * 64, row_v, &full[st]);
        }
      }
    };
    // O += P_jj . V_jj, then refill the stage with tile jj + kTcNS
    auto do_pv = [&](int jj) -> bool {
      const int st = jj % kTcNS;
      int slot;
      bool okg;
      fetch(jj + kTcNS, slot, okg);
      // keys of a partial tile past the unit's last key: their V rows hold
      // stale data (the page's unwritten rows, or an earlier tile where no
      // box was loaded) and P is 0 there, but 0 x NaN is NaN in the product,
      // so the rows are zeroed (the tile's TMA bytes have landed: QK waited)
      const int vend = kv_u - (t_begin + jj) * kTcTile;
      if (vend < kTcTile) {
        uint8_t* vt = skv + st * L::kStageBytes + L::kTileBytes;
        const int per_row = L::kBoxes * 8;  // 16-byte chunks of a key row
        for (int idx = lane; idx < (kTcTile - vend) * per_row; idx += 32) {
          const int row = vend + idx / per_row, c = idx - (idx / per_row) * per_row;
          *reinterpret_cast<uint4*>(vt + (c >> 3) * L::kKVHalf + row * 128 + (c & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
      }
      if (!warp_wait(&bar_p[jj & 1], (jj >> 1) & 1)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t vaddr = skv_addr + st * L::kStageBytes + L::kTileBytes;
#pragma unroll
        for (int kt = 0; kt < kTcTile / 16; ++kt)
          umma_ts(tmem + kColO, tmem + kColP + (jj & 1) * 32 + kt * 8,
                  umma_desc(vaddr + kt * 2048, L::kKVHalf, 1024), kIdescPV,
                  (jj > 0 || kt > 0) ? 1u : 0u);
        umma_commit(&bar_o[jj & 1]);
        umma_commit(&empty[st]);
      }
      __syncwarp();
      if (jj + kTcNS < n) {
        if (!warp_wait(&empty[st], (jj / kTcNS) & 1)) return false;
        issue(jj + kTcNS, slot, okg);
        ++loads_issued;
      }
      return true;
    };
    if (n > 0) {
      prefetch_tensormap(&tmap);
      for (int i = 0; i < kTcNS && i < n; ++i) {
        int slot;
        bool okg;
        fetch(i, slot, okg);
        issue(i, slot, okg);
        ++loads_issued;
      }
    }
    for (int j = 0; j < n; ++j) {
      const int st = j % kTcNS;
      if (!warp_wait(&full[st], (j / kTcNS) & 1)) {
        ok = false;
        break;
      }
      loads_seen = j + 1;
      if (j > 0 && !warp_wait(bar_sfree, (j - 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t kaddr = skv_addr + st * L::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < L::KS; ++kk) {
          const uint32_t off = (kk & 3) * 32;  // 16 elements = 32 B along K
          umma_ss(tmem + kColS,
                  umma_desc(sq_addr + (kk >> 2) * L::kQHalf + off, 16, 1024),
                  umma_desc(kaddr + (kk >> 2) * L::kKVHalf + off, 16, 1024), kIdescQK,
                  kk > 0 ? 1u : 0u);
        }
        umma_commit(bar_s);
      }
      mma_issued = true;
      __syncwarp();
      if (j > 0 && !do_pv(j - 1)) {
        ok = false;
        break;
      }
    }
    if (ok && n > 0) {
      ok = do_pv(n - 1);
      // the row warps wait for this last P.V before reading O; wait here as
      // well so that tensor memory is idle before it is released
      if (ok) ok = warp_wait(&bar_o[(n - 1) & 1], ((n - 1) >> 1) & 1);
    }
    if (!ok) {
      // a wait was abandoned (reported): before the CTA releases its tensor
      // memory and exits, wait (bounded) for the MMAs and TMA loads it issued
      if (mma_issued) {
        if (lane == 0) umma_commit(bar_fin);
        __syncwarp();
        warp_wait(bar_fin, 0);
      }
      for (int i = loads_seen; i < loads_issued; ++i)
        warp_wait(&full[i % kTcNS], (i / kTcNS) & 1);
    }
  } else {
    // ================================ row warps ================================
    const uint32_t lane_off = static_cast<uint32_t>(32 * warp) << 16;
    const int kv_len = min(a.kv_lens[b], a.max_pages * a.page_size);
    const int pos = kv_len - a.q_len + s_pos;  // absolute position of this row's query
    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; j < n; ++j) {
      if (!warp_wait(bar_s, j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t ra[32], rb2[32];
      tmem_ld32(tmem + lane_off + kColS, ra);
      tmem_ld32(tmem + lane_off + kColS + 32, rb2);
      tmem_wait_ld(ra);
      tmem_wait_ld(rb2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_sfree);  // S may now be overwritten

      const int j0 = (t_begin + j) * kTcTile;
      const int vend = kv_u - j0;
      float x[64];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        x[c] = __uint_as_float(ra[c]);
        x[32 + c] = __uint_as_float(rb2[c]);
      }
      const bool all_in = okr && vend >= kTcTile && j0 >= k_lo &&
                          (!a.causal || j0 + kTcTile - 1 <= pos);
      if (a.softcap > 0.f) {
#pragma unroll
        for (int c = 0; c < 64; ++c) x[c] = a.softcap * tanhf(x[c] * a.scale / a.softcap) * kLog2e;
      } else {
#pragma unroll
        for (int c = 0; c < 64; ++c) x[c] *= a.scale_log2;
      }
      if (a.mask != nullptr && okr)
        add_mask_row(a, b, s_pos, j0, all_in ? kTcTile : min(vend, kTcTile), x);
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const bool in =
            all_in || (okr && c < vend && j0 + c >= k_lo && (!a.causal || j0 + c <= pos));
        x[c] = in ? x[c] : -INFINITY;
        mx = fmaxf(mx, x[c]);
      }
      // reference max: moves only when the row's max grows by more than 2^8
      const bool need = mx > m_ref + kRescaleLog2 || (m_ref == -INFINITY && mx > -INFINITY);
      const float m_new = need ? mx : m_ref;
      const float alpha = need ? exp2f(m_ref - m_new) : 1.f;  // 0 while m_ref is -inf
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      m_ref = m_new;
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O holds the previous tiles: rescale this warp's rows once P.V of
        // tile j-1 has completed
        if (!warp_wait(&bar_o[(j - 1) & 1], ((j - 1) >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_off + kColO + c0, o);
          tmem_wait_ld(o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tmem + lane_off + kColO + c0, o);
        }
        tmem_wait_st();
      }
      // P buffer (j & 1) was last read by P.V of tile j-2
      if (j >= 2 && !warp_wait(&bar_o[j & 1], ((j - 2) >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sum = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const float p0 = exp2f(x[2 * c] - m_use), p1 = exp2f(x[2 * c + 1] - m_use);
        sum += p0 + p1;
        pk[c] = MmaOp<T>::pack(p0, p1);
      }
      l = l * alpha + sum;
      tmem_st32(tmem + lane_off + kColP + (j & 1) * 32, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_p[j & 1]);
    }
    if (ok && n > 0) {
      ok = warp_wait(&bar_o[(n - 1) & 1], ((n - 1) >> 1) & 1);
      tc_fence_after();
    }
    if (ok) {
      if (a.splits == 1) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* orow = static_cast<T*>(a.out) + static_cast<int64_t>(b) * a.o_sb +
                  static_cast<int64_t>(qh) * a.o_sh + static_cast<int64_t>(s_pos) * a.o_ss;
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (n > 0) {
            tmem_ld32(tmem + lane_off + kColO + c0, o);
            tmem_wait_ld(o);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pk[e] = MmaOp<T>::pack(__uint_as_float(o[2 * e]) * inv,
                                   __uint_as_float(o[2 * e + 1]) * inv);
          if (okr) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              *reinterpret_cast<uint4*>(orow + c0 + 8 * e) =
                  make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
          }
        }
      } else {
        const int64_t part = (static_cast<int64_t>(pair) * a.row_blocks + rb) * a.splits + split;
        const int64_t rec = part * kTcRows + threadIdx.x;
        float* po = a.part_o + rec * D;
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (n > 0) {
            tmem_ld32(tmem + lane_off + kColO + c0, o);
            tmem_wait_ld(o);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
#pragma unroll
          for (int e = 0; e < 8; ++e)
            *reinterpret_cast<float4*>(po + c0 + 4 * e) =
                make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                            __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
        }
        *reinterpret_cast<float2*>(a.part_ml + rec * 2) = make_float2(m_ref, l);
      }
    }
  }
  // all tensor-memory traffic of the CTA is complete: release the columns
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// 2^x by the hardware approximation (PTX ex2.approx.ftz.f32: relative error
// ~2^-22, results below 2^-126 flushed to 0; probabilities that small vanish
// in the bf16/fp16 P operand anyway).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------- two query tiles per CTA (default) --
// The same computation with two 128-row query tiles per CTA sharing every K/V
// tile (one CTA per SM, all 512 tensor-memory columns), so that the tensor
// core works on one tile while the other tile's rows turn scores into
// probabilities:
//   warps 0-3 / 4-7   softmax rows of query tile 0 / 1 (one row per thread)
//   warp 8            one elected lane issues every tcgen05.mma: per K/V tile
//                     S0 = Q0.K^T, S1 = Q1.K^T, then O0 += P0.V, O1 += P1.V of
//                     the previous tile (P written meanwhile by the row warps)
//   warp 9            TMA loads of the K/V tiles into an NS-stage ring, a stage
//                     refilled once both P.V products of its tile completed
// Tensor memory of query tile t: S [256t, 256t + 64), P double buffer
// [256t + 64, 256t + 128), O [256t + 128, 256t + 128 + D).  K/V reads from L2
// and HBM halve against the one-tile kernel (each tile serves 256 rows).
// The row warps' common case (every key of the tile visible, no mask, no
// soft-cap) takes each probability as one FMA and one ex2 of the raw score.
constexpr int kT2Q = 2;
constexpr int kT2Rows = kT2Q * kTcRows;
constexpr int kT2SoftWarps = kT2Q * kTcSoftWarps;
constexpr int kT2MmaWarp = kT2SoftWarps, kT2LoadWarp = kT2SoftWarps + 1;
constexpr int kT2Threads = (kT2SoftWarps + 2) * 32;
constexpr uint32_t kT2TmemCols = 512;
constexpr uint32_t kT2TileCols = 256;   // tensor-memory columns of one query tile

template <int D>
struct Tc2Layout {
  static constexpr int KS = D / 16;
  static constexpr int kQHalf = kTcRows * 128;
  static constexpr int kQBytes = kTcRows * D * 2;     // one query tile
  static constexpr int kKVHalf = kTcTile * 128;
  static constexpr int kTileBytes = kTcTile * D * 2;
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int kBoxes = D / 64;
  static constexpr int NS = D <= 64 ? 8 : 4;
  static constexpr int kBars = 2 * NS + 6 * kT2Q + 1;
  static constexpr size_t smem_bytes() {
    return 1024 + kT2Q * kQBytes + NS * kStageBytes + kBars * sizeof(uint64_t);
  }
};

template <typename T, int D>
__global__ void __launch_bounds__(kT2Threads, 1)
    paged_prefill_tc2_kernel(const __grid_constant__ CUtensorMap tmap, const PrefillArgs a) {
  using L = Tc2Layout<D>;
  constexpr int NS = L::NS;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdescQK = umma_idesc(kBf16, kTcRows, kTcTile, false);
  constexpr uint32_t kIdescPV = umma_idesc(kBf16, kTcRows, D, true);

  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t s_tmem;
  uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint8_t* sq = smem;                              // [kT2Q][kQBytes]
  uint8_t* skv = smem + kT2Q * L::kQBytes;         // [NS][K tile | V tile]
  uint64_t* bars = reinterpret_cast<uint64_t*>(skv + NS * L::kStageBytes);
  uint64_t* full = bars;                 // [NS] K/V tile landed (TMA bytes)
  uint64_t* empty = bars + NS;           // [NS] both P.V of the stage's tile completed
  // per query tile t, at tb + 6 t: S written, S read (4 row warps), P buffer
  // 0/1 written (4 row warps), P.V of tiles with parity 0/1 completed
  uint64_t* tb = bars + 2 * NS;
  uint64_t* bar_fin = tb + 6 * kT2Q;     // drain after an abandoned wait

  // blockIdx.x = ((b * hkv + h) * splits + split) * row_blocks + rb (256-row blocks)
  const int rb = blockIdx.x % a.row_blocks;
  const int rest = blockIdx.x / a.row_blocks;
  const int split = rest % a.splits;
  const int pair = rest / a.splits;
  const int b = pair / a.hkv, h = pair - (pair / a.hkv) * a.hkv;
  const int kv_u = unit_keys(a, b, rb, kT2Rows);
  const int k_lo = unit_first_key(a, b, kv_u);
  const int t_lo = k_lo / kTcTile;
  const int n_tiles = (kv_u + kTcTile - 1) / kTcTile - t_lo;
  const int t_begin = t_lo + static_cast<int>(static_cast<int64_t>(n_tiles) * split / a.splits);
  const int t_end = t_lo + static_cast<int>(static_cast<int64_t>(n_tiles) * (split + 1) / a.splits);
  const int n = t_end - t_begin;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int t = 0; t < kT2Q; ++t) {
      mbar_init(tb + 6 * t + 0, 1);              // S written (tcgen05.commit)
      mbar_init(tb + 6 * t + 1, kTcSoftWarps);   // S read
      mbar_init(tb + 6 * t + 2, kTcSoftWarps);   // P buffer 0 written
      mbar_init(tb + 6 * t + 3, kTcSoftWarps);   // P buffer 1 written
      mbar_init(tb + 6 * t + 4, 1);              // P.V of even tiles completed
      mbar_init(tb + 6 * t + 5, 1);              // P.V of odd tiles completed
    }
    mbar_init(bar_fin, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(&s_tmem)),
                 "r"(kT2TmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }

  // row of this thread (warps 0-7): query tile qt, tensor-memory lane tr
  const int qt = warp / kTcSoftWarps;
  const int tr = threadIdx.x - qt * kTcRows;
  const int r = rb * kT2Rows + qt * kTcRows + tr;
  const bool okr = warp < kT2SoftWarps && r < a.rows;
  const int s_pos = okr ? r / a.group : 0;
  const int qh = h * a.group + (okr ? r - s_pos * a.group : 0);
  if (warp < kT2SoftWarps) {
    // Q row -> its tile's slab, K-major 128-byte swizzle (as the one-tile kernel)
    const T* qrow = static_cast<const T*>(a.q) + static_cast<int64_t>(b) * a.q_sb +
                    static_cast<int64_t>(qh) * a.q_sh + static_cast<int64_t>(s_pos) * a.q_ss;
    uint8_t* sqt = sq + qt * L::kQBytes;
#pragma unroll
    for (int c = 0; c < D / 8; ++c) {
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (okr) v = *reinterpret_cast<const uint4*>(qrow + c * 8);
      *reinterpret_cast<uint4*>(sqt + (c >> 3) * L::kQHalf + tr * 128 + (((c & 7) ^ (tr & 7)) << 4)) = v;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  asm volatile("griddepcontrol.launch_dependents;");

  bool ok = true;
  if (warp == kT2LoadWarp) {
    // ================================== loads ==================================
    const int64_t kv_rows = static_cast<int64_t>(a.hkv) * a.page_size;
    int issued = 0;
    if (n > 0) prefetch_tensormap(&tmap);
    for (int i = 0; i < n; ++i) {
      const int st = i % NS;
      if (i >= NS && !warp_wait(&empty[st], ((i / NS) - 1) & 1)) {
        ok = false;
        break;
      }
      const int j = (t_begin + i) * kTcTile + lane * 16;
      const bool okg = lane < 4 && j < kv_u;
      int slot = okg ? a.page_table[static_cast<int64_t>(b) * a.pt_sb + j / a.page_size] : 0;
      const unsigned issuing = __ballot_sync(0xffffffffu, okg);
      if (lane == 0) mbar_arrive_expect_tx(&full[st], __popc(issuing) * 2 * L::kBoxes * 2048);
      __syncwarp();
      if (okg) {
        if (slot < 0 || slot >= a.pool_pages) {
          report_status(HELM_DEV_BAD_PAGE);
          slot = 0;
        }
        const int row_off = j - (j / a.page_size) * a.page_size;
        const int row_k = static_cast<int>(
            (static_cast<int64_t>(slot) * 2 * a.hkv + h) * a.page_size + row_off);
        const int row_v = static_cast<int>(row_k + kv_rows);
        uint8_t* kdst = skv + st * L::kStageBytes + lane * 2048;
#pragma unroll
        for (int hb = 0; hb < L::kBoxes; ++hb) {
          tma_load_2d(kdst + hb * L::kKVHalf, &tmap, hb * 64, row_k, &full[st]);
          tma_load_2d(kdst + L::kTileBytes + hb * L::kKVHalf, &tmap, hb * 64, row_v, &full[st]);
        }
      }
      ++issued;
    }
    if (!ok) {   // the last use of every stage: wait (bounded) for its bytes to land
      for (int i = issued > NS ? issued - NS : 0; i < issued; ++i)
        warp_wait(&full[i % NS], (i / NS) & 1);
    }
  } else if (warp == kT2MmaWarp) {
    // ================================== MMAs ===================================
    bool mma_issued = false;
    const uint32_t sq_addr = smem_addr(sq), skv_addr = smem_addr(skv);
    auto do_pv = [&](int jj) -> bool {
      const int st = jj % NS;
      // keys of a partial tile past the unit's last key: zero their V rows
      // (P is 0 there, but 0 x NaN would be NaN; the tile's bytes have landed)
      const int vend = kv_u - (t_begin + jj) * kTcTile;
      if (vend < kTcTile) {
        uint8_t* vt = skv + st * L::kStageBytes + L::kTileBytes;
        const int per_row = L::kBoxes * 8;
        for (int idx = lane; idx < (kTcTile - vend) * per_row; idx += 32) {
          const int row = vend + idx / per_row, c = idx - (idx / per_row) * per_row;
          *reinterpret_cast<uint4*>(vt + (c >> 3) * L::kKVHalf + row * 128 + (c & 7) * 16) =
              make_uint4(0u, 0u, 0u, 0u);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
      }
      const uint32_t vaddr = skv_addr + st * L::kStageBytes + L::kTileBytes;
      for (int t = 0; t < kT2Q; ++t) {
        uint64_t* tbt = tb + 6 * t;
        if (!warp_wait(tbt + 2 + (jj & 1), (jj >> 1) & 1)) return false;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t cols = tmem + t * kT2TileCols;
#pragma unroll
          for (int kt = 0; kt < kTcTile / 16; ++kt)
            umma_ts(cols + kColO, cols + kColP + (jj & 1) * 32 + kt * 8,
                    umma_desc(vaddr + kt * 2048, L::kKVHalf, 1024), kIdescPV,
                    (jj > 0 || kt > 0) ? 1u : 0u);
          umma_commit(tbt + 4 + (jj & 1));
        }
        __syncwarp();
      }
      if (lane == 0) umma_commit(&empty[st]);
      __syncwarp();
      return true;
    };
    for (int j = 0; j < n && ok; ++j) {
      const int st = j % NS;
      if (!warp_wait(&full[st], (j / NS) & 1)) {
        ok = false;
        break;
      }
      const uint32_t kaddr = skv_addr + st * L::kStageBytes;
      for (int t = 0; t < kT2Q; ++t) {
        uint64_t* tbt = tb + 6 * t;
        if (j > 0 && !warp_wait(tbt + 1, (j - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t qaddr = sq_addr + t * L::kQBytes;
#pragma unroll
          for (int kk = 0; kk < L::KS; ++kk) {
            const uint32_t off = (kk & 3) * 32;  // 16 elements = 32 B along K
            umma_ss(tmem + t * kT2TileCols + kColS,
                    umma_desc(qaddr + (kk >> 2) * L::kQHalf + off, 16, 1024),
                    umma_desc(kaddr + (kk >> 2) * L::kKVHalf + off, 16, 1024), kIdescQK,
                    kk > 0 ? 1u : 0u);
          }
          umma_commit(tbt + 0);
        }
        mma_issued = true;
        __syncwarp();
      }
      if (ok && j > 0 && !do_pv(j - 1)) ok = false;
    }
    if (ok && n > 0) {
      ok = do_pv(n - 1);
      // tensor memory must be idle before it is released
      for (int t = 0; ok && t < kT2Q; ++t)
        ok = warp_wait(tb + 6 * t + 4 + ((n - 1) & 1), ((n - 1) >> 1) & 1);
    }
    if (!ok && mma_issued) {
      // a wait was abandoned (reported): wait (bounded) for the MMAs issued
      if (lane == 0) umma_commit(bar_fin);
      __syncwarp();
      warp_wait(bar_fin, 0);
    }
  } else {
    // ================================ row warps ================================
    uint64_t* tbt = tb + 6 * qt;
    const uint32_t lane_off = static_cast<uint32_t>(32 * (warp & 3)) << 16;
    const uint32_t cols = tmem + lane_off + qt * kT2TileCols;
    const int kv_len = min(a.kv_lens[b], a.max_pages * a.page_size);
    const int pos = kv_len - a.q_len + s_pos;  // absolute position of this row's query
    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; j < n; ++j) {
      if (!warp_wait(tbt + 0, j & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t ra[32], rb2[32];
      tmem_ld32(cols + kColS, ra);
      tmem_ld32(cols + kColS + 32, rb2);
      tmem_wait_ld(ra);
      tmem_wait_ld(rb2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tbt + 1);  // S may now be overwritten

      const int j0 = (t_begin + j) * kTcTile;
      const int vend = kv_u - j0;
      float x[64];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        x[c] = __uint_as_float(ra[c]);
        x[32 + c] = __uint_as_float(rb2[c]);
      }
      const bool all_in = okr && vend >= kTcTile && j0 >= k_lo &&
                          (!a.causal || j0 + kTcTile - 1 <= pos);
      // Most tiles: every key of every row of the warp is visible, no mask and
      // no soft-cap.  Then the row max is taken on the raw scores (the scale is
      // positive, so the order and the rounded scaled max are the same) and
      // each probability is one FMA and one exp2: ex2(x * scale - m).
      const bool fast = a.softcap <= 0.f && a.mask == nullptr && a.scale_log2 > 0.f &&
                        __all_sync(0xffffffffu, all_in);
      float mx = -INFINITY;
      if (fast) {
#pragma unroll
        for (int c = 0; c < 64; ++c) mx = fmaxf(mx, x[c]);
        mx *= a.scale_log2;
      } else {
        if (a.softcap > 0.f) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            x[c] = a.softcap * tanhf(x[c] * a.scale / a.softcap) * kLog2e;
        } else {
#pragma unroll
          for (int c = 0; c < 64; ++c) x[c] *= a.scale_log2;
        }
        if (a.mask != nullptr && okr)
          add_mask_row(a, b, s_pos, j0, all_in ? kTcTile : min(vend, kTcTile), x);
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const bool in =
              all_in || (okr && c < vend && j0 + c >= k_lo && (!a.causal || j0 + c <= pos));
          x[c] = in ? x[c] : -INFINITY;
          mx = fmaxf(mx, x[c]);
        }
      }
      // reference max: moves only when the row's max grows by more than 2^8
      const bool need = mx > m_ref + kRescaleLog2 || (m_ref == -INFINITY && mx > -INFINITY);
      const float m_new = need ? mx : m_ref;
      const float alpha = need ? exp2f(m_ref - m_new) : 1.f;  // 0 while m_ref is -inf
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      m_ref = m_new;
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O holds the previous tiles: rescale once P.V of tile j-1 completed
        if (!warp_wait(tbt + 4 + ((j - 1) & 1), ((j - 1) >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          tmem_ld32(cols + kColO + c0, o);
          tmem_wait_ld(o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(cols + kColO + c0, o);
        }
        tmem_wait_st();
      }
      // P buffer (j & 1) was last read by P.V of tile j-2
      if (j >= 2 && !warp_wait(tbt + 4 + (j & 1), ((j - 2) >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sum = 0.f;
      uint32_t pk[32];
      if (fast) {
        const float sl = a.scale_log2;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p0 = ex2_approx(fmaf(x[2 * c], sl, -m_use));
          const float p1 = ex2_approx(fmaf(x[2 * c + 1], sl, -m_use));
          sum += p0 + p1;
          pk[c] = MmaOp<T>::pack(p0, p1);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float p0 = exp2f(x[2 * c] - m_use), p1 = exp2f(x[2 * c + 1] - m_use);
          sum += p0 + p1;
          pk[c] = MmaOp<T>::pack(p0, p1);
        }
      }
      l = l * alpha + sum;
      tmem_st32(cols + kColP + (j & 1) * 32, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tbt + 2 + (j & 1));
    }
    if (ok && n > 0) {
      ok = warp_wait(tbt + 4 + ((n - 1) & 1), ((n - 1) >> 1) & 1);
      tc_fence_after();
    }
    if (ok) {
      if (a.splits == 1) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        T* orow = static_cast<T*>(a.out) + static_cast<int64_t>(b) * a.o_sb +
                  static_cast<int64_t>(qh) * a.o_sh + static_cast<int64_t>(s_pos) * a.o_ss;
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (n > 0) {
            tmem_ld32(cols + kColO + c0, o);
            tmem_wait_ld(o);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pk[e] = MmaOp<T>::pack(__uint_as_float(o[2 * e]) * inv,
                                   __uint_as_float(o[2 * e + 1]) * inv);
          if (okr) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              *reinterpret_cast<uint4*>(orow + c0 + 8 * e) =
                  make_uint4(pk[4 * e], pk[4 * e + 1], pk[4 * e + 2], pk[4 * e + 3]);
          }
        }
      } else {
        const int64_t part = (static_cast<int64_t>(pair) * a.row_blocks + rb) * a.splits + split;
        const int64_t rec = part * kT2Rows + qt * kTcRows + tr;
        float* po = a.part_o + rec * D;
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          uint32_t o[32];
          if (n > 0) {
            tmem_ld32(cols + kColO + c0, o);
            tmem_wait_ld(o);
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = 0u;
          }
#pragma unroll
          for (int e = 0; e < 8; ++e)
            *reinterpret_cast<float4*>(po + c0 + 4 * e) =
                make_float4(__uint_as_float(o[4 * e]), __uint_as_float(o[4 * e + 1]),
                            __uint_as_float(o[4 * e + 2]), __uint_as_float(o[4 * e + 3]));
        }
        *reinterpret_cast<float2*>(a.part_ml + rec * 2) = make_float2(m_ref, l);
      }
    }
  }
  // all tensor-memory traffic of the CTA is complete: release the columns
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kT2TmemCols)
                 : "memory");
  }
}

template <typename T, int D>
int launch_prefill_tc2(PrefillArgs a, const void* pool, int64_t pool_rows, int max_kv_len,
                       void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  static bool configured[64][2] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return HELM_ERR_CUDA;
  if (!configured[dev][D == 128]) {
    if (cudaFuncSetAttribute(paged_prefill_tc2_kernel<T, D>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(Tc2Layout<D>::smem_bytes())) != cudaSuccess)
      return HELM_ERR_CUDA;
    configured[dev][D == 128] = true;
  }
  const PrefillPlan plan =
      plan_prefill(a.batch, a.q_len, a.hq, a.hkv, D, max_kv_len, 1, kT2Rows);
  if (workspace_bytes < plan.total()) return HELM_ERR_WORKSPACE;
  if (plan.total() > 0 && workspace == nullptr) return HELM_ERR_WORKSPACE;
  a.row_blocks = plan.row_blocks;
  a.splits = plan.splits;
  uint8_t* wsp = static_cast<uint8_t*>(workspace);
  a.part_o = plan.splits > 1 ? reinterpret_cast<float*>(wsp) : nullptr;
  a.part_ml = plan.splits > 1 ? reinterpret_cast<float*>(wsp + plan.o_bytes) : nullptr;
  const int64_t grid = plan.units * plan.splits;
  if (grid <= 0) return HELM_OK;
  if (grid >= (int64_t(1) << 31)) return HELM_ERR_UNSUPPORTED;
  CUtensorMap map;
  if (!encode_pool_map<T, D>(pool, pool_rows, &map)) return HELM_ERR_CUDA;
  paged_prefill_tc2_kernel<T, D><<<static_cast<unsigned>(grid), kT2Threads,
                                   Tc2Layout<D>::smem_bytes(), stream>>>(map, a);
  if (cudaGetLastError() != cudaSuccess) return HELM_ERR_CUDA;
  if (plan.splits == 1) return HELM_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(plan.units),
                     static_cast<unsigned>((kT2Rows * D / 4 + kPfMergeThreads - 1) / kPfMergeThreads));
  cfg.blockDim = dim3(kPfMergeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, merge_prefill_splits_kernel<T, D, kT2Rows>, a) != cudaSuccess)
    return HELM_ERR_CUDA;
  return HELM_OK;
}

template <typename T, int D>
int tc_ctas_per_sm() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  if (cached[dev] == 0) {
    int nb = 0;
    if (cudaFuncSetAttribute(paged_prefill_tc_kernel<T, D>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(TcLayout<D>::smem_bytes())) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, paged_prefill_tc_kernel<T, D>,
                                                      kTcThreads,
                                                      TcLayout<D>::smem_bytes()) != cudaSuccess ||
        nb <= 0)
      nb = 1;
    // two CTAs share an SM's 512 tensor-memory columns
    cached[dev] = std::min(nb, 2);
  }
  return cached[dev];
}

template <typename T, int D>
int launch_prefill_tc(PrefillArgs a, const void* pool, int64_t pool_rows, int max_kv_len,
                      void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  const int ctas = tc_ctas_per_sm<T, D>();
  const PrefillPlan plan =
      plan_prefill(a.batch, a.q_len, a.hq, a.hkv, D, max_kv_len, ctas, kTcRows);
  if (workspace_bytes < plan.total()) return HELM_ERR_WORKSPACE;
  if (plan.total() > 0 && workspace == nullptr) return HELM_ERR_WORKSPACE;
  a.row_blocks = plan.row_blocks;
  a.splits = plan.splits;
  uint8_t* wsp = static_cast<uint8_t*>(workspace);
  a.part_o = plan.splits > 1 ? reinterpret_cast<float*>(wsp) : nullptr;
  a.part_ml = plan.splits > 1 ? reinterpret_cast<float*>(wsp + plan.o_bytes) : nullptr;
  const int64_t grid = plan.units * plan.splits;
  if (grid <= 0) return HELM_OK;
  if (grid >= (int64_t(1) << 31)) return HELM_ERR_UNSUPPORTED;
  CUtensorMap map;
  if (!encode_pool_map<T, D>(pool, pool_rows, &map)) return HELM_ERR_CUDA;
  paged_prefill_tc_kernel<T, D><<<static_cast<unsigned>(grid), kTcThreads,
                                  TcLayout<D>::smem_bytes(), stream>>>(map, a);
  if (cudaGetLastError() != cudaSuccess) return HELM_ERR_CUDA;
  if (plan.splits == 1) return HELM_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(plan.units),
                     static_cast<unsigned>((kTcRows * D / 4 + kPfMergeThreads - 1) / kPfMergeThreads));
  cfg.blockDim = dim3(kPfMergeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, merge_prefill_splits_kernel<T, D, kTcRows>, a) != cudaSuccess)
    return HELM_ERR_CUDA;
  return HELM_OK;
}

// Which kernel serves a call: 0 the mma.sync kernel, 1 the one-tile tcgen05
// kernel, 2 the two-tile tcgen05 kernel (the default).  HELM_B200_PREFILL_KERNEL
// = "mma" / "tc1" selects the first two; query / output rows that are not
// 16-byte aligned take the mma.sync kernel (the tcgen05 kernels move whole
// 16-byte chunks of a row).
int prefill_kernel_choice(const void* q, int64_t q_sb, int64_t q_sh, int64_t q_ss,
                          const void* out, int64_t o_sb, int64_t o_sh, int64_t o_ss) {
  const char* env = std::getenv("HELM_B200_PREFILL_KERNEL");
  if (env != nullptr && std::strcmp(env, "mma") == 0) return 0;
  const bool q_ok = (reinterpret_cast<uintptr_t>(q) & 15) == 0 && q_sb % 8 == 0 &&
                    q_sh % 8 == 0 && q_ss % 8 == 0;
  const bool o_ok = out == nullptr || ((reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                                       o_sb % 8 == 0 && o_sh % 8 == 0 && o_ss % 8 == 0);
  if (!(q_ok && o_ok)) return 0;
  return (env != nullptr && std::strcmp(env, "tc1") == 0) ? 1 : 2;
}

template <typename T>
int prefill_tc_dispatch(int kernel, int head_dim, const PrefillArgs& a, const void* pool,
                        int64_t rows, int max_kv_len, void* ws, int64_t ws_bytes,
                        cudaStream_t s) {
  switch (head_dim) {
    case 64:
      return kernel == 2 ? launch_prefill_tc2<T, 64>(a, pool, rows, max_kv_len, ws, ws_bytes, s)
                         : launch_prefill_tc<T, 64>(a, pool, rows, max_kv_len, ws, ws_bytes, s);
    case 128:
      return kernel == 2 ? launch_prefill_tc2<T, 128>(a, pool, rows, max_kv_len, ws, ws_bytes, s)
                         : launch_prefill_tc<T, 128>(a, pool, rows, max_kv_len, ws, ws_bytes, s);
    default:
      return HELM_ERR_UNSUPPORTED;
  }
}

}  // namespace

}  // namespace helm

// ------------------------------------------------------------- C entry points --
// The workspace covers either kernel (the split plan differs between them):
// the larger of the two sizes.
extern "C" int64_t helm_paged_prefill_workspace_bytes(int batch, int q_len, int num_q_heads,
                                                      int num_kv_heads, int head_dim, int dtype,
                                                      int max_kv_len) {
  using namespace helm;
  if (batch <= 0 || q_len <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 ||
      num_q_heads % num_kv_heads != 0 || max_kv_len < 0)
    return 0;
  const bool bf = dtype == HELM_DTYPE_BF16;
  int c_mma = 1, c_tc = 1;
  if (head_dim == 64) {
    c_mma = bf ? prefill_ctas_per_sm<__nv_bfloat16, 64>() : prefill_ctas_per_sm<__half, 64>();
    c_tc = bf ? tc_ctas_per_sm<__nv_bfloat16, 64>() : tc_ctas_per_sm<__half, 64>();
  } else if (head_dim == 128) {
    c_mma = bf ? prefill_ctas_per_sm<__nv_bfloat16, 128>() : prefill_ctas_per_sm<__half, 128>();
    c_tc = bf ? tc_ctas_per_sm<__nv_bfloat16, 128>() : tc_ctas_per_sm<__half, 128>();
  } else {
    return 0;
  }
  const int64_t w_mma =
      plan_prefill(batch, q_len, num_q_heads, num_kv_heads, head_dim, max_kv_len, c_mma, kPfRows)
          .total();
  const int64_t w_tc =
      plan_prefill(batch, q_len, num_q_heads, num_kv_heads, head_dim, max_kv_len, c_tc, kTcRows)
          .total();
  const int64_t w_tc2 =
      plan_prefill(batch, q_len, num_q_heads, num_kv_heads, head_dim, max_kv_len, 1, kT2Rows)
          .total();
  return std::max(std::max(w_mma, w_tc), w_tc2);
}

extern "C" int helm_paged_prefill_attention(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, int64_t q_stride_s, const void* kv_pool,
    int64_t pool_pages, const int32_t* page_table, int64_t pt_stride_b, int max_pages,
    const int32_t* kv_lens, const int32_t* kv_starts, const void* mask, int mask_dtype,
    int64_t mask_stride_b, int64_t mask_stride_q, void* out, int64_t out_stride_b,
    int64_t out_stride_h,
    int64_t out_stride_s, void* workspace, int64_t workspace_bytes, int batch, int q_len,
    int num_q_heads, int num_kv_heads, int head_dim, int page_size, int dtype, int causal,
    float scale, float softcap, int max_kv_len, void* stream) {
  using namespace helm;
  if (q == nullptr || kv_pool == nullptr || page_table == nullptr || kv_lens == nullptr ||
      out == nullptr)
    return HELM_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || q_len <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || page_size <= 0 ||
      max_pages < 0 || pool_pages <= 0 || max_kv_len < 0)
    return HELM_ERR_INVALID_ARGUMENT;
  if (num_q_heads % num_kv_heads != 0) return HELM_ERR_INVALID_ARGUMENT;
  if (dtype != HELM_DTYPE_BF16 && dtype != HELM_DTYPE_FP16) return HELM_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return HELM_ERR_UNSUPPORTED;
  if (page_size % 16 != 0) return HELM_ERR_UNSUPPORTED;  // 16-key boxes stay inside a page
  if (mask != nullptr && mask_dtype != HELM_DTYPE_FP32 && mask_dtype != HELM_DTYPE_BF16 &&
      mask_dtype != HELM_DTYPE_FP16)
    return HELM_ERR_INVALID_ARGUMENT;
  // q and out are accessed as 32-bit words (16-byte chunks on the tcgen05
  // path), the pool through TMA (16-byte rule)
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (q_stride_b & 1) || (q_stride_h & 1) ||
      (q_stride_s & 1))
    return HELM_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(out) & 7) || (out_stride_b & 3) || (out_stride_h & 3) ||
      (out_stride_s & 3))
    return HELM_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(kv_pool) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return HELM_ERR_ALIGNMENT;
  const int64_t pool_rows = pool_pages * 2 * num_kv_heads * static_cast<int64_t>(page_size);
  if (pool_rows >= (int64_t(1) << 31)) return HELM_ERR_UNSUPPORTED;
  if (static_cast<int64_t>(max_pages) * page_size >= (int64_t(1) << 30)) return HELM_ERR_UNSUPPORTED;

  PrefillArgs a;
  a.q = q;
  a.q_sb = q_stride_b;
  a.q_sh = q_stride_h;
  a.q_ss = q_stride_s;
  a.pool_pages = pool_pages;
  a.page_table = page_table;
  a.pt_sb = pt_stride_b;
  a.max_pages = max_pages;
  a.kv_lens = kv_lens;
  a.kv_starts = kv_starts;
  a.mask = mask;
  a.mask_dtype = mask_dtype;
  a.mask_sb = mask_stride_b;
  a.mask_sq = mask_stride_q;
  a.out = out;
  a.o_sb = out_stride_b;
  a.o_sh = out_stride_h;
  a.o_ss = out_stride_s;
  a.part_o = nullptr;
  a.part_ml = nullptr;
  a.batch = batch;
  a.q_len = q_len;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.group = num_q_heads / num_kv_heads;
  a.page_size = page_size;
  a.rows = q_len * a.group;
  a.row_blocks = 0;
  a.splits = 1;
  a.causal = causal != 0 ? 1 : 0;
  a.scale = scale;
  a.scale_log2 = scale * kLog2e;
  a.softcap = softcap;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int kernel = prefill_kernel_choice(q, q_stride_b, q_stride_h, q_stride_s, out,
                                           out_stride_b, out_stride_h, out_stride_s);
  int rc;
  if (dtype == HELM_DTYPE_BF16)
    rc = kernel ? prefill_tc_dispatch<__nv_bfloat16>(kernel, head_dim, a, kv_pool, pool_rows,
                                                     max_kv_len, workspace, workspace_bytes, s)
                : prefill_dispatch<__nv_bfloat16>(head_dim, a, kv_pool, pool_rows, max_kv_len,
                                                  workspace, workspace_bytes, s);
  else
    rc = kernel ? prefill_tc_dispatch<__half>(kernel, head_dim, a, kv_pool, pool_rows, max_kv_len,
                                              workspace, workspace_bytes, s)
                : prefill_dispatch<__half>(head_dim, a, kv_pool, pool_rows, max_kv_len, workspace,
                                           workspace_bytes, s);
  if (rc == HELM_ERR_CUDA) set_last_cuda_error(cudaGetLastError());
  return rc;
}
