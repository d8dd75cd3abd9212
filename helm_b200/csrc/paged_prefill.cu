// Paged chunk-prefill attention for sm_100a (B200).
//
// Replaces the q_len > 1 branch of HELM's perform_streaming_attention
// (helm/runtime/kv_cache.py:469-555: per-page fp32 matmuls, softcap, additive
// mask and an online softmax over the concatenated pages), as called by
// _stream_prefill_batched (helm/runtime/kv_offload.py:206-227) for a prefill
// chunk that attends over every cached page of its sequence, with one launch
// that reads K/V straight from the page pool.
//
// Rows: the chunk's (query position, query head of the GQA group) pairs of one
// (sequence, kv head), head fastest, so one K/V tile in shared memory serves
// all G query heads of its kv head.  A ROW BLOCK is 64 rows; a UNIT is one row
// block of one (sequence, kv head).  A unit's keys (64-token tiles) are cut
// into `splits` equal parts and CTA (unit, split) streams its part:
//
//   TMA loads of each tile into a ring of NS stages (per K and per V four
//   16-row boxes, each inside one page found in the page table, x D/64 column
//   boxes, 128-byte swizzled), issued by warp 0, which refills a stage once
//   every warp has released it
//   4 warps, 16 rows each, tensor cores (mma.sync m16n8k16, fp32 accumulate):
//                     S[16 x 64] = Q[16 x D] . K^T
//                     scale (or softcap), + mask, causal limit; online softmax
//                     per row in the exp2 domain
//                     O[16 x D] += P[16 x 64] . V   (P from the S accumulators)
//
// With one split a CTA writes the normalised output; otherwise each split
// writes an fp32 partial (m, l, unnormalised O) and a second kernel, launched
// as a programmatic dependent, merges the splits of every row.  The split
// count is chosen on the host so that units x splits fills whole waves of
// CTAs (the chunk's rows alone give too few CTAs for long contexts); CTAs
// next to each other in launch order read the same K/V range, so the K/V
// bytes are fetched from HBM about once per wave and re-read from L2.
//
// This file is part of the single translation unit helm_b200.cu and uses the
// helpers of paged_attention.cu (get_encode_fn, mask_log2, kLog2e), which is
// included before it.  paged_prefill_tc.cu, included after it, holds the
// tensor-memory (tcgen05) form of the same computation and the C entry points
// that choose between the two.

namespace helm {

namespace {

constexpr int kPfRows = 64;       // query rows per CTA (4 warps x 16)
constexpr int kPfTile = 64;       // keys per tile
constexpr int kPfNCW = 4;         // warps per CTA
constexpr int kPfThreads = kPfNCW * 32;
constexpr int kPfMaxSplits = 32;
constexpr int64_t kPfMaxPartialBytes = int64_t(256) << 20;
constexpr int kPfMergeThreads = 256;

struct PrefillArgs {
  const void* q;
  int64_t q_sb, q_sh, q_ss;
  int64_t pool_pages;
  const int32_t* page_table;
  int64_t pt_sb;
  int max_pages;
  const int32_t* kv_lens;
  const int32_t* kv_starts;  // optional [batch]: first key each sequence's rows may see
  const void* mask;
  int mask_dtype;
  int64_t mask_sb, mask_sq;
  void* out;
  int64_t o_sb, o_sh, o_ss;
  float* part_o;   // [units * splits][64 rows][D]   unnormalised O
  float* part_ml;  // [units * splits][64 rows][2]   (m in log2 units, l)
  int batch, q_len, hq, hkv, group, page_size;
  int rows;        // q_len * group
  int row_blocks;  // ceil(rows / 64)
  int splits;
  int causal;
  float scale, scale_log2, softcap;
};

template <int D>
struct PfLayout {
  static constexpr int kBoxes = D / 64;                // 64-column TMA boxes per row
  static constexpr int kHalf = kPfTile * 128;          // bytes of one 64-column slab
  static constexpr int kTileBytes = kPfTile * D * 2;   // K (or V) of one tile
  static constexpr int kStageBytes = 2 * kTileBytes;
  static constexpr int NS = D <= 64 ? 4 : 3;
  static constexpr size_t smem_bytes() {
    return 1024 + NS * kStageBytes + 2 * NS * sizeof(uint64_t);
  }
};

// Keys of unit (b, rb) that any of its rows may see: the sequence's length,
// clamped to its page-table row, and with the causal limit of the block's
// last row (row blocks of `rpu` rows).
__device__ __forceinline__ int unit_keys(const PrefillArgs& a, int b, int rb, int rpu) {
  int kv = a.kv_lens[b];
  const int64_t cap = static_cast<int64_t>(a.max_pages) * a.page_size;
  if (kv < 0) kv = 0;
  if (kv > cap) {
    report_status(HELM_DEV_BAD_PAGE);
    kv = static_cast<int>(cap);
  }
  if (a.causal) {
    const int r_last = min(a.rows, (rb + 1) * rpu) - 1;
    const int lim = kv - a.q_len + r_last / a.group + 1;
    kv = max(0, min(kv, lim));
  }
  return kv;
}

// First key the rows of sequence b may see: kv_starts[b] clamped to [0, kv_u]
// (0 without kv_starts).  Keys before it are masked like keys past the causal
// limit, and whole tiles before it are not visited, so HELM's left-padding
// mask becomes a per-sequence key range instead of a mask read per element.
__device__ __forceinline__ int unit_first_key(const PrefillArgs& a, int b, int kv_u) {
  if (a.kv_starts == nullptr) return 0;
  return min(max(a.kv_starts[b], 0), kv_u);
}

template <typename T>
__device__ __forceinline__ float pf_mask(const PrefillArgs& a, int b, int s, int j) {
  const int64_t off = static_cast<int64_t>(b) * a.mask_sb + static_cast<int64_t>(s) * a.mask_sq + j;
  if (a.mask_dtype == HELM_DTYPE_FP32) return static_cast<const float*>(a.mask)[off];
  if (a.mask_dtype == HELM_DTYPE_BF16)
    return __bfloat162float(static_cast<const __nv_bfloat16*>(a.mask)[off]);
  return __half2float(static_cast<const __half*>(a.mask)[off]);
}

template <typename T, int D>
__global__ void __launch_bounds__(kPfThreads, 2)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tmap, const PrefillArgs a) {
  using L = PfLayout<D>;
  constexpr int NS = L::NS;
  constexpr int KS = D / 16;  // k-steps of Q.K^T
  constexpr int NO = D / 8;   // 8-column tiles of O

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * L::kStageBytes);
  uint64_t* empty = full + NS;

  // blockIdx.x = ((b * hkv + h) * splits + split) * row_blocks + rb
  const int rb = blockIdx.x % a.row_blocks;
  const int rest = blockIdx.x / a.row_blocks;
  const int split = rest % a.splits;
  const int pair = rest / a.splits;
  const int b = pair / a.hkv, h = pair - (pair / a.hkv) * a.hkv;
  const int kv_u = unit_keys(a, b, rb, kPfRows);
  const int k_lo = unit_first_key(a, b, kv_u);
  const int t_lo = k_lo / kPfTile;
  const int n_tiles = (kv_u + kPfTile - 1) / kPfTile - t_lo;
  const int t_begin = t_lo + static_cast<int>(static_cast<int64_t>(n_tiles) * split / a.splits);
  const int t_end = t_lo + static_cast<int>(static_cast<int64_t>(n_tiles) * (split + 1) / a.splits);
  const int n = t_end - t_begin;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kPfNCW);
    }
    fence_barrier_init();
  }
  __syncthreads();
  // the merge kernel may be placed once every CTA of this grid has started;
  // it waits (griddepcontrol.wait) for this grid to complete
  asm volatile("griddepcontrol.launch_dependents;");

  // Loads are issued by warp 0: lane g < 4 owns the tile's 16-key group g
  // (inside one page).  fetch() reads the group's page-table entry (issued a
  // tile ahead, so its latency hides under the math); issue() posts the
  // transaction count and the TMA boxes of tile i into stage i % NS.
  const int64_t kv_rows = static_cast<int64_t>(a.hkv) * a.page_size;
  auto fetch = [&](int i, int& slot, bool& okg) {
    const int j = (t_begin + i) * kPfTile + lane * 16;
    okg = lane < 4 && i < n && j < kv_u;
    slot = okg ? a.page_table[static_cast<int64_t>(b) * a.pt_sb + j / a.page_size] : 0;
  };
  auto issue = [&](int i, int slot, bool okg) {
    const int buf = i % NS;
    const unsigned issuing = __ballot_sync(0xffffffffu, okg);
    if (lane == 0) mbar_arrive_expect_tx(&full[buf], __popc(issuing) * 2 * L::kBoxes * 2048);
    __syncwarp();
    if (okg) {
      if (slot < 0 || slot >= a.pool_pages) {
        report_status(HELM_DEV_BAD_PAGE);
        slot = 0;
      }
      const int j = (t_begin + i) * kPfTile + lane * 16;
      const int row_off = j - (j / a.page_size) * a.page_size;
      const int row_k = static_cast<int>(
          (static_cast<int64_t>(slot) * 2 * a.hkv + h) * a.page_size + row_off);
      const int row_v = static_cast<int>(row_k + kv_rows);
      uint8_t* kdst = smem + buf * L::kStageBytes + lane * 2048;
      uint8_t* vdst = kdst + L::kTileBytes;
#pragma unroll
      for (int hb = 0; hb < L::kBoxes; ++hb) {
        tma_load_2d(kdst + hb * L::kHalf, &tmap, hb * 64, row_k, &full[buf]);
        tma_load_2d(vdst + hb * L::kHalf, &tmap, hb * 64, row_v, &full[buf]);
      }
    }
  };
  if (warp == 0 && n > 0) {
    prefetch_tensormap(&tmap);
    for (int i = 0; i < NS && i < n; ++i) {
      int slot;
      bool okg;
      fetch(i, slot, okg);
      issue(i, slot, okg);
    }
  }

  // ================================ per warp ==================================
  const int g = lane >> 2, t = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  const int r0 = rb * kPfRows + warp * 16;
  const int rA = r0 + g, rB = r0 + g + 8;
  const bool okA = rA < a.rows, okB = rB < a.rows;
  const int sA = okA ? rA / a.group : 0, sB = okB ? rB / a.group : 0;
  const int qhA = h * a.group + (okA ? rA - sA * a.group : 0);
  const int qhB = h * a.group + (okB ? rB - sB * a.group : 0);
  const int kv_len = min(a.kv_lens[b], a.max_pages * a.page_size);
  const int posA = kv_len - a.q_len + sA, posB = kv_len - a.q_len + sB;  // absolute positions

  // Q fragments (A operand, row-major 16 x 16 per k-step) straight from global
  uint32_t qa[KS][4];
  {
    const T* q = static_cast<const T*>(a.q);
    const T* pA = q + static_cast<int64_t>(b) * a.q_sb + static_cast<int64_t>(qhA) * a.q_sh +
                  static_cast<int64_t>(sA) * a.q_ss + 2 * t;
    const T* pB = q + static_cast<int64_t>(b) * a.q_sb + static_cast<int64_t>(qhB) * a.q_sh +
                  static_cast<int64_t>(sB) * a.q_ss + 2 * t;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      qa[kk][0] = okA ? *reinterpret_cast<const uint32_t*>(pA + kk * 16) : 0u;
      qa[kk][1] = okB ? *reinterpret_cast<const uint32_t*>(pB + kk * 16) : 0u;
      qa[kk][2] = okA ? *reinterpret_cast<const uint32_t*>(pA + kk * 16 + 8) : 0u;
      qa[kk][3] = okB ? *reinterpret_cast<const uint32_t*>(pB + kk * 16 + 8) : 0u;
    }
  }

  float o[NO][4];
#pragma unroll
  for (int i = 0; i < NO; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.f, lB = 0.f;
  const uint32_t ring = smem_addr(smem);
  bool ok = true;

  for (int i = 0; i < n; ++i) {
    const int buf = i % NS;
    int next_slot = 0;
    bool next_ok = false;
    if (warp == 0) fetch(i + NS, next_slot, next_ok);
    if (!mbar_wait(&full[buf], (i / NS) & 1)) {
      ok = false;
      break;
    }
    const int j0 = (t_begin + i) * kPfTile;
    const int vend = kv_u - j0;  // keys of this tile that hold data (>= 1)
    const uint32_t kb = ring + buf * L::kStageBytes;
    const uint32_t vb = kb + L::kTileBytes;

    // ---- S = Q . K^T ----------------------------------------------------------
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      const int c = kk * 2 + (mi & 1);  // 16-byte chunk of the head dim
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int tok = np * 16 + (mi >> 1) * 8 + r8;
        const uint32_t addr = kb + (c >> 3) * L::kHalf + tok * 128 + (((c & 7) ^ r8) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        MmaOp<T>::run(s[2 * np], qa[kk], b0, b1);
        MmaOp<T>::run(s[2 * np + 1], qa[kk], b2, b3);
      }
    }

    // ---- scale / softcap, mask, causal limit; online softmax (log2) ----------
    float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = nt * 8 + 2 * t + e;  // key within the tile
        const int jj = j0 + c;
        float xA = s[nt][e], xB = s[nt][2 + e];
        if (a.softcap > 0.f) {
          xA = a.softcap * tanhf(xA * a.scale / a.softcap) * kLog2e;
          xB = a.softcap * tanhf(xB * a.scale / a.softcap) * kLog2e;
        } else {
          xA *= a.scale_log2;
          xB *= a.scale_log2;
        }
        const bool inA = okA && c < vend && jj >= k_lo && (!a.causal || jj <= posA);
        const bool inB = okB && c < vend && jj >= k_lo && (!a.causal || jj <= posB);
        if (a.mask != nullptr) {
          if (inA) xA += mask_log2(pf_mask<T>(a, b, sA, jj));
          if (inB) xB += mask_log2(pf_mask<T>(a, b, sB, jj));
        }
        xA = inA ? xA : -INFINITY;
        xB = inB ? xB : -INFINITY;
        s[nt][e] = xA;
        s[nt][2 + e] = xB;
        mxA = fmaxf(mxA, xA);
        mxB = fmaxf(mxB, xB);
      }
    }
    mxA = warp_max_xor(mxA, 1, 2);
    mxB = warp_max_xor(mxB, 1, 2);
    const float mnA = fmaxf(mA, mxA), mnB = fmaxf(mB, mxB);
    const float muA = mnA == -INFINITY ? 0.f : mnA, muB = mnB == -INFINITY ? 0.f : mnB;
    const float alA = exp2f(mA - muA), alB = exp2f(mB - muB);
    mA = mnA;
    mB = mnB;
    float sumA = 0.f, sumB = 0.f;
    uint32_t pa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - muA), p1 = exp2f(s[nt][1] - muA);
      const float p2 = exp2f(s[nt][2] - muB), p3 = exp2f(s[nt][3] - muB);
      sumA += p0 + p1;
      sumB += p2 + p3;
      // A operand of P.V for k-step nt/2: regs {rowA lo, rowB lo, rowA hi, rowB hi}
      pa[nt >> 1][(nt & 1) * 2 + 0] = MmaOp<T>::pack(p0, p1);
      pa[nt >> 1][(nt & 1) * 2 + 1] = MmaOp<T>::pack(p2, p3);
    }
    lA = lA * alA + sumA;
    lB = lB * alB + sumB;
#pragma unroll
    for (int i2 = 0; i2 < NO; ++i2) {
      o[i2][0] *= alA;
      o[i2][1] *= alA;
      o[i2][2] *= alB;
      o[i2][3] *= alB;
    }

    // ---- O += P . V ------------------------------------------------------------
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) {
      // keys of this k-step that hold no data (stale shared memory past the
      // sequence, or key groups that were not loaded) are zeroed in the V operand
      uint32_t keep_lo = 0xffffffffu, keep_hi = 0xffffffffu;
      if (vend < kPfTile) {
        const int k0 = kt * 16 + 2 * t;
        keep_lo = (k0 < vend ? 0x0000ffffu : 0u) | (k0 + 1 < vend ? 0xffff0000u : 0u);
        keep_hi = (k0 + 8 < vend ? 0x0000ffffu : 0u) | (k0 + 9 < vend ? 0xffff0000u : 0u);
      }
      const int tok = kt * 16 + (mi & 1) * 8 + r8;
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int c = dp * 2 + (mi >> 1);
        const uint32_t addr = vb + (c >> 3) * L::kHalf + tok * 128 + (((c & 7) ^ r8) << 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(addr, b0, b1, b2, b3);
        b0 &= keep_lo;
        b1 &= keep_hi;
        b2 &= keep_lo;
        b3 &= keep_hi;
        MmaOp<T>::run(o[2 * dp], pa[kt], b0, b1);
        MmaOp<T>::run(o[2 * dp + 1], pa[kt], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[buf]);
    if (warp == 0 && i + NS < n) {
      // refill this stage with tile i + NS once every warp is done with it
      int alive = 1;
      if (lane == 0) alive = mbar_wait(&empty[buf], (i / NS) & 1) ? 1 : 0;
      alive = __shfl_sync(0xffffffffu, alive, 0);
      if (!alive) {
        ok = false;
        break;
      }
      issue(i + NS, next_slot, next_ok);
    }
  }
  if (!ok) return;  // a wait ran out (reported); nothing is written

  lA = warp_sum_xor(lA, 1, 2);
  lB = warp_sum_xor(lB, 1, 2);
  if (a.splits == 1) {
    T* out = static_cast<T*>(a.out);
    const float invA = lA > 0.f ? 1.f / lA : 0.f, invB = lB > 0.f ? 1.f / lB : 0.f;
    T* oA = out + static_cast<int64_t>(b) * a.o_sb + static_cast<int64_t>(qhA) * a.o_sh +
            static_cast<int64_t>(sA) * a.o_ss + 2 * t;
    T* oB = out + static_cast<int64_t>(b) * a.o_sb + static_cast<int64_t>(qhB) * a.o_sh +
            static_cast<int64_t>(sB) * a.o_ss + 2 * t;
#pragma unroll
    for (int i2 = 0; i2 < NO; ++i2) {
      if (okA)
        *reinterpret_cast<uint32_t*>(oA + i2 * 8) = MmaOp<T>::pack(o[i2][0] * invA, o[i2][1] * invA);
      if (okB)
        *reinterpret_cast<uint32_t*>(oB + i2 * 8) = MmaOp<T>::pack(o[i2][2] * invB, o[i2][3] * invB);
    }
  } else {
    const int64_t part = (static_cast<int64_t>(pair) * a.row_blocks + rb) * a.splits + split;
    const int rowA = warp * 16 + g, rowB = rowA + 8;
    float* pA = a.part_o + (part * kPfRows + rowA) * D + 2 * t;
    float* pB = a.part_o + (part * kPfRows + rowB) * D + 2 * t;
#pragma unroll
    for (int i2 = 0; i2 < NO; ++i2) {
      *reinterpret_cast<float2*>(pA + i2 * 8) = make_float2(o[i2][0], o[i2][1]);
      *reinterpret_cast<float2*>(pB + i2 * 8) = make_float2(o[i2][2], o[i2][3]);
    }
    if (t == 0) {
      *reinterpret_cast<float2*>(a.part_ml + (part * kPfRows + rowA) * 2) = make_float2(mA, lA);
      *reinterpret_cast<float2*>(a.part_ml + (part * kPfRows + rowB) * 2) = make_float2(mB, lB);
    }
  }
}

// Merges the splits of every unit: CTA (unit, chunk) owns 256 (row, 4-column)
// elements of the unit's RPU x D block and combines the `splits` partial
// states of each (running rescaled sum, the loads of kPfMergeBatch splits in
// flight per thread).  Partials are [unit * splits + split][RPU rows][D].
constexpr int kPfMergeBatch = 4;

template <typename T, int D, int RPU>
__global__ void __launch_bounds__(kPfMergeThreads) merge_prefill_splits_kernel(const PrefillArgs a) {
  constexpr int D4 = D / 4;
  // every thread waits for the prefill kernel (complete and visible)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int unit = blockIdx.x;  // (b * hkv + h) * row_blocks + rb
  const int rb = unit % a.row_blocks, pair = unit / a.row_blocks;
  const int e = blockIdx.y * kPfMergeThreads + threadIdx.x;
  const int row = e / D4, d4 = e - (e / D4) * D4;
  if (row >= RPU) return;
  const int r = rb * RPU + row;
  if (r >= a.rows) return;
  const int b = pair / a.hkv, h = pair - (pair / a.hkv) * a.hkv;
  const int s = r / a.group, qh = h * a.group + (r - s * a.group);
  const int64_t part0 = static_cast<int64_t>(unit) * a.splits;
  float M = -INFINITY, Lsum = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k0 = 0; k0 < a.splits; k0 += kPfMergeBatch) {
    float2 ml[kPfMergeBatch];
    float4 ov[kPfMergeBatch];
#pragma unroll
    for (int i = 0; i < kPfMergeBatch; ++i) {
      ml[i] = make_float2(-INFINITY, 0.f);
      ov[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k0 + i < a.splits) {
        const int64_t rec = (part0 + k0 + i) * RPU + row;
        ml[i] = __ldcg(reinterpret_cast<const float2*>(a.part_ml + rec * 2));
        ov[i] = __ldcg(reinterpret_cast<const float4*>(a.part_o + rec * D + d4 * 4));
      }
    }
    float Mb = M;
#pragma unroll
    for (int i = 0; i < kPfMergeBatch; ++i) Mb = fmaxf(Mb, ml[i].x);
    if (Mb == -INFINITY) continue;  // no visible key in any split so far
    const float rs = exp2f(M - Mb);  // 0 while M is -inf
    Lsum *= rs;
    acc.x *= rs;
    acc.y *= rs;
    acc.z *= rs;
    acc.w *= rs;
#pragma unroll
    for (int i = 0; i < kPfMergeBatch; ++i) {
      const float w = exp2f(ml[i].x - Mb);
      Lsum += ml[i].y * w;
      acc.x += w * ov[i].x;
      acc.y += w * ov[i].y;
      acc.z += w * ov[i].z;
      acc.w += w * ov[i].w;
    }
    M = Mb;
  }
  const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
  T* o = static_cast<T*>(a.out) + static_cast<int64_t>(b) * a.o_sb +
         static_cast<int64_t>(qh) * a.o_sh + static_cast<int64_t>(s) * a.o_ss + d4 * 4;
  reinterpret_cast<uint32_t*>(o)[0] = MmaOp<T>::pack(acc.x * inv, acc.y * inv);
  reinterpret_cast<uint32_t*>(o)[1] = MmaOp<T>::pack(acc.z * inv, acc.w * inv);
}

// CTAs of the prefill kernel resident per SM (cached per device and head size).
template <typename T, int D>
int prefill_ctas_per_sm() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 1;
  if (cached[dev] == 0) {
    int nb = 0;
    if (cudaFuncSetAttribute(paged_prefill_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(PfLayout<D>::smem_bytes())) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, paged_prefill_kernel<T, D>, kPfThreads,
                                                      PfLayout<D>::smem_bytes()) != cudaSuccess ||
        nb <= 0)
      nb = 1;
    cached[dev] = nb;
  }
  return cached[dev];
}

struct PrefillPlan {
  int row_blocks = 0, splits = 1;
  int64_t units = 0, o_bytes = 0, ml_bytes = 0;
  int64_t total() const { return splits > 1 ? o_bytes + ml_bytes : 0; }
};

// Split count: the one (<= kPfMaxSplits, partials <= kPfMaxPartialBytes) that
// minimises whole waves x tiles per split, plus two tiles' worth per extra
// pass (the partial write and the merge).
PrefillPlan plan_prefill(int batch, int q_len, int hq, int hkv, int d, int max_kv_len,
                         int ctas_per_sm, int rpu) {
  PrefillPlan p;
  const int group = hq / hkv;
  const int64_t rows = static_cast<int64_t>(q_len) * group;
  p.row_blocks = static_cast<int>((rows + rpu - 1) / rpu);
  p.units = static_cast<int64_t>(batch) * hkv * p.row_blocks;
  const int64_t slots = static_cast<int64_t>(num_sms_current_device()) * std::max(1, ctas_per_sm);
  const int64_t tiles = std::max<int64_t>(1, (static_cast<int64_t>(max_kv_len) + kPfTile - 1) / kPfTile);
  int64_t best_cost = -1;
  for (int sp = 1; sp <= kPfMaxSplits && sp <= tiles; ++sp) {
    if (sp > 1 && p.units * sp * rpu * d * 4 > kPfMaxPartialBytes) break;
    const int64_t waves = (p.units * sp + slots - 1) / slots;
    const int64_t cost = waves * ((tiles + sp - 1) / sp) + (sp > 1 ? 2 : 0);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      p.splits = sp;
    }
  }
  auto up = [](int64_t x) { return ((x + 255) / 256) * 256; };
  p.o_bytes = up(p.units * p.splits * rpu * d * 4);
  p.ml_bytes = up(p.units * p.splits * rpu * 2 * 4);
  return p;
}

// TMA map over the pool viewed as [slots * 2 * Hkv * page_size rows, D]:
// boxes of 16 rows x 64 columns, 128-byte swizzle.
template <typename T, int D>
bool encode_pool_map(const void* pool, int64_t pool_rows, CUtensorMap* map) {
  EncodeTiledFn encode = get_encode_fn();
  if (encode == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(pool_rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(D) * 2};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t estride[2] = {1, 1};
  const CUtensorMapDataType dt = std::is_same<T, __nv_bfloat16>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode(map, dt, 2, const_cast<void*>(pool), dims, strides, box, estride,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

template <typename T, int D>
int launch_prefill(PrefillArgs a, const void* pool, int64_t pool_rows, int max_kv_len,
                   void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  const int ctas = prefill_ctas_per_sm<T, D>();
  const PrefillPlan plan = plan_prefill(a.batch, a.q_len, a.hq, a.hkv, D, max_kv_len, ctas, kPfRows);
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
  paged_prefill_kernel<T, D><<<static_cast<unsigned>(grid), kPfThreads,
                               PfLayout<D>::smem_bytes(), stream>>>(map, a);
  if (cudaGetLastError() != cudaSuccess) return HELM_ERR_CUDA;
  if (plan.splits == 1) return HELM_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(plan.units),
                     static_cast<unsigned>((kPfRows * D / 4 + kPfMergeThreads - 1) / kPfMergeThreads));
  cfg.blockDim = dim3(kPfMergeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, merge_prefill_splits_kernel<T, D, kPfRows>, a) != cudaSuccess)
    return HELM_ERR_CUDA;
  return HELM_OK;
}

template <typename T>
int prefill_dispatch(int head_dim, const PrefillArgs& a, const void* pool, int64_t rows,
                     int max_kv_len, void* ws, int64_t ws_bytes, cudaStream_t s) {
  switch (head_dim) {
    case 64:
      return launch_prefill<T, 64>(a, pool, rows, max_kv_len, ws, ws_bytes, s);
    case 128:
      return launch_prefill<T, 128>(a, pool, rows, max_kv_len, ws, ws_bytes, s);
    default:
      return HELM_ERR_UNSUPPORTED;
  }
}

}  // namespace

}  // namespace helm

