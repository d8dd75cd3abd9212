// Paged decode attention for sm_100a (B200).
//
// Replaces the per-page eager loop / torch.cat+SDPA of HELM's
// perform_streaming_attention (helm/runtime/kv_cache.py:405-662) and the paged
// branches of _decode_batched (helm/runtime/kv_offload.py:144-186) with one
// persistent kernel launch.
//
// Work unit: a TILE = 16 consecutive token rows of one page of one KV head
// (K: 16 x D, V: 16 x D).  All tiles of all (sequence, kv-head) PAIRS are laid
// out in one flattened order (sequence-major, then kv head, then tile) and cut
// into equal contiguous ranges, one per WORKER (a consumer warp).  A worker
// walks its range, keeps an online-softmax state for the G query heads of the
// current pair, and when its range leaves a pair either writes the final
// output (it covered the whole pair) or an fp32 partial state (m, l,
// unnormalised O) at the unique slot worker + pair.  After its loop, a CTA
// combines the states of its warps that end in the same pair: the final
// output when the CTA covered the whole pair, else one CTA partial.  A second
// kernel, launched as a programmatic dependent (its CTAs are placed while the
// first still runs and wait in griddepcontrol.wait), merges the pairs split
// across CTAs, every split pair at once, each thread with the loads of all
// its sources in flight together.
//
// Per CTA: one producer warp issues TMA tile loads (two 64-column boxes per K
// or V tile, 128-byte swizzled so ldmatrix reads are bank-conflict free) into
// a ring of NS stages; stage s holds tile s of each of the CTA's NCW workers.
// Full/empty mbarriers hand stages between producer and consumers.
//
// Math per tile (tensor cores, mma.sync m16n8k16, fp32 accumulate):
//   S^T[16 tok x 8 heads] = K[16 x D] . Q^T[D x 8]        (tokens fill M)
//   online softmax over tokens per head (warp shuffles, exp2 domain)
//   O^T[D x 8] += V^T[D x 16] . P^T[16 x 8]               (P^T via movmatrix)
// The GQA group (G <= 16 query heads per KV head) is the N dimension.
#include "common.cuh"

namespace helm {

namespace {

constexpr int kTileRows = 16;
constexpr int kMaxNCW = 8;                   // most consumer warps (= workers) per CTA
constexpr int kStageBudget = 196608;         // bytes of tile ring per CTA
constexpr int kMaxBatch = 2048;              // prefix table held in shared memory
// With a length hint, the grid is cut to one CTA per kMinTilesPerWorker tiles
// of each worker warp: short contexts then use fewer SMs.  One tile per worker
// is fastest on the short contexts of a decode step (configs[0], 576 tokens x
// 8 KV heads: 1.06 ms per step against 1.29 ms at four tiles and 1.43 ms at
// eight; the 4.4k-token configs[2] step is bound by its host copies either way).
constexpr int kMinTilesPerWorker = 1;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct DecodeArgs {
  const void* q;
  int64_t q_sb, q_sh;
  int64_t pool_pages;
  const int32_t* page_table;
  int64_t pt_sb;
  int max_pages;
  const int32_t* kv_lens;
  const int32_t* num_pages;   // ragged page lists (nullable, with the next two)
  const int32_t* page_used;
  const int32_t* page_start;
  const void* mask;
  int mask_dtype;
  int64_t mask_sb;
  void* out;
  int64_t out_sb, out_sh;
  float* lse;
  float* part_o;    // warp partials [num_workers + pairs][G][D]
  float* part_ml;   // warp partials [num_workers + pairs][G][2]  (m in log2 units, l)
  float* cta_o;     // CTA partials [grid + pairs][G][D]
  float* cta_ml;    // CTA partials [grid + pairs][G][2]
  int batch, hq, hkv, group, page_size, tiles_per_page;
  int out_fp32;  // O written as fp32 (partial states for a cross-device merge)
  float scale;
  float scale_log2;
  float softcap;
  int num_workers;
};

__device__ __forceinline__ int div_up(int a, int b) { return (a + b - 1) / b; }

// Number of tiles of every pair of sequence b.  Out-of-range page counts are
// clamped (and reported) so that no page-table read leaves its row.
__device__ __forceinline__ int tiles_of_seq(const DecodeArgs& a, int b) {
  int n;
  if (a.num_pages != nullptr) {
    n = a.num_pages[b];
  } else {
    const int len = a.kv_lens[b];
    n = len > 0 ? div_up(len, a.page_size) : 0;
  }
  if (n < 0) n = 0;
  if (n > a.max_pages) {
    report_status(HELM_DEV_BAD_PAGE);
    n = a.max_pages;
  }
  return n * a.tiles_per_page;
}

// Fills s_cum[0..B] with the prefix sum of tiles per sequence (one warp).
__device__ void build_prefix(const DecodeArgs& a, int* s_cum, int lane) {
  int carry = 0;
  if (lane == 0) s_cum[0] = 0;
  for (int base = 0; base < a.batch; base += 32) {
    const int b = base + lane;
    int v = b < a.batch ? tiles_of_seq(a, b) : 0;
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, off);
      if (lane >= off) v += n;
    }
    if (b < a.batch) s_cum[b + 1] = carry + v;
    carry += __shfl_sync(0xffffffffu, v, 31);
  }
}

struct TilePos {
  int b, h, t;  // sequence, kv head, tile within the pair
};

// Maps a flattened tile index x (< total) to its (sequence, head, tile).
__device__ __forceinline__ TilePos locate(const int* s_cum, int batch, int hkv, int x) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {  // largest b with s_cum[b] * hkv <= x
    const int mid = (lo + hi + 1) >> 1;
    if (s_cum[mid] * hkv <= x)
      lo = mid;
    else
      hi = mid - 1;
  }
  const int tb = s_cum[lo + 1] - s_cum[lo];
  const int r = x - s_cum[lo] * hkv;
  TilePos p;
  p.b = lo;
  p.h = r / tb;
  p.t = r - p.h * tb;
  return p;
}

__device__ __forceinline__ void advance(TilePos& p, const int* s_cum, int batch, int hkv) {
  const int tb = s_cum[p.b + 1] - s_cum[p.b];
  if (++p.t < tb) return;
  p.t = 0;
  if (++p.h < hkv) return;
  p.h = 0;
  do {
    ++p.b;
  } while (p.b < batch && s_cum[p.b + 1] == s_cum[p.b]);
}

template <typename T>
__device__ __forceinline__ float load_mask(const DecodeArgs& a, int b, int tok) {
  const int64_t off = static_cast<int64_t>(b) * a.mask_sb + tok;
  if (a.mask_dtype == HELM_DTYPE_FP32) return static_cast<const float*>(a.mask)[off];
  if (a.mask_dtype == HELM_DTYPE_BF16)
    return __bfloat162float(static_cast<const __nv_bfloat16*>(a.mask)[off]);
  return __half2float(static_cast<const __half*>(a.mask)[off]);
}

// Writes one element of O (sequence b, query head qh, dim d).
template <typename T>
__device__ __forceinline__ void store_out(const DecodeArgs& a, int b, int qh, int d, float v) {
  const int64_t off =
      static_cast<int64_t>(b) * a.out_sb + static_cast<int64_t>(qh) * a.out_sh + d;
  if (a.out_fp32)
    static_cast<float*>(a.out)[off] = v;
  else
    static_cast<T*>(a.out)[off] = from_float<T>(v);
}

// Additive mask value in log2 units.  A finite mask (e.g. finfo(float32).min)
// stays finite instead of overflowing to -inf, so a row whose every key is
// masked with a finite value behaves as in eager fp32 arithmetic.
__device__ __forceinline__ float mask_log2(float m) {
  return m == -INFINITY ? -INFINITY : fmaxf(m * kLog2e, -3.0e38f);
}

template <typename T, int D, int NT>
struct Worker {
  static constexpr int KS = D / 16;  // k-steps over the head dim, = m-tiles of O^T
  float m[NT][2];
  float l[NT][2];
  float o[NT][KS][4];
  uint32_t qf[NT][KS][2];
  int cur_b = -1, cur_h = -1;
  int cur_len = 0;  // kv_len of the current sequence (dense page lists)

  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        m[nt][j] = -INFINITY;
        l[nt][j] = 0.f;
      }
#pragma unroll
      for (int mt = 0; mt < KS; ++mt)
#pragma unroll
        for (int e = 0; e < 4; ++e) o[nt][mt][e] = 0.f;
    }
  }

  __device__ __forceinline__ void load_q(const DecodeArgs& a, int b, int h, int lane) {
    const int g = lane >> 2, t = lane & 3;
    const T* qb = static_cast<const T*>(a.q) + static_cast<int64_t>(b) * a.q_sb;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int hg = nt * 8 + g;
      const bool ok = hg < a.group;
      const T* qh = qb + static_cast<int64_t>(h * a.group + (ok ? hg : 0)) * a.q_sh;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const uint32_t w0 = ok ? *reinterpret_cast<const uint32_t*>(qh + kk * 16 + 2 * t) : 0u;
        const uint32_t w1 =
            ok ? *reinterpret_cast<const uint32_t*>(qh + kk * 16 + 8 + 2 * t) : 0u;
        qf[nt][kk][0] = w0;
        qf[nt][kk][1] = w1;
      }
    }
  }

  // Ends the current pair: when this worker covered the whole pair it writes
  // the normalised output and LSE; otherwise its partial state goes to slot
  // worker + pair for the merge.
  __device__ __forceinline__ void flush(const DecodeArgs& a, const int* s_cum, int W, int v,
                                        int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int b = cur_b, h = cur_h, p = b * a.hkv + h;
    const int tb = s_cum[b + 1] - s_cum[b];
    const int st = s_cum[b] * a.hkv + h * tb;
    const bool alone = (st / W) == ((st + tb - 1) / W);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float lt = warp_sum_xor(l[nt][j], 4, 16);
        const int hg = nt * 8 + 2 * t + j;
        if (hg >= a.group) continue;
        if (alone) {
          const float inv = 1.f / fmaxf(lt, 1e-12f);
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            store_out<T>(a, b, h * a.group + hg, mt * 16 + g, o[nt][mt][j] * inv);
            store_out<T>(a, b, h * a.group + hg, mt * 16 + 8 + g, o[nt][mt][2 + j] * inv);
          }
          if (g == 0 && a.lse != nullptr)
            a.lse[static_cast<int64_t>(b) * a.hq + h * a.group + hg] =
                (m[nt][j] == -INFINITY || lt <= 0.f) ? -INFINITY : m[nt][j] * kLn2 + logf(lt);
        } else {
          const int64_t slot = static_cast<int64_t>(v + p) * a.group + hg;
          float* po = a.part_o + slot * D;
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            po[mt * 16 + g] = o[nt][mt][j];
            po[mt * 16 + 8 + g] = o[nt][mt][2 + j];
          }
          if (g == 0)
            *reinterpret_cast<float2*>(a.part_ml + slot * 2) = make_float2(m[nt][j], lt);
        }
      }
    }
  }

  // Raw state (m, lane-reduced l, unnormalised O) into a shared-memory record
  // laid out as m[16] | l[16] | O[16][D].
  __device__ __forceinline__ void save(float* rec, int group, int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float lt = warp_sum_xor(l[nt][j], 4, 16);
        const int hg = nt * 8 + 2 * t + j;
        if (hg >= group) continue;
        float* o_rec = rec + 32 + hg * D;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          o_rec[mt * 16 + g] = o[nt][mt][j];
          o_rec[mt * 16 + 8 + g] = o[nt][mt][2 + j];
        }
        if (g == 0) {
          rec[hg] = m[nt][j];
          rec[16 + hg] = lt;
        }
      }
    }
  }

  __device__ __forceinline__ void tile(const DecodeArgs& a, uint32_t kbase, uint32_t vbase,
                                       int valid, int tok0, int b, int lane) {
    const int g = lane >> 2, t = lane & 3, mi = lane >> 3, r7 = lane & 7;
    // ---- S^T = K . Q^T, two independent accumulation chains -----------------
    float s[NT][4], s2[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = s2[nt][e] = 0.f;
    {
      const int r = r7 + ((mi & 1) << 3);
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const int c = ((kk & 3) << 1) + (mi >> 1);
        const uint32_t addr = kbase + (kk >> 2) * 2048 + r * 128 + ((c ^ r7) << 4);
        uint32_t af[4];
        ldsm_x4(addr, af[0], af[1], af[2], af[3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (kk & 1)
            MmaOp<T>::run(s2[nt], af, qf[nt][kk][0], qf[nt][kk][1]);
          else
            MmaOp<T>::run(s[nt], af, qf[nt][kk][0], qf[nt][kk][1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] += s2[nt][e];
    }
    // ---- online softmax (log2 domain) ---------------------------------------
    const bool v0 = g < valid, v1 = g + 8 < valid;
    float madd0 = 0.f, madd1 = 0.f;
    if (a.mask != nullptr) {
      if (v0) madd0 = mask_log2(load_mask<T>(a, b, tok0 + g));
      if (v1) madd1 = mask_log2(load_mask<T>(a, b, tok0 + g + 8));
    }
    uint32_t pb0[NT], pb1[NT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float p[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float x0 = s[nt][j], x1 = s[nt][2 + j];
        if (a.softcap > 0.f) {
          x0 = a.softcap * tanhf(x0 * a.scale / a.softcap) * kLog2e;
          x1 = a.softcap * tanhf(x1 * a.scale / a.softcap) * kLog2e;
        } else {
          x0 *= a.scale_log2;
          x1 *= a.scale_log2;
        }
        x0 = v0 ? x0 + madd0 : -INFINITY;
        x1 = v1 ? x1 + madd1 : -INFINITY;
        const float mx = warp_max_xor(fmaxf(x0, x1), 4, 16);
        const float m_new = fmaxf(m[nt][j], mx);
        const float m_use = m_new == -INFINITY ? 0.f : m_new;
        const float alpha = exp2f(m[nt][j] - m_use);
        const float p0 = exp2f(x0 - m_use), p1 = exp2f(x1 - m_use);
        l[nt][j] = l[nt][j] * alpha + p0 + p1;
        m[nt][j] = m_new;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          o[nt][mt][j] *= alpha;
          o[nt][mt][2 + j] *= alpha;
        }
        p[j] = p0;
        p[2 + j] = p1;
      }
      pb0[nt] = movmatrix_trans(MmaOp<T>::pack(p[0], p[1]));
      pb1[nt] = movmatrix_trans(MmaOp<T>::pack(p[2], p[3]));
    }
    // ---- O^T += V^T . P^T ----------------------------------------------------
    uint32_t keep01 = 0xffffffffu, keep23 = 0xffffffffu;
    if (valid < kTileRows) {
      keep01 = (2 * t < valid ? 0x0000ffffu : 0u) | (2 * t + 1 < valid ? 0xffff0000u : 0u);
      keep23 = (2 * t + 8 < valid ? 0x0000ffffu : 0u) | (2 * t + 9 < valid ? 0xffff0000u : 0u);
    }
    const int r = r7 + ((mi >> 1) << 3);
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      const int c = ((mt & 3) << 1) + (mi & 1);
      const uint32_t addr = vbase + (mt >> 2) * 2048 + r * 128 + ((c ^ r7) << 4);
      uint32_t af[4];
      ldsm_x4_trans(addr, af[0], af[1], af[2], af[3]);
      af[0] &= keep01;
      af[1] &= keep01;
      af[2] &= keep23;
      af[3] &= keep23;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) MmaOp<T>::run(o[nt][mt], af, pb0[nt], pb1[nt]);
    }
  }
};

__device__ __forceinline__ void consumer_barrier(int threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// Pair geometry in the flattened tile order: the workers (warps) that cover it
// and whether the last of them goes on past it (then that worker flushed its
// state for the pair to the warp-partial slot in mid-range).
struct PairSpan {
  int tiles, vf, vl;
  bool last_continues;
};

__device__ __forceinline__ PairSpan pair_span(const DecodeArgs& a, const int* s_cum, int W,
                                              int total, int p) {
  const int b = p / a.hkv, h = p - (p / a.hkv) * a.hkv;
  PairSpan ps;
  ps.tiles = s_cum[b + 1] - s_cum[b];
  ps.vf = ps.vl = 0;
  ps.last_continues = false;
  if (ps.tiles > 0) {
    const int st = s_cum[b] * a.hkv + h * ps.tiles, en = st + ps.tiles;
    ps.vf = st / W;
    ps.vl = (en - 1) / W;
    ps.last_continues = min((ps.vl + 1) * W, total) > en;
  }
  return ps;
}

// Combines the end states of warps w0 .. w0+nw-1 of this CTA (shared-memory
// records m[16] | l[16] | O[16][D]), which all end in pair p, plus, when
// warp_slot >= 0, the warp partial at global slot warp_slot + p (written by a
// warp of this CTA before the preceding barrier).  Writes the normalised
// output and LSE (final) or a CTA partial at slot cta_out + p.  One pass, no
// barriers: each thread owns float4 output elements and reads the (m, l) and
// O values of all sources of its element together.
template <typename T, int D, int NCW>
__device__ void merge_group(const DecodeArgs& a, int p, const float* s_states, int w0, int nw,
                            int warp_slot, bool final_out, int cta_out) {
  constexpr int kConsumers = NCW * 32;
  constexpr int kRec = 32 + 16 * D;
  constexpr int D4 = D / 4;
  constexpr int kMaxK = NCW + 1;
  const int G = a.group;
  const int b = p / a.hkv, h = p - (p / a.hkv) * a.hkv;
  for (int e = threadIdx.x; e < G * D4; e += kConsumers) {
    const int hg = e / D4, d4 = e - (e / D4) * D4;
    float mk[kMaxK], lk[kMaxK];
    float4 ok[kMaxK];
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) {
      mk[k] = -INFINITY;
      lk[k] = 0.f;
      ok[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < nw) {
        const float* rec = s_states + (w0 + k) * kRec;
        mk[k] = rec[hg];
        lk[k] = rec[16 + hg];
        ok[k] = *reinterpret_cast<const float4*>(rec + 32 + hg * D + d4 * 4);
      } else if (k == nw && warp_slot >= 0) {
        const int64_t slot = static_cast<int64_t>(warp_slot + p) * G + hg;
        const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.part_ml + slot * 2));
        mk[k] = ml.x;
        lk[k] = ml.y;
        ok[k] = __ldcg(reinterpret_cast<const float4*>(a.part_o + slot * D + d4 * 4));
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) M = fmaxf(M, mk[k]);
    const float m_use = M == -INFINITY ? 0.f : M;
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) {
      const float w = exp2f(mk[k] - m_use);
      L += lk[k] * w;
      acc.x += w * ok[k].x;
      acc.y += w * ok[k].y;
      acc.z += w * ok[k].z;
      acc.w += w * ok[k].w;
    }
    if (final_out) {
      const float inv = 1.f / fmaxf(L, 1e-12f);
      store_out<T>(a, b, h * G + hg, d4 * 4 + 0, acc.x * inv);
      store_out<T>(a, b, h * G + hg, d4 * 4 + 1, acc.y * inv);
      store_out<T>(a, b, h * G + hg, d4 * 4 + 2, acc.z * inv);
      store_out<T>(a, b, h * G + hg, d4 * 4 + 3, acc.w * inv);
      if (d4 == 0 && a.lse != nullptr)
        a.lse[static_cast<int64_t>(b) * a.hq + h * G + hg] =
            (M == -INFINITY || L <= 0.f) ? -INFINITY : M * kLn2 + logf(L);
    } else {
      const int64_t slot = static_cast<int64_t>(cta_out + p) * G + hg;
      *reinterpret_cast<float4*>(a.cta_o + slot * D + d4 * 4) = acc;
      if (d4 == 0) *reinterpret_cast<float2*>(a.cta_ml + slot * 2) = make_float2(M, L);
    }
  }
}

template <int D>
struct Layout {
  static constexpr int NCW = D <= 128 ? 8 : 4;  // consumer warps (= workers) per CTA
  static constexpr int kThreads = (NCW + 1) * 32;
  static constexpr int kTileBytes = kTileRows * D * 2;
  static constexpr int kStageBytes = NCW * 2 * kTileBytes;
  static constexpr int NS = kStageBudget / kStageBytes;
  static_assert(NS >= 2, "tile ring needs at least two stages");
  static constexpr size_t smem_bytes(int batch) {
    return 1024 + NS * kStageBytes + 2 * NS * sizeof(uint64_t) + (batch + 1) * sizeof(int);
  }
};

template <typename T, int D, int NT>
__global__ void __launch_bounds__(Layout<D>::kThreads, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap tmap, const DecodeArgs a) {
  using L = Layout<D>;
  constexpr int NCW = L::NCW;
  constexpr int kTileBytes = L::kTileBytes;
  constexpr int kStageBytes = L::kStageBytes;
  constexpr int NS = L::NS;
  constexpr int kBoxes = D / 64;
  constexpr int kConsumers = NCW * 32;

  extern __shared__ uint8_t smem_raw[];
  __shared__ int s_abort;
  uint8_t* smem = smem_raw + ((1024 - (smem_addr(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * kStageBytes);
  uint64_t* empty = full + NS;
  int* s_cum = reinterpret_cast<int*>(empty + NS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) build_prefix(a, s_cum, lane);
  if (threadIdx.x == 32) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NCW);
    }
    fence_barrier_init();
    s_abort = 0;
  }
  __syncthreads();
  // the merge kernel may be placed now; it waits for this grid to complete
  asm volatile("griddepcontrol.launch_dependents;");

  // Launched as a programmatic dependent (decode overlap), this grid may run
  // before the previous kernel on the stream has finished: up to here it read
  // only the lengths; the page table is read next, and every thread waits
  // (griddepcontrol.wait) before it reads q or the pool or writes anything.
  // Launched normally, the waits return at once.

  // Pairs without tokens: zero output, LSE = -inf.
  bool waited = false;
  for (int p = blockIdx.x; p < a.batch * a.hkv; p += gridDim.x) {
    const int b = p / a.hkv, h = p - (p / a.hkv) * a.hkv;
    if (s_cum[b + 1] != s_cum[b]) continue;
    if (!waited) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      waited = true;
    }
    for (int e = threadIdx.x; e < a.group * D; e += blockDim.x)
      store_out<T>(a, b, h * a.group + e / D, e % D, 0.f);
    if (a.lse != nullptr && threadIdx.x < a.group)
      a.lse[static_cast<int64_t>(b) * a.hq + h * a.group + threadIdx.x] = -INFINITY;
  }

  const int total = s_cum[a.batch] * a.hkv;
  const int W = total > 0 ? div_up(total, a.num_workers) : 0;
  const int v0 = blockIdx.x * NCW;
  const int n_stages = total > 0 ? max(0, min(W, total - v0 * W)) : 0;
  if (n_stages == 0) {
    // nothing to stream; still wait, so that this grid cannot complete before
    // the kernel it depends on (later kernels rely on that ordering)
    if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");
    return;
  }

  if (warp == NCW) {
    // ================================ producer ================================
    prefetch_tensormap(&tmap);
    const int w = lane % NCW, j = lane / NCW;  // this lane's worker / stage in window
    constexpr int kWin = 32 / NCW;
    const int worker_first = (v0 + w) * W;
    const int worker_len = max(0, min(W, total - worker_first));
    const int64_t kv_rows = static_cast<int64_t>(a.hkv) * a.page_size;

    // row_k: pool row of the tile's K; tail: the tile is in its sequence's last
    // page (the one a preceding append kernel may still be writing)
    auto rows_of = [&](int s, int& row_k, bool& ok, bool& tail) {
      ok = s < worker_len;
      row_k = 0;
      tail = false;
      if (!ok) return;
      const TilePos p = locate(s_cum, a.batch, a.hkv, worker_first + s);
      const int page = p.t / a.tiles_per_page;
      tail = page == (s_cum[p.b + 1] - s_cum[p.b]) / a.tiles_per_page - 1;
      const int row_off = (p.t - page * a.tiles_per_page) * kTileRows;
      int slot = a.page_table[static_cast<int64_t>(p.b) * a.pt_sb + page];
      if (slot < 0 || slot >= a.pool_pages) {
        report_status(HELM_DEV_BAD_PAGE);
        slot = 0;
      }
      row_k = static_cast<int>((static_cast<int64_t>(slot) * 2 * a.hkv + p.h) * a.page_size +
                               row_off);
    };

    auto issue_tile = [&](int buf, int row_k) {
      uint8_t* kdst = smem + buf * kStageBytes + w * 2 * kTileBytes;
      uint8_t* vdst = kdst + kTileBytes;
      const int row_v = static_cast<int>(row_k + kv_rows);
#pragma unroll
      for (int hb = 0; hb < kBoxes; ++hb) {
        tma_load_2d(kdst + hb * 2048, &tmap, hb * 64, row_k, &full[buf]);
        tma_load_2d(vdst + hb * 2048, &tmap, hb * 64, row_v, &full[buf]);
      }
    };

    int row_cur, row_nxt;
    bool ok_cur, ok_nxt, tail_cur, tail_nxt;
    rows_of(j, row_cur, ok_cur, tail_cur);
    // The first `pre` stages (free ring slots) are posted before waiting for the
    // kernel before this one: their transaction counts, and the TMA loads of
    // tiles outside their sequence's last page (with decode overlap the only
    // page that kernel may write); last-page tiles are loaded after the wait.
    const int pre = min(min(NS, kWin), n_stages);
    for (int jj = 0; jj < pre; ++jj) {
      const bool mine = (j == jj) && ok_cur;
      const unsigned issuing = __ballot_sync(0xffffffffu, mine);
      if (lane == 0) mbar_arrive_expect_tx(&full[jj], __popc(issuing) * 2 * kTileBytes);
      __syncwarp();
      if (mine && !tail_cur) issue_tile(jj, row_cur);
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    for (int win = 0; win * kWin < n_stages; ++win) {
      rows_of((win + 1) * kWin + j, row_nxt, ok_nxt, tail_nxt);  // next window's page table
      for (int jj = 0; jj < kWin; ++jj) {
        const int s = win * kWin + jj;
        if (s >= n_stages) break;
        if (s < pre) {  // posted above; its last-page tiles go now
          if (j == jj && ok_cur && tail_cur) issue_tile(s, row_cur);
          continue;
        }
        const int buf = s % NS, n = s / NS;
        int alive = 1;
        if (lane == 0 && n > 0) alive = mbar_wait(&empty[buf], (n - 1) & 1) ? 1 : 0;
        alive = __shfl_sync(0xffffffffu, alive, 0);
        if (!alive) return;
        const bool mine = (j == jj) && ok_cur;
        const unsigned issuing = __ballot_sync(0xffffffffu, mine);
        if (lane == 0) mbar_arrive_expect_tx(&full[buf], __popc(issuing) * 2 * kTileBytes);
        __syncwarp();
        if (mine) issue_tile(buf, row_cur);
      }
      row_cur = row_nxt;
      ok_cur = ok_nxt;
      tail_cur = tail_nxt;
    }
    return;
  }

  // ================================= consumers ================================
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int v = v0 + warp;
  const int first = v * W;
  const int my_len = max(0, min(W, total - first));
  Worker<T, D, NT> st;
  TilePos pos;
  if (my_len > 0) pos = locate(s_cum, a.batch, a.hkv, first);
  const uint32_t ring = smem_addr(smem);
  bool ok = true;

  for (int s = 0; s < n_stages; ++s) {
    const int buf = s % NS, n = s / NS;
    if (!mbar_wait(&full[buf], n & 1)) {
      ok = false;
      break;
    }
    if (s < my_len) {
      if (pos.b != st.cur_b || pos.h != st.cur_h) {
        if (st.cur_b >= 0) st.flush(a, s_cum, W, v, lane);
        st.cur_b = pos.b;
        st.cur_h = pos.h;
        st.cur_len = a.num_pages != nullptr ? 0 : a.kv_lens[pos.b];
        st.reset();
        st.load_q(a, pos.b, pos.h, lane);
      }
      const int page = pos.t / a.tiles_per_page;
      const int row_off = (pos.t - page * a.tiles_per_page) * kTileRows;
      int page_tokens, tok0;
      if (a.num_pages != nullptr) {
        const int64_t e = static_cast<int64_t>(pos.b) * a.pt_sb + page;
        page_tokens = min(a.page_used[e], a.page_size);
        tok0 = a.page_start[e] + row_off;
      } else {
        page_tokens = min(a.page_size, st.cur_len - page * a.page_size);
        tok0 = page * a.page_size + row_off;
      }
      const int valid = max(0, min(kTileRows, page_tokens - row_off));
      const uint32_t kb = ring + buf * kStageBytes + warp * 2 * kTileBytes;
      st.tile(a, kb, kb + kTileBytes, valid, tok0, pos.b, lane);
      advance(pos, s_cum, a.batch, a.hkv);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[buf]);
  }
  // ============ merge ============
  // 1. each warp's end-of-range state (if it does not cover its pair alone)
  //    goes to a shared-memory record (the tile ring is idle now);
  // 2. warps of this CTA ending in the same pair are combined: the final
  //    output when this CTA covers the whole pair, else one CTA partial;
  // 3. pairs split across CTAs are merged by merge_split_pairs_kernel.
  constexpr int kRec = 32 + 16 * D;
  float* s_states = reinterpret_cast<float*>(smem);
  __shared__ int s_endpair[NCW];
  int end_pair = -1;
  if (!ok) {
    if (lane == 0) s_abort = 1;
  } else if (st.cur_b >= 0) {
    end_pair = st.cur_b * a.hkv + st.cur_h;
    const PairSpan ps = pair_span(a, s_cum, W, total, end_pair);
    if (ps.vf == ps.vl) {
      st.flush(a, s_cum, W, v, lane);  // covered alone: final output
      end_pair = -1;
    } else {
      st.save(s_states + warp * kRec, a.group, lane);
    }
  }
  if (lane == 0) s_endpair[warp] = end_pair;
  consumer_barrier(kConsumers);
  if (s_abort) return;  // every consumer warp reads the same flag after the barrier
  const int cta = blockIdx.x;
  for (int w0 = 0; w0 < NCW;) {
    const int p = s_endpair[w0];
    int w1 = w0 + 1;
    while (w1 < NCW && s_endpair[w1] == p) ++w1;
    if (p >= 0) {
      const PairSpan ps = pair_span(a, s_cum, W, total, p);
      const int cf = ps.vf / NCW, cl = ps.vl / NCW;
      if (cf == cl)  // the whole pair is in this CTA
        merge_group<T, D, NCW>(a, p, s_states, w0, w1 - w0, ps.last_continues ? ps.vl : -1,
                               true, 0);
      else
        merge_group<T, D, NCW>(a, p, s_states, w0, w1 - w0, -1, false, cta);
    }
    w0 = w1;
  }
}

// Merges the pairs whose tiles were split across CTAs (second kernel of a
// call).  CTA (pair p, chunk) owns 16 float4 elements of p's G x D output
// block; each half-warp covers those 16 elements for one group of sources.  Its sources are the CTA partials of CTAs
// vf/NCW .. vl_end/NCW (slots c + p) and, when the pair's last worker
// continues into the next pair, that worker's partial (slot vl + p).  The
// kMergeGroups half-warps take disjoint subsets of the sources (loads of up
// to kMergeBatch sources in flight per lane, a running rescaled state between
// batches); their states meet in shared memory.  With few long sequences a
// pair has up to ~150 sources (one per CTA), so spreading them over 16 groups
// keeps the merge at one or two L2 round trips.
constexpr int kMergeWarps = 8;
constexpr int kMergeThreads = kMergeWarps * 32;
constexpr int kMergeGroups = kMergeWarps * 2;
constexpr int kMergeElems = 16;  // float4 elements per CTA
constexpr int kMergeBatch = 6;

template <typename T, int D, int NCW>
__global__ void __launch_bounds__(kMergeThreads, 4) merge_split_pairs_kernel(const DecodeArgs a) {
  extern __shared__ int s_cum_m[];
  __shared__ float s_st[kMergeGroups][6][kMergeElems];  // per group: M, L, acc.xyzw
  asm volatile("griddepcontrol.launch_dependents;");
  const int p = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == 0) build_prefix(a, s_cum_m, lane);
  __syncthreads();
  // every thread waits for the decode kernel (complete and visible), also the
  // ones with nothing to merge: this grid must not complete before it
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int total = s_cum_m[a.batch] * a.hkv;
  if (total == 0) return;
  const int W = div_up(total, a.num_workers);
  const PairSpan ps = pair_span(a, s_cum_m, W, total, p);
  if (ps.tiles == 0 || ps.vf == ps.vl || ps.vf / NCW == ps.vl / NCW) return;  // not split
  const int vl_end = ps.last_continues ? ps.vl - 1 : ps.vl;
  const int c0 = ps.vf / NCW, n_cta = vl_end / NCW - c0 + 1;
  const int K = n_cta + (ps.last_continues ? 1 : 0);
  const int G = a.group;
  constexpr int D4 = D / 4;
  const int el = lane & (kMergeElems - 1);
  const int grp = warp * 2 + (lane >> 4);  // source group of this half-warp
  const int e = blockIdx.y * kMergeElems + el;
  const bool active = e < G * D4;
  const int hg = active ? e / D4 : 0, d4 = active ? e - (e / D4) * D4 : 0;
  float M = -INFINITY, Lsum = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  // group q: sources q, q + kMergeGroups, ...
  for (int k0 = grp; active && k0 < K; k0 += kMergeGroups * kMergeBatch) {
    float2 ml[kMergeBatch];
    float4 o[kMergeBatch];
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i) {  // issue the whole batch first
      const int k = k0 + i * kMergeGroups;
      ml[i] = make_float2(-INFINITY, 0.f);
      o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < K) {
        const bool cta_src = k < n_cta;
        const int64_t slot = cta_src ? static_cast<int64_t>(c0 + k + p)
                                     : static_cast<int64_t>(ps.vl + p);
        const float* mlp = (cta_src ? a.cta_ml : a.part_ml) + (slot * G + hg) * 2;
        const float* op = (cta_src ? a.cta_o : a.part_o) + (slot * G + hg) * D + d4 * 4;
        ml[i] = __ldcg(reinterpret_cast<const float2*>(mlp));
        o[i] = __ldcg(reinterpret_cast<const float4*>(op));
      }
    }
    float Mb = M;
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i) Mb = fmaxf(Mb, ml[i].x);
    if (Mb == -INFINITY) continue;  // no valid token in any source so far
    const float r = exp2f(M - Mb);   // 0 while M is -inf
    Lsum *= r;
    acc.x *= r;
    acc.y *= r;
    acc.z *= r;
    acc.w *= r;
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i) {
      const float w = exp2f(ml[i].x - Mb);
      Lsum += ml[i].y * w;
      acc.x += w * o[i].x;
      acc.y += w * o[i].y;
      acc.z += w * o[i].z;
      acc.w += w * o[i].w;
    }
    M = Mb;
  }
  s_st[grp][0][el] = M;
  s_st[grp][1][el] = Lsum;
  s_st[grp][2][el] = acc.x;
  s_st[grp][3][el] = acc.y;
  s_st[grp][4][el] = acc.z;
  s_st[grp][5][el] = acc.w;
  __syncthreads();
  if (threadIdx.x >= kMergeElems || !active) return;
  float Mt = -INFINITY;
#pragma unroll
  for (int q = 0; q < kMergeGroups; ++q) Mt = fmaxf(Mt, s_st[q][0][el]);
  const float m_use = Mt == -INFINITY ? 0.f : Mt;
  float L = 0.f, ox = 0.f, oy = 0.f, oz = 0.f, ow = 0.f;
#pragma unroll
  for (int q = 0; q < kMergeGroups; ++q) {
    const float f = exp2f(s_st[q][0][el] - m_use);  // 0 for groups without sources
    L += s_st[q][1][el] * f;
    ox += s_st[q][2][el] * f;
    oy += s_st[q][3][el] * f;
    oz += s_st[q][4][el] * f;
    ow += s_st[q][5][el] * f;
  }
  const int b = p / a.hkv, h = p - (p / a.hkv) * a.hkv;
  const float inv = 1.f / fmaxf(L, 1e-12f);
  store_out<T>(a, b, h * G + hg, d4 * 4 + 0, ox * inv);
  store_out<T>(a, b, h * G + hg, d4 * 4 + 1, oy * inv);
  store_out<T>(a, b, h * G + hg, d4 * 4 + 2, oz * inv);
  store_out<T>(a, b, h * G + hg, d4 * 4 + 3, ow * inv);
  if (d4 == 0 && a.lse != nullptr)
    a.lse[static_cast<int64_t>(b) * a.hq + h * G + hg] =
        (Mt == -INFINITY || L <= 0.f) ? -INFINITY : Mt * kLn2 + logf(L);
}

// ----------------------------------------------------------------- host side --
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

template <typename T, int D, int NT>
int launch(const DecodeArgs& a, const void* pool, int64_t pool_rows, int grid,
           cudaStream_t stream) {
  using L = Layout<D>;
  static unsigned long long configured = 0;  // one bit per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return HELM_ERR_CUDA;
  if (dev >= 64) return HELM_ERR_UNSUPPORTED;
  if (!(configured & (1ull << dev))) {
    if (cudaFuncSetAttribute(paged_decode_kernel<T, D, NT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(L::smem_bytes(kMaxBatch))) != cudaSuccess)
      return HELM_ERR_CUDA;
    configured |= 1ull << dev;
  }
  EncodeTiledFn encode = get_encode_fn();
  if (encode == nullptr) return HELM_ERR_CUDA;
  CUtensorMap map;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(pool_rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(D) * 2};
  cuuint32_t box[2] = {64, kTileRows};
  cuuint32_t estride[2] = {1, 1};
  const CUtensorMapDataType dt = std::is_same<T, __nv_bfloat16>::value
                                     ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (encode(&map, dt, 2, const_cast<void*>(pool), dims, strides, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return HELM_ERR_CUDA;
  DecodeArgs args = a;
  args.num_workers = grid * L::NCW;
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(L::kThreads);
    cfg.dynamicSmemBytes = L::smem_bytes(a.batch);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = decode_overlap_enabled() ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, paged_decode_kernel<T, D, NT>, map, args) != cudaSuccess)
      return HELM_ERR_CUDA;
  }
  // merge of split pairs: a programmatic dependent of the decode kernel
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.batch * a.hkv),
                     static_cast<unsigned>((a.group * (D / 4) + kMergeElems - 1) / kMergeElems));
  cfg.blockDim = dim3(kMergeThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(a.batch + 1) * sizeof(int);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, merge_split_pairs_kernel<T, D, L::NCW>, args) != cudaSuccess)
    return HELM_ERR_CUDA;
  return HELM_OK;
}

template <typename T, int D>
int dispatch_nt(const DecodeArgs& a, const void* pool, int64_t rows, int grid, cudaStream_t s) {
  if (a.group <= 8) return launch<T, D, 1>(a, pool, rows, grid, s);
  return launch<T, D, 2>(a, pool, rows, grid, s);
}

template <typename T>
int dispatch_d(int head_dim, const DecodeArgs& a, const void* pool, int64_t rows, int grid,
               cudaStream_t s) {
  switch (head_dim) {
    case 64:
      return dispatch_nt<T, 64>(a, pool, rows, grid, s);
    case 128:
      return dispatch_nt<T, 128>(a, pool, rows, grid, s);
    case 256:
      return dispatch_nt<T, 256>(a, pool, rows, grid, s);
    default:
      return HELM_ERR_UNSUPPORTED;
  }
}

}  // namespace

int64_t paged_decode_slots(int batch, int num_kv_heads) {
  return static_cast<int64_t>(num_sms_current_device()) * kMaxNCW +
         static_cast<int64_t>(batch) * num_kv_heads;
}

// Workspace: reserved [B*Hkv] int32 | partial O [slots][G][D] fp32 |
// partial (m, l) [slots][G][2] fp32, each region 256-byte aligned.  The
// reserved region (the first roundup(4*B*Hkv, 256) bytes) is neither read
// nor written.
struct WorkspaceLayout {
  int64_t cnt_bytes, o_bytes, ml_bytes, cta_o_bytes, cta_ml_bytes;
  WorkspaceLayout(int batch, int hq, int hkv, int d) {
    auto up = [](int64_t x) { return ((x + 255) / 256) * 256; };
    const int64_t group = hq / hkv;
    const int64_t pairs = static_cast<int64_t>(batch) * hkv;
    const int64_t slots = paged_decode_slots(batch, hkv);            // warp partials
    const int64_t cta_slots = num_sms_current_device() + pairs;      // CTA partials
    cnt_bytes = up(pairs * 4);
    o_bytes = up(slots * group * d * 4);
    ml_bytes = up(slots * group * 2 * 4);
    cta_o_bytes = up(cta_slots * group * d * 4);
    cta_ml_bytes = up(cta_slots * group * 2 * 4);
  }
  int64_t total() const { return cnt_bytes + o_bytes + ml_bytes + cta_o_bytes + cta_ml_bytes; }
};

}  // namespace helm

using helm::DecodeArgs;

extern "C" int64_t helm_paged_decode_workspace_bytes(int batch, int num_q_heads,
                                                     int num_kv_heads, int head_dim) {
  if (batch <= 0 || num_kv_heads <= 0 || num_q_heads <= 0 || head_dim <= 0) return 0;
  return helm::WorkspaceLayout(batch, num_q_heads, num_kv_heads, head_dim).total();
}

extern "C" int helm_paged_decode_attention(
    const void* q, int64_t q_stride_b, int64_t q_stride_h, const void* kv_pool, int64_t pool_pages,
    const int32_t* page_table, int64_t pt_stride_b, int max_pages, const int32_t* kv_lens,
    const int32_t* num_pages, const int32_t* page_used, const int32_t* page_start,
    const void* mask, int mask_dtype, int64_t mask_stride_b, void* out, int64_t out_stride_b,
    int64_t out_stride_h, float* lse, void* workspace, int64_t workspace_bytes, int batch,
    int num_q_heads, int num_kv_heads, int head_dim, int page_size, int dtype, int out_dtype,
    float scale, float softcap, int max_kv_len_hint, void* stream) {
  using namespace helm;
  if (q == nullptr || kv_pool == nullptr || page_table == nullptr || kv_lens == nullptr ||
      out == nullptr || workspace == nullptr)
    return HELM_ERR_INVALID_ARGUMENT;
  if (batch <= 0 || num_q_heads <= 0 || num_kv_heads <= 0 || page_size <= 0 || max_pages < 0 ||
      pool_pages <= 0)
    return HELM_ERR_INVALID_ARGUMENT;
  if (num_q_heads % num_kv_heads != 0) return HELM_ERR_INVALID_ARGUMENT;
  const int group = num_q_heads / num_kv_heads;
  if (group > 16) return HELM_ERR_UNSUPPORTED;
  if (batch > kMaxBatch) return HELM_ERR_UNSUPPORTED;
  if (dtype != HELM_DTYPE_BF16 && dtype != HELM_DTYPE_FP16) return HELM_ERR_UNSUPPORTED;
  if (out_dtype != dtype && out_dtype != HELM_DTYPE_FP32) return HELM_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return HELM_ERR_UNSUPPORTED;
  const bool ragged = num_pages != nullptr;
  if (ragged != (page_used != nullptr) || ragged != (page_start != nullptr))
    return HELM_ERR_INVALID_ARGUMENT;
  if (mask != nullptr && mask_dtype != HELM_DTYPE_FP32 && mask_dtype != HELM_DTYPE_BF16 &&
      mask_dtype != HELM_DTYPE_FP16)
    return HELM_ERR_INVALID_ARGUMENT;
  // q rows are read as 32-bit words, the pool through TMA (16-byte rule).
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (q_stride_b & 1) || (q_stride_h & 1))
    return HELM_ERR_ALIGNMENT;
  if ((reinterpret_cast<uintptr_t>(kv_pool) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return HELM_ERR_ALIGNMENT;
  const int64_t pool_rows = pool_pages * 2 * num_kv_heads * static_cast<int64_t>(page_size);
  if (pool_rows >= (int64_t(1) << 31)) return HELM_ERR_UNSUPPORTED;
  if (workspace_bytes <
      helm_paged_decode_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim))
    return HELM_ERR_WORKSPACE;

  const WorkspaceLayout ws(batch, num_q_heads, num_kv_heads, head_dim);
  DecodeArgs a;
  a.q = q;
  a.q_sb = q_stride_b;
  a.q_sh = q_stride_h;
  a.pool_pages = pool_pages;
  a.page_table = page_table;
  a.pt_sb = pt_stride_b;
  a.max_pages = max_pages;
  a.kv_lens = kv_lens;
  a.num_pages = num_pages;
  a.page_used = page_used;
  a.page_start = page_start;
  a.mask = mask;
  a.mask_dtype = mask_dtype;
  a.mask_sb = mask_stride_b;
  a.out = out;
  a.out_sb = out_stride_b;
  a.out_sh = out_stride_h;
  a.lse = lse;
  uint8_t* wsp = static_cast<uint8_t*>(workspace);
  a.part_o = reinterpret_cast<float*>(wsp + ws.cnt_bytes);
  a.part_ml = reinterpret_cast<float*>(wsp + ws.cnt_bytes + ws.o_bytes);
  a.cta_o = reinterpret_cast<float*>(wsp + ws.cnt_bytes + ws.o_bytes + ws.ml_bytes);
  a.cta_ml =
      reinterpret_cast<float*>(wsp + ws.cnt_bytes + ws.o_bytes + ws.ml_bytes + ws.cta_o_bytes);
  a.batch = batch;
  a.hq = num_q_heads;
  a.hkv = num_kv_heads;
  a.group = group;
  a.page_size = page_size;
  a.tiles_per_page = (page_size + kTileRows - 1) / kTileRows;
  a.out_fp32 = out_dtype == HELM_DTYPE_FP32 ? 1 : 0;
  a.scale = scale;
  a.scale_log2 = scale * kLog2e;
  a.softcap = softcap;

  const int sms = num_sms_current_device();
  int grid = sms;
  if (max_kv_len_hint > 0) {
    const int64_t pages = (static_cast<int64_t>(max_kv_len_hint) + page_size - 1) / page_size;
    const int64_t tiles = pages * a.tiles_per_page * batch * num_kv_heads;
    const int ncw = head_dim <= 128 ? 8 : 4;
    const int64_t want = (tiles + ncw * kMinTilesPerWorker - 1) / (ncw * kMinTilesPerWorker);
    grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(sms, want)));
  }
  a.num_workers = 0;  // set by launch() from the CTA shape of the head_dim
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = dtype == HELM_DTYPE_BF16
               ? dispatch_d<__nv_bfloat16>(head_dim, a, kv_pool, pool_rows, grid, s)
               : dispatch_d<__half>(head_dim, a, kv_pool, pool_rows, grid, s);
  if (rc == HELM_ERR_CUDA) set_last_cuda_error(cudaGetLastError());
  return rc;
}
