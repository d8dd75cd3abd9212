/*
 * ORACLE — test infrastructure only; never part of the product path.
 *
 * Plain-C restatement of HELM's paged streaming decode attention, used by the
 * tests as the CPU checker of the CUDA kernels and by bench.py as the timed
 * CPU baseline ("port" of the reference algorithm).
 *
 * It follows helm/runtime/kv_cache.py perform_streaming_attention, masked /
 * softcapped branch (kv_cache.py:468-555), which is also the exact math of the
 * unmasked branches (single softmax over the concatenated pages):
 *   - pages with used_tokens == 0 are skipped                (kv_cache.py:439)
 *   - no active page: output zeros                           (kv_cache.py:441-442)
 *   - GQA: query head h reads KV head h / (Hq/Hkv)           (kv_cache.py:459-466)
 *   - per page: scores = (q . k) * scale; softcap tanh(s/c)*c; + mask[token]
 *     block_max, new_max = max(running_max, block_max),
 *     old_scale = exp(running_max - new_max) (NaN -> 0),
 *     out = out*old_scale + sum_t exp(s_t - new_max) v_t,
 *     running_sum = running_sum*old_scale + sum_t exp(s_t - new_max)
 *                                                           (kv_cache.py:519-530)
 *   - out / max(running_sum, 1e-12)                          (kv_cache.py:554)
 * LSE is not produced by the reference; it is restated as
 * running_max + log(running_sum), the logsumexp of the same scores.
 * All arithmetic is fp32, as in the reference (q.float(), page.float()).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_F32 0
#define ORACLE_F16 1
#define ORACLE_BF16 2

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while (!(man & 0x400));
      man &= 0x3ff;
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (man << 13);
  } else {
    u = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static void load_row(const void* base, int dtype, int64_t off, int d, float* dst) {
  if (dtype == ORACLE_F32) {
    memcpy(dst, (const float*)base + off, sizeof(float) * d);
  } else if (dtype == ORACLE_BF16) {
    const uint16_t* p = (const uint16_t*)base + off;
    for (int i = 0; i < d; ++i) dst[i] = bf16_to_f32(p[i]);
  } else {
    const uint16_t* p = (const uint16_t*)base + off;
    for (int i = 0; i < d; ++i) dst[i] = f16_to_f32(p[i]);
  }
}

typedef struct {
  const float* q;       /* [B, Hq, D] fp32 */
  int B, Hq, Hkv, D, P;
  const void* pool;     /* [slots, 2, Hkv, P, D] */
  int dtype;
  const int32_t* page_table; /* [B, pt_stride] */
  int64_t pt_stride;
  const int32_t* num_pages;  /* [B] */
  const int32_t* page_used;  /* [B, pt_stride] */
  const float* mask;         /* [B, mask_stride] or NULL */
  int64_t mask_stride;
  float scale, softcap;
  float* out;  /* [B, Hq, D] */
  float* lse;  /* [B, Hq] or NULL */
  int next_row; /* work counter (rows = B*Hq) */
  pthread_mutex_t lock;
} Job;

static void one_row(const Job* j, int row, float* kbuf, float* vbuf, float* acc, float* sc) {
  const int b = row / j->Hq, h = row % j->Hq;
  const int group = j->Hq / j->Hkv;
  const int kvh = h / group;
  const int D = j->D, P = j->P;
  const float* q = j->q + (int64_t)row * D;
  float* out = j->out + (int64_t)row * D;
  float running_max = -INFINITY, running_sum = 0.f;
  int any = 0, cursor = 0;
  for (int d = 0; d < D; ++d) acc[d] = 0.f;
  for (int pg = 0; pg < j->num_pages[b]; ++pg) {
    const int used = j->page_used[(int64_t)b * j->pt_stride + pg];
    if (used <= 0) continue;
    any = 1;
    const int64_t slot = j->page_table[(int64_t)b * j->pt_stride + pg];
    const int64_t head_elems = (int64_t)P * D;
    const int64_t kbase = (slot * 2 * j->Hkv + kvh) * head_elems;
    const int64_t vbase = kbase + (int64_t)j->Hkv * head_elems;
    float block_max = -INFINITY;
    for (int t = 0; t < used; ++t) {
      load_row(j->pool, j->dtype, kbase + (int64_t)t * D, D, kbuf);
      float s = 0.f;
      for (int d = 0; d < D; ++d) s += q[d] * kbuf[d];
      s *= j->scale;
      if (j->softcap > 0.f) s = tanhf(s / j->softcap) * j->softcap;
      if (j->mask) s += j->mask[(int64_t)b * j->mask_stride + cursor + t];
      sc[t] = s;
      if (s > block_max) block_max = s;
    }
    const float new_max = running_max > block_max ? running_max : block_max;
    float old_scale = expf(running_max - new_max);
    if (isnan(old_scale)) old_scale = 0.f;
    float block_sum = 0.f;
    for (int d = 0; d < D; ++d) acc[d] *= old_scale;
    for (int t = 0; t < used; ++t) {
      const float e = expf(sc[t] - new_max);
      block_sum += e;
      load_row(j->pool, j->dtype, vbase + (int64_t)t * D, D, vbuf);
      for (int d = 0; d < D; ++d) acc[d] += e * vbuf[d];
    }
    running_sum = running_sum * old_scale + block_sum;
    running_max = new_max;
    cursor += used;
  }
  if (!any) {
    for (int d = 0; d < D; ++d) out[d] = 0.f;
    if (j->lse) j->lse[row] = -INFINITY;
    return;
  }
  const float denom = running_sum > 1e-12f ? running_sum : 1e-12f;
  for (int d = 0; d < D; ++d) out[d] = acc[d] / denom;
  if (j->lse) j->lse[row] = running_max + logf(running_sum);
}

static void* worker(void* arg) {
  Job* j = (Job*)arg;
  const int max_used = j->P;
  float* kbuf = (float*)malloc(sizeof(float) * j->D);
  float* vbuf = (float*)malloc(sizeof(float) * j->D);
  float* acc = (float*)malloc(sizeof(float) * j->D);
  float* sc = (float*)malloc(sizeof(float) * (max_used > 0 ? max_used : 1));
  const int rows = j->B * j->Hq;
  for (;;) {
    pthread_mutex_lock(&j->lock);
    const int row = j->next_row++;
    pthread_mutex_unlock(&j->lock);
    if (row >= rows) break;
    one_row(j, row, kbuf, vbuf, acc, sc);
  }
  free(kbuf);
  free(vbuf);
  free(acc);
  free(sc);
  return NULL;
}

/* Returns 0 on success.  page_used[b, i] must be <= P for every listed page. */
int oracle_paged_attention(const float* q, int B, int Hq, int Hkv, int D, const void* pool,
                           int dtype, int P, const int32_t* page_table, int64_t pt_stride,
                           const int32_t* num_pages, const int32_t* page_used, const float* mask,
                           int64_t mask_stride, float scale, float softcap, float* out, float* lse,
                           int threads) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || P <= 0 || Hq % Hkv) return 1;
  Job j;
  j.q = q;
  j.B = B;
  j.Hq = Hq;
  j.Hkv = Hkv;
  j.D = D;
  j.P = P;
  j.pool = pool;
  j.dtype = dtype;
  j.page_table = page_table;
  j.pt_stride = pt_stride;
  j.num_pages = num_pages;
  j.page_used = page_used;
  j.mask = mask;
  j.mask_stride = mask_stride;
  j.scale = scale;
  j.softcap = softcap;
  j.out = out;
  j.lse = lse;
  j.next_row = 0;
  pthread_mutex_init(&j.lock, NULL);
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  for (int i = 1; i < threads; ++i) pthread_create(&tid[i], NULL, worker, &j);
  worker(&j);
  for (int i = 1; i < threads; ++i) pthread_join(tid[i], NULL);
  pthread_mutex_destroy(&j.lock);
  return 0;
}
