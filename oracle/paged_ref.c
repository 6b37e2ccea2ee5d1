/*
 * CPU restatement of the reference PagedAttention forward (C, pthreads).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for large parity cases and the timed CPU baseline of
 * bench.py.  Nothing in the product links or calls it.
 *
 * Follows the same algorithm as oracle/paged_ref.py (float caches, no RoPE / norm / integer
 * codec): reference operator rust/src/ops/attention.rs:3857-4382 and its numpy oracle
 * tests/ops/test_paged_attention.py:63-158.
 *   1. KV append in token order (attention.rs:4064-4120): slot = slot_mapping[t] or
 *      block_table[b, (past+j)/bs]*bs + (past+j)%bs; slot < 0 skips; later tokens win.
 *   2. Per (sequence, kv head), every query row i and q head of the group: keys [0, past) from
 *      the updated cache through the block table, keys [past, total) from the new rows;
 *      scores = scale * q.k in fp32, optional softcap, causal / left-window masks, softmax
 *      with an optional sink in the denominator, output = softmax . V rounded to T.
 * Conversions: bf16 by bit shift / round-to-nearest-even; fp16 through the compiler's IEEE
 * _Float16 type.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define DT_F16 10
#define DT_BF16 16

static inline float bf16_to_f(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint16_t f_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
static inline float f16_to_f(uint16_t h) {
  _Float16 x;
  memcpy(&x, &h, 2);
  return (float)x;
}
static inline uint16_t f_to_f16(float f) {
  _Float16 x = (_Float16)f;
  uint16_t h;
  memcpy(&h, &x, 2);
  return h;
}
static inline float ld(const uint16_t* p, int64_t i, int dt) { return dt == DT_BF16 ? bf16_to_f(p[i]) : f16_to_f(p[i]); }
static inline uint16_t st(float x, int dt) { return dt == DT_BF16 ? f_to_bf16(x) : f_to_f16(x); }

typedef struct Job {
  int dtype, H, KV, D, B, bs, maxb, causal, window, seq_begin, seq_end;
  const uint16_t *q, *k, *v, *kc, *vc;
  const int32_t *cum, *past, *bt;
  float scale, softcap;
  const float* sink;
  uint16_t* out;
  int next; /* next (sequence, kv head) work item, taken with __atomic_fetch_add */
} Job;

static void* worker(void* arg) {
  Job* J = (Job*)arg;
  const int dtype = J->dtype, H = J->H, KV = J->KV, D = J->D, bs = J->bs, maxb = J->maxb;
  const int g = H / KV;
  const int64_t row = (int64_t)KV * D;
  const uint16_t *q = J->q, *k = J->k, *v = J->v, *kc = J->kc, *vc = J->vc;
  const int32_t *cum = J->cum, *past = J->past, *bt = J->bt;
  const float scale = J->scale, softcap = J->softcap;
  const float* sink = J->sink;
  const int causal = J->causal, window = J->window;
  uint16_t* out = J->out;
  const int items = (J->seq_end - J->seq_begin) * KV;
  int64_t cap = 0;
  float* scores = NULL;
  float* acc = (float*)malloc(sizeof(float) * D);
  float* qf = (float*)malloc(sizeof(float) * D);
  for (;;) {
    int item = __atomic_fetch_add(&J->next, 1, __ATOMIC_RELAXED);
    if (item >= items) break;
    const int b = J->seq_begin + item / KV, kh = item % KV;
    const int c0 = cum[b], nq = cum[b + 1] - cum[b], pb = past[b];
    const int total = pb + nq;
    if (nq <= 0) continue;
    if (total > cap) {
      free(scores);
      cap = total;
      scores = (float*)malloc(sizeof(float) * cap);
    }
    for (int i = 0; i < nq; ++i) {
      const int lo = window > 0 ? (pb + i - window + 1 > 0 ? pb + i - window + 1 : 0) : 0;
      const int hi = causal ? pb + i + 1 : total;
      for (int hl = 0; hl < g; ++hl) {
        const int h = kh * g + hl;
        for (int d = 0; d < D; ++d) qf[d] = ld(q, (int64_t)(c0 + i) * H * D + (int64_t)h * D + d, dtype);
        float mx = -INFINITY;
        for (int c = lo; c < hi; ++c) {
          const uint16_t* krow;
          if (c < pb) {
            int64_t slot = (int64_t)bt[(int64_t)b * maxb + c / bs] * bs + c % bs;
            krow = kc + slot * row + (int64_t)kh * D;
          } else {
            krow = k + (int64_t)(c0 + c - pb) * row + (int64_t)kh * D;
          }
          float s = 0.f;
          for (int d = 0; d < D; ++d) s += qf[d] * ld(krow, d, dtype);
          s *= scale;
          if (softcap > 0.f) s = softcap * tanhf(s / softcap);
          scores[c] = s;
          if (s > mx) mx = s;
        }
        float m2 = mx;
        if (sink && sink[h] > m2) m2 = sink[h];
        float denom = sink ? expf(sink[h] - m2) : 0.f;
        for (int c = lo; c < hi; ++c) {
          scores[c] = expf(scores[c] - m2);
          denom += scores[c];
        }
        for (int d = 0; d < D; ++d) acc[d] = 0.f;
        for (int c = lo; c < hi; ++c) {
          const uint16_t* vrow;
          if (c < pb) {
            int64_t slot = (int64_t)bt[(int64_t)b * maxb + c / bs] * bs + c % bs;
            vrow = vc + slot * row + (int64_t)kh * D;
          } else {
            vrow = v + (int64_t)(c0 + c - pb) * row + (int64_t)kh * D;
          }
          const float p = scores[c];
          for (int d = 0; d < D; ++d) acc[d] += p * ld(vrow, d, dtype);
        }
        for (int d = 0; d < D; ++d)
          out[(int64_t)(c0 + i) * H * D + (int64_t)h * D + d] = st(acc[d] / denom, dtype);
      }
    }
  }
  free(scores);
  free(acc);
  free(qf);
  return NULL;
}

int oracle_paged_attention(int dtype, int H, int KV, int D, int nt, int B, int NB, int bs, int maxb,
                           const void* qv, const void* kv_, const void* vv, void* kcv, void* vcv,
                           const int32_t* cum, const int32_t* past, const int32_t* bt, const int32_t* slots,
                           float scale, int causal, int window, float softcap, const float* sink,
                           void* outv, int threads, int do_append, int seq_begin, int seq_end) {
  const uint16_t* q = (const uint16_t*)qv;
  const uint16_t* k = (const uint16_t*)kv_;
  const uint16_t* v = (const uint16_t*)vv;
  uint16_t* kc = (uint16_t*)kcv;
  uint16_t* vc = (uint16_t*)vcv;
  uint16_t* out = (uint16_t*)outv;
  const int64_t row = (int64_t)KV * D;
  if (seq_end <= 0 || seq_end > B) seq_end = B;
  if (scale == 0.f) scale = 1.0f / sqrtf((float)D);

  if (do_append) {
    for (int b = 0; b < B; ++b) {
      for (int t = cum[b]; t < cum[b + 1]; ++t) {
        int64_t slot;
        if (slots) {
          slot = slots[t];
        } else {
          int64_t logical = (int64_t)past[b] + (t - cum[b]);
          slot = (int64_t)bt[(int64_t)b * maxb + logical / bs] * bs + logical % bs;
        }
        if (slot < 0 || slot >= (int64_t)NB * bs) continue;
        memcpy(kc + slot * row, k + (int64_t)t * row, sizeof(uint16_t) * row);
        memcpy(vc + slot * row, v + (int64_t)t * row, sizeof(uint16_t) * row);
      }
    }
  }

  Job job = {dtype, H, KV, D, B, bs, maxb, causal, window, seq_begin, seq_end, q, k, v, kc, vc,
             cum, past, bt, scale, softcap, sink, out, 0};
  if (threads < 1) threads = 1;
  pthread_t* tids = (pthread_t*)malloc(sizeof(pthread_t) * threads);
  int started = 0;
  for (int i = 1; i < threads; ++i)
    if (pthread_create(&tids[i], NULL, worker, &job) == 0) ++started; else break;
  worker(&job);
  for (int i = 1; i <= started; ++i) pthread_join(tids[i], NULL);
  free(tids);
  return 0;
}
