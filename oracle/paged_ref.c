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
 *      with an optional sink in the denominator, output = softmax . V rounded to T (or kept
 *      in fp32 when the caller asks for the unrounded output, for tolerance checks).
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

/* Row kernels over d channels (d % 8 == 0 takes the 8-lane form, which the compiler maps onto
 * SIMD registers: eight independent fp32 partial sums, combined pairwise at the end).  The sum
 * order differs from a sequential loop only by fp32 rounding, well inside the parity
 * tolerances this checker is used with. */
typedef uint16_t v8u16 __attribute__((vector_size(16)));
typedef uint32_t v8u32 __attribute__((vector_size(32)));
typedef _Float16 v8h __attribute__((vector_size(16)));
typedef float v8f __attribute__((vector_size(32)));

/* One row of d 16-bit values to fp32: bf16 is the high half of an fp32, fp16 widens exactly. */
static inline void row_to_f32(float* restrict dst, const uint16_t* restrict src, int D, int dt) {
  int d = 0;
  if (dt == DT_BF16) {
    for (; d + 8 <= D; d += 8) {
      v8u16 x;
      memcpy(&x, src + d, sizeof(x));
      v8u32 y = __builtin_convertvector(x, v8u32) << 16;
      memcpy(dst + d, &y, sizeof(y));
    }
    for (; d < D; ++d) dst[d] = bf16_to_f(src[d]);
  } else {
    for (; d + 8 <= D; d += 8) {
      v8h x;
      memcpy(&x, src + d, sizeof(x));
      v8f y = __builtin_convertvector(x, v8f);
      memcpy(dst + d, &y, sizeof(y));
    }
    for (; d < D; ++d) dst[d] = f16_to_f(src[d]);
  }
}

/* Four 8-lane fp32 vectors (GCC / Clang vector extension) hold 32 independent partial sums of
 * a dot product. */

static inline v8f v8_load(const float* p) {
  v8f x;
  memcpy(&x, p, sizeof(x));
  return x;
}

static inline float dot8(const float* restrict a, const float* restrict b, int D) {
  if (D % 32) {
    float s = 0.f;
    for (int d = 0; d < D; ++d) s += a[d] * b[d];
    return s;
  }
  v8f s0 = {0}, s1 = {0}, s2 = {0}, s3 = {0};
  for (int d = 0; d < D; d += 32) {
    s0 += v8_load(a + d) * v8_load(b + d);
    s1 += v8_load(a + d + 8) * v8_load(b + d + 8);
    s2 += v8_load(a + d + 16) * v8_load(b + d + 16);
    s3 += v8_load(a + d + 24) * v8_load(b + d + 24);
  }
  v8f t = (s0 + s1) + (s2 + s3);
  return ((t[0] + t[4]) + (t[1] + t[5])) + ((t[2] + t[6]) + (t[3] + t[7]));
}

typedef struct Job {
  int dtype, H, KV, D, B, bs, maxb, causal, window, seq_begin, seq_end;
  const uint16_t *q, *k, *v, *kc, *vc;
  const int32_t *cum, *past, *bt;
  float scale, softcap;
  const float* sink;
  uint16_t* out;
  float* out_f32; /* when set, the fp32 output before rounding to T goes here instead */
  /* fp8 e4m3 caches (kc / vc then hold one byte per element): per-(block, kv head) scales
   * [NB, KV]; every position, the new rows' included, is read back from the cache */
  const float *k_scale8, *v_scale8;
  int next; /* next (sequence, kv head) work item, taken with __atomic_fetch_add */
} Job;

/* Keys (or values) [t0, t1) of one (sequence, kv head) converted to fp32 rows of `tile`:
 * positions below `past` through the block table from the cache, the others from the
 * sequence's new rows (which start at token c0). */
#define KT 64
/* e4m3fn (1 sign, 4 exponent bits with bias 7, 3 mantissa bits, no infinities, S.1111.111 is
 * NaN): value of every code, from the format's definition. */
static float g_e4m3[256];
static void e4m3_table(void) {
  for (int c = 0; c < 256; ++c) {
    const int e = (c >> 3) & 15, m = c & 7;
    float v = e == 0 ? ldexpf((float)m, -9) : ldexpf(1.0f + m / 8.0f, e - 7);
    if (e == 15 && m == 7) v = NAN;
    g_e4m3[c] = (c & 0x80) ? -v : v;
  }
}

/* fp32 -> e4m3fn, round to nearest even, saturating at +-448 (the largest finite code). */
static uint8_t f32_to_e4m3(float x) {
  if (isnan(x)) return 0x7f;
  const uint8_t sign = signbit(x) ? 0x80 : 0;
  float a = fabsf(x);
  if (a > 448.f) a = 448.f;
  int k;
  const float f = frexpf(a, &k); /* a = f * 2^k, f in [0.5, 1) */
  int e = k - 1;                 /* a = (2f) * 2^e, 2f in [1, 2) */
  if (a == 0.f) return sign;
  if (e < -6) { /* subnormal: m * 2^-9 */
    const int m = (int)rintf(ldexpf(a, 9));
    return sign | (uint8_t)(m >= 8 ? 0x08 : m);
  }
  int m = (int)rintf((2.f * f - 1.f) * 8.f);
  if (m == 8) {
    m = 0;
    ++e;
  }
  return sign | (uint8_t)(((e + 7) << 3) | m);
}

static inline void load_tile_fp8(float* tile, const uint8_t* cache, const float* scales, const int32_t* bt_row,
                                 int t0, int t1, int bs, int64_t row, int kh, int KV, int D) {
  for (int c = t0; c < t1; ++c) {
    const int64_t blk = bt_row[c / bs];
    const uint8_t* src = cache + (blk * bs + c % bs) * row + (int64_t)kh * D;
    const float sc = scales[blk * KV + kh];
    float* dst = tile + (int64_t)(c - t0) * D;
    for (int d = 0; d < D; ++d) dst[d] = g_e4m3[src[d]] * sc;
  }
}

static inline void load_tile(float* tile, const uint16_t* cache, const uint16_t* fresh, const int32_t* bt_row,
                             int t0, int t1, int pb, int c0, int bs, int64_t row, int kh, int D, int dtype) {
  for (int c = t0; c < t1; ++c) {
    const uint16_t* src = c < pb ? cache + ((int64_t)bt_row[c / bs] * bs + c % bs) * row + (int64_t)kh * D
                                 : fresh + (int64_t)(c0 + c - pb) * row + (int64_t)kh * D;
    row_to_f32(tile + (int64_t)(c - t0) * D, src, D, dtype);
  }
}

/* Query rows of one (sequence, kv head) are processed in blocks of ROWS (row r = query i, head
 * hl of the group, r = i * g + hl), so each key / value row is converted to fp32 once per block
 * per block, in tiles of KT keys, and used by every row of the block while the tile sits in
 * L1. */
#define ROWS 32

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
  float* out_f32 = J->out_f32;
  const int items = (J->seq_end - J->seq_begin) * KV;
  int64_t cap = 0;
  float* scores = NULL; /* [ROWS][cap] */
  float* qf = (float*)malloc(sizeof(float) * ROWS * D);
  float* acc = (float*)malloc(sizeof(float) * ROWS * D);
  float* tile = (float*)malloc(sizeof(float) * KT * D);
  int lo[ROWS], hi[ROWS];
  float mx[ROWS], denom[ROWS];
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
      scores = (float*)malloc(sizeof(float) * ROWS * cap);
    }
    const int nrows = nq * g;
    for (int r0 = 0; r0 < nrows; r0 += ROWS) {
      const int nr = nrows - r0 < ROWS ? nrows - r0 : ROWS;
      int cmin = total, cmax = 0;
      for (int r = 0; r < nr; ++r) {
        const int i = (r0 + r) / g, h = kh * g + (r0 + r) % g;
        lo[r] = window > 0 ? (pb + i - window + 1 > 0 ? pb + i - window + 1 : 0) : 0;
        hi[r] = causal ? pb + i + 1 : total;
        if (lo[r] < cmin) cmin = lo[r];
        if (hi[r] > cmax) cmax = hi[r];
        mx[r] = -INFINITY;
        row_to_f32(qf + (int64_t)r * D, q + (int64_t)(c0 + i) * H * D + (int64_t)h * D, D, dtype);
      }
      /* scores, a tile of KT keys at a time: keys [0, past) through the block table from the
       * cache, [past, total) from the sequence's new rows */
      for (int t0 = cmin; t0 < cmax; t0 += KT) {
        const int t1 = t0 + KT < cmax ? t0 + KT : cmax;
        if (J->k_scale8)
          load_tile_fp8(tile, (const uint8_t*)kc, J->k_scale8, bt + (int64_t)b * maxb, t0, t1, bs, row, kh, KV, D);
        else
          load_tile(tile, kc, k, bt + (int64_t)b * maxb, t0, t1, pb, c0, bs, row, kh, D, dtype);
        for (int r = 0; r < nr; ++r) {
          const int a0 = lo[r] > t0 ? lo[r] : t0, a1 = hi[r] < t1 ? hi[r] : t1;
          const float* qr = qf + (int64_t)r * D;
          float* sr = scores + (int64_t)r * cap;
          for (int c = a0; c < a1; ++c) {
            float sc = dot8(qr, tile + (int64_t)(c - t0) * D, D) * scale;
            if (softcap > 0.f) sc = softcap * tanhf(sc / softcap);
            sr[c] = sc;
            if (sc > mx[r]) mx[r] = sc;
          }
        }
      }
      for (int r = 0; r < nr; ++r) {
        const int h = kh * g + (r0 + r) % g;
        float m2 = mx[r];
        if (sink && sink[h] > m2) m2 = sink[h];
        float den = sink ? expf(sink[h] - m2) : 0.f;
        float* sr = scores + (int64_t)r * cap;
        for (int c = lo[r]; c < hi[r]; ++c) {
          sr[c] = expf(sr[c] - m2);
          den += sr[c];
        }
        denom[r] = den;
        for (int d = 0; d < D; ++d) acc[(int64_t)r * D + d] = 0.f;
      }
      for (int t0 = cmin; t0 < cmax; t0 += KT) {
        const int t1 = t0 + KT < cmax ? t0 + KT : cmax;
        if (J->v_scale8)
          load_tile_fp8(tile, (const uint8_t*)vc, J->v_scale8, bt + (int64_t)b * maxb, t0, t1, bs, row, kh, KV, D);
        else
          load_tile(tile, vc, v, bt + (int64_t)b * maxb, t0, t1, pb, c0, bs, row, kh, D, dtype);
        for (int r = 0; r < nr; ++r) {
          const int a0 = lo[r] > t0 ? lo[r] : t0, a1 = hi[r] < t1 ? hi[r] : t1;
          const float* sr = scores + (int64_t)r * cap;
          float* ar = acc + (int64_t)r * D;
          for (int c = a0; c < a1; ++c) {
            const float p = sr[c];
            const float* vr = tile + (int64_t)(c - t0) * D;
            for (int d = 0; d < D; ++d) ar[d] += p * vr[d];
          }
        }
      }
      for (int r = 0; r < nr; ++r) {
        const int i = (r0 + r) / g, h = kh * g + (r0 + r) % g;
        const int64_t o = (int64_t)(c0 + i) * H * D + (int64_t)h * D;
        const float* ar = acc + (int64_t)r * D;
        if (out_f32) {
          for (int d = 0; d < D; ++d) out_f32[o + d] = ar[d] / denom[r];
        } else {
          for (int d = 0; d < D; ++d) out[o + d] = st(ar[d] / denom[r], dtype);
        }
      }
    }
  }
  free(scores);
  free(qf);
  free(acc);
  free(tile);
  return NULL;
}

static int run(int dtype, int H, int KV, int D, int nt, int B, int NB, int bs, int maxb, const void* qv,
               const void* kv_, const void* vv, void* kcv, void* vcv, const int32_t* cum, const int32_t* past,
               const int32_t* bt, const int32_t* slots, float scale, int causal, int window, float softcap,
               const float* sink, void* outv, int threads, int do_append, int seq_begin, int seq_end,
               float* out_f32, const float* k_scale8, const float* v_scale8) {
  const uint16_t* q = (const uint16_t*)qv;
  const uint16_t* k = (const uint16_t*)kv_;
  const uint16_t* v = (const uint16_t*)vv;
  const int64_t row = (int64_t)KV * D;
  const int fp8 = k_scale8 != NULL;
  if (seq_end <= 0 || seq_end > B) seq_end = B;
  if (scale == 0.f) scale = 1.0f / sqrtf((float)D);
  if (fp8) e4m3_table();

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
        if (fp8) { /* encode with the slot's block scale */
          const int64_t blk = slot / bs;
          uint8_t* kd = (uint8_t*)kcv + slot * row;
          uint8_t* vd = (uint8_t*)vcv + slot * row;
          for (int h = 0; h < KV; ++h) {
            const float ks = k_scale8[blk * KV + h], vs = v_scale8[blk * KV + h];
            for (int d = 0; d < D; ++d) {
              kd[h * D + d] = f32_to_e4m3(ld(k, (int64_t)t * row + h * D + d, dtype) / ks);
              vd[h * D + d] = f32_to_e4m3(ld(v, (int64_t)t * row + h * D + d, dtype) / vs);
            }
          }
        } else {
          memcpy((uint16_t*)kcv + slot * row, k + (int64_t)t * row, sizeof(uint16_t) * row);
          memcpy((uint16_t*)vcv + slot * row, v + (int64_t)t * row, sizeof(uint16_t) * row);
        }
      }
    }
  }

  Job job = {dtype, H, KV, D, B, bs, maxb, causal, window, seq_begin, seq_end, q, k, v,
             (const uint16_t*)kcv, (const uint16_t*)vcv, cum, past, bt, scale, softcap, sink,
             (uint16_t*)outv, out_f32, k_scale8, v_scale8, 0};
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

/* 16-bit caches in the activation dtype. */
int oracle_paged_attention(int dtype, int H, int KV, int D, int nt, int B, int NB, int bs, int maxb,
                           const void* qv, const void* kv_, const void* vv, void* kcv, void* vcv,
                           const int32_t* cum, const int32_t* past, const int32_t* bt, const int32_t* slots,
                           float scale, int causal, int window, float softcap, const float* sink,
                           void* outv, int threads, int do_append, int seq_begin, int seq_end, float* out_f32) {
  return run(dtype, H, KV, D, nt, B, NB, bs, maxb, qv, kv_, vv, kcv, vcv, cum, past, bt, slots, scale, causal,
             window, softcap, sink, outv, threads, do_append, seq_begin, seq_end, out_f32, NULL, NULL);
}

/* fp8 e4m3 caches with per-(block, kv head) fp32 scales k_scale / v_scale [NB, KV]: the new
 * rows are encoded into their slots (x / scale, round to nearest even, saturating at 448), then
 * every position is read back from the cache and decoded (code value * scale). */
int oracle_paged_attention_fp8(int dtype, int H, int KV, int D, int nt, int B, int NB, int bs, int maxb,
                               const void* qv, const void* kv_, const void* vv, void* kcv, void* vcv,
                               const int32_t* cum, const int32_t* past, const int32_t* bt, const int32_t* slots,
                               const float* k_scale, const float* v_scale, float scale, int causal, int window,
                               float softcap, const float* sink, void* outv, int threads, int do_append,
                               int seq_begin, int seq_end, float* out_f32) {
  if (!k_scale || !v_scale) return 1;
  return run(dtype, H, KV, D, nt, B, NB, bs, maxb, qv, kv_, vv, kcv, vcv, cum, past, bt, slots, scale, causal,
             window, softcap, sink, outv, threads, do_append, seq_begin, seq_end, out_f32, k_scale, v_scale);
}

/* e4m3fn encode of n fp32 values (exposed so the tests can pin it against another encoder). */
void oracle_e4m3_encode(const float* x, uint8_t* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = f32_to_e4m3(x[i]);
}
