// com.microsoft.GroupQueryAttention over a contiguous [B, KV, cap, D] (BNSH) cache.
//
// Reference: group_query_attention_op (rust/src/ops/attention.rs:932-1454) and its per-batch
// form gqa_batched (:586-848); masks as pinned by the reference's NumPy oracle
// (tests/ops/test_gqa_position_cache.py:88-134): query row i of batch b sits at
// query_past + i and sees keys [start, end), end = min(query_past + i + 1, length) when causal,
// else length, start = max(0, end - window) for window > 0.  Softcap and sink follow the
// composed path (capped_attention_logits :79-97, attention_probs_with_sink :100-118).
//
// B200 design (fp32 compute for every activation type; the op is HBM- or latency-bound at the
// sizes it serves):
//  * a CTA owns (batch b, kv head, tile of 16 query rows, key split).  A row is (token, q head
//    of the kv head), so the g heads of a group share every K/V byte read;
//  * per 64-key chunk: scores (two threads per key, each half of the channels for all 16 rows,
//    combined by a shuffle), online softmax (a warp per 4 rows), P.V (a thread per channel);
//  * decode-sized tiles split the key range over CTAs; the last CTA of a group (atomic
//    counter) merges the fp32 partials, so there is no second launch;
//  * when one row tile covers every key (decode, no window), the attention CTAs also write
//    each K/V row they read into `present`: the growing cache (present = past ++ new) costs
//    one read and one write of the cache.  Otherwise a copy kernel builds `present`.
#include <atomic>
#include <cmath>
#include <cooperative_groups.h>
#include <map>
#include <mutex>
#include <tuple>
#include <type_traits>
#include <cstring>
#include <string>
#include <vector>

#include "b200_common.cuh"
#include "b200_kernels.h"

namespace b200 {
namespace {

constexpr int kMaxRows = 16;   // query rows per CTA: 4, 8 or 16 (template R, from seq * g)
constexpr int kKeys = 64;      // keys per chunk
constexpr int kThreads = 128;
constexpr int kMaxD = 256;
constexpr int kMaxSplits = 128;  // key splits per row tile (merge weights live in shared memory)
constexpr float kLog2e = 1.4426950408889634f;

struct GqaArgs {
  int H, KV, D, g, B, S, new_seq, cap, pcap, total;
  int causal, window, smooth, dtype;
  float scale, softcap;
  int64_t q_stride, k_stride, v_stride;
  const void* q;
  const void* k;
  const void* v;
  const void* pk;
  const void* pv;
  void* ok;
  void* ov;
  const int32_t* seqlens;
  const void* sink;
  const void* bias;                       // attention_bias [Bb, Hb, S, total] or null
  int64_t bias_bstride, bias_hstride;     // 0 for a broadcast (size-1) dimension
  void* qk_out;                           // qk_output diagnostics [B, H, S, total] or null
  int qk_mode;                            // 1 logits, 2 probabilities
  int cache_bits;                         // 0 float caches, 8 int8, 4 int4 (codes in pk / pv, ok / ov)
  int cache_w;                            // bytes per stored cache row (int caches)
  const float* kscale;                    // int caches: PER_TENSOR [1] or PER_CHANNEL [KV, D]
  const float* vscale;
  int kpc, vpc;                           // per-channel scales
  int sliding, slide_gap;                 // sliding_window_cache=1; gap = cap - window + 1
  void* out;
  int row_tiles, splits, fused_copy, present_separate;
  float* part_o;   // [groups][splits][R][D]
  float* part_ml;  // [groups][splits][R][2]
  int* counters;   // [groups]
  int* status;     // kStatus* bits (a bounded wait ran out); cleared by CTA 0 of every call
};

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Read-only element and 4-element vector loads (ld.global.nc).  Nothing the attention kernel
// reads is written during the call: in place, only the new-row positions of the past buffer are
// written, and those rows are read from the key/value inputs.
template <typename T> struct Vec4 { using raw = uint2; };  // 4 x 16-bit
template <> struct Vec4<float> { using raw = float4; };
template <typename T> __device__ __forceinline__ typename Vec4<T>::raw ld4(const T* p) {
  return __ldg(reinterpret_cast<const typename Vec4<T>::raw*>(p));
}
template <typename T> __device__ __forceinline__ void st4(T* p, const typename Vec4<T>::raw& v) {
  *reinterpret_cast<typename Vec4<T>::raw*>(p) = v;
}
__device__ __forceinline__ void unpack4(const float4& v, float (&x)[4]) {
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
template <typename T> __device__ __forceinline__ void unpack4(const uint2& v, float (&x)[4]);
template <> __device__ __forceinline__ void unpack4<__half>(const uint2& v, float (&x)[4]) {
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
template <> __device__ __forceinline__ void unpack4<__nv_bfloat16>(const uint2& v, float (&x)[4]) {
  const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.x));
  const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v.y));
  x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
}
template <typename T> __device__ __forceinline__ void unpack_raw(const typename Vec4<T>::raw& v, float (&x)[4]) {
  if constexpr (std::is_same<T, float>::value) unpack4(v, x);
  else unpack4<T>(v, x);
}
template <typename T> __device__ __forceinline__ T ldg1(const T* p) {
  if constexpr (std::is_same<T, float>::value) return __ldg(p);
  else {
    const unsigned short u = __ldg(reinterpret_cast<const unsigned short*>(p));
    T t;
    memcpy(&t, &u, sizeof(u));
    return t;
  }
}

// Rows a sliding-window cache of capacity cap keeps of a length-n sequence (attention.rs:
// 1173-1181): all of them up to the capacity, beyond it whole gaps reclaimed from the front.
__host__ __device__ __forceinline__ int slide_resident(int n, int cap, int gap) {
  return n <= cap ? n : n - gap * ((n - cap + gap - 1) / gap);
}

// Per batch row (:662-667): length, query_past, past (rows taken from the past cache) and
// origin, the absolute position of past-cache row 0: 0, or for a sliding cache
// past - resident(past) (:1186-1193), so key position pos < past is cache row pos - origin.
// The visible keys of every query row start at or above the origin: resident(past) is past
// itself up to the capacity and at least the window beyond it.
struct BatchGeom {
  int length, query_past, past, origin;
};
__device__ __forceinline__ BatchGeom batch_geom(const GqaArgs& a, int b) {
  BatchGeom g;
  g.length = a.seqlens[b] + 1;
  g.query_past = max(g.length - a.S, 0);
  g.past = a.new_seq == 0 ? g.length : g.query_past;
  g.origin = a.sliding ? g.past - slide_resident(g.past, a.cap, a.slide_gap) : 0;
  return g;
}

// Row `pos` of kv head kh of batch b: past cache below `past`, new input rows from there on.
template <typename T>
__device__ __forceinline__ const T* key_row(const GqaArgs& a, const BatchGeom& bg, int b, int kh, int pos, bool value) {
  if (pos < bg.past) {
    const T* base = static_cast<const T*>(value ? a.pv : a.pk);
    return base + (((int64_t)b * a.KV + kh) * a.cap + (pos - bg.origin)) * a.D;
  }
  const T* base = static_cast<const T*>(value ? a.v : a.k);
  const int64_t stride = value ? a.v_stride : a.k_stride;
  return base + ((int64_t)b * a.new_seq + (pos - bg.past)) * stride + (int64_t)kh * a.D;
}

template <typename T>
__device__ __forceinline__ T* present_row(const GqaArgs& a, int b, int kh, int pos, bool value) {
  T* base = static_cast<T*>(value ? a.ov : a.ok);
  return base + (((int64_t)b * a.KV + kh) * a.pcap + pos) * a.D;
}

template <typename T, int R, int NC>
__global__ void __launch_bounds__(kThreads) gqa_attention_kernel(const GqaArgs a) {
  __shared__ float qs[R][kMaxD];
  __shared__ float sc[R][kKeys + 1];
  __shared__ float m_run[R], l_run[R], alpha_s[R];
  __shared__ int row_pos[R];  // absolute position of each row, or -1 (padding row)
  __shared__ int row_end[R], row_start[R];
  __shared__ int64_t row_bias[R];  // attention_bias offset of each row's [total] bias row

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int idx = blockIdx.x;
  const int sp = idx % a.splits;
  idx /= a.splits;
  const int rt = idx % a.row_tiles;
  idx /= a.row_tiles;
  const int kh = idx % a.KV;
  const int b = idx / a.KV;
  const int group = (b * a.KV + kh) * a.row_tiles + rt;
  const BatchGeom bg = batch_geom(a, b);
  const int D = a.D, g = a.g;
  const int rows_total = a.S * g;
  if (blockIdx.x == 0 && tid == 0) *a.status = 0;

  // Query rows of this tile (fp32, pre-scaled into the log2 domain unless softcap is on).
  const float qmul = a.softcap > 0.f ? 1.f : a.scale * kLog2e;
  for (int i = tid; i < R * D; i += kThreads) {
    const int r = i / D, d = i % D, rho = rt * R + r;
    float x = 0.f;
    if (rho < rows_total) {
      const int s = rho / g, hl = rho % g;
      x = to_f(static_cast<const T*>(a.q)[((int64_t)b * a.S + s) * a.q_stride + (int64_t)(kh * g + hl) * D + d]) * qmul;
    }
    qs[r][d] = x;
  }
  if (tid < R) {
    const int rho = rt * R + tid;
    if (rho < rows_total) {
      const int pos = bg.query_past + rho / g;
      const int end = a.causal ? min(pos + 1, bg.length) : bg.length;
      row_pos[tid] = pos;
      row_end[tid] = end;
      row_start[tid] = a.window > 0 ? max(0, end - a.window) : 0;
      row_bias[tid] = b * a.bias_bstride + (int64_t)(kh * g + rho % g) * a.bias_hstride + (int64_t)(rho / g) * a.total;
    } else {
      row_pos[tid] = -1;
      row_end[tid] = 0;
      row_start[tid] = 0;
    }
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.f;
  }
  __syncthreads();

  // Key range of the tile, then this CTA's share of its chunks.
  int kmin = bg.length, kmax = 0;
  for (int r = 0; r < R; ++r)
    if (row_pos[r] >= 0) {
      kmin = min(kmin, row_start[r]);
      kmax = max(kmax, row_end[r]);
    }
  if (a.fused_copy) {
    kmin = 0;
    kmax = bg.length;
  }
  const int c_lo = kmin / kKeys, c_hi = kmax > kmin ? (kmax + kKeys - 1) / kKeys : c_lo;
  const int nch = c_hi - c_lo;
  const int my_lo = c_lo + (int)((int64_t)nch * sp / a.splits), my_hi = c_lo + (int)((int64_t)nch * (sp + 1) / a.splits);

  // Channels of this thread in P.V.
  float o[R][NC];  // channels d0 = tid and, when NC == 2 (D > 128), d1 = tid + 128
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int c = 0; c < NC; ++c) o[r][c] = 0.f;
  const int d0 = tid, d1 = tid + kThreads;

  for (int c = my_lo; c < my_hi; ++c) {
    const int kend = min(kKeys, bg.length - c * kKeys);
    // ---- scores: thread = (key kk, channel half)
    {
      const int kk = tid >> 1, half = tid & 1;
      const int pos = c * kKeys + kk;
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = 0.f;
      if (pos < bg.length && pos >= bg.origin) {  // below the origin: not resident, never visible
        const T* krow = key_row<T>(a, bg, b, kh, pos, false);
        const bool copy = a.fused_copy && (a.present_separate || pos >= bg.past);
        T* kdst = copy ? present_row<T>(a, b, kh, pos, false) : nullptr;
        const int dh = D / 2, dbeg = half * dh, dend = dbeg + dh;
        // groups of 16 vectors (64 channels): all loads of a group in flight before its stores
        for (int d = dbeg; d < dend; d += 64) {
          typename Vec4<T>::raw raw[16];
#pragma unroll
          for (int u = 0; u < 16; ++u)
            if (d + 4 * u < dend) raw[u] = ld4(krow + d + 4 * u);
          if (copy) {
#pragma unroll
            for (int u = 0; u < 16; ++u)
              if (d + 4 * u < dend) st4(kdst + d + 4 * u, raw[u]);
          }
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            if (d + 4 * u < dend) {
              float kx[4];
              unpack_raw<T>(raw[u], kx);
#pragma unroll
              for (int r = 0; r < R; ++r) {
                const float4 qv = *reinterpret_cast<const float4*>(&qs[r][d + 4 * u]);
                acc[r] = fmaf(qv.x, kx[0], fmaf(qv.y, kx[1], fmaf(qv.z, kx[2], fmaf(qv.w, kx[3], acc[r]))));
              }
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 1);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r / (R / 2) != half) continue;
        float s = -INFINITY;
        if (row_pos[r] >= 0 && pos >= row_start[r] && pos < row_end[r]) {
          s = acc[r];
          if (a.softcap > 0.f) s = a.softcap * tanhf(s * a.scale / a.softcap) * kLog2e;
          if (a.bias) s += to_f(static_cast<const T*>(a.bias)[row_bias[r] + pos]) * kLog2e;
        }
        sc[r][kk] = s;
      }
    }
    __syncthreads();
    // ---- online softmax: warp w owns rows 4w..4w+3, lane = keys 2*lane, 2*lane+1
#pragma unroll
    for (int rr = 0; rr < R / 4; ++rr) {
      const int r = warp * (R / 4) + rr;
      const float s0 = sc[r][2 * lane], s1 = sc[r][2 * lane + 1];
      float mx = fmaxf(s0, s1);
      for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = m_run[r];
      const float m_new = fmaxf(m_old, mx);
      const float mu = m_new == -INFINITY ? 0.f : m_new;
      const float p0 = exp2f(s0 - mu), p1 = exp2f(s1 - mu);
      float sum = p0 + p1;
      for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      sc[r][2 * lane] = p0;
      sc[r][2 * lane + 1] = p1;
      __syncwarp();
      if (lane == 0) {
        const float alpha = m_old == -INFINITY ? 0.f : exp2f(m_old - mu);
        alpha_s[r] = alpha;
        l_run[r] = l_run[r] * alpha + sum;
        m_run[r] = m_new;
      }
    }
    __syncthreads();
    // ---- P.V: thread = channels d0 (and d1 when D > 128)
    {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float al = alpha_s[r];
#pragma unroll
        for (int c = 0; c < NC; ++c) o[r][c] *= al;
      }
      constexpr int kGroup = 16;  // keys whose V loads are in flight together
      for (int k0 = 0; k0 < kend; k0 += kGroup) {
        T x0[kGroup], x1[kGroup];
#pragma unroll
        for (int u = 0; u < kGroup; ++u) {
          x0[u] = x1[u] = from_f<T>(0.f);
          if (k0 + u < kend && c * kKeys + k0 + u >= bg.origin) {
            const T* vrow = key_row<T>(a, bg, b, kh, c * kKeys + k0 + u, true);
            if (d0 < D) x0[u] = ldg1(vrow + d0);
            if (NC == 2 && d1 < D) x1[u] = ldg1(vrow + d1);
          }
        }
        if (a.fused_copy) {
#pragma unroll
          for (int u = 0; u < kGroup; ++u) {
            const int pos = c * kKeys + k0 + u;
            if (k0 + u < kend && (a.present_separate || pos >= bg.past)) {
              T* vdst = present_row<T>(a, b, kh, pos, true);
              if (d0 < D) vdst[d0] = x0[u];
              if (NC == 2 && d1 < D) vdst[d1] = x1[u];
            }
          }
        }
#pragma unroll
        for (int u = 0; u < kGroup; ++u) {
          const float v0 = to_f(x0[u]), v1 = to_f(x1[u]);
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const float p = sc[r][min(k0 + u, kKeys - 1)];
            o[r][0] = fmaf(p, v0, o[r][0]);
            if constexpr (NC == 2) o[r][NC - 1] = fmaf(p, v1, o[r][NC - 1]);
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- finish: direct output, or partial + last-CTA merge
  auto sink_log2 = [&](int r) -> float {
    if (a.sink == nullptr && !a.smooth) return -INFINITY;
    const int hl = (rt * R + r) % g;
    const float s = a.sink ? to_f(static_cast<const T*>(a.sink)[kh * g + hl]) : 0.f;
    return s * kLog2e;
  };
  auto store_row = [&](int r, int d, float v) {
    const int rho = rt * R + r;
    const int s = rho / g, hl = rho % g;
    static_cast<T*>(a.out)[((int64_t)b * a.S + s) * a.H * D + (int64_t)(kh * g + hl) * D + d] = from_f<T>(v);
  };
  if (a.splits == 1) {
    for (int r = 0; r < R; ++r) {
      if (row_pos[r] < 0) continue;
      const float m = m_run[r], mu = m == -INFINITY ? 0.f : m;
      float L = l_run[r];
      const float sk = sink_log2(r);
      if (sk != -INFINITY) L += exp2f(sk - mu);
      const float inv = L > 0.f ? 1.f / L : 0.f;
      if (d0 < D) store_row(r, d0, o[r][0] * inv);
      if constexpr (NC == 2) {
        if (d1 < D) store_row(r, d1, o[r][NC - 1] * inv);
      }
    }
    return;
  }
  {
    float* po = a.part_o + ((int64_t)group * a.splits + sp) * R * D;
    float* pml = a.part_ml + ((int64_t)group * a.splits + sp) * R * 2;
    for (int r = 0; r < R; ++r) {
      if (row_pos[r] < 0) continue;
      if (d0 < D) po[r * D + d0] = o[r][0];
      if constexpr (NC == 2) {
        if (d1 < D) po[r * D + d1] = o[r][NC - 1];
      }
    }
    if (tid < R) {
      pml[tid * 2] = m_run[tid];
      pml[tid * 2 + 1] = l_run[tid];
    }
  }
  __threadfence();
  __shared__ int last;
  __syncthreads();
  if (tid == 0) last = atomicAdd(&a.counters[group], 1) == a.splits - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Merge, step 1: a warp per row (rows w, w+4, ...), lanes over splits: max, weights, sum.
  __shared__ float wts[R][kMaxSplits];
  __shared__ float inv_s[R];
  const float* pml_g = a.part_ml + (int64_t)group * a.splits * R * 2;
  for (int r = warp; r < R; r += kThreads / 32) {
    if (row_pos[r] < 0) continue;
    float M = -INFINITY;
    for (int j = lane; j < a.splits; j += 32) M = fmaxf(M, __ldcg(&pml_g[(j * R + r) * 2]));
    for (int off = 16; off; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const float mu = M == -INFINITY ? 0.f : M;
    float L = 0.f;
    for (int j = lane; j < a.splits; j += 32) {
      const float mj = __ldcg(&pml_g[(j * R + r) * 2]);
      const float w = mj == -INFINITY ? 0.f : exp2f(mj - mu);
      wts[r][j] = w;
      L += w * __ldcg(&pml_g[(j * R + r) * 2 + 1]);
    }
    for (int off = 16; off; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    if (lane == 0) {
      const float sk = sink_log2(r);
      if (sk != -INFINITY) L += exp2f(sk - mu);
      inv_s[r] = L > 0.f ? 1.f / L : 0.f;
    }
  }
  __syncthreads();
  // Step 2: each thread sums its channels over the splits for every row at once.
  float acc[R][NC];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int c = 0; c < NC; ++c) acc[r][c] = 0.f;
  const float* po_g = a.part_o + (int64_t)group * a.splits * R * D;
  for (int j0 = 0; j0 < a.splits; j0 += 8) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u;
      if (j >= a.splits) break;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (row_pos[r] < 0) continue;
        const float w = wts[r][j];
        const float* po = po_g + ((int64_t)j * R + r) * D;
        if (d0 < D) acc[r][0] = fmaf(w, __ldcg(&po[d0]), acc[r][0]);
        if constexpr (NC == 2) {
          if (d1 < D) acc[r][NC - 1] = fmaf(w, __ldcg(&po[d1]), acc[r][NC - 1]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (row_pos[r] < 0) continue;
    if (d0 < D) store_row(r, d0, acc[r][0] * inv_s[r]);
    if constexpr (NC == 2) {
      if (d1 < D) store_row(r, d1, acc[r][NC - 1] * inv_s[r]);
    }
  }
}

// Decode-shaped groups (one row tile covers every key, no window): a thread-block cluster per
// (batch, kv head).  Each CTA of the cluster owns a contiguous key range, stages its K and V
// rows in shared memory with one 1-D bulk copy each (the past rows of a BNSH head are
// contiguous; K and V on separate barriers, so the scores start while V is still arriving),
// writes the fused present rows from there, and keeps an fp32 partial (m, l, o).  The partials are merged through
// distributed shared memory: each CTA finishes a slice of the channels.  No workspace, no
// counters, one launch.
constexpr int kClThreads = 256;
constexpr int kClMaxCluster = 16;

// Dynamic shared memory of one CTA: K staging [kc][D] T (reused, after the last chunk, for the
// key-group reduction of P.V [1024/D][R][D] fp32), V staging [kc][D] T, probabilities [R][kc]
// and the CTA partial o [R][D] (fp32).
__host__ __device__ inline size_t cluster_kbuf_bytes(int R, int D, int esz, int kc) {
  const size_t k = (size_t)kc * D * esz, r = (size_t)1024 * R * 4;
  return k > r ? k : r;
}
__host__ __device__ inline size_t cluster_smem_bytes(int R, int D, int esz, int kc) {
  return cluster_kbuf_bytes(R, D, esz, kc) + (size_t)kc * D * esz + (size_t)R * kc * 4 + (size_t)R * D * 4;
}

template <typename T, int R, int D>
__global__ void __launch_bounds__(kClThreads) gqa_cluster_kernel(const GqaArgs a, int kc) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = (int)cluster.num_blocks();
  const int cr = (int)cluster.block_rank();
  extern __shared__ __align__(16) uint8_t cl_smem[];
  __shared__ float m_run[R], l_run[R], alpha_s[R];
  __shared__ int row_pos[R], row_end[R];
  __shared__ int64_t row_bias[R];  // attention_bias offset of each row's [total] bias row
  __shared__ __align__(8) uint64_t bar_k, bar_v;

  // Scores: LPK lanes per key, each holding the q values of UPL 4-channel units (units
  // j, j + LPK, ...: one 128-byte bank row per key and instruction) for all R rows.
  constexpr int kUnits = D / 4;
  constexpr int LPK = (R * D / 64) < 4 ? 4 : (R * D / 64) > 32 ? 32 : (R * D / 64);
  constexpr int UPL = kUnits / LPK;
  constexpr int KPP = kClThreads / LPK;  // keys per pass
  // P.V: thread = (4-channel unit, key group)
  constexpr int KG = kClThreads / kUnits;

  const int g = a.g, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = blockIdx.x / CL;  // (b, kh)
  const int kh = grp % a.KV, b = grp / a.KV;
  const BatchGeom bg = batch_geom(a, b);
  const int rows_total = a.S * g;

  T* kbuf = reinterpret_cast<T*>(cl_smem);
  T* vbuf = reinterpret_cast<T*>(cl_smem + cluster_kbuf_bytes(R, D, (int)sizeof(T), kc));
  float* sc = reinterpret_cast<float*>(vbuf + (size_t)kc * D);
  float* opart = sc + R * kc;
  float* red = reinterpret_cast<float*>(cl_smem);  // after the last chunk: K is no longer read

  if (tid < R) {
    if (tid < rows_total) {
      const int pos = bg.query_past + tid / g;
      row_pos[tid] = pos;
      row_end[tid] = a.causal ? min(pos + 1, bg.length) : bg.length;
      row_bias[tid] = b * a.bias_bstride + (int64_t)(kh * g + tid % g) * a.bias_hstride + (int64_t)(tid / g) * a.total;
    } else {
      row_pos[tid] = -1;
      row_end[tid] = 0;
    }
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.f;
  }
  const int k0 = (int)((int64_t)bg.length * cr / CL), k1 = (int)((int64_t)bg.length * (cr + 1) / CL);
  // Past rows of K and of V of the chunk at c0 (contiguous in the BNSH head): one bulk copy
  // each, on separate barriers so the scores start while V is in flight (thread 0).
  auto issue_chunk = [&](int c0) {
    const int nk = min(kc, k1 - c0);
    const int np = max(0, min(nk, bg.past - c0));
    if (np <= 0) return;
    const uint32_t pbytes = (uint32_t)np * D * sizeof(T);
    const T* kpast = static_cast<const T*>(a.pk) + (((int64_t)b * a.KV + kh) * a.cap + c0) * D;
    const T* vpast = static_cast<const T*>(a.pv) + (((int64_t)b * a.KV + kh) * a.cap + c0) * D;
    fence_proxy_async_smem();  // the previous chunk's generic reads and writes come first
    mbar_arrive_expect_tx(&bar_k, pbytes);
    bulk_load(kbuf, kpast, pbytes, &bar_k);
    mbar_arrive_expect_tx(&bar_v, pbytes);
    bulk_load(vbuf, vpast, pbytes, &bar_v);
  };
  if (tid == 0) {
    if (blockIdx.x == 0) *a.status = 0;
    mbar_init(&bar_k, 1);
    mbar_init(&bar_v, 1);
    fence_mbar_init();
    if (k0 < k1) issue_chunk(k0);  // the first chunk's copies go out before the q loads
  }
  uint32_t phase = 0;
  bool failed = false;  // a staging wait ran out: skip the math, still meet the cluster barriers
  // This lane's q units (fp32, scaled into the log2 domain unless softcap is on).
  const int sj = tid % LPK;
  float qr[R][UPL][4];
  {
    const float qmul = a.softcap > 0.f ? 1.f : a.scale * kLog2e;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const bool live = r < rows_total;
      const T* qrow = static_cast<const T*>(a.q) +
                      ((int64_t)b * a.S + (live ? r / g : 0)) * a.q_stride + (int64_t)(kh * g + (live ? r % g : 0)) * D;
#pragma unroll
      for (int i = 0; i < UPL; ++i) {
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        if (live) unpack_raw<T>(ld4(qrow + (sj + LPK * i) * 4), x);
#pragma unroll
        for (int e = 0; e < 4; ++e) qr[r][i][e] = x[e] * qmul;
      }
    }
  }

  const int cq = tid % kUnits, kgrp = tid / kUnits;
  float o[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) o[r][0] = o[r][1] = o[r][2] = o[r][3] = 0.f;
  __syncthreads();

  for (int c0 = k0; c0 < k1 && !failed; c0 += kc) {
    const int nk = min(kc, k1 - c0);
    const int np = max(0, min(nk, bg.past - c0));  // rows from the past cache
    // ---- stage: past rows by bulk copies (issued here for every chunk after the first), new
    // rows by plain loads
    if (tid == 0 && c0 != k0) issue_chunk(c0);
    for (int i = tid; i < (nk - np) * kUnits; i += kClThreads) {
      const int k = np + i / kUnits, d = (i % kUnits) * 4;
      st4(kbuf + (size_t)k * D + d, ld4(key_row<T>(a, bg, b, kh, c0 + k, false) + d));
      st4(vbuf + (size_t)k * D + d, ld4(key_row<T>(a, bg, b, kh, c0 + k, true) + d));
    }
    if (a.fused_copy) fence_proxy_async_smem();  // the new rows, for the bulk present stores
    if (np > 0 && !mbar_wait(&bar_k, phase)) failed = true;
    if (__syncthreads_or(failed)) {
      // one more bounded wait on each copy still in flight, then no further work
      if (tid == 0) {
        set_status(a.status, kStatusTimeout);
        mbar_wait(&bar_k, phase);
        mbar_wait(&bar_v, phase);
      }
      failed = true;
      break;
    }

    // ---- fused present rows of K (all rows when present is its own buffer, else the new ones):
    // contiguous in the BNSH present, so one bulk copy from the staging buffer
    if (a.fused_copy && tid == 0) {
      const int first = a.present_separate ? 0 : np;
      if (nk > first) {
        bulk_store(present_row<T>(a, b, kh, c0 + first, false), kbuf + (size_t)first * D,
                   (uint32_t)((nk - first) * D * (int)sizeof(T)));
        bulk_commit();
      }
    }

    // ---- scores
    for (int kb = 0; kb < nk; kb += KPP) {
      const int k = kb + tid / LPK;
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = 0.f;
      if (k < nk) {
        const T* krow = kbuf + (size_t)k * D;
#pragma unroll
        for (int i = 0; i < UPL; ++i) {
          float kx[4];
          unpack_raw<T>(*reinterpret_cast<const typename Vec4<T>::raw*>(krow + (sj + LPK * i) * 4), kx);
#pragma unroll
          for (int r = 0; r < R; ++r)
            acc[r] = fmaf(qr[r][i][0], kx[0], fmaf(qr[r][i][1], kx[1], fmaf(qr[r][i][2], kx[2], fmaf(qr[r][i][3], kx[3], acc[r]))));
        }
      }
#pragma unroll
      for (int off = 1; off < LPK; off <<= 1)
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
      if (k < nk && sj == 0) {
        const int pos = c0 + k;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float s = -INFINITY;
          if (row_pos[r] >= 0 && pos < row_end[r]) {
            s = acc[r];
            if (a.softcap > 0.f) s = a.softcap * tanhf(s * a.scale / a.softcap) * kLog2e;
            if (a.bias) s += to_f(static_cast<const T*>(a.bias)[row_bias[r] + pos]) * kLog2e;
          }
          sc[r * kc + k] = s;
        }
      }
    }
    __syncthreads();

    // ---- online softmax over the chunk: a warp per row
    for (int r = warp; r < R; r += kClThreads / 32) {
      float mx = -INFINITY;
      for (int k = lane; k < nk; k += 32) mx = fmaxf(mx, sc[r * kc + k]);
      for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_old = m_run[r], m_new = fmaxf(m_old, mx);
      const float mu = m_new == -INFINITY ? 0.f : m_new;
      float sum = 0.f;
      for (int k = lane; k < nk; k += 32) {
        const float p = exp2f(sc[r * kc + k] - mu);
        sc[r * kc + k] = p;
        sum += p;
      }
      for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0) {
        const float al = m_old == -INFINITY ? 0.f : exp2f(m_old - mu);
        alpha_s[r] = al;
        l_run[r] = l_run[r] * al + sum;
        m_run[r] = m_new;
      }
    }
    if (np > 0 && !mbar_wait(&bar_v, phase)) failed = true;
    if (np > 0) phase ^= 1u;
    if (__syncthreads_or(failed)) {
      if (tid == 0) {
        set_status(a.status, kStatusTimeout);
        mbar_wait(&bar_v, phase ^ 1u);
      }
      failed = true;
      break;
    }

    // ---- fused present rows of V, as for K
    if (a.fused_copy && tid == 0) {
      const int first = a.present_separate ? 0 : np;
      if (nk > first) {
        bulk_store(present_row<T>(a, b, kh, c0 + first, true), vbuf + (size_t)first * D,
                   (uint32_t)((nk - first) * D * (int)sizeof(T)));
        bulk_commit();
      }
    }

    // ---- P.V: thread = (4-channel unit cq, key group kgrp)
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float al = alpha_s[r];
      o[r][0] *= al; o[r][1] *= al; o[r][2] *= al; o[r][3] *= al;
    }
    for (int k = kgrp; k < nk; k += KG) {
      float vx[4];
      unpack_raw<T>(*reinterpret_cast<const typename Vec4<T>::raw*>(vbuf + (size_t)k * D + cq * 4), vx);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float p = sc[r * kc + k];
        o[r][0] = fmaf(p, vx[0], o[r][0]);
        o[r][1] = fmaf(p, vx[1], o[r][1]);
        o[r][2] = fmaf(p, vx[2], o[r][2]);
        o[r][3] = fmaf(p, vx[3], o[r][3]);
      }
    }
    if (tid == 0) bulk_wait_read();  // the present copies have read the staging buffers
    __syncthreads();  // the next chunk overwrites the staging buffers and the probabilities
  }
  if (tid == 0) bulk_wait_read();  // also after a failed wait (loop left early)

  // ---- CTA partial: sum the key groups
#pragma unroll
  for (int r = 0; r < R; ++r)
    *reinterpret_cast<float4*>(red + (kgrp * R + r) * D + cq * 4) = make_float4(o[r][0], o[r][1], o[r][2], o[r][3]);
  __syncthreads();
  for (int i = tid; i < R * D; i += kClThreads) {
    float s = 0.f;
#pragma unroll
    for (int q = 0; q < KG; ++q) s += red[q * R * D + i];
    opart[i] = s;
  }
  cluster.sync();  // every partial of the cluster is complete and visible

  // ---- merge: this CTA finishes channels [d_lo, d_hi) of every row from all CTAs' partials
  const int per = (D + CL - 1) / CL, d_lo = min(D, cr * per), d_hi = min(D, d_lo + per);
  for (int i = tid; i < R * (d_hi - d_lo); i += kClThreads) {
    const int r = i / (d_hi - d_lo), d = d_lo + i % (d_hi - d_lo);
    if (row_pos[r] < 0) continue;
    float mj[kClMaxCluster], lj[kClMaxCluster], oj[kClMaxCluster];
#pragma unroll
    for (int j = 0; j < kClMaxCluster; ++j) {
      if (j < CL) {
        mj[j] = *cluster.map_shared_rank(&m_run[r], j);
        lj[j] = *cluster.map_shared_rank(&l_run[r], j);
        oj[j] = *cluster.map_shared_rank(&opart[r * D + d], j);
      } else {
        mj[j] = -INFINITY;
        lj[j] = oj[j] = 0.f;
      }
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < kClMaxCluster; ++j) M = fmaxf(M, mj[j]);
    const float mu = M == -INFINITY ? 0.f : M;
    float L = 0.f, acc = 0.f;
#pragma unroll
    for (int j = 0; j < kClMaxCluster; ++j) {
      const float w = mj[j] == -INFINITY ? 0.f : exp2f(mj[j] - mu);
      L += w * lj[j];
      acc += w * oj[j];
    }
    if (a.sink != nullptr || a.smooth) {
      const int hl = r % g;
      const float sk = (a.sink ? to_f(static_cast<const T*>(a.sink)[kh * g + hl]) : 0.f) * kLog2e;
      L += exp2f(sk - mu);
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const int s = r / g, hl = r % g;
    static_cast<T*>(a.out)[((int64_t)b * a.S + s) * a.H * D + (int64_t)(kh * g + hl) * D + d] = from_f<T>(acc * inv);
  }
  cluster.sync();  // no CTA leaves while another still reads its shared memory
}

// present rows the attention kernel does not write: everything (copy mode) or the tail
// [length, pcap) (fused mode); in shared-buffer mode only the new rows.  One thread per element.
template <typename T>
__global__ void gqa_present_kernel(const GqaArgs a, int tail_only) {
  const int64_t n = (int64_t)a.B * a.KV * a.pcap * a.D;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % a.D);
    int64_t row = i / a.D;
    const int pos = (int)(row % a.pcap);
    row /= a.pcap;
    const int kh = (int)(row % a.KV), b = (int)(row / a.KV);
    const BatchGeom bg = batch_geom(a, b);
    const bool is_new = pos >= bg.past && pos < bg.length;
    if (tail_only && pos < bg.length) continue;
    if (!a.present_separate && !is_new) continue;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      T x;
      if (pos < bg.length) {
        x = key_row<T>(a, bg, b, kh, pos, which == 1)[d];
      } else if (pos < a.cap) {
        const T* base = static_cast<const T*>(which ? a.pv : a.pk);
        x = base[(((int64_t)b * a.KV + kh) * a.cap + pos) * a.D + d];
      } else {
        x = from_f<T>(0.f);
      }
      present_row<T>(a, b, kh, pos, which == 1)[d] = x;
    }
  }
}

// ------------------------------------------------------------------ q/k norm and rotary embedding
// The node's processed query and new key rows, written to workspace rows that the attention
// kernels then read.  Per head, in order:
//  * optional RMS norm (inputs 14 / 15, attention.rs:1070-1078): x / sqrt(mean(x^2) + eps) * w
//    in fp32, rounded to the activation type (the reference's rms_norm output has that type);
//  * optional RoPE (do_rotary=1, attention.rs:668-681): Q and K rotated at the query rows'
//    positions before K joins present, fp32 products and sum each rounded, one rounding to the
//    activation type (the reference oracle's _rotate, and gqa_rope_f32).
// One CTA per (batch, query row); the rows are staged in shared memory as fp32.
struct GqaRope {
  int H, KV, D, S, new_seq, half, interleaved, rows, first_prompt, do_rotary;
  float eps;
  int64_t q_stride, k_stride;
  const void* q;
  const void* k;
  const void* cos;
  const void* sin;
  const void* qw;          // [D] norm weights (both or neither)
  const void* kw;
  const int32_t* seqlens;
  const int64_t* pos_ids;  // NULL: positions query_past + s
  void* q_out;             // [B * S, H * D]
  void* k_out;             // [B * new_seq, KV * D]
};

size_t gqa_rope_smem(int H, int KV, int D) { return sizeof(float) * (size_t)(H + KV) * D; }

template <typename T>
__global__ void __launch_bounds__(256) gqa_rope_kernel(const GqaRope r) {
  extern __shared__ float rowbuf[];  // [(H + KV) * D]
  const int row = blockIdx.x;  // b * S + s
  const int b = row / r.S, s = row % r.S;
  const int nheads = r.H + (s < r.new_seq ? r.KV : 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  auto src_row = [&](int h) -> const T* {
    return h >= r.H ? static_cast<const T*>(r.k) + ((int64_t)b * r.new_seq + s) * r.k_stride + (int64_t)(h - r.H) * r.D
                    : static_cast<const T*>(r.q) + (int64_t)row * r.q_stride + (int64_t)h * r.D;
  };
  for (int h = warp; h < nheads; h += nwarps) {  // stage, and normalise, a head per warp
    const T* src = src_row(h);
    float* dst = rowbuf + (int64_t)h * r.D;
    float acc = 0.f;
    for (int d = lane; d < r.D; d += 32) {
      const float x = to_f<T>(src[d]);
      dst[d] = x;
      acc = __fadd_rn(acc, __fmul_rn(x, x));
    }
    if (r.qw) {
#pragma unroll
      for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      const float denom = sqrtf(__fdiv_rn(acc, (float)r.D) + r.eps);
      const T* w = static_cast<const T*>(h >= r.H ? r.kw : r.qw);
      for (int d = lane; d < r.D; d += 32)
        dst[d] = to_f<T>(from_f<T>(__fmul_rn(__fdiv_rn(dst[d], denom), to_f<T>(w[d]))));
    }
  }
  __syncthreads();
  const T* crow = nullptr;
  const T* srow = nullptr;
  if (r.do_rotary) {
    int64_t pos;
    if (r.pos_ids) pos = r.first_prompt ? r.pos_ids[0] + s : r.pos_ids[(int64_t)b * r.S + s];
    else pos = max(r.seqlens[b] + 1 - r.S, 0) + s;
    // the host rejected out-of-range positions before the launch; clamp so no read can stray
    pos = pos < 0 ? 0 : (pos >= r.rows ? r.rows - 1 : pos);
    crow = static_cast<const T*>(r.cos) + pos * r.half;
    srow = static_cast<const T*>(r.sin) + pos * r.half;
  }
  const int rot = r.do_rotary ? 2 * r.half : 0;
  for (int i = threadIdx.x; i < nheads * r.D; i += blockDim.x) {
    const int h = i / r.D, d = i - h * r.D;
    const bool is_k = h >= r.H;
    T* dst = is_k ? static_cast<T*>(r.k_out) + ((int64_t)b * r.new_seq + s) * ((int64_t)r.KV * r.D) + (int64_t)(h - r.H) * r.D
                  : static_cast<T*>(r.q_out) + (int64_t)row * ((int64_t)r.H * r.D) + (int64_t)h * r.D;
    const float* xrow = rowbuf + (int64_t)h * r.D;
    const float x = xrow[d];
    float y = x;
    if (d < rot) {
      int j, partner;
      bool first;
      if (r.interleaved) {  // pairs (2j, 2j + 1)
        j = d >> 1;
        partner = d ^ 1;
        first = (d & 1) == 0;
      } else {  // rotate-half: (j, j + half)
        j = d < r.half ? d : d - r.half;
        partner = d < r.half ? d + r.half : d - r.half;
        first = d < r.half;
      }
      const float c = to_f<T>(crow[j]), sn = to_f<T>(srow[j]), xp = xrow[partner];
      // two products and one sum, each rounded (no fused multiply-add), as the reference's
      // element-wise ops round them: fp32 caches match bit for bit
      y = __fadd_rn(__fmul_rn(x, c), __fmul_rn(first ? -xp : xp, sn));
    }
    dst[d] = from_f<T>(y);
  }
}

// ------------------------------------------------------------------ integer caches
// kv_cache_bit_width 8 / 4 (kv_cache.rs:16-108; test_quantized_kv.py:22-47 with paged = false):
// a code is rint(x * (1 / scale)) clipped to [-2^(bits-1), 2^(bits-1) - 1], a zero scale
// multiplying by 1; int4 codes are stored +8-biased, two per byte, the even channel in the low
// nibble.  A cached value is code * scale.  New rows go through the same encoding before the
// attention reads them, as the reference reads every key and value from the encoded cache.
__device__ __forceinline__ int gqa_code(float x, float scale, int bits) {
  const float inv = scale != 0.f ? __fdiv_rn(1.f, scale) : 1.f;
  const float lim = bits == 8 ? 128.f : 8.f;
  return (int)fminf(fmaxf(rintf(__fmul_rn(x, inv)), -lim), lim - 1.f);
}

__device__ __forceinline__ float gqa_scale(const GqaArgs& a, bool value, int kh, int d) {
  const float* sc = value ? a.vscale : a.kscale;
  return (value ? a.vpc : a.kpc) ? sc[(int64_t)kh * a.D + d] : sc[0];
}

// Channel d of key / value row `pos` of kv head kh of batch b, decoded: past rows from the
// integer past cache, new rows encoded and decoded on the fly.
template <typename T>
__device__ __forceinline__ float gqa_int_value(const GqaArgs& a, const BatchGeom& bg, int b, int kh, int pos, int d,
                                               bool value) {
  const float scale = gqa_scale(a, value, kh, d);
  int code;
  if (pos < bg.past) {
    const uint8_t* row =
        static_cast<const uint8_t*>(value ? a.pv : a.pk) + (((int64_t)b * a.KV + kh) * a.cap + (pos - bg.origin)) * a.cache_w;
    if (a.cache_bits == 8) {
      code = (int)reinterpret_cast<const int8_t*>(row)[d];
    } else {
      const uint8_t byte = row[d >> 1];
      code = (int)((d & 1) ? byte >> 4 : byte & 15) - 8;
    }
  } else {
    const T* src = static_cast<const T*>(value ? a.v : a.k);
    const int64_t stride = value ? a.v_stride : a.k_stride;
    code = gqa_code(to_f(src[((int64_t)b * a.new_seq + (pos - bg.past)) * stride + (int64_t)kh * a.D + d]), scale,
                    a.cache_bits);
  }
  return __fmul_rn((float)code, scale);
}

// Stored byte j of new row i (counted from the batch row's first new row) of kv head kh: an
// int8 code, or two +8-biased int4 codes (channel 2j low, 2j + 1 high).
template <typename T>
__device__ __forceinline__ uint8_t gqa_new_code_byte(const GqaArgs& a, int side, int b, int kh, int i, int j) {
  const T* x = static_cast<const T*>(side ? a.v : a.k) + ((int64_t)b * a.new_seq + i) * (side ? a.v_stride : a.k_stride) +
               (int64_t)kh * a.D;
  if (a.cache_bits == 8) return (uint8_t)(int8_t)gqa_code(to_f(x[j]), gqa_scale(a, side, kh, j), 8);
  const int d0 = 2 * j, d1 = 2 * j + 1;
  const int lo = gqa_code(to_f(x[d0]), gqa_scale(a, side, kh, d0), 4) + 8;
  const int hi = d1 < a.D ? gqa_code(to_f(x[d1]), gqa_scale(a, side, kh, d1), 4) + 8 : 8;
  return (uint8_t)(lo | (hi << 4));
}

// present rows of an integer cache: past rows copied (a separate present buffer), new rows
// encoded, the old buffer's rows past the length copied, then zero codes up to present_cap.
// One thread per stored byte of one row; grid (rows of B * KV heads).
template <typename T>
__global__ void __launch_bounds__(256) gqa_int_present_kernel(const GqaArgs a) {
  const int64_t row = blockIdx.x;  // (b * KV + kh) * pcap + r
  const int r = (int)(row % a.pcap), kh = (int)((row / a.pcap) % a.KV), b = (int)(row / ((int64_t)a.pcap * a.KV));
  const BatchGeom bg = batch_geom(a, b);
  const bool separate = a.present_separate != 0;
  const bool is_new = a.new_seq > 0 && r >= bg.past && r < bg.length;
  if (!separate && !is_new) return;  // shared buffer: only the new rows change
  const uint8_t zero = a.cache_bits == 8 ? 0 : 0x88;
  for (int side = 0; side < 2; ++side) {
    uint8_t* dst = static_cast<uint8_t*>(side ? a.ov : a.ok) + row * a.cache_w;
    const uint8_t* src = a.cap > 0 ? static_cast<const uint8_t*>(side ? a.pv : a.pk) +
                                         (((int64_t)b * a.KV + kh) * a.cap + r) * a.cache_w
                                   : nullptr;
    for (int j = threadIdx.x; j < a.cache_w; j += blockDim.x) {
      uint8_t byte = zero;
      if (is_new) {
        byte = gqa_new_code_byte<T>(a, side, b, kh, r - bg.past, j);
      } else if (r < a.cap) {
        byte = src[j];
      }
      dst[j] = byte;
    }
  }
}

// Attention over integer caches: one CTA (4 warps) per (batch, head, query row); the warps split
// the visible keys, the lanes the channels; online softmax per warp, merged in shared memory.
template <typename T, int EPL>
__global__ void __launch_bounds__(128) gqa_int_attention_kernel(const GqaArgs a) {
  constexpr int kWarps = 4;
  __shared__ float qs[32 * EPL];
  __shared__ float red_m[kWarps], red_l[kWarps];
  __shared__ float red_o[kWarps][32 * EPL];
  const int row = blockIdx.x;  // (b * H + h) * S + s
  const int s = row % a.S, h = (row / a.S) % a.H, b = row / (a.S * a.H);
  const int kh = h / a.g, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (blockIdx.x == 0 && threadIdx.x == 0) *a.status = 0;
  const BatchGeom bg = batch_geom(a, b);
  const int pos = bg.query_past + s;
  const int end = a.causal ? min(pos + 1, bg.length) : bg.length;
  const int start = max(a.window > 0 ? max(0, end - a.window) : 0, bg.origin);  // origin: see BatchGeom
  for (int d = threadIdx.x; d < 32 * EPL; d += blockDim.x)
    qs[d] = d < a.D ? to_f(static_cast<const T*>(a.q)[((int64_t)b * a.S + s) * a.q_stride + (int64_t)h * a.D + d]) : 0.f;
  __syncthreads();
  const T* bias = a.bias ? static_cast<const T*>(a.bias) + b * a.bias_bstride + (int64_t)h * a.bias_hstride +
                               (int64_t)s * a.total
                         : nullptr;
  float m = -INFINITY, l = 0.f, o[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) o[e] = 0.f;
  for (int j = start + warp; j < end; j += kWarps) {
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int d = lane + 32 * e;
      if (d < a.D) dot = fmaf(qs[d], gqa_int_value<T>(a, bg, b, kh, j, d, false), dot);
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    float x = dot * a.scale;
    if (a.softcap > 0.f) x = a.softcap * tanhf(x / a.softcap);
    if (bias) x += to_f(bias[j]);
    const float mn = fmaxf(m, x);
    const float alpha = expf(m - mn);  // m = -inf on the first key gives 0
    const float p = expf(x - mn);
    l = l * alpha + p;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int d = lane + 32 * e;
      const float vv = d < a.D ? gqa_int_value<T>(a, bg, b, kh, j, d, true) : 0.f;
      o[e] = o[e] * alpha + p * vv;
    }
    m = mn;
  }
  if (lane == 0) {
    red_m[warp] = m;
    red_l[warp] = l;
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) red_o[warp][lane + 32 * e] = o[e];
  __syncthreads();
  if (warp != 0) return;
  float M = -INFINITY;
  for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red_m[w]);
  float sink = -INFINITY;
  if (a.sink) sink = to_f(static_cast<const T*>(a.sink)[h]);
  else if (a.smooth) sink = 0.f;
  M = fmaxf(M, sink);
  float L = sink == -INFINITY ? 0.f : expf(sink - M), f[kWarps];
  for (int w = 0; w < kWarps; ++w) {
    f[w] = red_m[w] == -INFINITY ? 0.f : expf(red_m[w] - M);
    L += red_l[w] * f[w];
  }
  T* out = static_cast<T*>(a.out) + ((int64_t)b * a.S + s) * ((int64_t)a.H * a.D) + (int64_t)h * a.D;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const int d = lane + 32 * e;
    if (d >= a.D) continue;
    float acc = 0.f;
    for (int w = 0; w < kWarps; ++w) acc += red_o[w][d] * f[w];
    out[d] = from_f<T>(L > 0.f ? acc / L : 0.f);
  }
}

// present of a sliding cache (attention.rs:1341-1370): row r < after = resident(length) holds
// absolute position length - after + r, a resident past row (moved down by the reclaimed rows)
// or a new row (encoded for integer caches); rows from `after` on are zero (zero codes: 0, int4
// 0x88).  Runs after the attention, which still reads the old rows, into dk / dv: present
// itself, or workspace copies when present is the past buffer (rows move down, so an in-place
// copy would overwrite rows other CTAs have yet to read).  One CTA per (batch, kv head, row).
template <typename T>
__global__ void __launch_bounds__(128) gqa_slide_present_kernel(const GqaArgs a, void* dk, void* dv) {
  const int64_t row = blockIdx.x;  // (b * KV + kh) * cap + r
  const int r = (int)(row % a.cap), kh = (int)((row / a.cap) % a.KV), b = (int)(row / ((int64_t)a.cap * a.KV));
  const BatchGeom bg = batch_geom(a, b);
  const int after = slide_resident(bg.length, a.cap, a.slide_gap);
  const int pos = bg.length - after + r;  // absolute position held by row r < after
  for (int side = 0; side < 2; ++side) {
    if (a.cache_bits) {
      uint8_t* dst = static_cast<uint8_t*>(side ? dv : dk) + row * a.cache_w;
      const uint8_t zero = a.cache_bits == 8 ? 0 : 0x88;
      const uint8_t* src = pos < bg.past ? static_cast<const uint8_t*>(side ? a.pv : a.pk) +
                                               (((int64_t)b * a.KV + kh) * a.cap + (pos - bg.origin)) * a.cache_w
                                         : nullptr;
      for (int j = threadIdx.x; j < a.cache_w; j += blockDim.x) {
        uint8_t byte = zero;
        if (r < after) byte = src ? src[j] : gqa_new_code_byte<T>(a, side, b, kh, pos - bg.past, j);
        dst[j] = byte;
      }
    } else {
      T* dst = static_cast<T*>(side ? dv : dk) + row * a.D;
      const T* src = r < after ? key_row<T>(a, bg, b, kh, pos, side == 1) : nullptr;
      for (int d = threadIdx.x; d < a.D; d += blockDim.x) dst[d] = src ? src[d] : from_f<T>(0.f);
    }
  }
}

template <typename T>
cudaError_t launch_slide_present(const GqaArgs& a, void* dk, void* dv, cudaStream_t stream) {
  gqa_slide_present_kernel<T><<<(unsigned)((int64_t)a.B * a.KV * a.cap), 128, 0, stream>>>(a, dk, dv);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_int(const GqaArgs& a, cudaStream_t stream, int* launches) {
  if (a.ok && a.pcap > 0) {
    gqa_int_present_kernel<T><<<(unsigned)((int64_t)a.B * a.KV * a.pcap), 256, 0, stream>>>(a);
    ++*launches;
  }
  const unsigned grid = (unsigned)(a.B * a.H * a.S);
  const int epl = (a.D + 31) / 32;
  if (epl <= 2) gqa_int_attention_kernel<T, 2><<<grid, 128, 0, stream>>>(a);
  else if (epl <= 4) gqa_int_attention_kernel<T, 4><<<grid, 128, 0, stream>>>(a);
  else gqa_int_attention_kernel<T, 8><<<grid, 128, 0, stream>>>(a);
  ++*launches;
  return cudaGetLastError();
}

// ------------------------------------------------------------------ qk_output diagnostics
// attention.rs:756-787: for every (batch, head, query row) the logits of keys [0, length)
// (scale * q.k, soft-capped, plus attention_bias) where visible and 0 elsewhere (mode 1), or
// the softmax probabilities with the sink in the denominator (mode 2); columns [length, total)
// are 0.  A diagnostic path: one CTA per row recomputes the scores (twice for mode 2) from the
// query / key rows the attention kernels read.
template <typename T>
__global__ void __launch_bounds__(128) gqa_qk_kernel(const GqaArgs a) {
  extern __shared__ float qrow[];  // [D]
  __shared__ float red[2][4];
  const int row = blockIdx.x;  // (b * H + h) * S + s
  const int s = row % a.S, h = (row / a.S) % a.H, b = row / (a.S * a.H);
  const int kh = h / a.g, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const BatchGeom bg = batch_geom(a, b);
  const int pos = bg.query_past + s;
  const int end = a.causal ? min(pos + 1, bg.length) : bg.length;
  const int start = a.window > 0 ? max(0, end - a.window) : 0;
  for (int d = tid; d < a.D; d += blockDim.x)
    qrow[d] = to_f(static_cast<const T*>(a.q)[((int64_t)b * a.S + s) * a.q_stride + (int64_t)h * a.D + d]);
  __syncthreads();
  const T* bias = a.bias ? static_cast<const T*>(a.bias) + b * a.bias_bstride + (int64_t)h * a.bias_hstride +
                               (int64_t)s * a.total
                         : nullptr;
  auto logit = [&](int j) {
    float acc = 0.f;
    if (a.cache_bits) {
      for (int d = 0; d < a.D; ++d) acc = fmaf(qrow[d], gqa_int_value<T>(a, bg, b, kh, j, d, false), acc);
    } else {
      const T* krow = key_row<T>(a, bg, b, kh, j, false);
      for (int d = 0; d < a.D; ++d) acc = fmaf(qrow[d], to_f(krow[d]), acc);
    }
    float x = acc * a.scale;
    if (a.softcap > 0.f) x = a.softcap * tanhf(x / a.softcap);
    if (bias) x += to_f(bias[j]);
    return x;
  };
  T* out = static_cast<T*>(a.qk_out) + (int64_t)row * a.total;
  float M = -INFINITY, L = 0.f;
  if (a.qk_mode == 2) {  // max and sum over the visible keys (and the sink)
    float m = -INFINITY;
    for (int j = start + tid; j < end; j += blockDim.x) m = fmaxf(m, logit(j));
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[0][warp] = m;
    __syncthreads();
    M = fmaxf(fmaxf(red[0][0], red[0][1]), fmaxf(red[0][2], red[0][3]));
    float sink = -INFINITY;
    if (a.sink) sink = to_f(static_cast<const T*>(a.sink)[h]);
    else if (a.smooth) sink = 0.f;
    M = fmaxf(M, sink);
    float l = 0.f;
    for (int j = start + tid; j < end; j += blockDim.x) l += expf(logit(j) - M);
    for (int o = 16; o; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) red[1][warp] = l;
    __syncthreads();
    L = red[1][0] + red[1][1] + red[1][2] + red[1][3] + (sink == -INFINITY ? 0.f : expf(sink - M));
  }
  for (int j = tid; j < a.total; j += blockDim.x) {
    float y = 0.f;
    if (j >= start && j < end) {
      const float x = logit(j);
      y = a.qk_mode == 1 ? x : (L > 0.f ? expf(x - M) / L : 0.f);
    }
    out[j] = from_f<T>(y);
  }
}

template <typename T>
cudaError_t launch_qk(const GqaArgs& a, cudaStream_t stream) {
  gqa_qk_kernel<T><<<(unsigned)(a.B * a.H * a.S), 128, sizeof(float) * a.D, stream>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_rope(const GqaRope& r, dim3 grid, size_t smem, cudaStream_t stream) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(gqa_rope_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  gqa_rope_kernel<T><<<grid, 256, smem, stream>>>(r);
  return cudaSuccess;
}

// ------------------------------------------------------------------ host side
int gfail(int code, const std::string& msg) { return set_error(code, msg); }

int sm_count(const B200GqaParams* p) {
  if (p->num_sms > 0) return p->num_sms;
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    return 148;
  return n;
}

struct GqaPlan {
  int rows = kMaxRows, row_tiles = 1, splits = 1, fused = 0;
  size_t status = 0, counters = 0, part_o = 0, part_ml = 0, q_rot = 0, k_rot = 0, slide = 0, slide_bytes = 0,
         total = 0;
};

// Bytes of one stored cache row: integer codes (int8: D, int4: ceil(D / 2)) or D activations.
size_t cache_row_bytes(const B200GqaParams* p) {
  if (p->cache_dtype == B200_DTYPE_INT8) return (size_t)p->head_size;
  if (p->cache_dtype == B200_DTYPE_UINT8) return (size_t)(p->head_size + 1) / 2;
  return (size_t)p->head_size * (p->dtype == B200_DTYPE_FLOAT ? 4 : 2);
}

size_t act_size(int dtype) { return dtype == B200_DTYPE_FLOAT ? 4 : 2; }

GqaPlan gqa_plan(const B200GqaParams* p) {
  GqaPlan P;
  const int g = p->num_heads / p->kv_num_heads;
  const int rows_total = p->seq * g;
  P.rows = rows_total <= 4 ? 4 : rows_total <= 8 ? 8 : kMaxRows;
  P.row_tiles = (rows_total + P.rows - 1) / P.rows;
  const int64_t groups = (int64_t)p->batch * p->kv_num_heads * P.row_tiles;
  const int chunks = (std::max(p->total_sequence_length, 1) + kKeys - 1) / kKeys;
  const int target = 2 * sm_count(p);
  P.splits = groups >= target ? 1 : (int)std::min<int64_t>(std::min(chunks, kMaxSplits), (target + groups - 1) / groups);
  if (P.splits < 1) P.splits = 1;
  P.fused = P.row_tiles == 1 && !(p->local_window_size > 0);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = (off + bytes + 255) / 256 * 256;
    return at;
  };
  P.status = take(sizeof(int));
  if (p->do_rotary || p->q_norm_weight) {  // normalised / rotated query and key rows
    P.q_rot = take(act_size(p->dtype) * (size_t)p->batch * p->seq * p->num_heads * p->head_size);
    P.k_rot = take(act_size(p->dtype) * (size_t)p->batch * std::max(p->new_seq, 1) * p->kv_num_heads * p->head_size);
  }
  if (P.splits > 1) {
    P.counters = take(sizeof(int) * groups);
    P.part_o = take(sizeof(float) * groups * P.splits * P.rows * p->head_size);
    P.part_ml = take(sizeof(float) * groups * P.splits * P.rows * 2);
  }
  if (p->sliding_window_cache) {  // staged present K and V, for a present that is the past buffer
    P.slide_bytes = (size_t)p->batch * p->kv_num_heads * std::max(p->cap, 0) * cache_row_bytes(p);
    P.slide = take(2 * P.slide_bytes);
  }
  P.total = std::max<size_t>(off, 256);
  return P;
}

int check_gqa(const B200GqaParams* p) {
  if (!p) return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: null params");
  if (p->num_heads <= 0 || p->kv_num_heads <= 0 || p->num_heads % p->kv_num_heads)
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: num_heads must be a positive multiple of kv_num_heads");
  if (p->head_size <= 0 || p->head_size > kMaxD || p->head_size % 8)
    return gfail(B200_ERR_UNSUPPORTED, "GroupQueryAttention: head_size must be a multiple of 8 up to 256 on B200");
  if (!(p->dtype == B200_DTYPE_FLOAT || p->dtype == B200_DTYPE_FLOAT16 || p->dtype == B200_DTYPE_BFLOAT16))
    return gfail(B200_ERR_UNSUPPORTED, "GroupQueryAttention: activations must be float, float16 or bfloat16");
  if (p->batch < 1 || p->seq < 1 || p->new_seq < 0 || p->cap < 0)
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: bad batch / sequence / capacity");
  if (!p->query || !p->output || !p->seqlens_k || !p->host_seqlens_k)
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: missing query, output or seqlens_k");
  if (p->new_seq > 0 && (!p->key || !p->value))
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: missing key or value");
  if ((p->past_key == nullptr) != (p->past_value == nullptr) || (p->present_key == nullptr) != (p->present_value == nullptr))
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: past/present key and value must be provided together");
  if (p->cap > 0 && !p->past_key)
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: past capacity without past cache");
  if (!(p->softcap >= 0.f) || std::isinf(p->softcap))
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: softcap must be finite and non-negative");
  if (p->local_window_size < -1)
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: local_window_size must be -1 or positive");
  {
    // the kernels load K/V rows as 4-element vectors
    const size_t align = p->dtype == B200_DTYPE_FLOAT ? 16 : 8;
    const void* ptrs[] = {p->query, p->key, p->value, p->past_key, p->past_value, p->present_key, p->present_value};
    bool ok = true;
    for (const void* q : ptrs) ok &= (reinterpret_cast<uintptr_t>(q) % align) == 0;
    const int64_t strides[] = {p->query_row_stride, p->key_row_stride, p->value_row_stride};
    for (int64_t st : strides) ok &= st % 4 == 0;
    if (!ok)
      return gfail(B200_ERR_INVALID_ARGUMENT,
                   "GroupQueryAttention: tensors must be aligned to 4 elements (16 bytes for float, 8 for 16-bit)");
  }
  if (p->do_rotary) {
    if (!p->cos_cache || !p->sin_cache)
      return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: do_rotary=1 requires cos_cache and sin_cache");
    if (p->rotary_dim <= 0 || p->rotary_dim % 2 || p->rotary_dim > p->head_size || p->rotary_positions <= 0)
      return gfail(B200_ERR_INVALID_ARGUMENT,
                   "rotary caches must have matching [positions,rotary_dim/2] shapes within the head");
    if (p->position_ids && !p->host_position_ids)
      return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: position_ids need their host copy (host_position_ids)");
  }
  if (p->cache_dtype != 0 && p->cache_dtype != p->dtype && p->cache_dtype != B200_DTYPE_INT8 &&
      p->cache_dtype != B200_DTYPE_UINT8)
    return gfail(B200_ERR_UNSUPPORTED, "GroupQueryAttention: caches must be in the activation type, int8 or int4");
  if ((p->cache_dtype == B200_DTYPE_INT8 || p->cache_dtype == B200_DTYPE_UINT8)) {
    if (!p->k_scale || !p->v_scale)
      return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: integer caches require k_scale and v_scale");
    if (p->cache_dtype == B200_DTYPE_UINT8 && p->head_size % 2)
      return gfail(B200_ERR_INVALID_ARGUMENT,
                   "GQA packed INT4 requires an even logical head size (pinned CheckPast byte geometry)");
  }
  if (p->qk_output < 0 || p->qk_output > 2 || (p->qk_output != 0) != (p->output_qk != nullptr))
    return gfail(B200_ERR_INVALID_ARGUMENT,
                 "qk_output must be 0, 1 or 2 and enabled exactly when output_qk is present");
  if ((p->q_norm_weight == nullptr) != (p->k_norm_weight == nullptr))
    return gfail(B200_ERR_INVALID_ARGUMENT, "q_norm_weight and k_norm_weight must be provided together");
  if ((p->do_rotary || p->q_norm_weight) &&
      gqa_rope_smem(p->num_heads, p->kv_num_heads, p->head_size) > 227 * 1024)
    return gfail(B200_ERR_UNSUPPORTED, "GroupQueryAttention: the query and key heads of one row exceed the prologue's "
                                       "shared memory");
  // attention.rs:637-652 (a sliding cache checks the bias with its own message, at run time)
  if (p->attention_bias && !p->sliding_window_cache &&
      ((p->bias_batch != 1 && p->bias_batch != p->batch) || (p->bias_heads != 1 && p->bias_heads != p->num_heads) ||
       p->bias_seq != p->seq || p->bias_total != p->total_sequence_length))
    return gfail(B200_ERR_FAIL, "GroupQueryAttention: attention_bias must broadcast to [batch,heads,sequence,total]");
  // attention.rs:992-997
  if (p->new_seq != p->seq && (p->new_seq != 0 || !p->past_key || p->sliding_window_cache))
    return gfail(B200_ERR_FAIL, "GroupQueryAttention: K/V must match Q sequence or be empty with paired non-sliding past");
  if (p->sliding_window_cache) {  // attention.rs:2455-2475, :2735-2738
    if (!p->present_key)
      return gfail(B200_ERR_INVALID_ARGUMENT, "sliding_window_cache requires present key/value outputs");
    if (p->qk_output)
      return gfail(B200_ERR_UNSUPPORTED, "sliding_window_cache with QK diagnostics is unsupported");
    if ((int64_t)p->batch * p->kv_num_heads * std::max(p->cap, 1) > INT32_MAX)
      return gfail(B200_ERR_UNSUPPORTED, "GroupQueryAttention: sliding cache rows exceed one launch");
  }
  return B200_OK;
}

// Runtime checks of a sliding cache, in the reference's order and words (attention.rs:
// 1140-1171): every length in [seq - 1, total - 1] with the maximum total - 1; a bias with
// absolute [.., seq, total] columns; 0 < local_window_size <= capacity.  present keeps the
// past's capacity (the reference's present is that buffer).
int validate_sliding(const B200GqaParams* p) {
  const int64_t total = p->total_sequence_length;
  const int32_t* L = p->host_seqlens_k;
  bool bad = total <= 0;
  int64_t mx = -1;
  for (int b = 0; b < p->batch; ++b) {
    const int64_t n = L[b];
    if (n < 0 || n >= total || n + 1 < p->seq) bad = true;
    mx = std::max(mx, n);
  }
  if (bad || mx != total - 1) return gfail(B200_ERR_FAIL, "GroupQueryAttention: invalid sliding sequence lengths");
  if (p->attention_bias &&
      ((p->bias_batch != 1 && p->bias_batch != p->batch) || (p->bias_heads != 1 && p->bias_heads != p->num_heads) ||
       p->bias_seq != p->seq || p->bias_total != total))
    return gfail(B200_ERR_FAIL,
                 "GroupQueryAttention: sliding attention_bias requires absolute total_sequence_length columns");
  if (p->local_window_size <= 0 || p->cap < p->local_window_size)
    return gfail(B200_ERR_FAIL, "GroupQueryAttention: sliding cache requires 0 < local_window_size <= capacity");
  if (p->present_cap != p->cap)
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: a sliding present must have the past's capacity");
  return B200_OK;
}

// Runtime length checks with the reference's messages.  The single-batch route of the
// reference (:1014-1025, taken when b == 1 with a past, causal, no window, not composed and
// new rows present) checks seqlens_k == [total - 1] and 0 <= total - S <= cap; the batched
// route (:613-630, :668-673) checks every length and the past capacity.
int validate_lengths(const B200GqaParams* p) {
  const int64_t total = p->total_sequence_length;
  if (total < 0 || total > INT32_MAX)
    return gfail(B200_ERR_FAIL, "GroupQueryAttention: total_sequence_length is outside int32 range");
  const bool composed = p->softcap > 0.f || p->smooth_softmax == 1 || p->head_sink != nullptr;
  const bool single = p->batch == 1 && p->past_key && p->is_causal && p->local_window_size < 0 && !composed &&
                      p->new_seq != 0;
  const int32_t* L = p->host_seqlens_k;
  if (single) {
    const int64_t vp = total - p->new_seq;
    if ((int64_t)L[0] != total - 1 || vp < 0 || vp > p->cap)
      return gfail(B200_ERR_FAIL, "GroupQueryAttention: inconsistent sequence lengths or cache capacity");
  } else {
    bool bad = total <= 0;
    int64_t mx = -1;
    for (int b = 0; b < p->batch && !bad; ++b) {
      const int64_t n = L[b];
      if (n < 0 || n >= total || (total != p->seq && n + 1 < p->seq)) bad = true;
      mx = std::max(mx, n);
    }
    if (bad || mx != total - 1)
      return gfail(B200_ERR_FAIL, "GroupQueryAttention: invalid per-batch or maximum sequence lengths");
  }
  for (int b = 0; b < p->batch; ++b) {
    const int length = L[b] + 1;
    const int query_past = std::max(length - p->seq, 0);
    const int past = p->new_seq == 0 ? length : query_past;
    if (past > p->cap || (!p->past_key && past != 0))
      return gfail(B200_ERR_FAIL, "GroupQueryAttention: sequence length exceeds available past cache");
  }
  if (p->present_key && p->present_cap < std::max<int64_t>(p->cap, total))
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: present capacity must be max(cap, total_sequence_length)");
  if (p->present_key && p->present_key == p->past_key && p->present_cap != p->cap)
    return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: an in-place present must have the past's capacity");
  return B200_OK;
}

// Rotary positions (gqa_rotary_rows, attention.rs:538-585; cos_sin_row :525-536): without
// position_ids row s of batch b sits at query_past + s; with them, a first prompt (total ==
// seq) uses only the first id as an offset, later calls the first batch * seq flattened ids.
int validate_rotary(const B200GqaParams* p) {
  if (!p->do_rotary) return B200_OK;
  const int64_t rows = p->rotary_positions, seq = p->seq;
  if (!p->position_ids) {
    for (int b = 0; b < p->batch; ++b) {
      const int64_t query_past = std::max<int64_t>((int64_t)p->host_seqlens_k[b] + 1 - seq, 0);
      if (query_past > rows - seq)
        return gfail(B200_ERR_FAIL, "RotaryEmbedding: requested positions exceed the supplied cache");
    }
    return B200_OK;
  }
  if (p->position_ids_width < p->seq)
    return gfail(B200_ERR_FAIL, "GroupQueryAttention: position_ids must be int64 [batch,>=sequence]");
  const int64_t* ids = p->host_position_ids;
  if ((int64_t)p->total_sequence_length == seq) {
    if (ids[0] < 0 || ids[0] > rows - seq)
      return gfail(B200_ERR_FAIL, "GroupQueryAttention: position_ids exceed the supplied cache");
    return B200_OK;
  }
  for (int64_t i = 0; i < (int64_t)p->batch * seq; ++i)
    if (ids[i] < 0 || ids[i] >= rows)
      return gfail(B200_ERR_FAIL, "GroupQueryAttention: position_ids exceed the supplied cache");
  return B200_OK;
}

// Cluster path (decode-shaped groups: one row tile covers every key, no window).
constexpr size_t kClSmemBudget = 220 * 1024;

bool cluster_path(const B200GqaParams* p, const GqaPlan& P) {
  const int D = p->head_size;
  if (!P.fused || !(D == 64 || D == 128 || D == 256)) return false;
  for (const void* ptr : {(const void*)p->past_key, (const void*)p->past_value, (const void*)p->present_key,
                          (const void*)p->present_value})
    if (reinterpret_cast<uintptr_t>(ptr) % 16) return false;  // bulk copies move 16-byte units
  return true;
}

// Active clusters per (kernel, cluster size, shared memory, device), queried once each.
struct OccKey {
  const void* kern;
  int cl;
  size_t smem;
  int dev;
  bool operator<(const OccKey& o) const { return std::tie(kern, cl, smem, dev) < std::tie(o.kern, o.cl, o.smem, o.dev); }
};

template <typename T, int R, int D>
cudaError_t launch_cluster_rd(const GqaArgs& a, cudaStream_t stream) {
  static std::mutex mu;
  static std::map<OccKey, int> occ;
  static std::map<std::pair<const void*, int>, bool> prepared;
  auto kern = gqa_cluster_kernel<T, R, D>;
  const void* kp = reinterpret_cast<const void*>(kern);
  constexpr int esz = (int)sizeof(T);
  int kc_max = 0;  // the most keys per staging chunk that fit the shared-memory budget
  for (int kc = 16; kc <= 512; kc += 16)
    if (cluster_smem_bytes(R, D, esz, kc) <= kClSmemBudget) kc_max = kc;
  if (kc_max < 16) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;

  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kClThreads);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;

  // Cluster size: fewest waves of clusters times keys per CTA (each staging chunk also costs a
  // memory round trip, worth about 256 keys), from the device's own count of co-resident
  // clusters.
  const int64_t groups = (int64_t)a.B * a.KV;
  const int maxlen = std::max(a.total, 1);
  int best_cl = 0, best_kc = 0;
  double best_cost = 0.0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!prepared[{kp, dev}]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cluster_smem_bytes(R, D, esz, kc_max));
      if (e != cudaSuccess) return e;
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
      prepared[{kp, dev}] = true;
    }
    for (int cl = kClMaxCluster; cl >= 1; --cl) {
      const int per_cta = (maxlen + cl - 1) / cl;
      const int kc = std::min(kc_max, (per_cta + 15) / 16 * 16);
      const size_t smem = cluster_smem_bytes(R, D, esz, kc);
      const OccKey key{kp, cl, smem, dev};
      auto it = occ.find(key);
      int active = 0;
      if (it != occ.end()) {
        active = it->second;
      } else {
        attr[0].val.clusterDim.x = cl;
        cfg.gridDim = dim3((unsigned)cl);
        cfg.dynamicSmemBytes = smem;
        if (cudaOccupancyMaxActiveClusters(&active, kern, &cfg) != cudaSuccess) active = 0;
        cudaGetLastError();  // a refused size is not an error of the call
        occ[key] = active;
      }
      if (active <= 0) continue;
      const int64_t waves = (groups + active - 1) / active;
      const int chunks = (per_cta + kc - 1) / kc;
      const double cost = (double)waves * (per_cta + 256.0 * chunks);
      if (best_cl == 0 || cost < best_cost) {
        best_cl = cl;
        best_kc = kc;
        best_cost = cost;
      }
    }
  }
  if (best_cl == 0) return cudaErrorLaunchOutOfResources;
  attr[0].val.clusterDim.x = best_cl;
  cfg.gridDim = dim3((unsigned)(groups * best_cl));
  cfg.dynamicSmemBytes = cluster_smem_bytes(R, D, esz, best_kc);
  return cudaLaunchKernelEx(&cfg, kern, a, best_kc);
}

template <typename T, int R>
cudaError_t launch_cluster_r(const GqaArgs& a, cudaStream_t stream) {
  if (a.D == 64) return launch_cluster_rd<T, R, 64>(a, stream);
  if (a.D == 128) return launch_cluster_rd<T, R, 128>(a, stream);
  return launch_cluster_rd<T, R, 256>(a, stream);
}

template <typename T>
cudaError_t launch_cluster(const GqaArgs& a, const GqaPlan& P, cudaStream_t stream) {
  if (P.rows == 4) return launch_cluster_r<T, 4>(a, stream);
  if (P.rows == 8) return launch_cluster_r<T, 8>(a, stream);
  return launch_cluster_r<T, kMaxRows>(a, stream);
}

template <typename T>
cudaError_t launch_gqa(const GqaArgs& a, const GqaPlan& P, bool cluster, bool tail_rows, cudaStream_t stream,
                       int* launches) {
  if (cluster) {
    cudaError_t e = launch_cluster<T>(a, P, stream);
    ++*launches;
    if (e != cudaSuccess) return e;
    if (a.ok != nullptr && a.present_separate && tail_rows) {
      const int64_t n = (int64_t)a.B * a.KV * a.pcap * a.D;
      const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
      gqa_present_kernel<T><<<blocks, 256, 0, stream>>>(a, 1);
      ++*launches;
      e = cudaGetLastError();
    }
    return e;
  }
  const int64_t grid = (int64_t)a.B * a.KV * a.row_tiles * a.splits;
  if (P.splits > 1) {
    cudaError_t e = cudaMemsetAsync(a.counters, 0, sizeof(int) * (size_t)a.B * a.KV * a.row_tiles, stream);
    if (e != cudaSuccess) return e;
    ++*launches;
  }
  const bool two = a.D > kThreads;
  if (P.rows == 4) {
    if (two) gqa_attention_kernel<T, 4, 2><<<(unsigned)grid, kThreads, 0, stream>>>(a);
    else gqa_attention_kernel<T, 4, 1><<<(unsigned)grid, kThreads, 0, stream>>>(a);
  } else if (P.rows == 8) {
    if (two) gqa_attention_kernel<T, 8, 2><<<(unsigned)grid, kThreads, 0, stream>>>(a);
    else gqa_attention_kernel<T, 8, 1><<<(unsigned)grid, kThreads, 0, stream>>>(a);
  } else {
    if (two) gqa_attention_kernel<T, kMaxRows, 2><<<(unsigned)grid, kThreads, 0, stream>>>(a);
    else gqa_attention_kernel<T, kMaxRows, 1><<<(unsigned)grid, kThreads, 0, stream>>>(a);
  }
  ++*launches;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const bool need_copy = a.ok != nullptr && (!a.fused_copy || (a.present_separate && tail_rows));
  if (need_copy) {
    const int64_t n = (int64_t)a.B * a.KV * a.pcap * a.D;
    const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 16);
    gqa_present_kernel<T><<<blocks, 256, 0, stream>>>(a, a.fused_copy);
    ++*launches;
    e = cudaGetLastError();
  }
  return e;
}

}  // namespace
}  // namespace b200

extern "C" {

int b200_gqa_params_size(void) { return (int)sizeof(B200GqaParams); }

int b200_group_query_attention_workspace_size(const B200GqaParams* p, size_t* bytes) {
  int rc = b200::check_gqa(p);
  if (rc) return rc;
  if (!bytes) return b200::gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: null bytes pointer");
  *bytes = b200::gqa_plan(p).total;
  return B200_OK;
}

int b200_group_query_attention(const B200GqaParams* p, void* stream_ptr) {
  using namespace b200;
  try {
    int rc = check_gqa(p);
    if (rc) return rc;
    rc = p->sliding_window_cache ? validate_sliding(p) : validate_lengths(p);
    if (rc) return rc;
    rc = validate_rotary(p);
    if (rc) return rc;
    const GqaPlan P = gqa_plan(p);
    if (!p->workspace || p->workspace_bytes < P.total)
      return gfail(B200_ERR_WORKSPACE, "GroupQueryAttention: workspace missing or smaller than b200_group_query_attention_workspace_size()");
    GqaArgs a{};
    a.H = p->num_heads;
    a.KV = p->kv_num_heads;
    a.D = p->head_size;
    a.g = a.H / a.KV;
    a.B = p->batch;
    a.S = p->seq;
    a.new_seq = p->new_seq;
    a.cap = p->cap;
    a.pcap = p->present_key ? p->present_cap : 0;
    a.total = p->total_sequence_length;
    a.causal = p->is_causal;
    a.window = p->local_window_size > 0 ? p->local_window_size : 0;
    a.smooth = p->smooth_softmax == 1;
    a.dtype = p->dtype;
    a.scale = p->scale != 0.f ? p->scale : 1.0f / std::sqrt((float)p->head_size);
    a.softcap = p->softcap;
    a.q_stride = p->query_row_stride ? p->query_row_stride : (int64_t)a.H * a.D;
    a.k_stride = p->key_row_stride ? p->key_row_stride : (int64_t)a.KV * a.D;
    a.v_stride = p->value_row_stride ? p->value_row_stride : (int64_t)a.KV * a.D;
    a.q = p->query;
    a.k = p->key;
    a.v = p->value;
    a.pk = p->past_key;
    a.pv = p->past_value;
    a.ok = p->present_key;
    a.ov = p->present_value;
    a.seqlens = p->seqlens_k;
    a.sink = p->head_sink;
    if (p->attention_bias) {
      a.bias = p->attention_bias;
      const int64_t plane = (int64_t)p->seq * p->bias_total;
      a.bias_hstride = p->bias_heads == 1 ? 0 : plane;
      a.bias_bstride = p->bias_batch == 1 ? 0 : plane * p->bias_heads;
    }
    a.out = p->output;
    a.row_tiles = P.row_tiles;
    a.splits = P.splits;
    a.fused_copy = P.fused && p->present_key != nullptr;
    a.present_separate = p->present_key != nullptr && p->present_key != p->past_key;
    if (p->cache_dtype == B200_DTYPE_INT8 || p->cache_dtype == B200_DTYPE_UINT8) {
      a.cache_bits = p->cache_dtype == B200_DTYPE_INT8 ? 8 : 4;
      a.cache_w = a.cache_bits == 8 ? a.D : (a.D + 1) / 2;
      a.kscale = p->k_scale;
      a.vscale = p->v_scale;
      a.kpc = p->k_quant_per_channel != 0;
      a.vpc = p->v_quant_per_channel != 0;
    }
    if (p->sliding_window_cache) {
      a.sliding = 1;
      a.slide_gap = p->cap - p->local_window_size + 1;
    }
    char* ws = static_cast<char*>(p->workspace);
    a.status = reinterpret_cast<int*>(ws + P.status);
    if (P.splits > 1) {
      a.counters = reinterpret_cast<int*>(ws + P.counters);
      a.part_o = reinterpret_cast<float*>(ws + P.part_o);
      a.part_ml = reinterpret_cast<float*>(ws + P.part_ml);
    }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    int launches = 0;
    cudaError_t e;
    if (p->do_rotary || p->q_norm_weight) {  // normalise / rotate the new rows first; the attention
                                             // kernels read the processed copies
      GqaRope r{};
      r.H = a.H;
      r.KV = a.KV;
      r.D = a.D;
      r.S = a.S;
      r.new_seq = a.new_seq;
      r.do_rotary = p->do_rotary != 0;
      r.qw = p->q_norm_weight;
      r.kw = p->k_norm_weight;
      r.eps = p->qk_norm_epsilon > 0.f ? p->qk_norm_epsilon : 1e-6f;
      r.half = p->rotary_dim / 2;
      r.interleaved = p->rotary_interleaved != 0;
      r.rows = p->rotary_positions;
      r.first_prompt = p->total_sequence_length == p->seq;
      r.q_stride = a.q_stride;
      r.k_stride = a.k_stride;
      r.q = a.q;
      r.k = a.k;
      r.cos = p->cos_cache;
      r.sin = p->sin_cache;
      r.seqlens = p->seqlens_k;
      r.pos_ids = p->position_ids;
      r.q_out = ws + P.q_rot;
      r.k_out = ws + P.k_rot;
      const dim3 grid((unsigned)(a.B * a.S));
      const size_t smem = gqa_rope_smem(a.H, a.KV, a.D);
      if (a.dtype == B200_DTYPE_FLOAT) e = launch_rope<float>(r, grid, smem, stream);
      else if (a.dtype == B200_DTYPE_FLOAT16) e = launch_rope<__half>(r, grid, smem, stream);
      else e = launch_rope<__nv_bfloat16>(r, grid, smem, stream);
      if (e == cudaSuccess) e = cudaGetLastError();
      if (e != cudaSuccess) return gfail(B200_ERR_CUDA, std::string("GroupQueryAttention: CUDA error: ") + cudaGetErrorString(e));
      add_launches(1);
      a.q = r.q_out;
      a.q_stride = (int64_t)a.H * a.D;
      if (a.new_seq > 0) {
        a.k = r.k_out;
        a.k_stride = (int64_t)a.KV * a.D;
      }
    }
    // A sliding cache's present is written after the attention (its rows move), so the
    // attention launches see no present.
    GqaArgs run = a;
    if (a.sliding) {
      run.ok = run.ov = nullptr;
      run.fused_copy = 0;
    }
    if (a.cache_bits) {  // integer caches: the codec kernels (a correctness path)
      if (a.dtype == B200_DTYPE_FLOAT) e = launch_int<float>(run, stream, &launches);
      else if (a.dtype == B200_DTYPE_FLOAT16) e = launch_int<__half>(run, stream, &launches);
      else e = launch_int<__nv_bfloat16>(run, stream, &launches);
    } else {
      // Rows past some batch's length exist in present only when a length is below its capacity.
      bool tail_rows = false;
      for (int b = 0; b < p->batch; ++b) tail_rows |= p->host_seqlens_k[b] + 1 < a.pcap;
      const bool cluster = cluster_path(p, P);
      if (a.dtype == B200_DTYPE_FLOAT) e = launch_gqa<float>(run, P, cluster, tail_rows, stream, &launches);
      else if (a.dtype == B200_DTYPE_FLOAT16) e = launch_gqa<__half>(run, P, cluster, tail_rows, stream, &launches);
      else e = launch_gqa<__nv_bfloat16>(run, P, cluster, tail_rows, stream, &launches);
    }
    if (e == cudaSuccess && a.sliding && a.cap > 0) {
      const bool in_place = p->present_key == p->past_key || p->present_value == p->past_value ||
                            p->present_key == p->past_value || p->present_value == p->past_key;
      void* dk = in_place ? static_cast<void*>(ws + P.slide) : a.ok;
      void* dv = in_place ? static_cast<void*>(ws + P.slide + P.slide_bytes) : a.ov;
      if (a.dtype == B200_DTYPE_FLOAT) e = launch_slide_present<float>(a, dk, dv, stream);
      else if (a.dtype == B200_DTYPE_FLOAT16) e = launch_slide_present<__half>(a, dk, dv, stream);
      else e = launch_slide_present<__nv_bfloat16>(a, dk, dv, stream);
      ++launches;
      if (e == cudaSuccess && in_place) {
        e = cudaMemcpyAsync(a.ok, dk, P.slide_bytes, cudaMemcpyDeviceToDevice, stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(a.ov, dv, P.slide_bytes, cudaMemcpyDeviceToDevice, stream);
      }
    }
    add_launches(launches);
    if (e == cudaSuccess && p->qk_output) {  // diagnostics after the attention of the call
      a.qk_out = p->output_qk;
      a.qk_mode = p->qk_output;
      if (a.dtype == B200_DTYPE_FLOAT) e = launch_qk<float>(a, stream);
      else if (a.dtype == B200_DTYPE_FLOAT16) e = launch_qk<__half>(a, stream);
      else e = launch_qk<__nv_bfloat16>(a, stream);
      add_launches(1);
    }
    if (e != cudaSuccess)
      return gfail(B200_ERR_CUDA, std::string("GroupQueryAttention: CUDA error: ") + cudaGetErrorString(e));
    return B200_OK;
  } catch (const std::exception& ex) {
    return gfail(B200_ERR_FAIL, std::string("GroupQueryAttention: ") + ex.what());
  } catch (...) {
    return gfail(B200_ERR_FAIL, "GroupQueryAttention: unknown failure");
  }
}

int b200_group_query_attention_read_status(const B200GqaParams* p, void* stream_ptr) {
  using namespace b200;
  if (!p || !p->workspace) return gfail(B200_ERR_INVALID_ARGUMENT, "GroupQueryAttention: no workspace");
  const GqaPlan P = gqa_plan(p);
  int bits = 0;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  cudaError_t e = cudaMemcpyAsync(&bits, static_cast<char*>(p->workspace) + P.status, sizeof(int),
                                  cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess)
    return gfail(B200_ERR_CUDA, std::string("GroupQueryAttention: CUDA error: ") + cudaGetErrorString(e));
  if (bits == 0) return B200_OK;
  if (bits & kStatusTimeout)
    return gfail(B200_ERR_DEVICE, "GroupQueryAttention: a device wait timed out (bulk copy did not complete)");
  return gfail(B200_ERR_DEVICE, "GroupQueryAttention: device status " + std::to_string(bits));
}

}  // extern "C"
