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
#include <cstring>
#include <string>
#include <vector>

#include "b200_common.cuh"
#include "b200_kernels.h"

namespace b200 {
namespace {

constexpr int kRows = 16;      // query rows per CTA
constexpr int kKeys = 64;      // keys per chunk
constexpr int kThreads = 128;
constexpr int kMaxD = 256;
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
  void* out;
  int row_tiles, splits, fused_copy, present_separate;
  float* part_o;   // [groups][splits][kRows][D]
  float* part_ml;  // [groups][splits][kRows][2]
  int* counters;   // [groups]
};

template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// Per batch row (:662-667): length, query_past, past (rows taken from the past cache).
struct BatchGeom {
  int length, query_past, past;
};
__device__ __forceinline__ BatchGeom batch_geom(const GqaArgs& a, int b) {
  BatchGeom g;
  g.length = a.seqlens[b] + 1;
  g.query_past = max(g.length - a.S, 0);
  g.past = a.new_seq == 0 ? g.length : g.query_past;
  return g;
}

// Row `pos` of kv head kh of batch b: past cache below `past`, new input rows from there on.
template <typename T>
__device__ __forceinline__ const T* key_row(const GqaArgs& a, const BatchGeom& bg, int b, int kh, int pos, bool value) {
  if (pos < bg.past) {
    const T* base = static_cast<const T*>(value ? a.pv : a.pk);
    return base + (((int64_t)b * a.KV + kh) * a.cap + pos) * a.D;
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

template <typename T>
__global__ void __launch_bounds__(kThreads) gqa_attention_kernel(const GqaArgs a) {
  __shared__ float qs[kRows][kMaxD];
  __shared__ float sc[kRows][kKeys + 1];
  __shared__ float m_run[kRows], l_run[kRows], alpha_s[kRows];
  __shared__ int row_pos[kRows];  // absolute position of each row, or -1 (padding row)
  __shared__ int row_end[kRows], row_start[kRows];

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

  // Query rows of this tile (fp32, pre-scaled into the log2 domain unless softcap is on).
  const float qmul = a.softcap > 0.f ? 1.f : a.scale * kLog2e;
  for (int i = tid; i < kRows * D; i += kThreads) {
    const int r = i / D, d = i % D, rho = rt * kRows + r;
    float x = 0.f;
    if (rho < rows_total) {
      const int s = rho / g, hl = rho % g;
      x = to_f(static_cast<const T*>(a.q)[((int64_t)b * a.S + s) * a.q_stride + (int64_t)(kh * g + hl) * D + d]) * qmul;
    }
    qs[r][d] = x;
  }
  if (tid < kRows) {
    const int rho = rt * kRows + tid;
    if (rho < rows_total) {
      const int pos = bg.query_past + rho / g;
      const int end = a.causal ? min(pos + 1, bg.length) : bg.length;
      row_pos[tid] = pos;
      row_end[tid] = end;
      row_start[tid] = a.window > 0 ? max(0, end - a.window) : 0;
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
  for (int r = 0; r < kRows; ++r)
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
  float o[kRows][2];
#pragma unroll
  for (int r = 0; r < kRows; ++r) o[r][0] = o[r][1] = 0.f;
  const int d0 = tid, d1 = tid + kThreads;

  for (int c = my_lo; c < my_hi; ++c) {
    // ---- scores: thread = (key kk, channel half)
    {
      const int kk = tid >> 1, half = tid & 1;
      const int pos = c * kKeys + kk;
      float acc[kRows];
#pragma unroll
      for (int r = 0; r < kRows; ++r) acc[r] = 0.f;
      if (pos < bg.length) {
        const T* krow = key_row<T>(a, bg, b, kh, pos, false);
        const bool copy = a.fused_copy && (a.present_separate || pos >= bg.past);
        T* kdst = copy ? present_row<T>(a, b, kh, pos, false) : nullptr;
        const int dh = D / 2, dbeg = half * dh;
        for (int d = dbeg; d < dbeg + dh; d += 4) {
          float kx[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const T kv = krow[d + e];
            kx[e] = to_f(kv);
            if (copy) kdst[d + e] = kv;
          }
#pragma unroll
          for (int r = 0; r < kRows; ++r) {
            const float4 qv = *reinterpret_cast<const float4*>(&qs[r][d]);
            acc[r] = fmaf(qv.x, kx[0], fmaf(qv.y, kx[1], fmaf(qv.z, kx[2], fmaf(qv.w, kx[3], acc[r]))));
          }
        }
      }
#pragma unroll
      for (int r = 0; r < kRows; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], 1);
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        if ((r >> 3) != half) continue;
        float s = -INFINITY;
        if (row_pos[r] >= 0 && pos >= row_start[r] && pos < row_end[r]) {
          s = acc[r];
          if (a.softcap > 0.f) s = a.softcap * tanhf(s * a.scale / a.softcap) * kLog2e;
        }
        sc[r][kk] = s;
      }
    }
    __syncthreads();
    // ---- online softmax: warp w owns rows 4w..4w+3, lane = keys 2*lane, 2*lane+1
#pragma unroll
    for (int rr = 0; rr < kRows / 4; ++rr) {
      const int r = warp * (kRows / 4) + rr;
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
      for (int r = 0; r < kRows; ++r) {
        const float al = alpha_s[r];
        o[r][0] *= al;
        o[r][1] *= al;
      }
      const int kend = min(kKeys, bg.length - c * kKeys);
      for (int kk = 0; kk < kend; ++kk) {
        const int pos = c * kKeys + kk;
        const T* vrow = key_row<T>(a, bg, b, kh, pos, true);
        const bool copy = a.fused_copy && (a.present_separate || pos >= bg.past);
        T* vdst = copy ? present_row<T>(a, b, kh, pos, true) : nullptr;
        float v0 = 0.f, v1 = 0.f;
        if (d0 < D) {
          const T x = vrow[d0];
          v0 = to_f(x);
          if (copy) vdst[d0] = x;
        }
        if (d1 < D) {
          const T x = vrow[d1];
          v1 = to_f(x);
          if (copy) vdst[d1] = x;
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          const float p = sc[r][kk];
          o[r][0] = fmaf(p, v0, o[r][0]);
          o[r][1] = fmaf(p, v1, o[r][1]);
        }
      }
    }
    __syncthreads();
  }

  // ---- finish: direct output, or partial + last-CTA merge
  auto sink_log2 = [&](int r) -> float {
    if (a.sink == nullptr && !a.smooth) return -INFINITY;
    const int hl = (rt * kRows + r) % g;
    const float s = a.sink ? to_f(static_cast<const T*>(a.sink)[kh * g + hl]) : 0.f;
    return s * kLog2e;
  };
  auto store_row = [&](int r, int d, float v) {
    const int rho = rt * kRows + r;
    const int s = rho / g, hl = rho % g;
    static_cast<T*>(a.out)[((int64_t)b * a.S + s) * a.H * D + (int64_t)(kh * g + hl) * D + d] = from_f<T>(v);
  };
  if (a.splits == 1) {
    for (int r = 0; r < kRows; ++r) {
      if (row_pos[r] < 0) continue;
      const float m = m_run[r], mu = m == -INFINITY ? 0.f : m;
      float L = l_run[r];
      const float sk = sink_log2(r);
      if (sk != -INFINITY) L += exp2f(sk - mu);
      const float inv = L > 0.f ? 1.f / L : 0.f;
      if (d0 < D) store_row(r, d0, o[r][0] * inv);
      if (d1 < D) store_row(r, d1, o[r][1] * inv);
    }
    return;
  }
  {
    float* po = a.part_o + ((int64_t)group * a.splits + sp) * kRows * D;
    float* pml = a.part_ml + ((int64_t)group * a.splits + sp) * kRows * 2;
    for (int r = 0; r < kRows; ++r) {
      if (d0 < D) po[r * D + d0] = o[r][0];
      if (d1 < D) po[r * D + d1] = o[r][1];
    }
    if (tid < kRows) {
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
  for (int r = 0; r < kRows; ++r) {
    if (row_pos[r] < 0) continue;
    const float* pml = a.part_ml + (int64_t)group * a.splits * kRows * 2;
    float M = -INFINITY;
    for (int j = 0; j < a.splits; ++j) M = fmaxf(M, __ldcg(&pml[(j * kRows + r) * 2]));
    const float mu = M == -INFINITY ? 0.f : M;
    float L = 0.f, acc0 = 0.f, acc1 = 0.f;
    for (int j = 0; j < a.splits; ++j) {
      const float mj = __ldcg(&pml[(j * kRows + r) * 2]);
      const float w = mj == -INFINITY ? 0.f : exp2f(mj - mu);
      L += w * __ldcg(&pml[(j * kRows + r) * 2 + 1]);
      const float* po = a.part_o + ((int64_t)group * a.splits + j) * kRows * D + r * D;
      if (d0 < D) acc0 += w * __ldcg(&po[d0]);
      if (d1 < D) acc1 += w * __ldcg(&po[d1]);
    }
    const float sk = sink_log2(r);
    if (sk != -INFINITY) L += exp2f(sk - mu);
    const float inv = L > 0.f ? 1.f / L : 0.f;
    if (d0 < D) store_row(r, d0, acc0 * inv);
    if (d1 < D) store_row(r, d1, acc1 * inv);
  }
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
  int row_tiles = 1, splits = 1, fused = 0;
  size_t counters = 0, part_o = 0, part_ml = 0, total = 0;
};

GqaPlan gqa_plan(const B200GqaParams* p) {
  GqaPlan P;
  const int g = p->num_heads / p->kv_num_heads;
  P.row_tiles = (p->seq * g + kRows - 1) / kRows;
  const int64_t groups = (int64_t)p->batch * p->kv_num_heads * P.row_tiles;
  const int chunks = (std::max(p->total_sequence_length, 1) + kKeys - 1) / kKeys;
  const int target = 2 * sm_count(p);
  P.splits = groups >= target ? 1 : (int)std::min<int64_t>(chunks, (target + groups - 1) / groups);
  if (P.splits < 1) P.splits = 1;
  P.fused = P.row_tiles == 1 && !(p->local_window_size > 0);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = (off + bytes + 255) / 256 * 256;
    return at;
  };
  if (P.splits > 1) {
    P.counters = take(sizeof(int) * groups);
    P.part_o = take(sizeof(float) * groups * P.splits * kRows * p->head_size);
    P.part_ml = take(sizeof(float) * groups * P.splits * kRows * 2);
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
  // attention.rs:992-997
  if (p->new_seq != p->seq && (p->new_seq != 0 || !p->past_key))
    return gfail(B200_ERR_FAIL, "GroupQueryAttention: K/V must match Q sequence or be empty with paired non-sliding past");
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

template <typename T>
cudaError_t launch_gqa(const GqaArgs& a, const GqaPlan& P, bool tail_rows, cudaStream_t stream, int* launches) {
  const int64_t grid = (int64_t)a.B * a.KV * a.row_tiles * a.splits;
  if (P.splits > 1) {
    cudaError_t e = cudaMemsetAsync(a.counters, 0, sizeof(int) * (size_t)a.B * a.KV * a.row_tiles, stream);
    if (e != cudaSuccess) return e;
    ++*launches;
  }
  gqa_attention_kernel<T><<<(unsigned)grid, kThreads, 0, stream>>>(a);
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
    rc = validate_lengths(p);
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
    a.out = p->output;
    a.row_tiles = P.row_tiles;
    a.splits = P.splits;
    a.fused_copy = P.fused && p->present_key != nullptr;
    a.present_separate = p->present_key != nullptr && p->present_key != p->past_key;
    char* ws = static_cast<char*>(p->workspace);
    if (P.splits > 1) {
      a.counters = reinterpret_cast<int*>(ws + P.counters);
      a.part_o = reinterpret_cast<float*>(ws + P.part_o);
      a.part_ml = reinterpret_cast<float*>(ws + P.part_ml);
    }
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    int launches = 0;
    cudaError_t e;
    // Rows past some batch's length exist in present only when a length is below its capacity.
    bool tail_rows = false;
    for (int b = 0; b < p->batch; ++b) tail_rows |= p->host_seqlens_k[b] + 1 < a.pcap;
    if (a.dtype == B200_DTYPE_FLOAT) e = launch_gqa<float>(a, P, tail_rows, stream, &launches);
    else if (a.dtype == B200_DTYPE_FLOAT16) e = launch_gqa<__half>(a, P, tail_rows, stream, &launches);
    else e = launch_gqa<__nv_bfloat16>(a, P, tail_rows, stream, &launches);
    add_launches(launches);
    if (e != cudaSuccess)
      return gfail(B200_ERR_CUDA, std::string("GroupQueryAttention: CUDA error: ") + cudaGetErrorString(e));
    return B200_OK;
  } catch (const std::exception& ex) {
    return gfail(B200_ERR_FAIL, std::string("GroupQueryAttention: ") + ex.what());
  } catch (...) {
    return gfail(B200_ERR_FAIL, "GroupQueryAttention: unknown failure");
  }
}

}  // extern "C"
