// Generic paged attention: every form the claim accepts, any head size up to 640, any block
// size, float / int8 / int4 / fp8 caches, SEPARATE or LATENT layout.  One CTA (4 warps) per (query token, query head);
// the warps split the visible keys and merge their online-softmax states in shared memory.
//
// Semantics (rust/src/ops/attention.rs:4124-4320, oracle test_paged_attention.py:119-157):
//  * query row i of sequence b sits at absolute position past+i; key c is visible iff
//    c <= past+i (causal) and c >= past+i-window+1 (window > 0); is_causal=0 shows all keys;
//  * keys [0, past) come from the (already appended) cache through the block table, keys
//    [past, total) from the sequence's own new rows; integer / fp8 caches read every key from
//    the decoded cache (attention.rs:4190-4192);
//  * scores = scale * q.k, optional softcap * tanh(s / softcap), fp32 softmax with an optional
//    per-head sink in the denominator (attention.rs:99-118), fp32 accumulation, output in T;
//  * LATENT layout (attention.rs:4058-4062, :4210-4212): one kv head, and the values are the
//    first v_head channels of the key rows (the host points the value views at the key rows);
//    the output has v_head channels per head.
// This kernel is the reference-semantics path used for prefill rows and for shapes the fast
// kernels do not cover.
#include "b200_common.cuh"
#include "b200_kernels.h"

namespace b200 {

template <int EPL>
__global__ void __launch_bounds__(128) generic_attention_kernel(AttnArgs a) {
  constexpr int kWarps = 4;
  __shared__ float red_m[kWarps], red_l[kWarps];
  __shared__ float red_o[kWarps][32 * EPL];
  __shared__ float qs[32 * EPL];

  const int t = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = seq_of_token(a.cum, a.batch, t);
  const int c0 = a.cum[b];
  const int nq = a.cum[b + 1] - c0;
  if (a.route && a.route[b] != kRouteGeneric) return;  // another kernel owns this sequence
  const int D = a.head_size, VD = a.v_head;
  const int i = t - c0;
  const int past = a.past[b];
  // invalid metadata (flagged by the check kernel): never index outside the new rows
  if (past < 0 || i < 0 || i >= nq || c0 < 0 || a.cum[b + 1] > a.num_tokens) return;
  const int total = past + nq;
  const int kh = h / a.group;
  const bool quant = a.cache_dtype != a.act_dtype;

  for (int d = threadIdx.x; d < 32 * EPL; d += blockDim.x)
    qs[d] = d < D ? load_act(a.q, (int64_t)t * a.q_stride + (int64_t)h * D + d, a.act_dtype) : 0.f;
  __syncthreads();

  int lo = 0, hi = a.is_causal ? past + i + 1 : total;
  if (a.window > 0) lo = max(0, past + i - a.window + 1);

  CacheView kc{a.key_cache, a.cache_dtype, a.cache_dtype == B200_DTYPE_UINT8 ? (D + 1) / 2 : D, a.k_scale,
               a.k_per_channel};
  CacheView vc{a.value_cache, a.cache_dtype, kc.width, a.v_scale, a.v_per_channel};

  float m = -INFINITY, l = 0.f, o[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) o[e] = 0.f;

  for (int c = lo + warp; c < hi; c += kWarps) {
    bool from_new = !quant && c >= past;
    int64_t slot = 0, new_row = 0;
    if (from_new) {
      new_row = c0 + (c - past);
    } else {
      int64_t page = c / a.block_size;
      int32_t blk = page < a.max_blocks ? a.block_table[(int64_t)b * a.max_blocks + page] : -1;
      if (blk < 0 || blk >= a.num_blocks) {
        if (lane == 0) set_status(a.status, kStatusBadBlock);
        continue;
      }
      slot = (int64_t)blk * a.block_size + c % a.block_size;
    }
    float dot = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      int d = lane + 32 * e;
      if (d < D) {
        float kv = from_new ? load_act(a.k_new, new_row * a.k_stride + (int64_t)kh * D + d, a.act_dtype)
                            : cache_value(kc, slot, a.kv_heads, kh, d, D, a.block_size);
        dot += qs[d] * kv;
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    float s = dot * a.scale;
    if (a.softcap > 0.f) s = a.softcap * tanhf(s / a.softcap);
    float m_new = fmaxf(m, s);
    float alpha = expf(m - m_new);  // m = -inf on the first key gives 0
    float p = expf(s - m_new);
    l = l * alpha + p;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      int d = lane + 32 * e;
      float vv = 0.f;
      if (d < VD)
        vv = from_new ? load_act(a.v_new, new_row * a.v_stride + (int64_t)kh * D + d, a.act_dtype)
                      : cache_value(vc, slot, a.kv_heads, kh, d, D, a.block_size);
      o[e] = o[e] * alpha + p * vv;
    }
    m = m_new;
  }

  if (lane == 0) { red_m[warp] = m; red_l[warp] = l; }
#pragma unroll
  for (int e = 0; e < EPL; ++e) red_o[warp][lane + 32 * e] = o[e];
  __syncthreads();
  if (warp != 0) return;
  float M = -INFINITY;
  for (int w = 0; w < kWarps; ++w) M = fmaxf(M, red_m[w]);
  float sink_term = 0.f;
  if (a.head_sink) {
    float sink = load_act(a.head_sink, h, a.act_dtype);
    float M2 = fmaxf(M, sink);
    sink_term = expf(sink - M2);
    M = M2;
  }
  float L = sink_term, f[kWarps];
  for (int w = 0; w < kWarps; ++w) {
    f[w] = red_m[w] == -INFINITY ? 0.f : expf(red_m[w] - M);
    L += red_l[w] * f[w];
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    int d = lane + 32 * e;
    if (d >= VD) continue;
    float acc = 0.f;
    for (int w = 0; w < kWarps; ++w) acc += red_o[w][d] * f[w];
    float y = L > 0.f ? acc / L : 0.f;
    store_act(a.out, (int64_t)t * a.num_heads * VD + (int64_t)h * VD + d, y, a.act_dtype);
  }
}

cudaError_t launch_generic(const AttnArgs& a, cudaStream_t stream) {
  if (a.num_tokens <= 0) return cudaSuccess;
  dim3 grid(a.num_tokens, a.num_heads);
  int epl = (a.head_size + 31) / 32;
  if (epl <= 1) generic_attention_kernel<1><<<grid, 128, 0, stream>>>(a);
  else if (epl <= 2) generic_attention_kernel<2><<<grid, 128, 0, stream>>>(a);
  else if (epl <= 4) generic_attention_kernel<4><<<grid, 128, 0, stream>>>(a);
  else if (epl <= 8) generic_attention_kernel<8><<<grid, 128, 0, stream>>>(a);
  else if (epl <= 12) generic_attention_kernel<12><<<grid, 128, 0, stream>>>(a);
  else if (epl <= 16) generic_attention_kernel<16><<<grid, 128, 0, stream>>>(a);
  else if (epl <= 20) generic_attention_kernel<20><<<grid, 128, 0, stream>>>(a);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace b200
