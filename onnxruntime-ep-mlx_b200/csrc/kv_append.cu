// KV append ("reshape and cache") and the per-call metadata checks.
//
// Reference behaviour (rust/src/ops/attention.rs):
//  * :4064-4079  slot of new token j of sequence b: slot_mapping[token] if given, else
//                block_table[b, (past+j)/bs] * bs + (past+j) % bs; slot < 0 skips the write
//  * :4045-4057  optional per-head RMS norm of new Q/K, then RoPE at positions [past, total)
//  * :4080-4120  scatter of the (optionally integer-encoded, kv_cache.rs:170-220) rows into the
//                flattened [NB*bs, KV, d] caches, applied in token order so a later token
//                overwrites an earlier one at the same slot
//  * engine.rs:1212-1364  the updated rows land in the caller's input cache buffers
//
// B200 design: one CTA per token row.  The plain path (no norm/RoPE, float cache) is a 16-byte
// vectorised copy of the token's whole [KV*d] row, which is contiguous in both the packed input
// and the [NB, bs, KV, d] pool.  Duplicate slots are resolved deterministically: a per-call
// open-addressing table maps slot -> largest token index (atomicMax), and only that token
// writes.  The table is skipped when the host proved the slots unique.
#include "b200_common.cuh"
#include "b200_kernels.h"

namespace b200 {

__device__ __forceinline__ uint32_t slot_hash(int32_t slot) {
  uint32_t x = static_cast<uint32_t>(slot);
  x ^= x >> 16;
  x *= 0x7feb352dU;
  x ^= x >> 15;
  x *= 0x846ca68bU;
  x ^= x >> 16;
  return x;
}

// Slot of token t, or -1 (skip).  Returns false when the metadata makes it invalid.
__device__ __forceinline__ bool token_slot(const PrologueArgs& a, int t, int b, int64_t& slot) {
  if (a.slot_mapping) {
    slot = a.slot_mapping[t];
    return slot >= -1 && slot < (int64_t)a.num_blocks * a.block_size;
  }
  int64_t logical = (int64_t)a.past[b] + (t - a.cum[b]);
  if (logical < 0) return false;
  int64_t page = logical / a.block_size;
  if (page >= a.max_blocks) return false;
  int32_t blk = a.block_table[(int64_t)b * a.max_blocks + page];
  if (blk < 0 || blk >= a.num_blocks) return false;
  slot = (int64_t)blk * a.block_size + logical % a.block_size;
  return true;
}

// Device-side metadata validation (the checks of attention.rs:3934-3990) and, when asked,
// the slot -> last-token table.  Thread i checks sequence i, block-table entry i (sequence
// i / max_blocks, entry i % max_blocks, if the sequence needs it) and token i, so no thread
// walks a whole block-table row.
__device__ __forceinline__ void check_sequence_and_table(const PrologueArgs& a, int64_t i) {
  if (i < a.batch) {
    int c0 = a.cum[i], c1 = a.cum[i + 1];
    int bits = 0;
    if ((i == 0 && c0 != 0) || c0 < 0 || c0 > c1 || (i == a.batch - 1 && c1 != a.num_tokens)) bits |= kStatusBadCumulative;
    int p = a.past[i];
    if (p < 0) bits |= kStatusBadPast;
    int64_t total = (int64_t)p + (c1 - c0);
    if (total > (int64_t)a.max_blocks * a.block_size) bits |= kStatusBadCapacity;
    if (a.rotary_positions > 0 && total > a.rotary_positions) bits |= kStatusBadPosition;
    if (bits) set_status(a.status, bits);
  }
  if (a.max_blocks > 0 && i < (int64_t)a.batch * a.max_blocks) {
    const int b = (int)(i / a.max_blocks);
    const int j = (int)(i % a.max_blocks);
    const int c0 = a.cum[b], c1 = a.cum[b + 1], p = a.past[b];
    const int64_t total = (int64_t)p + (c1 - c0);
    if (p >= 0 && c1 >= c0 && total <= (int64_t)a.max_blocks * a.block_size &&
        j < (total + a.block_size - 1) / a.block_size) {
      const int32_t blk = a.block_table[i];
      if (blk < 0 || blk >= a.num_blocks) set_status(a.status, kStatusBadBlock);
    }
  }
}

__global__ void meta_check_kernel(PrologueArgs a) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  check_sequence_and_table(a, i);
  if (i < a.num_tokens) {
    const int t = (int)i;
    int b = seq_of_token(a.cum, a.batch, t);
    int64_t slot;
    if (!token_slot(a, t, b, slot)) {
      set_status(a.status, a.slot_mapping ? kStatusBadSlot : kStatusBadBlock);
      return;
    }
    if (slot < 0 || !a.owner_keys) return;
    uint32_t mask = a.owner_capacity - 1;
    uint32_t h = slot_hash((int32_t)slot) & mask;
    for (uint32_t probe = 0; probe < a.owner_capacity; ++probe) {
      int prev = atomicCAS(&a.owner_keys[h], -1, (int)slot);
      if (prev == -1 || prev == (int)slot) {
        atomicMax(&a.owner_vals[h], t);
        return;
      }
      h = (h + 1) & mask;
    }
  }
}

__device__ __forceinline__ bool owns_slot(const PrologueArgs& a, int t, int64_t slot) {
  if (!a.owner_keys) return true;
  uint32_t mask = a.owner_capacity - 1;
  uint32_t h = slot_hash((int32_t)slot) & mask;
  for (uint32_t probe = 0; probe < a.owner_capacity; ++probe) {
    int key = a.owner_keys[h];
    if (key == (int)slot) return a.owner_vals[h] == t;
    if (key == -1) return true;
    h = (h + 1) & mask;
  }
  return true;
}

// Encode one [d] row (fp32 values in `src`, stride 1) of kv head `kh` into the cache slot.
__device__ void write_cache_row(const PrologueArgs& a, bool is_key, int64_t slot, int kh, const float* src,
                                int tid, int nthreads) {
  const int d = a.head_size;
  const int dtype = a.cache_dtype;
  void* cache = is_key ? a.key_cache : a.value_cache;
  const float* scale = is_key ? a.k_scale : a.v_scale;
  const int per_channel = is_key ? a.k_per_channel : a.v_per_channel;
  if (dtype == B200_DTYPE_UINT8) {
    int width = (d + 1) / 2;
    uint8_t* row = reinterpret_cast<uint8_t*>(cache) + (slot * a.kv_heads + kh) * (int64_t)width;
    for (int j = tid; j < width; j += nthreads) {
      int d0 = 2 * j, d1 = 2 * j + 1;
      float s0 = per_channel ? scale[kh * d + d0] : scale[0];
      int lo = quant_code(src[d0], s0, 4) + 8;
      int hi = 8;
      if (d1 < d) {
        float s1 = per_channel ? scale[kh * d + d1] : scale[0];
        hi = quant_code(src[d1], s1, 4) + 8;
      }
      row[j] = (uint8_t)(lo | (hi << 4));
    }
    return;
  }
  int64_t base = (slot * a.kv_heads + kh) * (int64_t)d;
  for (int j = tid; j < d; j += nthreads) {
    float x = src[j];
    if (dtype == B200_DTYPE_INT8) {
      float s = per_channel ? scale[kh * d + j] : scale[0];
      reinterpret_cast<int8_t*>(cache)[base + j] = (int8_t)quant_code(x, s, 8);
    } else if (dtype == B200_DTYPE_FLOAT8E4M3FN) {
      int64_t blk = slot / a.block_size;
      float s = scale[blk * a.kv_heads + kh];
      reinterpret_cast<uint8_t*>(cache)[base + j] = fp8_code(x, s);
    } else {
      store_act(cache, base + j, x, dtype);
    }
  }
}

// The prefill kernel reads this call's new keys back from the cache; a prefill sequence may
// stay on it only when every new row lands in its own block-table slot.
__device__ __forceinline__ void refine_route(const PrologueArgs& a, int t, int b, int64_t slot, bool write) {
  if (!a.route || a.route[b] != kRoutePrefill) return;
  bool canonical = write;
  if (canonical && a.slot_mapping) {
    const int64_t logical = (int64_t)a.past[b] + (t - a.cum[b]);
    const int64_t page = logical / a.block_size;
    canonical = page < a.max_blocks &&
                slot == (int64_t)a.block_table[(int64_t)b * a.max_blocks + page] * a.block_size +
                            logical % a.block_size;
  }
  if (!canonical) a.route[b] = kRouteGeneric;
}

// Plain reshape-and-cache (no norm / RoPE, cache in the activation type): one warp per token,
// kCopyTokensPerCta tokens per CTA.  The token's [KV*d] K and V rows are contiguous in the
// input and in the pool; each lane issues all its 16-byte loads of both rows before storing, and
// with a slot_mapping the first group of loads goes out before the slot's owner is resolved.
constexpr int kCopyTokensPerCta = 8;
constexpr int kCopyUnroll = 4;

__global__ void __launch_bounds__(32 * kCopyTokensPerCta) kv_copy_kernel(PrologueArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kCopyTokensPerCta + warp;
  if (t >= a.num_tokens) return;  // whole warp
  const int64_t bytes = (int64_t)a.kv_heads * a.head_size * 2;
  const int64_t n16 = bytes / 16;
  const char* ksrc = reinterpret_cast<const char*>(a.key) + (int64_t)t * a.key_stride * 2;
  const char* vsrc = reinterpret_cast<const char*>(a.value) + (int64_t)t * a.value_stride * 2;
  const bool src_vec = ((reinterpret_cast<uintptr_t>(ksrc) | reinterpret_cast<uintptr_t>(vsrc) | bytes) & 15) == 0;
  // With a slot_mapping, the row's first group of loads is in flight during the sequence search and
  // the owner-table probe below (not for padding tokens, slot -1); the stores still wait for them.
  uint4 kr[kCopyUnroll], vr[kCopyUnroll];
  const bool pre = src_vec && a.slot_mapping && __ldg(a.slot_mapping + t) >= 0;  // warp-uniform
  if (pre) {
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
      const int64_t j = u * 32 + lane;
      if (j < n16) {
        kr[u] = __ldg(reinterpret_cast<const uint4*>(ksrc) + j);
        vr[u] = __ldg(reinterpret_cast<const uint4*>(vsrc) + j);
      }
    }
  }
  const int b = seq_of_token(a.cum, a.batch, t);
  int64_t slot = -1;
  const bool valid = token_slot(a, t, b, slot);
  const bool write = valid && slot >= 0 && owns_slot(a, t, slot);
  if (lane == 0) {
    if (!valid) set_status(a.status, a.slot_mapping ? kStatusBadSlot : kStatusBadBlock);
    refine_route(a, t, b, slot, write);
  }
  if (!write) return;  // whole warp
  char* kdst = reinterpret_cast<char*>(a.key_cache) + slot * bytes;
  char* vdst = reinterpret_cast<char*>(a.value_cache) + slot * bytes;
  const bool vec = src_vec && ((reinterpret_cast<uintptr_t>(kdst) | reinterpret_cast<uintptr_t>(vdst)) & 15) == 0;
  if (vec) {
    for (int64_t j0 = 0; j0 < n16; j0 += 32 * kCopyUnroll) {
      if (j0 > 0 || !pre) {
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u) {
          const int64_t j = j0 + u * 32 + lane;
          if (j < n16) {
            kr[u] = __ldg(reinterpret_cast<const uint4*>(ksrc) + j);
            vr[u] = __ldg(reinterpret_cast<const uint4*>(vsrc) + j);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t j = j0 + u * 32 + lane;
        if (j < n16) {
          reinterpret_cast<uint4*>(kdst)[j] = kr[u];
          reinterpret_cast<uint4*>(vdst)[j] = vr[u];
        }
      }
    }
  } else {
    for (int64_t j = lane; j < bytes / 2; j += 32) {
      reinterpret_cast<uint16_t*>(kdst)[j] = reinterpret_cast<const uint16_t*>(ksrc)[j];
      reinterpret_cast<uint16_t*>(vdst)[j] = reinterpret_cast<const uint16_t*>(vsrc)[j];
    }
  }
}

// Small plain append with a device slot_mapping, in one launch: the metadata checks of
// meta_check_kernel (grid-stride), then a warp per token.  Every CTA stages the whole
// slot_mapping (at most kAppendFusedMaxTokens entries) in shared memory, and a token writes only
// when no later token names the same slot, which is the reference's token-order scatter
// (the last writer wins) without the slot table and its reset.
__global__ void __launch_bounds__(32 * kCopyTokensPerCta) kv_append_fused_kernel(PrologueArgs a) {
  __shared__ int32_t slots[kAppendFusedMaxTokens];
  const int nt = a.num_tokens;
  const int64_t checks = max((int64_t)a.batch * max(a.max_blocks, 0), (int64_t)a.batch);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < checks; i += (int64_t)gridDim.x * blockDim.x)
    check_sequence_and_table(a, i);
  for (int i = threadIdx.x; i < nt; i += blockDim.x) slots[i] = __ldg(a.slot_mapping + i);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kCopyTokensPerCta + warp;
  if (t >= nt) return;  // whole warp
  const int32_t slot = slots[t];
  if (slot < -1 || (int64_t)slot >= (int64_t)a.num_blocks * a.block_size) {
    if (lane == 0) set_status(a.status, kStatusBadSlot);
    return;
  }
  if (slot < 0) return;
  bool later = false;
  for (int u = t + 1 + lane; u < nt && !later; u += 32) later = slots[u] == slot;
  if (__any_sync(0xffffffffu, later)) return;  // a later token writes this slot
  const int64_t bytes = (int64_t)a.kv_heads * a.head_size * 2;
  char* kdst = reinterpret_cast<char*>(a.key_cache) + (int64_t)slot * bytes;
  char* vdst = reinterpret_cast<char*>(a.value_cache) + (int64_t)slot * bytes;
  const char* ksrc = reinterpret_cast<const char*>(a.key) + (int64_t)t * a.key_stride * 2;
  const char* vsrc = reinterpret_cast<const char*>(a.value) + (int64_t)t * a.value_stride * 2;
  const bool vec = ((reinterpret_cast<uintptr_t>(kdst) | reinterpret_cast<uintptr_t>(vdst) |
                     reinterpret_cast<uintptr_t>(ksrc) | reinterpret_cast<uintptr_t>(vsrc) | bytes) & 15) == 0;
  if (vec) {
    const int64_t n16 = bytes / 16;
    for (int64_t j0 = 0; j0 < n16; j0 += 32 * kCopyUnroll) {
      uint4 kr[kCopyUnroll], vr[kCopyUnroll];
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t j = j0 + u * 32 + lane;
        if (j < n16) {
          kr[u] = __ldg(reinterpret_cast<const uint4*>(ksrc) + j);
          vr[u] = __ldg(reinterpret_cast<const uint4*>(vsrc) + j);
        }
      }
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t j = j0 + u * 32 + lane;
        if (j < n16) {
          reinterpret_cast<uint4*>(kdst)[j] = kr[u];
          reinterpret_cast<uint4*>(vdst)[j] = vr[u];
        }
      }
    }
  } else {
    for (int64_t j = lane; j < bytes / 2; j += 32) {
      reinterpret_cast<uint16_t*>(kdst)[j] = reinterpret_cast<const uint16_t*>(ksrc)[j];
      reinterpret_cast<uint16_t*>(vdst)[j] = reinterpret_cast<const uint16_t*>(vsrc)[j];
    }
  }
}

bool append_fused_eligible(const PrologueArgs& a) {
  return a.kv_only && !a.latent && a.slot_mapping != nullptr && !(a.do_norm || a.do_rotary) &&
         a.cache_dtype == a.act_dtype && a.num_tokens > 0 && a.num_tokens <= kAppendFusedMaxTokens && a.route == nullptr;
}

cudaError_t launch_append_fused(const PrologueArgs& a, cudaStream_t stream) {
  kv_append_fused_kernel<<<(a.num_tokens + kCopyTokensPerCta - 1) / kCopyTokensPerCta, 32 * kCopyTokensPerCta, 0,
                           stream>>>(a);
  return cudaGetLastError();
}

// One CTA per token, for the processing paths (RMS norm / RoPE, integer or fp8 caches).  Shared
// memory: fp32 rows [H*d] for Q and [KV*d] for K, plus [KV*d] for V when the cache is encoded.
__global__ void kv_prologue_kernel(PrologueArgs a) {
  extern __shared__ float smem[];
  const int t = blockIdx.x;
  const int b = seq_of_token(a.cum, a.batch, t);
  const int H = a.num_heads, KV = a.kv_heads, d = a.head_size;
  const int tid = threadIdx.x, nthreads = blockDim.x;
  const int dt = a.act_dtype;

  int64_t slot = -1;
  bool valid = token_slot(a, t, b, slot);
  bool write = valid && slot >= 0 && owns_slot(a, t, slot);
  if (!valid && tid == 0) set_status(a.status, a.slot_mapping ? kStatusBadSlot : kStatusBadBlock);
  if (tid == 0) refine_route(a, t, b, slot, write);
  if (a.kv_only && !write) return;

  const bool process = a.do_norm || a.do_rotary;

  // Staged rows: Q (processing path only) then K and V; sized by prologue_smem_bytes().
  const int nq_heads = process && !a.kv_only ? H : 0;
  float* qs = smem;                        // [nq_heads*d]
  float* ks = qs + (int64_t)nq_heads * d;  // [KV*d]
  float* vs = ks + (int64_t)KV * d;        // [KV*d]
  const int64_t seq_pos = (int64_t)a.past[b] + (t - a.cum[b]);

  for (int j = tid; j < nq_heads * d; j += nthreads)
    qs[j] = load_act(a.query, (int64_t)t * a.query_stride + j, dt);
  for (int j = tid; j < KV * d; j += nthreads) {
    ks[j] = load_act(a.key, (int64_t)t * a.key_stride + j, dt);
    if (!a.latent) vs[j] = load_act(a.value, (int64_t)t * a.value_stride + j, dt);
  }
  __syncthreads();

  if (a.do_norm) {
    // RMS norm per head (attention.rs:4045-4049): x / sqrt(mean(x^2) + eps) * w, rounded to T.
    const int warp = tid >> 5, lane = tid & 31, nwarps = nthreads >> 5;
    for (int hh = warp; hh < nq_heads + KV; hh += nwarps) {
      float* row = hh < nq_heads ? qs + (int64_t)hh * d : ks + (int64_t)(hh - nq_heads) * d;
      const void* w = hh < nq_heads ? a.q_norm : a.k_norm;
      float acc = 0.f;
      for (int j = lane; j < d; j += 32) acc += row[j] * row[j];
      for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      float denom = sqrtf(__fdiv_rn(acc, (float)d) + a.norm_eps);
      for (int j = lane; j < d; j += 32)
        row[j] = round_act(__fmul_rn(__fdiv_rn(row[j], denom), load_act(w, j, dt)), dt);
    }
    __syncthreads();
  }
  if (a.do_rotary) {
    // RoPE over channels [offset, offset + rot) at position past + j
    // (test_paged_attention.py:27-58 / attention.rs:3812-3855), products not fused.
    if (seq_pos < a.rotary_positions) {
      const int half = a.rotary_dim / 2;
      const int pairs = (nq_heads + KV) * half;
      for (int pidx = tid; pidx < pairs; pidx += nthreads) {
        int hh = pidx / half, i = pidx % half;
        float* row = hh < nq_heads ? qs + (int64_t)hh * d : ks + (int64_t)(hh - nq_heads) * d;
        int i0, i1;
        if (a.rotary_interleaved) { i0 = a.rotary_offset + 2 * i; i1 = i0 + 1; }
        else { i0 = a.rotary_offset + i; i1 = i0 + half; }
        float c = load_act(a.cos_cache, seq_pos * half + i, dt);
        float s = load_act(a.sin_cache, seq_pos * half + i, dt);
        float x0 = row[i0], x1 = row[i1];
        row[i0] = round_act(__fadd_rn(__fmul_rn(x0, c), __fmul_rn(-x1, s)), dt);
        row[i1] = round_act(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s)), dt);
      }
    } else if (tid == 0) {
      set_status(a.status, kStatusBadPosition);
    }
    __syncthreads();
  }
  if (process && !a.kv_only) {
    for (int j = tid; j < H * d; j += nthreads) store_act(a.q_proc, (int64_t)t * H * d + j, qs[j], dt);
    for (int j = tid; j < KV * d; j += nthreads) store_act(a.k_proc, (int64_t)t * KV * d + j, ks[j], dt);
  }
  if (!write) return;
  const int warp = tid >> 5, lane = tid & 31, nwarps = nthreads >> 5;
  for (int hh = warp; hh < (a.latent ? KV : 2 * KV); hh += nwarps) {  // LATENT: key rows only
    bool is_key = hh < KV;
    int kh = is_key ? hh : hh - KV;
    write_cache_row(a, is_key, slot, kh, (is_key ? ks : vs) + (int64_t)kh * d, lane, 32);
  }
}

void launch_meta_check(const PrologueArgs& a, cudaStream_t stream) {
  int64_t n = a.batch > a.num_tokens ? a.batch : a.num_tokens;
  const int64_t entries = (int64_t)a.batch * (a.max_blocks > 0 ? a.max_blocks : 0);
  if (entries > n) n = entries;
  if (n <= 0) return;
  meta_check_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(a);
}

size_t prologue_smem_bytes(const PrologueArgs& a) {
  const bool process = a.do_norm || a.do_rotary;
  if (!process && a.cache_dtype == a.act_dtype && !a.latent) return 0;  // kv_copy_kernel stages nothing
  int qheads = process && !a.kv_only ? a.num_heads : 0;
  return sizeof(float) * (size_t)a.head_size * (qheads + 2 * a.kv_heads);
}

cudaError_t launch_prologue(const PrologueArgs& a, cudaStream_t stream) {
  if (a.num_tokens <= 0) return cudaSuccess;
  size_t smem = prologue_smem_bytes(a);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kv_prologue_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  if (!(a.do_norm || a.do_rotary) && a.cache_dtype == a.act_dtype && !a.latent) {
    kv_copy_kernel<<<(a.num_tokens + kCopyTokensPerCta - 1) / kCopyTokensPerCta, 32 * kCopyTokensPerCta, 0, stream>>>(a);
    return cudaGetLastError();
  }
  kv_prologue_kernel<<<a.num_tokens, 128, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace b200
