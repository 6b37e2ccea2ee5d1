// Ragged causal chunked prefill over the paged cache on the 5th-generation tensor core.
//
// Replaces the reference's per-sequence gather + SDPA for prefill chunks
// (rust/src/ops/attention.rs:4192-4319, native grouped-query prefill :4235-4253): same
// mathematics as the decode kernel (scale*q.k, softcap, top-left causal and left-window masks,
// fp32 softmax with optional sink, fp32 accumulation).
//
// B200 design:
//  * work item = (sequence, kv head, q tile).  A q tile is 128 rows = 128/g query tokens x the
//    g query heads of the kv head, so each K/V tile serves the whole head group (native GQA);
//  * persistent CTAs (one per SM: 225 KB of shared memory and all 512 tensor-memory columns)
//    take items round-robin, longest (latest q tile) first;
//  * warp-specialised, the roles synchronised only through mbarriers:
//      - warp 4 (TMA producer): Q tile [128 x 128] by a 3-D box pair from the [nt, H, d] query
//        view; K/V tiles of 128 keys = 8 pages of 16 slots, one 64-channel box per lane (32
//        boxes per tile issued in parallel), 3 stages; pages past the sequence end load from an
//        out-of-range coordinate (TMA zero fill);
//      - warp 5 (MMA issuer): S = Q K^T (8 x tcgen05.mma kind::f16, M=128, N=128, K=16) into one
//        of two tensor-memory S buffers, then O += P V with P read from tensor memory and V as
//        the MN-major operand (the cache's [key][channel] layout); QK of tile j+1 runs while the
//        softmax works on tile j;
//      - warps 0-3 (softmax, one q row per thread = tensor-memory lane): exp2-domain softmax
//        with a lazily rescaled running max (O is rescaled in tensor memory only when the max
//        grows by more than 2^8); P goes back over the S columns as a hi + lo pair of 16-bit
//        values (~16 mantissa bits); epilogue normalises (sink) and stores the rows.
//  * every mbarrier wait is bounded (%globaltimer); a timeout sets the status word and the CTA
//    drains and stops instead of hanging.
#include <type_traits>

#include "b200_common.cuh"
#include "b200_kernels.h"
#include "b200_tcgen05.cuh"

namespace b200 {

namespace {

constexpr int kBM = 128;             // q rows per tile
constexpr int kBN = 128;             // keys per tile
constexpr int kD = 128;              // head size of this kernel
constexpr int kStages = 3;           // K/V pipeline depth
constexpr int kBoxBytes = 128 * 128; // one [128 rows][64 channels] 16-bit box: 16 KB
constexpr int kTileBytes = 2 * kBoxBytes;  // [128][128] 16-bit tile: 32 KB
constexpr float kLog2eP = 1.4426950408889634f;

// shared-memory map (offsets from the 1024-aligned base)
constexpr int kSmemQ = 0;
constexpr int kSmemK = kSmemQ + kTileBytes;              // kStages K tiles
constexpr int kSmemV = kSmemK + kStages * kTileBytes;    // kStages V tiles
constexpr int kSmemBytes = kSmemV + kStages * kTileBytes;  // 224 KB

// Roles: warps 0-3 softmax / epilogue (one q row per thread), warp 4 TMA producer, warp 5 MMA.
constexpr int kSoftmaxThreads = 128;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kThreads = 192;

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t kv_full[kStages], kv_empty[kStages];
  uint64_t s_full[2], p_full[2], o_done[2];
  uint64_t o_free;
};

// One item of the prefill work list, as every role decodes it.
struct Item {
  int skip, b, kh, c0, nq, past, total, q0, q1, kv_lo, nkv;
};

__device__ __forceinline__ Item decode_item(const AttnArgs& a, const DecodePlan& plan, int64_t it) {
  Item m{};
  const int KV = a.kv_heads, TQ = a.prefill_tq;
  const int64_t qtiles_total = *plan.pf_total / KV;
  const int64_t qt_global = qtiles_total - 1 - it / KV;  // latest q tiles (most keys) first
  m.kh = (int)(it % KV);
  int lo = 0, hi = a.batch - 1;  // sequence: largest b with pf_tile_off[b] <= qt_global
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (plan.pf_tile_off[mid] <= qt_global) lo = mid; else hi = mid - 1;
  }
  m.b = lo;
  m.skip = a.route[m.b] != kRoutePrefill;  // moved to the generic kernel by the prologue
  if (m.skip) return m;
  const int qt = (int)(qt_global - plan.pf_tile_off[m.b]);
  m.c0 = a.cum[m.b];
  m.nq = a.cum[m.b + 1] - m.c0;
  m.past = a.past[m.b];
  m.total = m.past + m.nq;
  m.q0 = qt * TQ;
  m.q1 = min(m.q0 + TQ, m.nq);
  const int kv_hi = a.is_causal ? m.past + m.q1 : m.total;
  m.kv_lo = a.window > 0 ? max(0, m.past + m.q0 - a.window + 1) : 0;
  m.kv_lo &= ~(kTile - 1);
  m.nkv = (kv_hi - m.kv_lo + kBN - 1) / kBN;
  return m;
}

}  // namespace

bool prefill_supported(int head_size, int block_size, int group, int act_dtype, int cache_dtype) {
  return head_size == kD && block_size % kTile == 0 && act_dtype == cache_dtype &&
         (act_dtype == B200_DTYPE_FLOAT16 || act_dtype == B200_DTYPE_BFLOAT16) &&
         (group == 1 || group == 2 || group == 4 || group == 8 || group == 16);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) paged_prefill_kernel(const __grid_constant__ AttnArgs a,
                                                                     const __grid_constant__ PrefillMaps maps,
                                                                     const DecodePlan plan) {
  using MMA = mma_op<T>;  // packing helpers only
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdQK = tc::idesc_f16(kBM, kBN, kBF16, false, false);
  constexpr uint32_t kIdPV = tc::idesc_f16(kBM, kD, kBF16, false, true);

  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) Bars bars;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int s_failed;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = a.group, H = a.num_heads;
  const int64_t n_items = *plan.pf_total;
  if (n_items == 0) return;

  if (warp == kMmaWarp) tc::alloc(&tmem_slot, 512);
  if (tid == 0) {
    mbar_init(&bars.q_full, 1);
    mbar_init(&bars.q_empty, 1);
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bars.kv_full[i], 1);
      mbar_init(&bars.kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.s_full[i], 1);
      mbar_init(&bars.p_full[i], kSoftmaxThreads);
      mbar_init(&bars.o_done[i], 1);
    }
    mbar_init(&bars.o_free, kSoftmaxThreads);
    fence_mbar_init();
    s_failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t tO = tmem + 256;  // S/P buffers at columns [0,128) and [128,256)

  // Bounded wait on completion `index` of an mbarrier (parity = index & 1).
  auto wait_idx = [&](uint64_t* bar, uint32_t index) -> bool {
    if (s_failed) return false;
    if (mbar_wait(bar, index & 1u)) return true;
    set_status(a.status, kStatusTimeout);
    s_failed = 1;
    return false;
  };

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------------ TMA producer
    uint32_t tile = 0, items = 0;
    const int64_t oob_z = (int64_t)a.num_blocks * a.block_size;  // past the cache: zero fill
    for (int64_t it = blockIdx.x; it < n_items && !s_failed; it += gridDim.x) {
      const Item m = decode_item(a, plan, it);
      if (m.skip) continue;
      if (items > 0 && !wait_idx(&bars.q_empty, items - 1)) break;
      if (lane == 0) mbar_arrive_expect_tx(&bars.q_full, kTileBytes);
      __syncwarp();
      if (lane < 2)
        tma_load_3d(smem + kSmemQ + lane * kBoxBytes, &maps.q_map, &bars.q_full, lane * 64, m.kh * g, m.c0 + m.q0);
      const int32_t* bt = a.block_table + (int64_t)m.b * a.max_blocks;
      for (int j = 0; j < m.nkv; ++j, ++tile) {
        const int st = tile % kStages;
        const uint32_t use = tile / kStages;
        if (use > 0 && !wait_idx(&bars.kv_empty[st], use - 1)) break;
        // lane l: page l/4, channel half (l/2)%2, K (even l) or V (odd l)
        const int page = lane >> 2, half = (lane >> 1) & 1, is_v = lane & 1;
        const int pos0 = m.kv_lo + j * kBN + page * kTile;
        const int32_t blk = pos0 < m.total ? __ldg(bt + pos0 / a.block_size) : -1;
        const bool blk_ok = blk >= 0 && blk < a.num_blocks;
        if (pos0 < m.total && !blk_ok) set_status(a.status, kStatusBadBlock);
        const int z = blk_ok ? blk * a.block_size + pos0 % a.block_size : (int)oob_z;
        if (lane == 0) mbar_arrive_expect_tx(&bars.kv_full[st], 2 * kTileBytes);
        __syncwarp();
        uint8_t* dst = smem + (is_v ? kSmemV : kSmemK) + st * kTileBytes + half * kBoxBytes + page * (kTile * 128);
        tma_load_3d(dst, is_v ? &maps.v_map : &maps.k_map, &bars.kv_full[st], half * 64, m.kh, z);
      }
      ++items;
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t tile = 0, items = 0;
      for (int64_t it = blockIdx.x; it < n_items && !s_failed; it += gridDim.x) {
        const Item m = decode_item(a, plan, it);
        if (m.skip) continue;
        if (!wait_idx(&bars.q_full, items)) break;
        tc::fence_after_sync();
        bool first_pv = true;
        auto issue_pv = [&](uint32_t t) -> bool {  // O (+)= P_t . V_t, then release stage and buffer
          if (!wait_idx(&bars.p_full[t & 1], t >> 1)) return false;
          if (first_pv && items > 0 && !wait_idx(&bars.o_free, items - 1)) return false;
          tc::fence_after_sync();
          const uint32_t pbuf = tmem + (t & 1) * 128;
          const uint32_t vbase = sbase + kSmemV + (t % kStages) * kTileBytes;
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint64_t vdesc = tc::smem_desc(vbase + kk * 2048, kBoxBytes, 1024);
            tc::mma_ts(tO, pbuf + kk * 8, vdesc, kIdPV, (first_pv && kk == 0) ? 0u : 1u);
            tc::mma_ts(tO, pbuf + 64 + kk * 8, vdesc, kIdPV, 1u);
          }
          tc::commit(&bars.o_done[t & 1]);
          tc::commit(&bars.kv_empty[t % kStages]);
          first_pv = false;
          return true;
        };
        bool ok = true;
        for (int j = 0; j < m.nkv && ok; ++j, ++tile) {
          const int st = tile % kStages;
          if (!(ok = wait_idx(&bars.kv_full[st], tile / kStages))) break;
          tc::fence_after_sync();
          const uint32_t sbuf = tmem + (tile & 1) * 128;
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
            tc::mma_ss(sbuf, tc::smem_desc(sbase + kSmemQ + off, 16, 1024),
                       tc::smem_desc(sbase + kSmemK + st * kTileBytes + off, 16, 1024), kIdQK, kk > 0);
          }
          tc::commit(&bars.s_full[tile & 1]);
          if (j > 0) ok = issue_pv(tile - 1);
        }
        if (ok) ok = issue_pv(tile - 1);
        tc::commit(&bars.q_empty);
        if (!ok) break;
        ++items;
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int row = tid;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const float qk_scale = a.softcap > 0.f ? a.scale : a.scale * kLog2eP;
    uint32_t tile = 0;
    for (int64_t it = blockIdx.x; it < n_items && !s_failed; it += gridDim.x) {
      const Item m = decode_item(a, plan, it);
      if (m.skip) continue;
      const int tl = row / g, hl = row % g;
      const bool row_ok = m.q0 + tl < m.q1;
      const int qpos = m.past + m.q0 + tl;
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int j = 0; j < m.nkv; ++j, ++tile) {
        if (!(ok = wait_idx(&bars.s_full[tile & 1], tile >> 1))) break;
        tc::fence_after_sync();
        const uint32_t sbuf = tmem + (tile & 1) * 128 + lane_off;
        float sv[kBN / 32][32];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) tc::ld32(sbuf + c * 32, sv[c]);
        tc::wait_ld();
        const int kbase = m.kv_lo + j * kBN;
        // Masks only where a key can be invisible to this row (diagonal tile, sequence end, window).
        const bool full = row_ok && kbase + kBN <= m.total && (!a.is_causal || kbase + kBN - 1 <= qpos) &&
                          (a.window <= 0 || kbase >= qpos - a.window + 1) && a.softcap <= 0.f;
        // In the unmasked case the scores stay raw and scale folds into the exponent's FMA
        // (qk_scale > 0); masked tiles are rewritten to scaled log2 values (-inf = masked).
        const bool raw = full && qk_scale > 0.f;
        float m_tile;
        if (raw) {
          float mx[8];
#pragma unroll
          for (int r = 0; r < 8; ++r) mx[r] = -INFINITY;
#pragma unroll
          for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) mx[i & 7] = fmaxf(mx[i & 7], sv[c][i]);
          m_tile = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
          m_tile *= qk_scale;
        } else {
          // Keys this row sees, as a column range [vlo, vhi] of the tile (empty for padding rows).
          const int vhi = row_ok ? min(m.total - 1, a.is_causal ? qpos : m.total - 1) - kbase : -1;
          const int vlo = (a.window > 0 ? qpos - a.window + 1 : 0) - kbase;
          if (a.softcap > 0.f) {
            // cap * tanh(y / cap) in the log2 domain, tanh(u) = 1 - 2 / (1 + e^(2u)).
            const float two_log2e_over_cap = 2.f * kLog2eP / a.softcap, cap_log2e = a.softcap * kLog2eP;
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float e = tc::ex2(fminf(sv[c][i] * qk_scale * two_log2e_over_cap, 126.f));
                sv[c][i] = cap_log2e * (1.f - __fdividef(2.f, 1.f + e));
              }
          } else {
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
              for (int i = 0; i < 32; ++i) sv[c][i] *= qk_scale;
          }
          float mx[8];
#pragma unroll
          for (int r = 0; r < 8; ++r) mx[r] = -INFINITY;
#pragma unroll
          for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = c * 32 + i;
              sv[c][i] = (col >= vlo && col <= vhi) ? sv[c][i] : -INFINITY;
              mx[i & 7] = fmaxf(mx[i & 7], sv[c][i]);
            }
          m_tile = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        }
        // Lazy rescale: the reference max moves only when the row max grows by more than 2^8.
        const float m_new = fmaxf(m_run, m_tile);
        const bool grow = m_new > m_run + 8.0f;
        const float alpha = (grow && m_run != -INFINITY) ? tc::ex2(m_run - m_new) : 1.0f;
        if (grow) {
          l_run *= (m_run == -INFINITY ? 0.f : alpha);
          m_run = m_new;
        }
        if (j > 0 && __any_sync(0xffffffffu, grow && alpha != 1.0f)) {
          // O holds tiles < j: wait for PV of tile j-1, then scale this warp's rows in place.
          if (!(ok = wait_idx(&bars.o_done[(tile - 1) & 1], (tile - 1) >> 1))) break;
          tc::fence_after_sync();
#pragma unroll 1
          for (int c = 0; c < kD / 16; ++c) {
            float r[16];
            tc::ld16(tO + lane_off + c * 16, r);
            tc::wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] *= alpha;
            tc::st16(tO + lane_off + c * 16, r);
          }
          tc::wait_st();
        }
        // P = 2^(s - m_run) as hi + lo 16-bit halves over the S columns: hi in [0,64), lo in [64,128)
        const float mu = m_run == -INFINITY ? 0.f : m_run;
        const float kscale = raw ? qk_scale : 1.0f;  // p = 2^(s * kscale - mu)
        float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = tc::ex2(fmaf(sv[c][2 * i], kscale, -mu));
            const float p1 = tc::ex2(fmaf(sv[c][2 * i + 1], kscale, -mu));
            ls[i & 3] += p0 + p1;
            hi[i] = MMA::pack(p0, p1);
            const float2 h = MMA::unpack(hi[i]);
            lo[i] = MMA::pack(p0 - h.x, p1 - h.y);
          }
          tc::st16u(sbuf + c * 16, hi);
          tc::st16u(sbuf + 64 + c * 16, lo);
        }
        const float lsum = (ls[0] + ls[1]) + (ls[2] + ls[3]);
        l_run += lsum;
        tc::wait_st();
        tc::fence_before_sync();
        mbar_arrive(&bars.p_full[tile & 1]);
      }
      if (!ok) break;
      // ---- epilogue: last PV done -> normalise -> store this row
      if (!wait_idx(&bars.o_done[(tile - 1) & 1], (tile - 1) >> 1)) break;
      tc::fence_after_sync();
      float L = l_run;
      if (a.head_sink) {  // l is relative to the reference max m_run; fold the sink in that frame
        const float sink = load_act(a.head_sink, m.kh * g + hl, a.act_dtype) * kLog2eP;
        L += tc::ex2(sink - (m_run == -INFINITY ? 0.f : m_run));
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      T* orow = reinterpret_cast<T*>(a.out) + (int64_t)(m.c0 + m.q0 + tl) * H * kD + (int64_t)(m.kh * g + hl) * kD;
#pragma unroll 1
      for (int c = 0; c < kD / 16; ++c) {
        float r[16];
        tc::ld16(tO + lane_off + c * 16, r);
        tc::wait_ld();
        if (row_ok) {
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) w[i] = MMA::pack(r[2 * i] * inv, r[2 * i + 1] * inv);
          reinterpret_cast<uint4*>(orow + c * 16)[0] = make_uint4(w[0], w[1], w[2], w[3]);
          reinterpret_cast<uint4*>(orow + c * 16)[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      tc::fence_before_sync();
      mbar_arrive(&bars.o_free);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == kMmaWarp) tc::dealloc(tmem, 512);
}

cudaError_t launch_prefill(const AttnArgs& a, const DecodePlan& plan, const PrefillMaps& maps, int num_sms,
                           cudaStream_t stream) {
  const size_t smem = kSmemBytes + 1024;
  const bool bf = a.act_dtype == B200_DTYPE_BFLOAT16;
  static bool attr_set[2] = {false, false};
  cudaError_t e = cudaSuccess;
  if (bf) {
    if (!attr_set[1]) {
      e = cudaFuncSetAttribute(paged_prefill_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      attr_set[1] = true;
    }
    paged_prefill_kernel<__nv_bfloat16><<<num_sms, kThreads, smem, stream>>>(a, maps, plan);
  } else {
    if (!attr_set[0]) {
      e = cudaFuncSetAttribute(paged_prefill_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      attr_set[0] = true;
    }
    paged_prefill_kernel<__half><<<num_sms, kThreads, smem, stream>>>(a, maps, plan);
  }
  return cudaGetLastError();
}

}  // namespace b200
