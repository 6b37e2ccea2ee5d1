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
//  * thread 0 issues TMA and tcgen05.mma; the 4 warps (one row per thread, tensor-memory lane
//    = row) run the softmax:
//      - Q tile [128 x 128] by one 3-D TMA box pair from the [nt, H, d] query view;
//      - K/V tiles of 128 keys = 8 pages of 16 slots, 2 TMA boxes (64 channels) per page,
//        double-buffered; pages past the sequence end load from an out-of-range coordinate
//        (TMA zero fill);
//      - S = Q K^T: 8 x tcgen05.mma kind::f16 (M=128, N=128, K=16) into one of two tensor-memory
//        S buffers, so QK of tile j+1 overlaps the softmax of tile j;
//      - softmax per row in the exp2 domain with a lazily rescaled running max (O is rescaled
//        in tensor memory only when the max grows by more than 2^8); P is written to 128B-
//        swizzled shared memory as a hi + lo pair of 16-bit values (~16 mantissa bits);
//      - O += P V: tcgen05.mma with P K-major and V MN-major (the cache's [key][channel]
//        layout), accumulating in tensor memory;
//      - epilogue: tcgen05.ld of O, normalise (sink), store the rows.
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
constexpr int kBoxBytes = 128 * 128; // one [128 rows][64 channels] 16-bit box: 16 KB
constexpr int kTileBytes = 2 * kBoxBytes;  // [128][128] 16-bit tile: 32 KB
constexpr float kLog2eP = 1.4426950408889634f;

// shared-memory map (offsets from the 1024-aligned base)
constexpr int kSmemQ = 0;
constexpr int kSmemK = kSmemQ + kTileBytes;        // 2 stages
constexpr int kSmemV = kSmemK + 2 * kTileBytes;    // 2 stages
constexpr int kSmemPhi = kSmemV + 2 * kTileBytes;
constexpr int kSmemPlo = kSmemPhi + kTileBytes;
constexpr int kSmemBytes = kSmemPlo + kTileBytes;  // 224 KB

struct Bars {
  uint64_t q, k[2], v[2], s[2], o;
};

__device__ __forceinline__ void tma3(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  tma_load_3d(dst, map, bar, x, y, z);
}

}  // namespace

bool prefill_supported(int head_size, int block_size, int group, int act_dtype, int cache_dtype) {
  return head_size == kD && block_size % kTile == 0 && act_dtype == cache_dtype &&
         (act_dtype == B200_DTYPE_FLOAT16 || act_dtype == B200_DTYPE_BFLOAT16) &&
         (group == 1 || group == 2 || group == 4 || group == 8 || group == 16);
}

template <typename T>
__global__ void __launch_bounds__(128, 1) paged_prefill_kernel(const __grid_constant__ AttnArgs a,
                                                               const __grid_constant__ PrefillMaps maps,
                                                               const DecodePlan plan) {
  using MMA = mma_op<T>;  // packing helpers only
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kIdQK = tc::idesc_f16(kBM, kBN, kBF16, false, false);
  constexpr uint32_t kIdPV = tc::idesc_f16(kBM, kD, kBF16, false, true);

  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) Bars bars;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_failed;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int g = a.group, TQ = a.prefill_tq, KV = a.kv_heads, H = a.num_heads;
  const int64_t n_items = *plan.pf_total;
  if (n_items == 0) return;

  if (warp == 0) tc::alloc(&tmem_slot, 512);
  if (tid == 0) {
    mbar_init(&bars.q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.k[i], 1);
      mbar_init(&bars.v[i], 1);
      mbar_init(&bars.s[i], 1);
    }
    mbar_init(&bars.o, 1);
    fence_mbar_init();
    s_failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO = tmem + 256;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;

  // mbarrier parities (bit = next parity to wait for)
  uint32_t ph_q = 0, ph_k = 0, ph_v = 0, ph_s = 0, ph_o = 0;
  const float qk_scale = a.softcap > 0.f ? a.scale : a.scale * kLog2eP;
  const int64_t oob_z = (int64_t)a.num_blocks * a.block_size;  // past the cache: TMA zero fill

  auto wait = [&](uint64_t* bar, uint32_t& ph, int bit) -> bool {
    const bool ok = mbar_wait(bar, (ph >> bit) & 1u);
    ph ^= 1u << bit;
    if (!ok) {
      set_status(a.status, kStatusTimeout);
      s_failed = 1;
    }
    return ok;
  };

  for (int64_t it = blockIdx.x; it < n_items && !s_failed; it += gridDim.x) {
    // ---- item -> (sequence, kv head, q tile); latest q tiles first (the most keys)
    const int64_t qtiles_total = *plan.pf_total / KV;
    const int64_t qt_global = qtiles_total - 1 - it / KV;
    const int kh = (int)(it % KV);
    int lo = 0, hi = a.batch - 1;  // sequence: largest b with pf_tile_off[b] <= qt_global
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (plan.pf_tile_off[mid] <= qt_global) lo = mid; else hi = mid - 1;
    }
    const int b = lo;
    if (a.route[b] != kRoutePrefill) continue;  // moved to the generic kernel by the prologue
    const int qt = (int)(qt_global - plan.pf_tile_off[b]);
    const int c0 = a.cum[b], nq = a.cum[b + 1] - c0, past = a.past[b];
    const int total = past + nq;
    const int q0 = qt * TQ, q1 = min(q0 + TQ, nq);
    int kv_hi = a.is_causal ? past + q1 : total;
    int kv_lo = a.window > 0 ? max(0, past + q0 - a.window + 1) : 0;
    kv_lo &= ~(kTile - 1);
    const int nkv = (kv_hi - kv_lo + kBN - 1) / kBN;
    const int32_t* bt = a.block_table + (int64_t)b * a.max_blocks;

    // ---- loaders (thread 0)
    auto load_kv = [&](bool is_k, int j, int stage) {
      uint64_t* bar = is_k ? &bars.k[stage] : &bars.v[stage];
      const CUtensorMap* map = is_k ? &maps.k_map : &maps.v_map;
      uint8_t* dst = smem + (is_k ? kSmemK : kSmemV) + stage * kTileBytes;
      // Block ids of the 8 pages first (independent loads, one round trip), then the copies.
      int zs[kBN / kTile];
#pragma unroll
      for (int p = 0; p < kBN / kTile; ++p) {
        const int pos0 = kv_lo + j * kBN + p * kTile;
        const int32_t blk = pos0 < total ? __ldg(bt + pos0 / a.block_size) : -1;
        zs[p] = (blk >= 0 && blk < a.num_blocks) ? blk * a.block_size + pos0 % a.block_size : (int)oob_z;
        if (pos0 < total && !(blk >= 0 && blk < a.num_blocks)) set_status(a.status, kStatusBadBlock);
      }
      mbar_arrive_expect_tx(bar, kTileBytes);
#pragma unroll
      for (int p = 0; p < kBN / kTile; ++p)
        for (int h = 0; h < 2; ++h) tma3(dst + h * kBoxBytes + p * (kTile * 128), map, bar, h * 64, kh, zs[p]);
    };
    auto issue_qk = [&](int j) {  // S[j&1] = Q . K_j^T
      const int st = j & 1;
      for (int kk = 0; kk < kD / 16; ++kk) {
        const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
        tc::mma_ss(tS[st], tc::smem_desc(sbase + kSmemQ + off, 16, 1024),
                   tc::smem_desc(sbase + kSmemK + st * kTileBytes + off, 16, 1024), kIdQK, kk > 0);
      }
      tc::commit(&bars.s[st]);
    };

    if (tid == 0) {
      mbar_arrive_expect_tx(&bars.q, kTileBytes);
      for (int h = 0; h < 2; ++h) tma3(smem + kSmemQ + h * kBoxBytes, &maps.q_map, &bars.q, h * 64, kh * g, c0 + q0);
      load_kv(true, 0, 0);
      load_kv(false, 0, 0);
      if (nkv > 1) {
        load_kv(true, 1, 1);
        load_kv(false, 1, 1);
      }
      if (wait(&bars.q, ph_q, 0) && wait(&bars.k[0], ph_k, 0)) {
        tc::fence_after_sync();
        issue_qk(0);
      }
    }

    // ---- per-row state (thread = row = tensor-memory lane)
    const int row = tid;
    const int tl = row / g, hl = row % g;
    const bool row_ok = q0 + tl < q1;
    const int qpos = past + q0 + tl;
    float m_run = -INFINITY, l_run = 0.f;

    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      if (tid == 0 && !s_failed && j + 1 < nkv) {
        tc::fence_after_sync();
        if (wait(&bars.k[(j + 1) & 1], ph_k, (j + 1) & 1)) issue_qk(j + 1);
      }
      // S_j ready; PV_{j-1} done (P buffers free, O stable, V stage (j+1)&1 free)
      const bool ok_s = mbar_wait(&bars.s[st], (ph_s >> st) & 1u);
      ph_s ^= 1u << st;
      bool ok_o = true;
      if (j > 0) {
        ok_o = mbar_wait(&bars.o, ph_o & 1u);
        ph_o ^= 1u;
      }
      if (!ok_s || !ok_o) {
        if (tid == 0) set_status(a.status, kStatusTimeout);
        s_failed = 1;
      }
      tc::fence_after_sync();
      if (tid == 0 && !s_failed) {
        if (j + 2 < nkv) load_kv(true, j + 2, st);           // K_j consumed by S_j
        if (j >= 1 && j + 1 < nkv) load_kv(false, j + 1, (j + 1) & 1);  // V_{j-1} consumed by PV_{j-1}
      }

      // S_j row -> registers (4 x 32 columns, one wait)
      const int kbase = kv_lo + j * kBN;
      float sv[kBN / 32][32];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) tc::ld32(tS[st] + lane_off + c * 32, sv[c]);
      tc::wait_ld();
      // Masks are needed only where a key can be invisible to this row: the diagonal tile,
      // the sequence end, a left window; elsewhere scale only.
      const bool full = row_ok && kbase + kBN <= total && (!a.is_causal || kbase + kBN - 1 <= qpos) &&
                        (a.window <= 0 || kbase >= qpos - a.window + 1) && a.softcap <= 0.f;
      float m_tile = -INFINITY;
      if (full) {
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            sv[c][i] *= qk_scale;
            m_tile = fmaxf(m_tile, sv[c][i]);
          }
      } else {
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int kp = kbase + c * 32 + i;
            bool vis = row_ok && kp < total;
            if (a.is_causal) vis = vis && kp <= qpos;
            if (a.window > 0) vis = vis && kp >= qpos - a.window + 1;
            float y = sv[c][i] * qk_scale;
            if (a.softcap > 0.f) y = a.softcap * tanhf(y / a.softcap) * kLog2eP;
            sv[c][i] = vis ? y : -INFINITY;
            m_tile = fmaxf(m_tile, sv[c][i]);
          }
      }
      // lazy rescale: move the reference max only when it grows by more than 2^8
      const float m_new = fmaxf(m_run, m_tile);
      const bool grow = m_new > m_run + 8.0f;
      const float alpha = (grow && m_run != -INFINITY) ? tc::ex2(m_run - m_new) : 1.0f;
      if (grow) {
        l_run *= (m_run == -INFINITY ? 0.f : alpha);
        m_run = m_new;
      }
      if (j > 0 && __any_sync(0xffffffffu, grow && alpha != 1.0f)) {
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
      // P = 2^(s - m_run) as hi + lo 16-bit halves into swizzled shared memory
      const float mu = m_run == -INFINITY ? 0.f : m_run;
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
#pragma unroll
        for (int q8 = 0; q8 < 4; ++q8) {  // 8 keys = one 16-byte chunk
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float p0 = tc::ex2(sv[c][q8 * 8 + 2 * i] - mu);
            const float p1 = tc::ex2(sv[c][q8 * 8 + 2 * i + 1] - mu);
            lsum += p0 + p1;
            hi[i] = MMA::pack(p0, p1);
            const float2 h = MMA::unpack(hi[i]);
            lo[i] = MMA::pack(p0 - h.x, p1 - h.y);
          }
          const int chunk = c * 4 + q8;  // 0..15 over the 128 keys
          const uint32_t off = (chunk >> 3) * kBoxBytes + tc::sw128(row, chunk & 7);
          *reinterpret_cast<uint4*>(smem + kSmemPhi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(smem + kSmemPlo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
      }
      l_run += lsum;
      fence_proxy_async_smem();
      tc::fence_before_sync();
      __syncthreads();
      if (s_failed) break;
      if (tid == 0) {
        tc::fence_after_sync();
        if (wait(&bars.v[st], ph_v, st)) {
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint32_t aoff = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
            const uint32_t voff = kk * 2048;  // 16 key rows further
            const uint64_t vdesc = tc::smem_desc(sbase + kSmemV + st * kTileBytes + voff, kBoxBytes, 1024);
            tc::mma_ss(tO, tc::smem_desc(sbase + kSmemPhi + aoff, 16, 1024), vdesc, kIdPV, (j > 0 || kk > 0) ? 1u : 0u);
            tc::mma_ss(tO, tc::smem_desc(sbase + kSmemPlo + aoff, 16, 1024), vdesc, kIdPV, 1u);
          }
          tc::commit(&bars.o);
        }
      }
    }

    // ---- epilogue: wait for the last PV, normalise, store
    if (!s_failed && nkv > 0) {
      const bool ok = mbar_wait(&bars.o, ph_o & 1u);
      ph_o ^= 1u;
      if (!ok) {
        if (tid == 0) set_status(a.status, kStatusTimeout);
        s_failed = 1;
      }
    }
    tc::fence_after_sync();
    if (!s_failed) {
      float M = m_run, L = l_run, f = 1.f;
      if (a.head_sink) {
        const float sink = load_act(a.head_sink, kh * g + hl, a.act_dtype) * kLog2eP;
        const float mref = M == -INFINITY ? 0.f : M;
        // l is relative to the (possibly stale) reference max; fold the sink in the same frame
        L += exp2f(sink - mref);
        (void)f;
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      T* orow = reinterpret_cast<T*>(a.out) + (int64_t)(c0 + q0 + tl) * H * kD + (int64_t)(kh * g + hl) * kD;
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
    }
    tc::fence_before_sync();
    __syncthreads();
  }

  // Drain: never leave the CTA with copies or MMAs in flight into its shared / tensor memory.
  if (s_failed && tid == 0) {
    mbar_wait(&bars.o, ph_o & 1u);
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::dealloc(tmem, 512);
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
    paged_prefill_kernel<__nv_bfloat16><<<num_sms, 128, smem, stream>>>(a, maps, plan);
  } else {
    if (!attr_set[0]) {
      e = cudaFuncSetAttribute(paged_prefill_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      attr_set[0] = true;
    }
    paged_prefill_kernel<__half><<<num_sms, 128, smem, stream>>>(a, maps, plan);
  }
  return cudaGetLastError();
}

}  // namespace b200
