// Ragged causal chunked prefill over the paged cache on the 5th-generation tensor core.
//
// Replaces the reference's per-sequence gather + SDPA for prefill chunks
// (rust/src/ops/attention.rs:4192-4319, native grouped-query prefill :4235-4253): same
// mathematics as the decode kernel (scale*q.k, softcap, top-left causal and left-window masks,
// fp32 softmax with optional sink, fp32 accumulation).
//
// B200 design:
//  * work item = (sequence, kv head, pair of q tiles).  A q tile is 128 rows = 128/g query
//    tokens x the g query heads of the kv head, so each K/V tile serves the whole head group
//    (native GQA), and the two q tiles of an item share every K/V tile they load;
//  * persistent CTAs (one per SM: 224 KB of shared memory and all 512 tensor-memory columns)
//    take items from the list (longest, i.e. latest q tiles, first) by an atomic counter when
//    ready for the next one;
//  * warp-specialised, the roles synchronised only through mbarriers:
//      - warp 8 (TMA producer): Q tiles [128 x 128] by a 3-D box pair from the [nt, H, d]
//        query view, one buffer per q tile; K tiles (2 stages) and V tiles (3 stages) of 128
//        keys = 8 pages of 16 slots, one 64-channel box per lane; pages past the sequence end
//        load from an out-of-range coordinate (TMA zero fill);
//      - warp 9 (MMA issuer, one thread): per K/V tile j, in order
//          PV0(j-1), S0(j), PV1(j-1), S1(j)
//        with S = Q K^T (tcgen05.mma kind::f16, M=N=128, K=16 steps, both operands in shared
//        memory) and O += P V (P from tensor memory, V as the MN-major operand in the cache's
//        [key][channel] layout).  While warpgroup 0 turns S0 into P0 the tensor core runs
//        PV1/S1, and the other way round (ping-pong);
//      - warpgroups 0 and 1 (softmax and epilogue of q tile 0 / 1, one row per thread =
//        tensor-memory lane): exp2-domain softmax with a lazily rescaled running max (O is
//        rescaled in tensor memory only when the max grows by more than 2^8); P goes back over
//        the S columns: fp16 P (11 significant bits, one P . V MMA per 16 keys) for fp16
//        activations; for bf16 a hi + lo pair of bf16 values (~16 bits, two MMAs), since one
//        bf16 P (8 bits) costs up to ~3e-3 on unit-scale data; the epilogue
//        normalises (sink) and stores the rows;
//  * tensor memory: S0/P0 columns [0,128), S1/P1 [128,256), O0 [256,384), O1 [384,512);
//  * registers: warpgroups 0-1 grow to 200 per thread and warpgroup 2 shrinks to 96
//    (setmaxnreg); together they stay within the 384 x 168 the block is launched with, which
//    the launcher checks before the first launch (a split above it would never complete);
//  * every mbarrier wait is bounded (%globaltimer); a timeout sets the status word, the CTA
//    waits (bounded) for its own copies and MMAs in flight, frees tensor memory and returns.
#include <algorithm>
#include <atomic>
#include <type_traits>

#include "b200_common.cuh"
#include "b200_kernels.h"
#include "b200_tcgen05.cuh"

namespace b200 {

// Optional per-event timestamps of CTA 0 (build with -DB200_PREFILL_TRACE): slot = 16 x counter +
// event, events 0/1 S0/S1 issued, 2/3 PV0/PV1 issued, 4 K resident, 5 V resident, 6/7/8 and
// 9/10/11 warpgroup 0/1 S loaded / P written / row stored, 12/13 K/V copy issued, 14/15 P0/P1
// seen by the MMA issuer.
#ifdef B200_PREFILL_TRACE
constexpr int kTraceSlots = 1 << 16;
__device__ long long g_prefill_trace[kTraceSlots];
#define PF_TRACE(slot)                                                  \
  do {                                                                  \
    const int _s = (slot);                                              \
    if (blockIdx.x == 0 && _s >= 0 && _s < kTraceSlots) g_prefill_trace[_s] = clock64(); \
  } while (0)
#else
#define PF_TRACE(slot) \
  do {                 \
  } while (0)
#endif

namespace {

constexpr int kBM = 128;             // q rows per tile
constexpr int kBN = 128;             // keys per tile
constexpr int kD = 128;              // head size of this kernel
constexpr int kQTiles = 2;           // q tiles per work item
constexpr int kKStages = 2;          // K pipeline depth
constexpr int kVStages = 3;          // V pipeline depth
constexpr int kBoxBytes = 128 * 128; // one [128 rows][64 channels] 16-bit box: 16 KB
constexpr int kTileBytes = 2 * kBoxBytes;  // [128][128] 16-bit tile: 32 KB
constexpr float kLog2eP = 1.4426950408889634f;
constexpr int kPolyEvery = 4;        // every 4th exponential pair of a softmax on the FMA pipe

// shared-memory map (offsets from the 1024-aligned base)
constexpr int kSmemQ = 0;                                   // kQTiles Q tiles
constexpr int kSmemK = kSmemQ + kQTiles * kTileBytes;       // kKStages K tiles
constexpr int kSmemV = kSmemK + kKStages * kTileBytes;      // kVStages V tiles
constexpr int kSmemBytes = kSmemV + kVStages * kTileBytes;  // 224 KB

// Roles: warpgroups 0-1 softmax / epilogue of q tile 0 / 1; warpgroup 2 = warp 8 TMA producer of
// Q and K, warp 9 MMA issuer, warp 10 TMA producer of V, warp 11 idle.
constexpr int kThreads = 384;
constexpr int kWgThreads = 128;
constexpr int kProducerWarp = 8;   // Q and K tiles
constexpr int kMmaWarp = 9;
constexpr int kVProducerWarp = 10; // V tiles: its own warp, so a V stage refills as soon as it frees
constexpr int kSoftmaxRegs = 200;  // setmaxnreg split: 2 x 128 x 200 + 128 x 96 = 63488
constexpr int kControlRegs = 96;
constexpr int kSplitRegs = 2 * kWgThreads * kSoftmaxRegs + kWgThreads * kControlRegs;
static_assert(kSplitRegs <= kThreads * 168, "register split exceeds the 384 x 168 launch allocation");
// Work items are handed out at run time: warp 8 takes the next item of the list with an atomicAdd
// on plan.pf_next when it is ready for it and passes it through a kSched-slot queue in shared
// memory to the other roles, so CTAs that finish early take more items (the list is longest
// first) instead of a fixed round-robin share.
constexpr int kSched = 4;
constexpr int kSchedTakers = 2 * kWgThreads / 32 + 2;  // softmax warps, MMA warp, V producer warp

struct Bars {
  uint64_t q_full[kQTiles], q_empty[kQTiles];
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full[kVStages], v_empty[kVStages];
  // o_done[w] completes once per item of q tile w, after its last P . V (the epilogue's wait).
  // Within an item no O wait is needed: S_w(j) is issued after PV_w(j-1) and a commit covers all
  // earlier MMAs, so s_full[w] for tile j also says that P . V of tile j-1 has landed in O.
  uint64_t s_full[kQTiles], p_full[kQTiles], o_done[kQTiles];
  uint64_t drain;
  uint64_t sched_full[kSched], sched_empty[kSched];  // item queue: published / taken by every taker warp
};

// One item of the prefill work list, as every role decodes it.
struct Item {
  int skip, b, kh, c0, nq, past, total, q0, kv_lo, n;
  int nkv[kQTiles];  // K/V tiles q tile w needs (0: the tile has no rows); n = max
};

__device__ __forceinline__ Item decode_item(const AttnArgs& a, const DecodePlan& plan, int64_t it) {
  Item m{};
  const int KV = a.kv_heads, TQ = a.prefill_tq / kQTiles;
  const int64_t items_total = *plan.pf_total / KV;
  const int64_t qt_global = items_total - 1 - it / KV;  // latest q tiles (most keys) first
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
  m.q0 = qt * a.prefill_tq;
  m.kv_lo = a.window > 0 ? max(0, m.past + m.q0 - a.window + 1) : 0;
  m.kv_lo &= ~(kTile - 1);
  m.n = 0;
#pragma unroll
  for (int w = 0; w < kQTiles; ++w) {
    const int t0 = m.q0 + w * TQ, t1 = min(t0 + TQ, m.nq);
    const int kv_hi = a.is_causal ? m.past + t1 : m.total;
    m.nkv[w] = t0 < m.nq ? (kv_hi - m.kv_lo + kBN - 1) / kBN : 0;
    m.n = max(m.n, m.nkv[w]);
  }
  return m;
}

// K/V tiles of q tile w, by select (an indexed read with a run-time w would put the Item in
// local memory)
__device__ __forceinline__ int nkv_of(const Item& m, int w) { return w ? m.nkv[1] : m.nkv[0]; }

// Rows of K/V tile j that hold the sequence's keys; fewer than kBN only for an item's last tile
// (earlier tiles end below kv_hi <= total).
__device__ __forceinline__ int tile_rows(const Item& m, int j) { return min(kBN, m.total - (m.kv_lo + j * kBN)); }

// Page `page` of a V stage (16 rows of both 64-channel boxes) by plain loads: rows [0, rows)
// from the cache (block `blk`, slots from position `pos0`), the rest zero.  The stores follow the
// TMA's 128B swizzle (16-byte piece c of row r at piece c ^ (r & 7); the stage is 1024-byte
// aligned), and a proxy fence orders them before the tensor core's reads.  A whole warp; `blk`
// out of range (already reported by the caller) fills zeros.  Out of line: it runs once per
// sequence end at most, and the producer's loop stays small.
__device__ __noinline__ void fill_tail_page(uint8_t* stage, const AttnArgs& a, int32_t blk, int pos0, int kh, int page,
                                            int rows, int lane) {
  const bool blk_ok = blk >= 0 && blk < a.num_blocks;
  const int D = a.head_size;
  const int64_t slot0 = (int64_t)blk * a.block_size + pos0 % a.block_size;
  for (int i = lane; i < kTile * 16; i += 32) {  // i = row (16) x box (2) x 16-byte piece (8)
    const int r = i >> 4, box = (i >> 3) & 1, piece = i & 7;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < rows && blk_ok) {
      const uint8_t* src = static_cast<const uint8_t*>(a.value_cache) +
                           (((slot0 + r) * a.kv_heads + kh) * D + box * 64) * 2 + piece * 16;
      v = *reinterpret_cast<const uint4*>(src);
    }
    const int row = page * kTile + r;
    *reinterpret_cast<uint4*>(stage + box * kBoxBytes + row * 128 + ((piece ^ (row & 7)) * 16)) = v;
  }
  fence_proxy_async_smem();
  __syncwarp();
}

}  // namespace

bool prefill_supported(int head_size, int block_size, int group, int act_dtype, int cache_dtype) {
  return head_size == kD && block_size % kTile == 0 && act_dtype == cache_dtype &&
         (act_dtype == B200_DTYPE_FLOAT16 || act_dtype == B200_DTYPE_BFLOAT16) &&
         (group == 1 || group == 2 || group == 4 || group == 8 || group == 16);
}

int prefill_tokens_per_item(int group) { return kQTiles * kBM / group; }

// SHADOW (bf16 only): V tiles come from an fp16 copy of the call's new V rows (maps.vs_map; every
// prefill sequence has no cached prefix), so P is one fp16 value as for fp16 activations.
template <typename T, bool SHADOW>
__global__ void __launch_bounds__(kThreads, 1) paged_prefill_kernel(const __grid_constant__ AttnArgs a,
                                                                     const __grid_constant__ PrefillMaps maps,
                                                                     const DecodePlan plan) {
  using MMA = mma_op<T>;  // packing helpers only
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr bool kHiLo = kBF16 && !SHADOW;  // P as a hi + lo pair of bf16 values
  constexpr uint32_t kIdQK = tc::idesc_f16(kBM, kBN, kBF16, false, false);
  constexpr uint32_t kIdPV = tc::idesc_f16(kBM, kD, kHiLo, false, true);
  // The shadow-V launch steps aside when the copy found a value beyond the fp16 range; the bf16
  // launch after it runs only then.
  if (a.v_shadow_wide && (SHADOW || a.prefill_fallback)) {
    const int wide = *a.v_shadow_wide;
    if (SHADOW ? wide != 0 : wide == 0) return;
  }

  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) Bars bars;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int s_failed;
  __shared__ volatile long long s_item[kSched];

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = a.group, H = a.num_heads, TQ = a.prefill_tq / kQTiles;
  const int64_t n_items = *plan.pf_total;
  if (n_items == 0) return;

  if (warp == kMmaWarp) tc::alloc(&tmem_slot, 512);
  if (tid == 0) {
    for (int w = 0; w < kQTiles; ++w) {
      mbar_init(&bars.q_full[w], 1);
      mbar_init(&bars.q_empty[w], 1);
      mbar_init(&bars.s_full[w], 1);
      mbar_init(&bars.p_full[w], kWgThreads);
      mbar_init(&bars.o_done[w], 1);
    }
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&bars.k_full[i], 1);
      mbar_init(&bars.k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(&bars.v_full[i], 1);
      mbar_init(&bars.v_empty[i], 1);
    }
    mbar_init(&bars.drain, 1);
    for (int i = 0; i < kSched; ++i) {
      mbar_init(&bars.sched_full[i], 1);
      mbar_init(&bars.sched_empty[i], kSchedTakers);
    }
    fence_mbar_init();
    s_failed = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;

  // Bounded wait on completion `index` of an mbarrier (parity = index & 1).
  auto wait_idx = [&](uint64_t* bar, uint32_t index) -> bool {
    if (s_failed) return false;
    if (mbar_wait(bar, index & 1u)) return true;
    set_status(a.status, kStatusTimeout);
    s_failed = 1;
    return false;
  };
  // Warp-uniform bounded wait: every lane waits, then the warp agrees, so warp-collective code
  // after it (tensor-memory loads/stores, __syncwarp) never runs with part of a warp.
  auto wait_warp = [&](uint64_t* bar, uint32_t index) -> bool {
    return __all_sync(0xffffffffu, wait_idx(bar, index));
  };
  auto failed_warp = [&]() -> bool { return __any_sync(0xffffffffu, s_failed != 0); };
  // After a failure: bounded wait for a copy or commit this CTA issued, without the early exit.
  auto drain_idx = [&](uint64_t* bar, uint32_t index) { mbar_wait(bar, index & 1u); };
  // k-th work item of this CTA (n_items or more: none left).  Warp 8 takes it from the list and
  // publishes it; every taker warp reads it and frees the slot.  False when a wait ran out.
  auto fetch_item = [&](uint32_t k, int64_t& it) -> bool {
    const uint32_t slot = k % kSched;
    if (k >= (uint32_t)kSched && !wait_warp(&bars.sched_empty[slot], k / kSched - 1)) return false;
    long long v = 0;
    if (lane == 0) {
      v = (long long)atomicAdd(plan.pf_next, 1ull);
      s_item[slot] = v;
      mbar_arrive(&bars.sched_full[slot]);
    }
    it = __shfl_sync(0xffffffffu, v, 0);
    return true;
  };
  auto take_item = [&](uint32_t k, int64_t& it) -> bool {
    const uint32_t slot = k % kSched;
    if (!wait_warp(&bars.sched_full[slot], k / kSched)) return false;
    it = s_item[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars.sched_empty[slot]);
    return true;
  };

  if (warp >= 2 * (kWgThreads / 32)) {
    // warpgroup 2: producers, MMA issuer and an idle warp give registers to the softmax
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kControlRegs));
    if (warp == kProducerWarp || warp == kVProducerWarp) {
      // ------------------------------------------------------------------ TMA producers
      // Warp 8 loads Q and K tiles, warp 10 V tiles; each ring refills as soon as its stage frees.
      // Lane l < 16 loads box (page l / 2, channel half l & 1) of each tile; its block id is
      // loaded one tile ahead, so the block-table read never sits between a free stage and its copy.
      const bool is_v = warp == kVProducerWarp;
      const int stages = is_v ? kVStages : kKStages;
      uint64_t* full_bar = is_v ? bars.v_full : bars.k_full;
      uint64_t* empty_bar = is_v ? bars.v_empty : bars.k_empty;
      const bool from_shadow = SHADOW && is_v;  // V rows of the call's fp16 copy: no pages
      const CUtensorMap* map = from_shadow ? &maps.vs_map : is_v ? &maps.v_map : &maps.k_map;
      const uint32_t ring = sbase + (is_v ? kSmemV : kSmemK);
      uint32_t qc0 = 0, qc1 = 0, c = 0;  // Q loads per buffer, tiles loaded on this ring (scalars: no local memory)
      const int64_t oob_z = (int64_t)a.num_blocks * a.block_size;  // past the cache: zero fill
      const int page = (lane & 15) >> 1, half = lane & 1;
      const bool loader = lane < 16;
      bool ok = true;
      for (uint32_t k = 0; ok && !failed_warp(); ++k) {
        int64_t it;
        if (!(ok = is_v ? take_item(k, it) : fetch_item(k, it)) || it >= n_items) break;
        const Item m = decode_item(a, plan, it);
        if (m.skip) continue;
        if (!is_v) {
          for (int w = 0; w < kQTiles && ok; ++w) {
            if (nkv_of(m, w) == 0) continue;
            const uint32_t qc = w ? qc1 : qc0;
            if (qc > 0 && !(ok = wait_warp(&bars.q_empty[w], qc - 1))) break;
            if (lane == 0) mbar_arrive_expect_tx(&bars.q_full[w], kTileBytes);
            __syncwarp();
            if (lane < 2)
              tma_load_3d(smem + kSmemQ + w * kTileBytes + lane * kBoxBytes, &maps.q_map, &bars.q_full[w], lane * 64,
                          m.kh * g, m.c0 + m.q0 + w * TQ);
            if (w) qc1 = qc + 1; else qc0 = qc + 1;
          }
        }
        const int32_t* bt = a.block_table + (int64_t)m.b * a.max_blocks;
        auto block_of = [&](int j) -> int32_t {
          const int pos = m.kv_lo + j * kBN + page * kTile;
          return loader && pos < m.total ? __ldg(bt + pos / a.block_size) : -1;
        };
        int32_t blk_next = m.n > 0 ? block_of(0) : -1;
        for (int j = 0; j < m.n && ok; ++j) {
          const int pos0 = m.kv_lo + j * kBN + page * kTile;
          const int32_t blk = blk_next;
          if (j + 1 < m.n) blk_next = block_of(j + 1);  // in flight during the stage wait below
          const bool blk_ok = blk >= 0 && blk < a.num_blocks;
          if (!is_v && loader && pos0 < m.total && !blk_ok) set_status(a.status, kStatusBadBlock);
          // copy row of position pos0 (no cached prefix): its token, or past the call's rows
          // (zero fill); rows past the sequence's end are the next sequence's, finite, and get P = 0
          const int z = from_shadow ? m.c0 + pos0 - m.past
                                    : blk_ok ? blk * a.block_size + pos0 % a.block_size : (int)oob_z;
          const int st = (int)(c % (uint32_t)stages);
          if (c >= (uint32_t)stages && !(ok = wait_warp(&empty_bar[st], c / stages - 1))) break;
          // A V page that reaches past the sequence's last key (rows `rows` of 16 are the
          // sequence's): its rows come by plain loads and its unused slots are zeroed, since
          // whatever they hold, NaN included, must not meet P = 0 in the MMA.  Pages wholly past
          // the end load zero-filled by TMA.
          const int rows = is_v && !from_shadow ? tile_rows(m, j) & (kTile - 1) : 0;
          const int tail_page = tile_rows(m, j) >> 4;
          if (rows) {
            const int32_t tblk = __shfl_sync(0xffffffffu, blk, 2 * tail_page);
            const int tpos = __shfl_sync(0xffffffffu, pos0, 2 * tail_page);
            fill_tail_page(smem + kSmemV + st * kTileBytes, a, tblk, tpos, m.kh, tail_page, rows, lane);
          }
          if (lane == 0) mbar_arrive_expect_tx(&full_bar[st], rows ? kTileBytes - kTile * 256 : kTileBytes);
          __syncwarp();
          if (loader && !(rows && page == tail_page))
            tma_load_3d(smem + (ring - sbase) + st * kTileBytes + half * kBoxBytes + page * (kTile * 128), map,
                        &full_bar[st], half * 64, m.kh, z);
          if (lane == 0) PF_TRACE(c * 16 + (is_v ? 13 : 12));
          ++c;
        }
      }
      // Every issued copy lands before the CTA can exit (immediate on the normal path).
      if (qc0 > 0) drain_idx(&bars.q_full[0], qc0 - 1);
      if (qc1 > 0) drain_idx(&bars.q_full[1], qc1 - 1);
      for (uint32_t i = (c > (uint32_t)stages ? c - stages : 0); i < c; ++i) drain_idx(&full_bar[i % stages], i / stages);
    } else if (warp == kMmaWarp) {
      // ------------------------------------------------------------------ MMA issuer
      // The whole warp runs the schedule (waits, counters, descriptors stay warp-uniform and in
      // uniform registers); one elected lane issues the MMAs and their commits.
      const bool leader = tc::elect_one();
      uint32_t qc0 = 0, qc1 = 0, pc0 = 0, pc1 = 0, kvc = 0;
      bool issued = false, ok = true;
      for (uint32_t k = 0; ok && !failed_warp(); ++k) {
        int64_t it;
        if (!(ok = take_item(k, it)) || it >= n_items) break;
        const Item m = decode_item(a, plan, it);
        if (m.skip) continue;
        // Step j issues PV0(j-1), S0(j), PV1(j-1), S1(j) (step n: the last PVs only), each from
        // one call site so the issuing loop stays small; a late K_j never holds back PV0(j-1).
#pragma unroll 1
        for (int j = 0; j <= m.n && ok; ++j) {
          const uint32_t ki = kvc + j, vi = ki - 1;
          if (j > 0) {
            if (!(ok = wait_warp(&bars.v_full[vi % kVStages], vi / kVStages))) break;
            PF_TRACE(vi * 16 + 5);
          }
          bool k_ready = false;
#pragma unroll 1
          for (int w = 0; w < kQTiles; ++w) {
            const uint32_t pc = w ? pc1 : pc0;  // values, not references: no local memory
            if (j > 0 && j - 1 < nkv_of(m, w)) {  // O_w (+)= P_w(j-1) . V_(j-1)
              if (!(ok = wait_warp(&bars.p_full[w], pc))) break;
              tc::fence_after_sync();  // P was written to tensor memory by the softmax threads
              PF_TRACE(pc * 16 + 14 + w);
              const uint32_t pbuf = tmem + w * 128, obuf = tmem + 256 + w * 128;
              // one descriptor per stage; a K step of 16 keys adds 2048 B = 128 in the address field
              const uint64_t vdesc0 = tc::smem_desc(sbase + kSmemV + (vi % kVStages) * kTileBytes, kBoxBytes, 1024);
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk) {
                const uint64_t vdesc = vdesc0 + (uint64_t)(kk * (2048 >> 4));
                // P of keys 16kk..16kk+15 at chunk kk/2's columns (kk%2)*8..; bf16: the lo halves
                // 16 columns on
                const uint32_t pcol = pbuf + (kk >> 1) * 32 + (kk & 1) * 8;
                if (leader) {
                  tc::mma_ts(obuf, pcol, vdesc, kIdPV, (j > 1 || kk > 0) ? 1u : 0u);
                  if (kHiLo) tc::mma_ts(obuf, pcol + 16, vdesc, kIdPV, 1u);
                }
              }
              if (leader && j == nkv_of(m, w)) tc::commit(&bars.o_done[w]);  // the item's last P . V
              PF_TRACE(pc * 16 + 2 + w);
              if (w) pc1 = pc + 1; else pc0 = pc + 1;
            }
            if (j < nkv_of(m, w)) {  // S_w(j) = Q_w . K_j^T into the S_w columns
              if (!k_ready) {  // K and Q arrive by TMA: the mbarrier wait orders them for the MMA
                if (!(ok = wait_warp(&bars.k_full[ki % kKStages], ki / kKStages))) break;
                PF_TRACE(ki * 16 + 4);
                k_ready = true;
              }
              if (j == 0 && !(ok = wait_warp(&bars.q_full[w], w ? qc1 : qc0))) break;
              // base descriptors once; the K step's byte offset goes straight into the address field
              const uint64_t kdesc0 = tc::smem_desc(sbase + kSmemK + (ki % kKStages) * kTileBytes, 16, 1024);
              const uint64_t qdesc0 = tc::smem_desc(sbase + kSmemQ + w * kTileBytes, 16, 1024);
#pragma unroll
              for (int kk = 0; kk < kD / 16; ++kk) {
                const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
                const uint64_t qdesc = qdesc0 + (uint64_t)(off >> 4), kdesc = kdesc0 + (uint64_t)(off >> 4);
                if (leader) tc::mma_ss(tmem + w * 128, qdesc, kdesc, kIdQK, kk > 0);
              }
              if (leader) tc::commit(&bars.s_full[w]);
              PF_TRACE((w ? pc1 : pc0) * 16 + w);
              if (j == nkv_of(m, w) - 1) {  // last use of Q_w in this item
                if (leader) tc::commit(&bars.q_empty[w]);
                if (w) ++qc1; else ++qc0;
              }
              issued = true;
            }
          }
          if (!ok) break;
          if (leader && j > 0) tc::commit(&bars.v_empty[vi % kVStages]);
          if (leader && k_ready) tc::commit(&bars.k_empty[ki % kKStages]);
        }
        kvc += m.n;
      }
      // Every issued MMA completes before tensor memory is freed (immediate on the normal path).
      if (issued) {
        if (leader) tc::commit(&bars.drain);
        drain_idx(&bars.drain, 0);
      }
      __syncwarp();
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    // ------------------------------------------------------------------ softmax + epilogue
    const int w = warp >> 2;           // q tile of this warpgroup
    const int row = tid & (kWgThreads - 1);
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t sbuf = tmem + w * 128 + lane_off, obuf = tmem + 256 + w * 128 + lane_off;
    const float qk_scale = a.softcap > 0.f ? a.scale : a.scale * kLog2eP;
    uint32_t t = 0;      // tiles this warpgroup has processed
    uint32_t items = 0;  // items this warpgroup has finished (o_done completions)
    for (uint32_t k = 0; !failed_warp(); ++k) {
      int64_t it;
      if (!take_item(k, it) || it >= n_items) break;
      const Item m = decode_item(a, plan, it);
      if (m.skip || nkv_of(m, w) == 0) continue;
      const int tl = row / g, hl = row % g;
      const int tok = m.q0 + w * TQ + tl;
      const bool row_ok = tl < TQ && tok < m.nq;
      const int qpos = m.past + tok;
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int j = 0; j < nkv_of(m, w); ++j, ++t) {
        if (!(ok = wait_warp(&bars.s_full[w], t))) break;
        tc::fence_after_sync();
        if (row == 0) PF_TRACE(t * 16 + 6 + 3 * w);
        const int kbase = m.kv_lo + j * kBN;
        // Masks only where a key can be invisible to this row (diagonal tile, sequence end, window).
        const bool full = row_ok && kbase + kBN <= m.total && (!a.is_causal || kbase + kBN - 1 <= qpos) &&
                          (a.window <= 0 || kbase >= qpos - a.window + 1) && a.softcap <= 0.f;
        // In the unmasked case the scores stay raw and scale folds into the exponent's FMA
        // (qk_scale > 0); masked tiles are rewritten in place to scaled log2 values (-inf = masked).
        // Warp-uniform: both paths use tensor-memory loads/stores, which the whole warp executes
        // together (the masked path is also exact for rows that see the whole tile).
        const bool raw = __all_sync(0xffffffffu, full && qk_scale > 0.f);
        float mx[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) mx[r] = -INFINITY;
        if (raw) {
          float sv[kBN / 32][32];
#pragma unroll
          for (int c = 0; c < kBN / 32; ++c) tc::ld32(sbuf + c * 32, sv[c]);
          tc::wait_ld();
#pragma unroll
          for (int c = 0; c < kBN / 32; ++c)
#pragma unroll
            for (int i = 0; i < 16; ++i) mx[i & 3] = tc::max3(mx[i & 3], sv[c][2 * i], sv[c][2 * i + 1]);
        } else {
          // Keys this row sees, as a column range [vlo, vhi] of the tile (empty for padding rows).
          const int vhi = row_ok ? min(m.total - 1, a.is_causal ? qpos : m.total - 1) - kbase : -1;
          const int vlo = (a.window > 0 ? qpos - a.window + 1 : 0) - kbase;
#pragma unroll 1
          for (int c = 0; c < kBN / 32; ++c) {
            float x[32];
            tc::ld32(sbuf + c * 32, x);
            tc::wait_ld();
            if (a.softcap > 0.f) {
              // cap * tanh(y / cap) in the log2 domain, tanh(u) = 1 - 2 / (1 + e^(2u)).
              const float two_log2e_over_cap = 2.f * kLog2eP / a.softcap, cap_log2e = a.softcap * kLog2eP;
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float e = tc::ex2(fminf(x[i] * qk_scale * two_log2e_over_cap, 126.f));
                x[i] = cap_log2e * (1.f - __fdividef(2.f, 1.f + e));
              }
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) x[i] *= qk_scale;
            }
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = c * 32 + i;
              x[i] = (col >= vlo && col <= vhi) ? x[i] : -INFINITY;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) mx[i & 3] = tc::max3(mx[i & 3], x[2 * i], x[2 * i + 1]);
            tc::st32(sbuf + c * 32, x);
          }
          tc::wait_st();
        }
        float m_tile = tc::max3(mx[0], mx[1], fmaxf(mx[2], mx[3]));
        if (raw) m_tile *= qk_scale;
        // Lazy rescale: the reference max moves only when the row max grows by more than 2^8.
        const float m_new = fmaxf(m_run, m_tile);
        const bool grow = m_new > m_run + 8.0f;
        const float alpha = (grow && m_run != -INFINITY) ? tc::ex2(m_run - m_new) : 1.0f;
        if (grow) {
          l_run *= (m_run == -INFINITY ? 0.f : alpha);
          m_run = m_new;
        }
        if (j > 0 && __any_sync(0xffffffffu, grow && alpha != 1.0f)) {
          // O holds tiles < j and P . V of tile j-1 has landed (s_full of tile j, waited above, covers
          // it): scale this warp's rows in place.
#pragma unroll 1
          for (int c = 0; c < kD / 16; ++c) {
            float r[16];
            tc::ld16(obuf + c * 16, r);
            tc::wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] *= alpha;
            tc::st16(obuf + c * 16, r);
          }
          tc::wait_st();
        }
        // P = 2^(s * kscale - mu) per 32-column chunk of S, over the chunk's first 16 columns (fp16,
        // or bf16 hi halves with the lo halves over its last 16; each chunk is read before it is
        // overwritten)
        const float mu = m_run == -INFINITY ? 0.f : m_run;
        const float kscale = raw ? qk_scale : 1.0f;
        const float2 ks2 = make_float2(kscale, kscale), nmu2 = make_float2(-mu, -mu);
        float2 ls[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        auto exp_chunk = [&](const float(&x)[32], int c) {
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 e = tc::fma2(make_float2(x[2 * i], x[2 * i + 1]), ks2, nmu2);
            // every kPolyEvery-th pair on the FMA pipe, the rest on the MUFU unit
            const float2 p = (kPolyEvery > 0 && i % kPolyEvery == kPolyEvery - 1) ? tc::exp2_poly2(e)
                                                                                   : make_float2(tc::ex2(e.x), tc::ex2(e.y));
            ls[i & 1] = tc::add2(ls[i & 1], p);
            if constexpr (kHiLo) {
              // hi = p truncated to bf16 (its upper 16 bits), lo = p - hi exactly, then rounded
              const uint32_t u0 = __float_as_uint(p.x), u1 = __float_as_uint(p.y);
              hi[i] = __byte_perm(u0, u1, 0x7632);
              const float2 l = tc::sub2(p, make_float2(__uint_as_float(u0 & 0xffff0000u), __uint_as_float(u1 & 0xffff0000u)));
              lo[i] = MMA::pack(l.x, l.y);
            } else if constexpr (kBF16) {  // shadow V: fp16 P
              const __half2 h = __floats2half2_rn(p.x, p.y);
              hi[i] = *reinterpret_cast<const uint32_t*>(&h);
            } else {
              hi[i] = MMA::pack(p.x, p.y);
            }
          }
          tc::st16u(sbuf + c * 32, hi);
          if constexpr (kHiLo) tc::st16u(sbuf + c * 32 + 16, lo);
        };
        // Chunk c+1's tensor-memory load is in flight while chunk c is exponentiated.
        float xa[32], xb[32];
        tc::ld32(sbuf, xa);
        tc::wait_ld();
#pragma unroll 1
        for (int c = 0; c < kBN / 32; c += 2) {
          tc::ld32(sbuf + (c + 1) * 32, xb);
          exp_chunk(xa, c);
          tc::wait_ld();
          if (c + 2 < kBN / 32) tc::ld32(sbuf + (c + 2) * 32, xa);
          exp_chunk(xb, c + 1);
          tc::wait_ld();
        }
        l_run += (ls[0].x + ls[1].x) + (ls[0].y + ls[1].y);
        tc::wait_st();
        tc::fence_before_sync();
        mbar_arrive(&bars.p_full[w]);
        if (row == 0) PF_TRACE(t * 16 + 7 + 3 * w);
      }
      if (!ok) break;
      // ---- epilogue: last PV done -> normalise -> store this row
      if (!wait_warp(&bars.o_done[w], items++)) break;
      tc::fence_after_sync();
      float L = l_run;
      if (a.head_sink) {  // l is relative to the reference max m_run; fold the sink in that frame
        const float sink = load_act(a.head_sink, m.kh * g + hl, a.act_dtype) * kLog2eP;
        L += tc::ex2(sink - (m_run == -INFINITY ? 0.f : m_run));
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      T* orow = reinterpret_cast<T*>(a.out) + (int64_t)(m.c0 + tok) * H * kD + (int64_t)(m.kh * g + hl) * kD;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float o[2][32];
        tc::ld32(obuf + h * 64, o[0]);
        tc::ld32(obuf + h * 64 + 32, o[1]);
        tc::wait_ld();
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint32_t v[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) v[i] = MMA::pack(o[c][q * 8 + 2 * i] * inv, o[c][q * 8 + 2 * i + 1] * inv);
              reinterpret_cast<uint4*>(orow + h * 64 + c * 32 + q * 8)[0] = make_uint4(v[0], v[1], v[2], v[3]);
            }
        }
      }
      if (row == 0) PF_TRACE((t - 1) * 16 + 8 + 3 * w);
      tc::fence_before_sync();
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == kMmaWarp) tc::dealloc(tmem, 512);
}

template <typename T, bool SHADOW>
cudaError_t launch_prefill_t(const AttnArgs& a, const DecodePlan& plan, const PrefillMaps& maps, int num_sms,
                             cudaStream_t stream) {
  const size_t smem = kSmemBytes + 1024;
  auto kernel = paged_prefill_kernel<T, SHADOW>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::atomic<uint32_t> ready[64];  // per device: attributes set and checked
  std::atomic<uint32_t>& flag = ready[dev & 63];
  if (!flag.load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // setmaxnreg.inc waits until the block's launch allocation can cover the split.
    cudaFuncAttributes attr;
    e = cudaFuncGetAttributes(&attr, kernel);
    if (e != cudaSuccess) return e;
    if (attr.numRegs * kThreads < kSplitRegs) return cudaErrorInvalidConfiguration;
    flag.store(1, std::memory_order_release);
  }
  kernel<<<num_sms, kThreads, smem, stream>>>(a, maps, plan);
  return cudaGetLastError();
}

cudaError_t launch_prefill(const AttnArgs& a, const DecodePlan& plan, const PrefillMaps& maps, int num_sms,
                           cudaStream_t stream, bool shadow_v) {
  if (a.act_dtype != B200_DTYPE_BFLOAT16) return launch_prefill_t<__half, false>(a, plan, maps, num_sms, stream);
  if (!shadow_v) return launch_prefill_t<__nv_bfloat16, false>(a, plan, maps, num_sms, stream);
  cudaError_t e = launch_prefill_t<__nv_bfloat16, true>(a, plan, maps, num_sms, stream);
  if (e != cudaSuccess) return e;
  AttnArgs fb = a;
  fb.prefill_fallback = 1;
  return launch_prefill_t<__nv_bfloat16, false>(fb, plan, maps, num_sms, stream);
}

// fp16 copy of the new V rows, 8 channels per thread; a value beyond the fp16 range (bf16
// magnitude bits >= 0x4780: bit 15 of (bits & 0x7fff) + 0x3880) sets the flag word.
__global__ void __launch_bounds__(256) v_shadow_kernel(const AttnArgs a, uint4* shadow) {
  const int vecs = a.kv_heads * a.head_size / 8;  // 16-byte pieces of one token's V row
  const int64_t n = (int64_t)a.num_tokens * vecs;
  uint32_t over = 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / vecs;
    const int c = (int)(i - t * vecs);
    const uint4 v = *reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.v_new) + t * a.v_stride + c * 8);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      over |= (w[k] & 0x7fff7fffu) + 0x38803880u;
      const __half2 h = __floats2half2_rn(__uint_as_float(w[k] << 16), __uint_as_float(w[k] & 0xffff0000u));
      o[k] = *reinterpret_cast<const uint32_t*>(&h);
    }
    shadow[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (__any_sync(0xffffffffu, (over & 0x80008000u) != 0) && (threadIdx.x & 31) == 0) atomicOr(a.v_shadow_wide, 1);
}

cudaError_t launch_v_shadow(const AttnArgs& a, void* shadow, cudaStream_t stream) {
  const int64_t n = (int64_t)a.num_tokens * a.kv_heads * a.head_size / 8;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 8));
  v_shadow_kernel<<<grid, 256, 0, stream>>>(a, static_cast<uint4*>(shadow));
  return cudaGetLastError();
}

#ifdef B200_PREFILL_TRACE
extern "C" __attribute__((visibility("default"))) int b200_prefill_trace_dump(long long* host, int clear) {
  cudaError_t e = cudaMemcpyFromSymbol(host, g_prefill_trace, sizeof(long long) * kTraceSlots);
  void* dev = nullptr;
  if (e == cudaSuccess && clear) e = cudaGetSymbolAddress(&dev, g_prefill_trace);
  if (e == cudaSuccess && clear) e = cudaMemset(dev, 0, sizeof(long long) * kTraceSlots);
  return (int)e;
}
#endif

}  // namespace b200
