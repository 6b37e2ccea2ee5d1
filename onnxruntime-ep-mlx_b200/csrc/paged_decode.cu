// Paged GQA decode: block-table gather fused with split-K flash-decode.
//
// Replaces the reference's direct Metal decode (rust/src/ops/paged_attention.rs:31-143,
// dispatched per sequence at :229-334) and the gather+SDPA fallback for decode rows
// (rust/src/ops/attention.rs:4192-4319).  Same mathematics: scale*q.k, optional softcap, causal
// and left-window masks, fp32 online softmax, optional sink, fp32 accumulation; keys at
// positions >= past come from the sequence's own new rows (the reference's overlay,
// paged_attention.rs:52-61).
//
// B200 design (one launch for the whole ragged batch, not one per sequence):
//  * decode_plan_kernel (1 CTA) routes every sequence (decode / tcgen05 prefill / generic) and
//    lays the decode work out as one stream of 16-token tiles: for each decode sequence, for
//    each kv head, its tiles (prefix offsets per sequence);
//  * paged_decode_kernel is persistent (grid = SMs x resident CTAs) and every warp owns an
//    equal contiguous range of that stream (stream-K: exact balance for ragged lengths, no
//    scheduling atomics).  A warp streams its tiles through a private STAGES-deep ring of
//    shared-memory stages filled by TMA (cp.async.bulk.tensor.3d, 128-byte swizzle,
//    single-CTA destination) from the [NB*bs, KV, d] cache view; the lookahead runs across (sequence, kv
//    head) boundaries, so the ring never drains;
//  * the g = H/KV query heads of a kv head (times the unit's queries, <= 8 rows) are batched
//    into one tensor-core tile: S^T[16 tok x 8 rows] = K_tile[16 x d] . Q^T via
//    mma.m16n8k16 (K from ldmatrix, Q fragments in registers), so every K/V byte is read once
//    per kv head, not once per query head as in the reference kernel;
//  * online softmax on the accumulator fragments (exp2 domain), P^T moved into the B operand
//    with movmatrix.trans, O^T[d x 8 rows] += V_tile^T . P^T with ldmatrix.trans; for 16-bit
//    caches P is carried as a hi + lo pair of 16-bit values so the PV product keeps ~16
//    mantissa bits; fp8 tiles (converted to fp16 in registers) use one fp16 P, a lazily moved
//    running max (P <= 2^8) and a V unit that keeps P's scale near 1;
//  * a (sequence, kv head) segment that lies inside one warp's range is written directly;
//    a segment cut by range boundaries leaves one fp32 partial (m, l, o) per warp, and the last
//    warp to finish it merges them (fused split-K combine, no extra launch).  A warp writes at
//    most two partials, so partial storage is 2 x 8 rows per warp.
#include "b200_common.cuh"
#include "b200_kernels.h"

namespace b200 {

constexpr int kDecodeWarps = kDecodeWarpsPerCta;
constexpr float kLog2e = 1.4426950408889634f;

bool decode_supported(int head_size, int block_size, int act_dtype, int cache_dtype) {
  const bool act16 = act_dtype == B200_DTYPE_FLOAT16 || act_dtype == B200_DTYPE_BFLOAT16;
  if (!act16 || block_size % kTile != 0) return false;
  if (cache_dtype == B200_DTYPE_FLOAT8E4M3FN) return head_size == 128 || head_size == 256;
  return (head_size == 64 || head_size == 128 || head_size == 256) && act_dtype == cache_dtype;
}

// ---------------------------------------------------------------------------------------
// Plan: one CTA scans the sequences (chunks of blockDim) and writes the tile-stream offsets.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive prefix of warp totals
  }
  __syncthreads();
  int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  total = warp_sums[nw - 1];
  __syncthreads();
  return before;
}

// Route of sequence b, with its decode tiles (per kv head) or prefill q tiles.
__device__ __forceinline__ int route_of(const AttnArgs& a, int b, int& dtiles, int& ptiles) {
  dtiles = ptiles = 0;
  const int c0 = a.cum[b], c1 = a.cum[b + 1], nq = c1 - c0, past = a.past[b];
  const int64_t total = (int64_t)past + nq;
  const bool valid = c0 >= 0 && c1 <= a.num_tokens && nq >= 1 && past >= 0 &&
                     total <= (int64_t)a.max_blocks * a.block_size;
  if (!valid) return kRouteGeneric;  // the generic kernel guards invalid metadata itself
  if (a.decode_on && nq * a.group <= kDecodeRows) {
    dtiles = (int)((total + a.decode_tile - 1) / a.decode_tile);
    return kRouteDecode;
  }
  if (a.prefill_tq > 0) {
    ptiles = (nq + a.prefill_tq - 1) / a.prefill_tq;
    return kRoutePrefill;
  }
  return kRouteGeneric;
}

__global__ void __launch_bounds__(1024) decode_plan_kernel(AttnArgs a, DecodePlan plan) {
  __shared__ int warp_sums[32];
  if (threadIdx.x == 0 && a.status) *a.status = 0;  // first kernel of every call clears status
  if (threadIdx.x == 0 && a.v_shadow_wide) *a.v_shadow_wide = 0;
  int carry = 0, pcarry = 0;
  for (int base = 0; base < a.batch; base += blockDim.x) {
    const int b = base + threadIdx.x;
    int dtiles = 0, ptiles = 0, route = kRouteGeneric;
    if (b < a.batch) route = route_of(a, b, dtiles, ptiles);
    int tot, ptot;
    const int off = block_exclusive_scan(dtiles, warp_sums, tot);
    const int poff = block_exclusive_scan(ptiles, warp_sums, ptot);
    if (b < a.batch) {
      a.route[b] = route;
      plan.seq_tile_off[b] = carry + off;
      plan.pf_tile_off[b] = pcarry + poff;
      for (int kh = 0; kh < a.kv_heads; ++kh) plan.done[(int64_t)b * a.kv_heads + kh] = 0;
    }
    carry += tot;
    pcarry += ptot;
  }
  if (threadIdx.x == 0) {
    plan.seq_tile_off[a.batch] = carry;
    plan.pf_tile_off[a.batch] = pcarry;
    *plan.total_tiles = (int64_t)carry * a.kv_heads;
    *plan.pf_total = (int64_t)pcarry * a.kv_heads;
    if (plan.pf_next) *plan.pf_next = 0;
  }
}

// ---------------------------------------------------------------------------------------
// Decode kernel
// ---------------------------------------------------------------------------------------
// A decode tile is kHalves half-tiles of kTile (16) tokens: one for 16-bit caches,
// kFp8HalfTiles for fp8 caches (two give 32 tokens per stage and per softmax step).  A half-tile
// never crosses a cache block (block_size % 16 == 0), so each has its own block id, TMA boxes
// and fp8 scales.
template <int D, bool FP8>
struct DecodeLayout {
  static constexpr int kElem = FP8 ? 1 : 2;              // stored bytes per element
  static constexpr int kBoxCols = 128 / kElem;           // elements per 128-byte TMA box row
  static constexpr int kBoxes = D / kBoxCols;            // TMA boxes per half-tile row
  static constexpr int kBoxBytes = kTile * 128;          // 16 rows x 128 B
  static constexpr int kHalves = FP8 ? kFp8HalfTiles : 1;
  static constexpr int kTileRows = kTile * kHalves;      // tokens per tile
  static constexpr int kHalfBytes = kTile * D * kElem;   // one tensor, one half-tile, as stored
  static constexpr int kTileBytes = kHalves * kHalfBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;     // K + V
};

// Four fp8 e4m3 values of `w` -> two fp16x2: lo = bytes 0, 1 and hi = bytes 2, 3 (exact: every
// e4m3 value is an fp16 value; the lower byte of a pair lands in the lower half).
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

// fp8 tiles feed the fp16 MMAs straight from registers:
//  * K: ldmatrix of the fp8 bytes as 16-bit pairs gives lane (g, t) channels 4t..4t+3 of its
//    row; the MMA's K index 2t+j is channel 4t+j and 2t+8+j is channel 4t+2+j within each
//    16-channel block, and Q's fragments are loaded with the same permutation;
//  * V: ldmatrix.trans gives lane (g, t) channels 2g, 2g+1 of tokens 2t, 2t+1; after the
//    conversion a byte permute regroups them per channel, so MMA row g is channel 2g and row
//    g+8 is channel 2g+1 of the 16-channel block (the output channel index follows).
__device__ __forceinline__ int out_channel(bool fp8, int mt, int dr, int hi) {
  return fp8 ? mt * 16 + 2 * dr + hi : mt * 16 + dr + 8 * hi;
}

// Byte offset of 16-byte chunk `chunk` (global over the d channels) of tile row `row` in a
// 128B-swizzled tile written by the TMA boxes.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  int box = chunk >> 3, c = chunk & 7;
  return (uint32_t)(box * (kTile * 128) + row * 128 + ((c ^ (row & 7)) << 4));
}

// A piece of one (sequence, kv head) segment of the tile stream, as a warp sees it.
struct Piece {
  int valid, b, kh, t0, t1, tiles, c0, nq, past, total;
  int64_t seg_start;  // stream index of the segment's first tile
};

// Stream layout: for each decode sequence b (in order), for each kv head, its tiles; sequence b
// starts at seq_tile_off[b] * KV.  Warp g of W owns stream range [g*T/W, (g+1)*T/W).
__device__ __forceinline__ int64_t range_start(int64_t g, int64_t T, int64_t W) { return g * T / W; }
__device__ __forceinline__ int64_t warp_of(int64_t x, int64_t T, int64_t W) { return ((x + 1) * W + T - 1) / T - 1; }

// T: the MMA type (the activation type; fp16 for fp8 caches, whose tiles are converted to fp16
// in shared memory and whose per-(block, kv head) scales multiply S and P per tile).
template <typename T, int D, int STAGES, bool FP8>
__global__ void __launch_bounds__(128) paged_decode_kernel(const __grid_constant__ AttnArgs a,
                                                           const __grid_constant__ DecodeMaps maps,
                                                           const DecodePlan plan) {
  using L = DecodeLayout<D, FP8>;
  constexpr int kWarpBytes = STAGES * L::kStageBytes;
  using MMA = mma_op<T>;
  constexpr int KSTEPS = D / 16;
  constexpr int RING = STAGES + 1;  // pieces live at once: one per in-flight tile + the newest
  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) uint64_t bars[kDecodeWarps][STAGES];
  __shared__ Piece ring[kDecodeWarps][RING];

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* wbase = smem + warp * kWarpBytes;
  const uint32_t wbase_u32 = smem_u32(wbase);
  Piece* myring = ring[warp];

  const int KV = a.kv_heads, g = a.group, H = a.num_heads;
  const int64_t Ttot = *plan.total_tiles;
  const int64_t Wmax = (int64_t)gridDim.x * kDecodeWarps;
  const int64_t W = max((int64_t)1, min(Wmax, (Ttot + plan.min_tiles_per_warp - 1) / plan.min_tiles_per_warp));
  const int64_t gw = (int64_t)blockIdx.x * kDecodeWarps + warp;
  if (Ttot == 0 || gw >= W) return;
  const int64_t r0 = range_start(gw, Ttot, W), r1 = range_start(gw + 1, Ttot, W);
  if (r0 >= r1) return;

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&bars[warp][s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const float qk_scale = a.softcap > 0.f ? a.scale : a.scale * kLog2e;

  // Piece of the stream starting at position x (< r1) into ring slot `slot` (all lanes).
  auto locate = [&](int slot, int64_t x) {
    Piece p{};
    if (x < r1) {
      int lo = 0, hi = a.batch - 1;  // largest b with seq_tile_off[b] * KV <= x
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if ((int64_t)plan.seq_tile_off[mid] * KV <= x) lo = mid; else hi = mid - 1;
      }
      const int b = lo;
      const int64_t sb = (int64_t)plan.seq_tile_off[b] * KV;
      const int tb = plan.seq_tile_off[b + 1] - plan.seq_tile_off[b];
      if (tb > 0) {
        const int64_t rel = x - sb;
        p.valid = 1;
        p.b = b;
        p.kh = (int)(rel / tb);
        p.tiles = tb;
        p.t0 = (int)(rel % tb);
        p.t1 = (int)min((int64_t)tb, p.t0 + (r1 - x));
        p.seg_start = sb + (int64_t)p.kh * tb;
        p.c0 = a.cum[b];
        p.nq = a.cum[b + 1] - p.c0;
        p.past = a.past[b];
        p.total = p.past + p.nq;
      }
    }
    __syncwarp();
    if (lane == 0) myring[slot] = p;
    __syncwarp();
  };

  // Issue the TMA loads of tile t of the piece in ring slot `slot` into stage s (lane 0).
  auto issue = [&](int s, int slot, int t) {
    if (lane != 0) return;
    const Piece& u = myring[slot];
    uint64_t* bar = &bars[warp][s];
    if constexpr (FP8) {
      // Half-tiles past the sequence load nothing (their tokens are masked); a half-tile with an
      // invalid block id loads nothing and reports it.
      int z[L::kHalves];
      uint32_t bytes = 0;
#pragma unroll
      for (int h = 0; h < L::kHalves; ++h) {
        const int pos = t * L::kTileRows + h * kTile;
        z[h] = -1;
        if (pos >= u.total) continue;
        const int32_t blk = a.block_table[(int64_t)u.b * a.max_blocks + pos / a.block_size];
        if (blk < 0 || blk >= a.num_blocks) {
          set_status(a.status, kStatusBadBlock);
          continue;
        }
        z[h] = blk * a.block_size + pos % a.block_size;
        bytes += 2 * L::kHalfBytes;
      }
      if (bytes == 0) {
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
        return;
      }
      uint8_t* kdst = wbase + s * L::kStageBytes;
      uint8_t* vdst = kdst + L::kTileBytes;
      mbar_arrive_expect_tx(bar, bytes);
#pragma unroll
      for (int h = 0; h < L::kHalves; ++h) {
        if (z[h] < 0) continue;
#pragma unroll
        for (int hb = 0; hb < L::kBoxes; ++hb) {
          tma_load_3d(kdst + h * L::kHalfBytes + hb * L::kBoxBytes, &maps.k_map, bar, hb * L::kBoxCols, u.kh, z[h]);
          tma_load_3d(vdst + h * L::kHalfBytes + hb * L::kBoxBytes, &maps.v_map, bar, hb * L::kBoxCols, u.kh, z[h]);
        }
      }
      return;
    }
    const int pos0 = t * kTile;
    const int32_t blk = a.block_table[(int64_t)u.b * a.max_blocks + pos0 / a.block_size];
    if (blk < 0 || blk >= a.num_blocks) {
      set_status(a.status, kStatusBadBlock);
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
      return;
    }
    const int z = blk * a.block_size + pos0 % a.block_size;
    uint8_t* kdst = wbase + s * L::kStageBytes;
    uint8_t* vdst = kdst + L::kTileBytes;
    mbar_arrive_expect_tx(bar, L::kStageBytes);
#pragma unroll
    for (int h = 0; h < L::kBoxes; ++h) {
      tma_load_3d(kdst + h * L::kBoxBytes, &maps.k_map, bar, h * L::kBoxCols, u.kh, z);
      tma_load_3d(vdst + h * L::kBoxBytes, &maps.v_map, bar, h * L::kBoxCols, u.kh, z);
    }
  };

  // Producer: ring slot ps, next tile pt of that piece.  The lookahead runs across pieces.
  int ps = 0, pt = 0;
  locate(0, r0);
  bool producing = myring[0].valid != 0;
  if (producing) pt = myring[0].t0;
  uint32_t phase = 0, pending = 0;
  int issued = 0, consumed = 0;
  bool failed = false;

  auto produce = [&]() {
    while (producing && pt >= myring[ps].t1) {
      const int64_t next = myring[ps].seg_start + myring[ps].t1;
      ps = (ps + 1) % RING;
      locate(ps, next);
      producing = myring[ps].valid != 0;
      if (producing) pt = myring[ps].t0;
    }
    if (!producing) return;
    const int s = issued % STAGES;
    issue(s, ps, pt);
    pending |= 1u << s;
    ++pt;
    ++issued;
  };

  for (int i = 0; i < STAGES; ++i) produce();
  __syncwarp();

  int cs = 0;
  int ct = myring[0].t0;
  const int col0 = (lane & 3) * 2;  // q rows held by this lane: col0, col0 + 1

  while (consumed < issued && !failed) {
    const Piece u = myring[cs];
    const int rows = u.nq * g;
    const int qi0 = col0 / g, qi1 = (col0 + 1) / g;

    // Q^T B-fragments: column n = lane/4 is q row r = (query i, head-in-group).
    uint32_t qf[KSTEPS][2];
    {
      const int r = lane >> 2, kq = (lane & 3) * 2;
      if (r < rows) {
        const int qi = r / g, hl = r % g;
        const T* qrow =
            reinterpret_cast<const T*>(a.q) + (int64_t)(u.c0 + qi) * a.q_stride + (int64_t)(u.kh * g + hl) * D;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          if constexpr (FP8) {
            // fp16 MMA on the fp8 channel permutation: K index 2t+j -> channel 4t+j, 2t+8+j -> 4t+2+j
            const int64_t e0 =
                (int64_t)(u.c0 + qi) * a.q_stride + (int64_t)(u.kh * g + hl) * D + kk * 16 + (lane & 3) * 4;
            qf[kk][0] = MMA::pack(load_act(a.q, e0, a.act_dtype), load_act(a.q, e0 + 1, a.act_dtype));
            qf[kk][1] = MMA::pack(load_act(a.q, e0 + 2, a.act_dtype), load_act(a.q, e0 + 3, a.act_dtype));
          } else {
            qf[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + kq);
            qf[kk][1] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + kq);
          }
        }
      } else {
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) qf[kk][0] = qf[kk][1] = 0u;
      }
    }

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[KSTEPS][4];
#pragma unroll
    for (int mt = 0; mt < KSTEPS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    // fp8: o is kept in units of vref, a V scale of the piece (P carries v_scale / vref, which
    // stays near 1 so the fp16 P keeps its precision); 16-bit caches: 1.
    float vref = FP8 ? 0.f : 1.f;

    if constexpr (FP8) {
      // Half-tile metadata in windows of 32 half-tiles (kWin tiles): lane i holds half-tile
      // kHalves * wb + i's block id and K / V scales; the next window's ids are loaded when a
      // window starts and its scales 4 tiles later.
      constexpr int kWin = 32 / L::kHalves;
      auto half_block = [&](int hidx) -> int32_t {
        const int t = hidx / L::kHalves, pos = t * L::kTileRows + (hidx % L::kHalves) * kTile;
        return t < u.t1 && pos < u.total
                   ? __ldg(a.block_table + (int64_t)u.b * a.max_blocks + pos / a.block_size)
                   : -1;
      };
      auto block_scale = [&](const float* sc, int32_t blk) -> float {
        return blk >= 0 && blk < a.num_blocks ? __ldg(sc + (int64_t)blk * KV + u.kh) : 0.f;
      };
      int wb = ct;
      int32_t w_blk = half_block(L::kHalves * wb + lane), n_blk = -1;
      float w_ks = block_scale(a.k_scale, w_blk), w_vs = block_scale(a.v_scale, w_blk);
      float n_ks = 0.f, n_vs = 0.f;
      const int full_end = a.is_causal ? min(u.total, u.past + 1) : u.total;
      const int full_begin = a.window > 0 ? u.past + u.nq - a.window : 0;

      for (; ct < u.t1; ++ct) {
        const int s = consumed % STAGES;
        const int pos0 = ct * L::kTileRows;
        int wi = ct - wb;
        if (wi == kWin) {
          wb = ct;
          wi = 0;
          w_blk = n_blk;
          w_ks = n_ks;
          w_vs = n_vs;
        }
        if (wi == 0) n_blk = half_block(L::kHalves * (wb + kWin) + lane);
        if (wi == 4) {
          n_ks = block_scale(a.k_scale, n_blk);
          n_vs = block_scale(a.v_scale, n_blk);
        }
        if (!mbar_wait(&bars[warp][s], (phase >> s) & 1u)) {
          if (lane == 0) set_status(a.status, kStatusTimeout);
          failed = true;
          for (int s2 = 0; s2 < STAGES; ++s2)
            if ((pending >> s2) & 1u) mbar_wait(&bars[warp][s2], (phase >> s2) & 1u);
          pending = 0;
          break;
        }
        phase ^= 1u << s;
        pending &= ~(1u << s);
        int32_t blk[L::kHalves];
        float k_sc[L::kHalves], v_sc[L::kHalves];
        bool blk_ok[L::kHalves];
#pragma unroll
        for (int h = 0; h < L::kHalves; ++h) {
          blk[h] = __shfl_sync(0xffffffffu, w_blk, L::kHalves * wi + h);
          k_sc[h] = __shfl_sync(0xffffffffu, w_ks, L::kHalves * wi + h);
          v_sc[h] = __shfl_sync(0xffffffffu, w_vs, L::kHalves * wi + h);
          blk_ok[h] = blk[h] >= 0 && blk[h] < a.num_blocks;
        }
        bool full = pos0 >= full_begin && pos0 + L::kTileRows <= full_end;
#pragma unroll
        for (int h = 0; h < L::kHalves; ++h) full = full && blk_ok[h];
        const uint32_t kbase = wbase_u32 + s * L::kStageBytes;
        const uint32_t vbase = kbase + L::kTileBytes;

        // S^T per half-tile = K_half . Q^T; two accumulators per half halve the MMA chains.
        float c[L::kHalves][2][4];
#pragma unroll
        for (int h = 0; h < L::kHalves; ++h)
#pragma unroll
          for (int j = 0; j < 2; ++j) c[h][j][0] = c[h][j][1] = c[h][j][2] = c[h][j][3] = 0.f;
        {
          const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
          const int half = lane >> 4;
#pragma unroll
          for (int kk = 0; kk < KSTEPS; kk += 2) {
#pragma unroll
            for (int h = 0; h < L::kHalves; ++h) {
              // 16-byte chunks kk, kk+1 = channel blocks of k-steps kk, kk+1
              uint32_t af[4], bf[4], d0, d1, d2, d3;
              ldsm_x4(kbase + h * L::kHalfBytes + swz(row, kk + half), d0, d1, d2, d3);
              e4m3x4_to_f16x2x2(d0, af[0], af[2]);
              e4m3x4_to_f16x2x2(d1, af[1], af[3]);
              e4m3x4_to_f16x2x2(d2, bf[0], bf[2]);
              e4m3x4_to_f16x2x2(d3, bf[1], bf[3]);
              MMA::run(c[h][0], af, qf[kk][0], qf[kk][1]);
              MMA::run(c[h][1], bf, qf[kk + 1][0], qf[kk + 1][1]);
            }
          }
        }

        // Masks, scale (log2 domain), online softmax per q-row column over the 32 tokens.
        float sc[L::kHalves][4];
#pragma unroll
        for (int h = 0; h < L::kHalves; ++h) {
          const float ksq = k_sc[h] * qk_scale;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = h * kTile + (lane >> 2) + ((e >> 1) << 3);
            const int col = col0 + (e & 1);
            const int qi = (e & 1) ? qi1 : qi0;
            const int pos = pos0 + tok;
            bool vis = col < rows;
            if (!full) {
              vis = vis && blk_ok[h] && pos < u.total;
              if (a.is_causal) vis = vis && pos <= u.past + qi;
              if (a.window > 0) vis = vis && pos >= u.past + qi - a.window + 1;
            }
            float x = (c[h][0][e] + c[h][1][e]) * ksq;
            if (a.softcap > 0.f) x = a.softcap * tanhf(x / a.softcap) * kLog2e;
            sc[h][e] = vis ? x : -INFINITY;
          }
        }
        float mx0 = fmaxf(sc[0][0], sc[0][2]), mx1 = fmaxf(sc[0][1], sc[0][3]);
#pragma unroll
        for (int h = 1; h < L::kHalves; ++h) {
          mx0 = fmaxf(mx0, fmaxf(sc[h][0], sc[h][2]));
          mx1 = fmaxf(mx1, fmaxf(sc[h][1], sc[h][3]));
        }
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        // Lazy rescale: the running max moves only when a score exceeds it by more than 2^8, so
        // P stays <= 256 (exact in fp16) and most tiles skip the O rescale.  The decision is
        // warp-uniform.
        if (__any_sync(0xffffffffu, mx0 > m0 + 8.f || mx1 > m1 + 8.f)) {
          const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
          const float al0 = exp2f(m0 - (mn0 == -INFINITY ? 0.f : mn0));
          const float al1 = exp2f(m1 - (mn1 == -INFINITY ? 0.f : mn1));
          l0 *= al0;
          l1 *= al1;
#pragma unroll
          for (int mt = 0; mt < KSTEPS; ++mt) {
            o[mt][0] *= al0; o[mt][2] *= al0;
            o[mt][1] *= al1; o[mt][3] *= al1;
          }
          m0 = mn0;
          m1 = mn1;
        }
        // The V unit moves when a half-tile's V scale exceeds it 64-fold (then P <= 256 * 64
        // stays inside fp16); the first tile with a nonzero scale sets it.
        float vmax = v_sc[0];
#pragma unroll
        for (int h = 1; h < L::kHalves; ++h) vmax = fmaxf(vmax, v_sc[h]);
        if (vmax > vref * 64.f) {  // warp-uniform: the scales are shuffled values
          const float f = vref / vmax;
#pragma unroll
          for (int mt = 0; mt < KSTEPS; ++mt) {
            o[mt][0] *= f; o[mt][1] *= f; o[mt][2] *= f; o[mt][3] *= f;
          }
          vref = vmax;
        }
        const float mu0 = m0 == -INFINITY ? 0.f : m0, mu1 = m1 == -INFINITY ? 0.f : m1;
        const float inv_vref = vref > 0.f ? 1.f / vref : 0.f;
        uint32_t bp[L::kHalves][2];  // P^T B-fragments per half-tile (fp16, V scale / vref folded in)
#pragma unroll
        for (int h = 0; h < L::kHalves; ++h) {
          const float p0 = exp2f(sc[h][0] - mu0), p1 = exp2f(sc[h][1] - mu1);
          const float p2 = exp2f(sc[h][2] - mu0), p3 = exp2f(sc[h][3] - mu1);
          l0 += p0 + p2;
          l1 += p1 + p3;
          const float vr = v_sc[h] * inv_vref;
          bp[h][0] = movm_t(MMA::pack(p0 * vr, p1 * vr));
          bp[h][1] = movm_t(MMA::pack(p2 * vr, p3 * vr));
        }

        // O^T += V_half^T . P_half^T for both half-tiles
        {
          const int jm = lane >> 3;
          const int row = (lane & 7) + (jm >> 1) * 8;
          const int sub = jm & 1;
          // tokens 2t, 2t+1 (and +8) of this lane; tokens past the sequence or of an invalid
          // block read as zeros (P is 0 there, and 0 x NaN from an unused slot would poison
          // O).  The byte permute [t0 c0, t0 c1, t1 c0, t1 c1] -> [t0 c0, t1 c0, t0 c1, t1 c1]
          // (selector 0x3120) regroups the bytes per channel; a masked token selects zeros.
          const int t2 = (lane & 3) * 2;
          auto perm_sel = [&](int h, int p) -> uint32_t {
            const int pos = pos0 + h * kTile + p;
            const bool ok0 = full || (blk_ok[h] && pos < u.total);
            const bool ok1 = full || (blk_ok[h] && pos + 1 < u.total);
            return (ok0 ? 0x0100u : 0x0404u) | (ok1 ? 0x3020u : 0x4040u);
          };
          uint32_t sel_lo[L::kHalves], sel_hi[L::kHalves];
#pragma unroll
          for (int h = 0; h < L::kHalves; ++h) {
            sel_lo[h] = perm_sel(h, t2);
            sel_hi[h] = perm_sel(h, t2 + 8);
          }
#pragma unroll
          for (int mt = 0; mt < KSTEPS; mt += 2) {
#pragma unroll
            for (int h = 0; h < L::kHalves; ++h) {
              uint32_t d[4];
              ldsm_x4_t(vbase + h * L::kHalfBytes + swz(row, mt + sub), d[0], d[1], d[2], d[3]);
#pragma unroll
              for (int blk2 = 0; blk2 < 2; ++blk2) {  // channel blocks mt, mt+1
                uint32_t af[4];
                e4m3x4_to_f16x2x2(__byte_perm(d[blk2], 0u, sel_lo[h]), af[0], af[1]);
                e4m3x4_to_f16x2x2(__byte_perm(d[blk2 + 2], 0u, sel_hi[h]), af[2], af[3]);
                MMA::run(o[mt + blk2], af, bp[h][0], bp[h][1]);
              }
            }
          }
        }
        __syncwarp();
        ++consumed;
        produce();  // refill the stage just freed (possibly with the next piece's first tile)
        __syncwarp();
      }
    } else {
      // Tile metadata in windows of 32 tiles: lane i holds tile wb + i's physical block; the
      // next window's entries are loaded when a window starts, so no tile waits on a dependent
      // global load.
      auto tile_block = [&](int t) -> int32_t {
        return t < u.t1 ? __ldg(a.block_table + (int64_t)u.b * a.max_blocks + (t * kTile) / a.block_size) : -1;
      };
      int wb = ct;
      int32_t w_blk = tile_block(wb + lane), n_blk = -1;
      // A tile needs no per-position mask when it lies inside the sequence, before every
      // query's causal limit and after every query's window start.
      const int full_end = a.is_causal ? min(u.total, u.past + 1) : u.total;
      const int full_begin = a.window > 0 ? u.past + u.nq - a.window : 0;

      for (; ct < u.t1; ++ct) {
        const int s = consumed % STAGES;
        const int pos0 = ct * kTile;
        int wi = ct - wb;
        if (wi == 32) {
          wb = ct;
          wi = 0;
          w_blk = n_blk;
        }
        if (wi == 0) n_blk = tile_block(wb + 32 + lane);
        if (!mbar_wait(&bars[warp][s], (phase >> s) & 1u)) {
          if (lane == 0) set_status(a.status, kStatusTimeout);
          failed = true;
          // One more bounded wait for the loads still in flight before the warp stops.
          for (int s2 = 0; s2 < STAGES; ++s2)
            if ((pending >> s2) & 1u) mbar_wait(&bars[warp][s2], (phase >> s2) & 1u);
          pending = 0;
          break;
        }
        phase ^= 1u << s;
        pending &= ~(1u << s);
        const int32_t blk = __shfl_sync(0xffffffffu, w_blk, wi);
        const bool blk_ok = blk >= 0 && blk < a.num_blocks;
        const bool full = blk_ok && pos0 >= full_begin && pos0 + kTile <= full_end;
        const uint32_t kbase = wbase_u32 + s * L::kStageBytes;
        const uint32_t vbase = kbase + L::kTileBytes;

        // Overlay: tile rows at positions >= past hold the sequence's own new K/V rows.
        const bool overlay = pos0 + kTile > u.past;
        if (overlay) {
          constexpr int CH = D / 8;  // 16-byte chunks per row
          for (int idx = lane; idx < kTile * CH; idx += 32) {
            const int row = idx / CH, chunk = idx % CH;
            const int pos = pos0 + row;
            if (pos >= u.total) {
              // rows past the sequence: V becomes zeros (P is 0 there; 0 x NaN from an unused
              // slot would still poison O)
              *reinterpret_cast<uint4*>(wbase + (vbase - wbase_u32) + swz(row, chunk)) = make_uint4(0u, 0u, 0u, 0u);
              continue;
            }
            if (pos < u.past) continue;
            const int64_t tok = u.c0 + (pos - u.past);
            const uint4 kv = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.k_new) + tok * a.k_stride +
                                                             (int64_t)u.kh * D + chunk * 8);
            const uint4 vv = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.v_new) + tok * a.v_stride +
                                                             (int64_t)u.kh * D + chunk * 8);
            *reinterpret_cast<uint4*>(wbase + (kbase - wbase_u32) + swz(row, chunk)) = kv;
            *reinterpret_cast<uint4*>(wbase + (vbase - wbase_u32) + swz(row, chunk)) = vv;
          }
          __syncwarp();
        }

        // S^T = K_tile . Q^T (two accumulators halve the dependent MMA chain)
        float c[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
        {
          const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
          const int half = lane >> 4;
#pragma unroll
          for (int kk = 0; kk < KSTEPS; kk += 2) {
            uint32_t af[4], bf[4];
            ldsm_x4(kbase + swz(row, kk * 2 + half), af[0], af[1], af[2], af[3]);
            ldsm_x4(kbase + swz(row, kk * 2 + 2 + half), bf[0], bf[1], bf[2], bf[3]);
            MMA::run(c, af, qf[kk][0], qf[kk][1]);
            MMA::run(c2, bf, qf[kk + 1][0], qf[kk + 1][1]);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) c[e] += c2[e];
        }

        // Masks, scale (log2 domain), online softmax per q-row column.
        float sc[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = (lane >> 2) + ((e >> 1) << 3);
          const int col = col0 + (e & 1);
          const int qi = (e & 1) ? qi1 : qi0;
          const int pos = pos0 + tok;
          bool vis = col < rows;
          if (!full) {
            vis = vis && blk_ok && pos < u.total;
            if (a.is_causal) vis = vis && pos <= u.past + qi;
            if (a.window > 0) vis = vis && pos >= u.past + qi - a.window + 1;
          }
          float x = c[e] * qk_scale;
          if (a.softcap > 0.f) x = a.softcap * tanhf(x / a.softcap) * kLog2e;
          sc[e] = vis ? x : -INFINITY;
        }
        float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
        const float al0 = exp2f(m0 - mu0), al1 = exp2f(m1 - mu1);
        const float p0 = exp2f(sc[0] - mu0), p1 = exp2f(sc[1] - mu1);
        const float p2 = exp2f(sc[2] - mu0), p3 = exp2f(sc[3] - mu1);
        l0 = l0 * al0 + p0 + p2;
        l1 = l1 * al1 + p1 + p3;
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int mt = 0; mt < KSTEPS; ++mt) {
          o[mt][0] *= al0; o[mt][2] *= al0;
          o[mt][1] *= al1; o[mt][3] *= al1;
        }

        // P^T -> B fragments (hi + lo 16-bit split, about 16 mantissa bits of P)
        const uint32_t x0 = MMA::pack(p0, p1), x1 = MMA::pack(p2, p3);
        const float2 h0 = MMA::unpack(x0), h1 = MMA::unpack(x1);
        const uint32_t y0 = MMA::pack(p0 - h0.x, p1 - h0.y), y1 = MMA::pack(p2 - h1.x, p3 - h1.y);
        const uint32_t bh0 = movm_t(x0), bh1 = movm_t(x1), bl0 = movm_t(y0), bl1 = movm_t(y1);

        // O^T += V_tile^T . P^T
        {
          const int jm = lane >> 3;
          const int row = (lane & 7) + (jm >> 1) * 8;
          const int sub = jm & 1;
#pragma unroll
          for (int mt = 0; mt < KSTEPS; ++mt) {
            uint32_t af[4];
            ldsm_x4_t(vbase + swz(row, mt * 2 + sub), af[0], af[1], af[2], af[3]);
            MMA::run(o[mt], af, bh0, bh1);
            MMA::run(o[mt], af, bl0, bl1);
          }
        }
        __syncwarp();
        if (overlay) fence_proxy_async_smem();
        ++consumed;
        produce();  // refill the stage just freed (possibly with the next piece's first tile)
        __syncwarp();
      }
    }
    if (failed) break;

    // ---- finish the piece: column sums of l, then output or partial (+ fused combine)
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const int dr = lane >> 2;
    if (u.t0 == 0 && u.t1 == u.tiles) {
      // Whole segment in this warp: normalise and write the output rows.
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = col0 + e;
        if (r >= rows) continue;
        float M = e ? m1 : m0, Ls = e ? l1 : l0, f = 1.f;
        const int qi = r / g, hl = r % g;
        if (a.head_sink) {
          const float sink = load_act(a.head_sink, u.kh * g + hl, a.act_dtype) * kLog2e;
          const float M2 = fmaxf(M, sink);
          f = M == -INFINITY ? 0.f : exp2f(M - M2);
          Ls = Ls * f + exp2f(sink - M2);
        }
        const float inv = Ls > 0.f ? f / Ls * vref : 0.f;
        T* orow = reinterpret_cast<T*>(a.out) + (int64_t)(u.c0 + qi) * H * D + (int64_t)(u.kh * g + hl) * D;
#pragma unroll
        for (int mt = 0; mt < KSTEPS; ++mt) {
          store_act(orow, out_channel(FP8, mt, dr, 0), o[mt][e] * inv, a.act_dtype);
          store_act(orow, out_channel(FP8, mt, dr, 1), o[mt][e + 2] * inv, a.act_dtype);
        }
      }
    } else {
      // Partial: slot 0 holds the warp's first piece, slot 1 its last (split) piece.
      const int64_t piece_start = u.seg_start + u.t0;
      const int slot = piece_start == r0 ? 0 : 1;
      const int64_t prow = (gw * 2 + slot) * kDecodeRows;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int r = col0 + e;
        if (r >= rows) continue;
        float* po = plan.part_o + (prow + r) * D;
        if (dr == 0) {
          plan.part_ml[(prow + r) * 2] = e ? m1 : m0;
          plan.part_ml[(prow + r) * 2 + 1] = e ? l1 : l0;
        }
#pragma unroll
        for (int mt = 0; mt < KSTEPS; ++mt) {
          po[out_channel(FP8, mt, dr, 0)] = o[mt][e] * vref;
          po[out_channel(FP8, mt, dr, 1)] = o[mt][e + 2] * vref;
        }
      }
      __threadfence();
      __syncwarp();
      const int64_t seg_end = u.seg_start + u.tiles;
      const int64_t w_first = warp_of(u.seg_start, Ttot, W);
      const int pieces = (int)(warp_of(seg_end - 1, Ttot, W) - w_first + 1);
      int prior = 0;
      if (lane == 0) prior = atomicAdd(&plan.done[(int64_t)u.b * KV + u.kh], 1);
      prior = __shfl_sync(0xffffffffu, prior, 0);
      if (prior == pieces - 1) {
        // Last piece of this (sequence, kv head) to finish: merge all pieces.
        __threadfence();
        const bool first_is_last_slot = u.seg_start > range_start(w_first, Ttot, W);
        for (int r = 0; r < rows; ++r) {
          float mloc = -INFINITY;
          for (int pc = lane; pc < pieces; pc += 32) {
            const int64_t row = ((w_first + pc) * 2 + (pc == 0 && first_is_last_slot ? 1 : 0)) * kDecodeRows + r;
            mloc = fmaxf(mloc, __ldcg(plan.part_ml + row * 2));
          }
#pragma unroll
          for (int off = 16; off; off >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, off));
          const float M = mloc;
          float lloc = 0.f;
          for (int pc = lane; pc < pieces; pc += 32) {
            const int64_t row = ((w_first + pc) * 2 + (pc == 0 && first_is_last_slot ? 1 : 0)) * kDecodeRows + r;
            const float mp = __ldcg(plan.part_ml + row * 2);
            lloc += mp == -INFINITY ? 0.f : __ldcg(plan.part_ml + row * 2 + 1) * exp2f(mp - M);
          }
#pragma unroll
          for (int off = 16; off; off >>= 1) lloc += __shfl_xor_sync(0xffffffffu, lloc, off);
          float Lsum = lloc, fo = 1.f;
          const int qi = r / g, hl = r % g;
          if (a.head_sink) {
            const float sink = load_act(a.head_sink, u.kh * g + hl, a.act_dtype) * kLog2e;
            const float M2 = fmaxf(M, sink);
            fo = M == -INFINITY ? 0.f : exp2f(M - M2);
            Lsum = Lsum * fo + exp2f(sink - M2);
          }
          const float inv = Lsum > 0.f ? fo / Lsum : 0.f;
          T* orow = reinterpret_cast<T*>(a.out) + (int64_t)(u.c0 + qi) * H * D + (int64_t)(u.kh * g + hl) * D;
          for (int d4 = lane; d4 < D / 4; d4 += 32) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int pc = 0; pc < pieces; ++pc) {
              const int64_t row = ((w_first + pc) * 2 + (pc == 0 && first_is_last_slot ? 1 : 0)) * kDecodeRows + r;
              const float mp = __ldcg(plan.part_ml + row * 2);
              const float f = mp == -INFINITY ? 0.f : exp2f(mp - M);
              const float4 v = __ldcg(reinterpret_cast<const float4*>(plan.part_o + row * D) + d4);
              acc.x += f * v.x; acc.y += f * v.y; acc.z += f * v.z; acc.w += f * v.w;
            }
            store_act(orow, d4 * 4 + 0, acc.x * inv, a.act_dtype);
            store_act(orow, d4 * 4 + 1, acc.y * inv, a.act_dtype);
            store_act(orow, d4 * 4 + 2, acc.z * inv, a.act_dtype);
            store_act(orow, d4 * 4 + 3, acc.w * inv, a.act_dtype);
          }
        }
      }
    }
    // next consumer piece
    cs = (cs + 1) % RING;
    ct = myring[cs].t0;
  }
}

// ---------------------------------------------------------------------------------------
// Launch
// ---------------------------------------------------------------------------------------
// Resident CTAs per SM of one decode instantiation on the current device (its shared-memory
// need decides it), capped at kDecodeMaxCtasPerSm.  Cached per device; the first query also sets
// the kernel's dynamic shared-memory limit.  The workspace sizing of the partial rows and the
// launch grid both use it, so the grid never has more warps than the partial rows cover.
template <typename T, int D, int STAGES, bool FP8 = false>
static int decode_occupancy_t(cudaError_t* err) {
  using L = DecodeLayout<D, FP8>;
  constexpr size_t smem = (size_t)kDecodeWarps * STAGES * L::kStageBytes + 1024;
  static int occupancy[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (occupancy[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(paged_decode_kernel<T, D, STAGES, FP8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    int occ = 0;
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, paged_decode_kernel<T, D, STAGES, FP8>, 128, smem);
    if (e != cudaSuccess) {
      if (err) *err = e;
      return kDecodeMaxCtasPerSm;
    }
    occupancy[dev] = occ < 1 ? 1 : (occ > kDecodeMaxCtasPerSm ? kDecodeMaxCtasPerSm : occ);
  }
  return occupancy[dev];
}

template <typename T, int D, int STAGES, bool FP8 = false>
static cudaError_t launch_decode_t(const AttnArgs& a, const DecodePlan& plan, const DecodeMaps& maps, int num_sms,
                                   cudaStream_t stream) {
  using L = DecodeLayout<D, FP8>;
  constexpr size_t smem = (size_t)kDecodeWarps * STAGES * L::kStageBytes + 1024;
  cudaError_t e = cudaSuccess;
  const int occ = decode_occupancy_t<T, D, STAGES, FP8>(&e);
  if (e != cudaSuccess) return e;
  paged_decode_kernel<T, D, STAGES, FP8><<<num_sms * occ, 128, smem, stream>>>(a, maps, plan);
  return cudaGetLastError();
}

int decode_ctas_per_sm(int head_size, int act_dtype, int cache_dtype) {
  const bool bf = act_dtype == B200_DTYPE_BFLOAT16;
  if (cache_dtype == B200_DTYPE_FLOAT8E4M3FN) {
    switch (head_size) {
      case 128: return decode_occupancy_t<__half, 128, 2, true>(nullptr);
      case 256: return decode_occupancy_t<__half, 256, 2, true>(nullptr);
      default: return kDecodeMaxCtasPerSm;
    }
  }
  switch (head_size) {
    case 64: return bf ? decode_occupancy_t<__nv_bfloat16, 64, 4>(nullptr) : decode_occupancy_t<__half, 64, 4>(nullptr);
    case 128: return bf ? decode_occupancy_t<__nv_bfloat16, 128, 3>(nullptr) : decode_occupancy_t<__half, 128, 3>(nullptr);
    case 256: return bf ? decode_occupancy_t<__nv_bfloat16, 256, 2>(nullptr) : decode_occupancy_t<__half, 256, 2>(nullptr);
    default: return kDecodeMaxCtasPerSm;
  }
}

cudaError_t launch_decode_plan(const AttnArgs& a, const DecodePlan& plan, cudaStream_t stream) {
  decode_plan_kernel<<<1, 1024, 0, stream>>>(a, plan);
  return cudaGetLastError();
}

cudaError_t launch_decode(const AttnArgs& a, const DecodePlan& plan, const DecodeMaps& maps, int num_sms,
                          cudaStream_t stream) {
  const bool bf = a.act_dtype == B200_DTYPE_BFLOAT16;
  if (a.cache_dtype == B200_DTYPE_FLOAT8E4M3FN) {
    switch (a.head_size) {
      case 128: return launch_decode_t<__half, 128, 2, true>(a, plan, maps, num_sms, stream);
      case 256: return launch_decode_t<__half, 256, 2, true>(a, plan, maps, num_sms, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (a.head_size) {
    case 64: return bf ? launch_decode_t<__nv_bfloat16, 64, 4>(a, plan, maps, num_sms, stream)
                       : launch_decode_t<__half, 64, 4>(a, plan, maps, num_sms, stream);
    case 128: return bf ? launch_decode_t<__nv_bfloat16, 128, 3>(a, plan, maps, num_sms, stream)
                        : launch_decode_t<__half, 128, 3>(a, plan, maps, num_sms, stream);
    case 256: return bf ? launch_decode_t<__nv_bfloat16, 256, 2>(a, plan, maps, num_sms, stream)
                        : launch_decode_t<__half, 256, 2>(a, plan, maps, num_sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace b200
