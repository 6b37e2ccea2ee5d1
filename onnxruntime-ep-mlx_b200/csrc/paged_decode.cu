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
//  * decode_plan_kernel (1 CTA) turns cum/past into a device work list of units
//    (sequence, split) x kv-head, each covering up to `tiles_per_split` 16-token tiles;
//  * paged_decode_kernel is persistent (grid = SMs x resident CTAs).  A unit is processed by 4
//    warps that take the unit's tiles round-robin.  Each warp owns a private STAGES-deep ring
//    of shared-memory stages filled by TMA (cp.async.bulk.tensor.3d, 128-byte swizzle, no
//    multicast) from the [NB*bs, KV, d] cache view: a 16-token tile of one kv head is one
//    box per 64 channels for K and for V, completion tracked by an mbarrier;
//  * the g = H/KV query heads of a kv head (times the unit's queries, <= 8 rows) are batched
//    into one tensor-core tile: S^T[16 tok x 8 rows] = K_tile[16 x d] . Q^T via
//    mma.m16n8k16 (K from ldmatrix, Q fragments in registers), so every K/V byte is read once
//    per kv head, not once per query head as in the reference kernel;
//  * online softmax on the accumulator fragments (exp2 domain), P^T moved into the B operand
//    with movmatrix.trans, O^T[d x 8 rows] += V_tile^T . P^T with ldmatrix.trans; P is carried
//    as a hi + lo pair of 16-bit values so the PV product keeps ~16 mantissa bits;
//  * the 4 warps merge in shared memory; a unit that covers its whole sequence writes the
//    output, otherwise an fp32 partial (m, l, o) that decode_combine_kernel reduces.
#include "b200_common.cuh"
#include "b200_kernels.h"

namespace b200 {

constexpr int kDecodeWarps = 4;
constexpr float kLog2e = 1.4426950408889634f;

bool decode_supported(int head_size, int block_size, int act_dtype, int cache_dtype) {
  return (head_size == 64 || head_size == 128 || head_size == 256) && block_size % kTile == 0 &&
         act_dtype == cache_dtype && (act_dtype == B200_DTYPE_FLOAT16 || act_dtype == B200_DTYPE_BFLOAT16);
}

// ---------------------------------------------------------------------------------------
// Plan: one CTA scans the sequences (chunks of 1024) and emits the unit list.
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

__global__ void __launch_bounds__(1024) decode_plan_kernel(AttnArgs a, DecodePlan plan) {
  __shared__ int warp_sums[32];
  if (threadIdx.x == 0 && a.status) *a.status = 0;  // first kernel of every call clears status
  int carry_items = 0, carry_rows = 0;
  const int P = plan.tiles_per_split;
  for (int base = 0; base < a.batch; base += blockDim.x) {
    int b = base + threadIdx.x;
    int ns = 0, rows = 0;
    if (b < a.batch) {
      int c0 = a.cum[b], c1 = a.cum[b + 1], nq = c1 - c0, past = a.past[b];
      int64_t total = (int64_t)past + nq;
      if (c0 >= 0 && c1 <= a.num_tokens && nq >= 1 && nq * a.group <= kDecodeRows && past >= 0 &&
          total <= (int64_t)a.max_blocks * a.block_size) {
        int tiles = (int)((total + kTile - 1) / kTile);
        ns = (tiles + P - 1) / P;
        rows = nq * a.group;
      }
    }
    int total_items, total_rows;
    int item_off = block_exclusive_scan(ns, warp_sums, total_items);
    int row_off = block_exclusive_scan(ns * rows * a.kv_heads, warp_sums, total_rows);
    if (b < a.batch) {
      plan.seq_nsplit[b] = ns;
      plan.seq_part_off[b] = carry_rows + row_off;
      for (int s = 0; s < ns; ++s) {
        int idx = carry_items + item_off + s;
        if (idx < plan.max_items) plan.units[idx] = make_int2(b, s);
      }
    }
    carry_items += total_items;
    carry_rows += total_rows;
  }
  if (threadIdx.x == 0) *plan.n_units = min(carry_items, plan.max_items);
}

// ---------------------------------------------------------------------------------------
// Decode kernel
// ---------------------------------------------------------------------------------------
template <int D>
struct DecodeLayout {
  static constexpr int kBoxes = D / 64;                 // 64-channel TMA boxes per tile row
  static constexpr int kBoxBytes = kTile * 128;         // 16 rows x 128 B
  static constexpr int kTileBytes = kTile * D * 2;      // one tensor, one tile
  static constexpr int kStageBytes = 2 * kTileBytes;    // K + V
};

// Byte offset of 16-byte chunk `chunk` (global over the d channels) of tile row `row` in a
// 128B-swizzled tile written by the TMA boxes.
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  int box = chunk >> 3, c = chunk & 7;
  return (uint32_t)(box * (kTile * 128) + row * 128 + ((c ^ (row & 7)) << 4));
}

template <typename T, int D, int STAGES>
__global__ void __launch_bounds__(128) paged_decode_kernel(const __grid_constant__ AttnArgs a,
                                                           const __grid_constant__ DecodeMaps maps,
                                                           const DecodePlan plan) {
  using L = DecodeLayout<D>;
  using MMA = mma_op<T>;
  constexpr int KSTEPS = D / 16;
  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) uint64_t bars[kDecodeWarps][STAGES];

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* wbase = smem + warp * STAGES * L::kStageBytes;
  const uint32_t wbase_u32 = smem_u32(wbase);

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&bars[warp][s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  uint32_t phase = 0;    // bit s: parity of the next completion of stage s
  uint32_t pending = 0;  // bit s: a load into stage s has been issued and not yet waited on
  bool failed = false;

  const int KV = a.kv_heads, g = a.group, H = a.num_heads;
  const int P = plan.tiles_per_split;
  const int n_units = *plan.n_units * KV;
  const float qk_scale = a.softcap > 0.f ? a.scale : a.scale * kLog2e;

  for (int u = blockIdx.x; u < n_units; u += gridDim.x) {
    const int2 it = plan.units[u / KV];
    const int kh = u % KV;
    const int b = it.x, split = it.y;
    const int c0 = a.cum[b], nq = a.cum[b + 1] - c0, past = a.past[b];
    const int total = past + nq;
    const int tiles = (total + kTile - 1) / kTile;
    const int t0 = split * P, t1 = min(t0 + P, tiles);
    const int rows = nq * g;
    const int32_t* bt = a.block_table + (int64_t)b * a.max_blocks;
    const int n_my = t1 - t0 > warp ? (t1 - t0 - warp + kDecodeWarps - 1) / kDecodeWarps : 0;

    // Q^T B-fragments: column n = lane/4 is q row r = (query i, head-in-group); k pairs.
    uint32_t qf[KSTEPS][2];
    {
      const int r = lane >> 2, kq = (lane & 3) * 2;
      if (r < rows) {
        const int qi = r / g, hl = r % g;
        const T* qrow = reinterpret_cast<const T*>(a.q) + (int64_t)(c0 + qi) * a.q_stride + (int64_t)(kh * g + hl) * D;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          qf[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + kq);
          qf[kk][1] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + kq);
        }
      } else {
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) qf[kk][0] = qf[kk][1] = 0u;
      }
    }

    // Issue the TMA loads of my j-th tile into stage j % STAGES (lane 0 only).
    auto issue = [&](int j) {
      const int s = j % STAGES;
      const int t = t0 + warp + kDecodeWarps * j;
      const int pos0 = t * kTile;
      const int32_t blk = bt[pos0 / a.block_size];
      uint64_t* bar = &bars[warp][s];
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
        tma_load_3d(kdst + h * L::kBoxBytes, &maps.k_map, bar, h * 64, kh, z);
        tma_load_3d(vdst + h * L::kBoxBytes, &maps.v_map, bar, h * 64, kh, z);
      }
    };

    if (!failed) {
      for (int j = 0; j < min(STAGES, n_my); ++j) {
        if (lane == 0) issue(j);
        pending |= 1u << (j % STAGES);
      }
    }
    __syncwarp();

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[KSTEPS][4];
#pragma unroll
    for (int mt = 0; mt < KSTEPS; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

    const int col0 = (lane & 3) * 2;          // q rows held by this lane: col0, col0 + 1
    const int qi0 = col0 / g, qi1 = (col0 + 1) / g;

    for (int j = 0; j < n_my && !failed; ++j) {
      const int s = j % STAGES;
      const int t = t0 + warp + kDecodeWarps * j;
      const int pos0 = t * kTile;
      if (!mbar_wait(&bars[warp][s], (phase >> s) & 1u)) {
        if (lane == 0) set_status(a.status, kStatusTimeout);
        failed = true;
        // Give the loads still in flight into this warp's stages one more bounded wait
        // before the shared memory is reused, then stop issuing.
        for (int s2 = 0; s2 < STAGES; ++s2)
          if ((pending >> s2) & 1u) mbar_wait(&bars[warp][s2], (phase >> s2) & 1u);
        pending = 0;
        break;
      }
      phase ^= 1u << s;
      pending &= ~(1u << s);
      const int32_t blk = bt[pos0 / a.block_size];
      const bool blk_ok = blk >= 0 && blk < a.num_blocks;
      const uint32_t kbase = wbase_u32 + s * L::kStageBytes;
      const uint32_t vbase = kbase + L::kTileBytes;

      // Overlay: tile rows at positions >= past hold the sequence's own new K/V rows.
      const bool overlay = pos0 + kTile > past;
      if (overlay) {
        constexpr int CH = D / 8;  // 16-byte chunks per row
        for (int idx = lane; idx < kTile * CH; idx += 32) {
          const int row = idx / CH, chunk = idx % CH;
          const int pos = pos0 + row;
          if (pos < past || pos >= total) continue;
          const int64_t tok = c0 + (pos - past);
          const uint4 kv = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.k_new) + tok * a.k_stride + (int64_t)kh * D + chunk * 8);
          const uint4 vv = *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.v_new) + tok * a.v_stride + (int64_t)kh * D + chunk * 8);
          *reinterpret_cast<uint4*>(wbase + (kbase - wbase_u32) + swz(row, chunk)) = kv;
          *reinterpret_cast<uint4*>(wbase + (vbase - wbase_u32) + swz(row, chunk)) = vv;
        }
        __syncwarp();
      }

      // S^T = K_tile . Q^T
      float c[4] = {0.f, 0.f, 0.f, 0.f};
      {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int half = lane >> 4;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          uint32_t af[4];
          ldsm_x4(kbase + swz(row, kk * 2 + half), af[0], af[1], af[2], af[3]);
          MMA::run(c, af, qf[kk][0], qf[kk][1]);
        }
      }

      // Masks, scale (log2 domain), online softmax per q-row column.
      float sc[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = (lane >> 2) + ((e >> 1) << 3);
        const int col = col0 + (e & 1);
        const int qi = (e & 1) ? qi1 : qi0;
        const int pos = pos0 + tok;
        bool vis = blk_ok && col < rows && pos < total;
        if (a.is_causal) vis = vis && pos <= past + qi;
        if (a.window > 0) vis = vis && pos >= past + qi - a.window + 1;
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

      // P^T -> B fragments (hi + lo 16-bit split).
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
      if (j + STAGES < n_my) {
        if (lane == 0) issue(j + STAGES);
        pending |= 1u << s;
      }
      __syncwarp();
    }

    // Column sums of l across the 8 lanes that share a column.
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }

    // Merge the 4 warps through shared memory (stage buffers are idle now).
    __syncthreads();
    float* mo = reinterpret_cast<float*>(smem);                  // [4][8][D]
    float* mm = mo + kDecodeWarps * kDecodeRows * D;             // [4][8]
    float* ml = mm + kDecodeWarps * kDecodeRows;                 // [4][8]
    if (lane < 4) {
      mm[warp * kDecodeRows + col0] = m0; mm[warp * kDecodeRows + col0 + 1] = m1;
      ml[warp * kDecodeRows + col0] = l0; ml[warp * kDecodeRows + col0 + 1] = l1;
    }
    {
      float* ow = mo + warp * kDecodeRows * D;
      const int dr = lane >> 2;
#pragma unroll
      for (int mt = 0; mt < KSTEPS; ++mt) {
        ow[col0 * D + mt * 16 + dr] = o[mt][0];
        ow[(col0 + 1) * D + mt * 16 + dr] = o[mt][1];
        ow[col0 * D + mt * 16 + dr + 8] = o[mt][2];
        ow[(col0 + 1) * D + mt * 16 + dr + 8] = o[mt][3];
      }
    }
    __syncthreads();
    const int nsplit = plan.seq_nsplit[b];
    for (int idx = threadIdx.x; idx < rows * D; idx += blockDim.x) {
      const int r = idx / D, d = idx % D;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kDecodeWarps; ++w) M = fmaxf(M, mm[w * kDecodeRows + r]);
      float Lsum = 0.f, Osum = 0.f;
#pragma unroll
      for (int w = 0; w < kDecodeWarps; ++w) {
        const float mw = mm[w * kDecodeRows + r];
        const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
        Lsum += ml[w * kDecodeRows + r] * f;
        Osum += mo[(w * kDecodeRows + r) * D + d] * f;
      }
      const int qi = r / g, hl = r % g;
      if (nsplit == 1) {
        if (a.head_sink) {
          const float sink = load_act(a.head_sink, kh * g + hl, a.act_dtype) * kLog2e;
          const float M2 = fmaxf(M, sink);
          const float f = M == -INFINITY ? 0.f : exp2f(M - M2);
          Lsum = Lsum * f + exp2f(sink - M2);
          Osum *= f;
        }
        const float y = Lsum > 0.f ? Osum / Lsum : 0.f;
        store_act(a.out, (int64_t)(c0 + qi) * H * D + (int64_t)(kh * g + hl) * D + d, y, a.act_dtype);
      } else {
        const int64_t pr = plan.seq_part_off[b] + ((int64_t)split * KV + kh) * rows + r;
        float* part = plan.partials + pr * (D + 2);
        part[2 + d] = Osum;
        if (d == 0) { part[0] = M; part[1] = Lsum; }
      }
    }
    __syncthreads();
  }
}

// Reduce the split partials of every (sequence, kv head) with more than one split.
__global__ void __launch_bounds__(128) decode_combine_kernel(AttnArgs a, DecodePlan plan) {
  const int b = blockIdx.x, kh = blockIdx.y;
  const int ns = plan.seq_nsplit[b];
  if (ns <= 1) return;
  const int D = a.head_size, KV = a.kv_heads, g = a.group, H = a.num_heads;
  const int c0 = a.cum[b], nq = a.cum[b + 1] - c0;
  const int rows = nq * g;
  const int64_t base = plan.seq_part_off[b];
  for (int idx = threadIdx.x; idx < rows * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D;
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, plan.partials[(base + ((int64_t)s * KV + kh) * rows + r) * (D + 2)]);
    float Lsum = 0.f, Osum = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float* part = plan.partials + (base + ((int64_t)s * KV + kh) * rows + r) * (D + 2);
      const float f = part[0] == -INFINITY ? 0.f : exp2f(part[0] - M);
      Lsum += part[1] * f;
      Osum += part[2 + d] * f;
    }
    const int qi = r / g, hl = r % g;
    if (a.head_sink) {
      const float sink = load_act(a.head_sink, kh * g + hl, a.act_dtype) * kLog2e;
      const float M2 = fmaxf(M, sink);
      const float f = M == -INFINITY ? 0.f : exp2f(M - M2);
      Lsum = Lsum * f + exp2f(sink - M2);
      Osum *= f;
    }
    const float y = Lsum > 0.f ? Osum / Lsum : 0.f;
    store_act(a.out, (int64_t)(c0 + qi) * H * D + (int64_t)(kh * g + hl) * D + d, y, a.act_dtype);
  }
}

// ---------------------------------------------------------------------------------------
// Launch
// ---------------------------------------------------------------------------------------
template <typename T, int D, int STAGES>
static cudaError_t launch_decode_t(const AttnArgs& a, const DecodePlan& plan, const DecodeMaps& maps, int num_sms,
                                   cudaStream_t stream) {
  using L = DecodeLayout<D>;
  constexpr size_t stage_smem = (size_t)kDecodeWarps * STAGES * L::kStageBytes;
  constexpr size_t merge_smem = sizeof(float) * (size_t)kDecodeWarps * kDecodeRows * (D + 2);
  constexpr size_t smem = (stage_smem > merge_smem ? stage_smem : merge_smem) + 1024;
  static int occupancy[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (occupancy[dev] == 0) {
    cudaError_t e = cudaFuncSetAttribute(paged_decode_kernel<T, D, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, paged_decode_kernel<T, D, STAGES>, 128, smem);
    if (e != cudaSuccess) return e;
    occupancy[dev] = occ > 0 ? occ : 1;
  }
  paged_decode_kernel<T, D, STAGES><<<num_sms * occupancy[dev], 128, smem, stream>>>(a, maps, plan);
  decode_combine_kernel<<<dim3(a.batch, a.kv_heads), 128, 0, stream>>>(a, plan);
  return cudaGetLastError();
}

cudaError_t launch_decode_plan(const AttnArgs& a, const DecodePlan& plan, cudaStream_t stream) {
  decode_plan_kernel<<<1, 1024, 0, stream>>>(a, plan);
  return cudaGetLastError();
}

cudaError_t launch_decode(const AttnArgs& a, const DecodePlan& plan, const DecodeMaps& maps, int num_sms,
                          cudaStream_t stream) {
  const bool bf = a.act_dtype == B200_DTYPE_BFLOAT16;
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
