// Internal kernel argument blocks and launchers (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

namespace b200 {

// Device status word.  Bit flags, OR-ed by any thread that detects a problem; the host maps
// them to the reference's error messages (attention.rs:3934-3990).
// ---------------------------------------------------------------------------------------
enum StatusBits : int {
  kStatusBadCumulative = 1 << 0,   // cum[0] != 0, not monotone, cum[B] != nt
  kStatusBadPast = 1 << 1,         // past < 0
  kStatusBadCapacity = 1 << 2,     // total > max_blocks * block_size
  kStatusBadBlock = 1 << 3,        // block id outside [0, num_blocks)
  kStatusBadSlot = 1 << 4,         // slot outside [-1, num_blocks * block_size)
  kStatusTimeout = 1 << 5,         // a bounded wait ran out
  kStatusBadPosition = 1 << 6,     // RoPE position outside the cos/sin cache
};


// Record `msg` as this thread's b200_last_error() and return `code` (capi.cu).
int set_error(int code, const std::string& msg);
// Add to the library's launch counter (b200_launch_count).
void add_launches(uint64_t n);

// KV append / Q-K preprocessing (kv_append.cu).
struct PrologueArgs {
  int num_heads, kv_heads, head_size;
  int num_tokens, batch, num_blocks, block_size, max_blocks;
  int act_dtype, cache_dtype, k_per_channel, v_per_channel;
  int do_norm, do_rotary, rotary_interleaved, rotary_offset, rotary_dim, rotary_positions;
  int kv_only;  // append alone: skip Q processing
  int latent;   // LATENT layout: no value rows or value cache (key rows only)
  float norm_eps;
  int64_t query_stride, key_stride, value_stride;
  const void* query; const void* key; const void* value;
  void* key_cache; void* value_cache;
  const int32_t* cum; const int32_t* past; const int32_t* block_table; const int32_t* slot_mapping;
  const void* cos_cache; const void* sin_cache; const void* q_norm; const void* k_norm;
  const float* k_scale; const float* v_scale;
  void* q_proc; void* k_proc;  // processed rows [nt, H*d], [nt, KV*d] in T (norm/RoPE only)
  int* owner_keys; int* owner_vals; uint32_t owner_capacity;  // duplicate-slot table or null
  int* status;
  int* route;  // per-sequence route; a prefill sequence whose new rows do not all land in their
               // block-table slots (slot_mapping elsewhere, -1, or overwritten) moves to generic
};

void launch_meta_check(const PrologueArgs& a, cudaStream_t stream);
size_t prologue_smem_bytes(const PrologueArgs& a);
cudaError_t launch_prologue(const PrologueArgs& a, cudaStream_t stream);
// Plain append with a device slot_mapping of at most kAppendFusedMaxTokens tokens: the metadata
// checks, the duplicate-slot resolution and the copy in one launch (no slot table).
constexpr int kAppendFusedMaxTokens = 4096;
bool append_fused_eligible(const PrologueArgs& a);
cudaError_t launch_append_fused(const PrologueArgs& a, cudaStream_t stream);

// Attention over the paged cache (paged_generic.cu, paged_decode.cu).
struct AttnArgs {
  int num_heads, kv_heads, head_size, group;
  int num_tokens, batch, num_blocks, block_size, max_blocks;
  int act_dtype, cache_dtype, k_per_channel, v_per_channel;
  int is_causal, window;
  float scale, softcap;
  // processed new rows (Q after norm/RoPE, K after norm/RoPE, V raw) and their row strides
  const void* q; const void* k_new; const void* v_new;
  int64_t q_stride, k_stride, v_stride;
  const void* key_cache; const void* value_cache;
  const float* k_scale; const float* v_scale;
  const int32_t* cum; const int32_t* past; const int32_t* block_table;
  const void* head_sink;
  void* out;
  int* status;
  // Per-sequence route (kRoute*), written by the plan kernel and refined by the prologue; null
  // means every sequence runs on the generic kernel.
  int* route;
  int v_head;      // value channels per head and output channels per head (head_size, or the
                   // LATENT v_head_size; LATENT values are read from the key rows)
  int decode_on;   // decode kernel enabled for this call (shape supported)
  int decode_tile; // tokens per decode tile: kTile, or kFp8HalfTiles * kTile for fp8 caches
  int prefill_tq;  // query tokens per prefill work item (2 x 128 rows / group) or 0 = prefill kernel off
  // bf16 prefill over an fp16 copy of this call's new V rows (every prefill sequence without a
  // cached prefix): *v_shadow_wide is cleared by the plan kernel and set by the copy kernel when
  // a value lies beyond the fp16 range; the shadow-V prefill then exits and the bf16 prefill,
  // launched after it with prefill_fallback = 1, runs instead (it exits when the word is clear).
  int* v_shadow_wide;
  int prefill_fallback;
};

enum Route : int { kRouteDecode = 0, kRoutePrefill = 1, kRouteGeneric = 2 };

constexpr int kDecodeRows = 8;   // q rows (query x head-in-group) one decode unit covers
constexpr int kTile = 16;        // tokens per decode tile (one mma M tile)
// Half-tiles of kTile tokens per fp8 decode tile (1 or 2).  Two halve the per-tile fixed costs
// but double the shared memory of a stage; on B200 both settle near 0.61-0.64 of HBM on
// config 5 (the kernel is bound by dependent-latency chains at 8-12 resident warps per SM), and
// one with two stages was the best measured.
constexpr int kFp8HalfTiles = 1;

cudaError_t launch_generic(const AttnArgs& a, cudaStream_t stream);

// Plan of one call, written by decode_plan_kernel into the workspace: per-sequence routes,
// the decode tile stream (stream-K layout) and the prefill tile list.
struct DecodePlan {
  int64_t* pf_total;     // [1]   prefill work items: q tiles x kv heads
  unsigned long long* pf_next;  // [1] next prefill work item to hand out (CTAs take items
                               //     by atomicAdd, in list order); zeroed by the plan kernel
  int* pf_tile_off;      // [B+1] exclusive prefix of prefill q tiles over sequences
  int64_t* total_tiles;  // [1]   tiles over all decode sequences x kv heads
  int* seq_tile_off;     // [B+1] exclusive prefix of decode tiles (per kv head) over sequences
  int* done;             // [B*KV] pieces finished per (sequence, kv head), for the fused combine
  float* part_o;         // [max_warps * 2 * 8][head_size] partial outputs (2 slots per warp)
  float* part_ml;        // [max_warps * 2 * 8][2]          partial (max, sum), log2 domain
  int min_tiles_per_warp;
};

constexpr int kDecodeMaxCtasPerSm = 4;  // grid cap of the decode kernel (bounds partial storage)
constexpr int kDecodeWarpsPerCta = 4;

struct DecodeMaps {
  CUtensorMap k_map;
  CUtensorMap v_map;
};

// Plan kernel; also clears the status word, so it must be the call's first launch.
cudaError_t launch_decode_plan(const AttnArgs& a, const DecodePlan& plan, cudaStream_t stream);
// Host: encode a tiled TMA tensor map (rank 2-5), 128B swizzle, no OOB fill.  `strides` are
// the byte strides of dims 1..rank-1.  Returns the CUresult.
int encode_tensor_map(CUtensorMap* map, bool bf16, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides, const uint32_t* box);
// Same, for 8-bit elements (fp8 caches).
int encode_tensor_map_u8(CUtensorMap* map, int rank, const void* base, const uint64_t* dims,
                         const uint64_t* strides, const uint32_t* box);

cudaError_t launch_decode(const AttnArgs& a, const DecodePlan& plan, const DecodeMaps& maps, int num_sms,
                          cudaStream_t stream);
// Resident decode CTAs per SM for this head size / dtype pair on the current device (at most
// kDecodeMaxCtasPerSm): the decode grid is num_sms times this, and the workspace's partial rows
// are sized from it.
int decode_ctas_per_sm(int head_size, int act_dtype, int cache_dtype);
struct PrefillMaps {
  CUtensorMap k_map;  // cache views, as DecodeMaps
  CUtensorMap v_map;
  CUtensorMap q_map;  // [nt, H, d] view of the (processed) queries: box {64, group, 128/group}
  CUtensorMap vs_map; // [nt, KV, d] fp16 copy of the new V rows (shadow-V prefill): box {64, 1, 16}
};
bool prefill_supported(int head_size, int block_size, int group, int act_dtype, int cache_dtype);
// Query tokens of one prefill work item (a pair of 128-row q tiles) for query-head group `group`.
int prefill_tokens_per_item(int group);
// shadow_v: the shadow-V instantiation first, then the bf16 one as its fallback (see AttnArgs).
cudaError_t launch_prefill(const AttnArgs& a, const DecodePlan& plan, const PrefillMaps& maps, int num_sms,
                           cudaStream_t stream, bool shadow_v = false);
// fp16 copy [nt, KV, d] of the new V rows (a.v_new, row stride a.v_stride), flagging values
// beyond the fp16 range (bf16 magnitude bits 0x4780 and above, inf and NaN included) in
// *a.v_shadow_wide.
cudaError_t launch_v_shadow(const AttnArgs& a, void* shadow, cudaStream_t stream);

cudaError_t launch_tc_selftest(bool bf16, const void* a, const void* b, const void* v, float* c_qk, float* c_pv,
                               float* c_ts, int* status, cudaStream_t stream, int* cu_result);
bool decode_supported(int head_size, int block_size, int act_dtype, int cache_dtype);

}  // namespace b200
