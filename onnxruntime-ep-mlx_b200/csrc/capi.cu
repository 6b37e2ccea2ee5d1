// C ABI: parameter checks, host metadata validation, workspace layout and launch sequence of
// one PagedAttention call.
//
// Host mirror of paged_attention_op (rust/src/ops/attention.rs:3857-4382):
//  * attribute / geometry errors          attention.rs:3866-3932
//  * runtime metadata validation          attention.rs:3934-3990 (same messages)
//  * append, then attention, then output  attention.rs:4021-4382
// Errors never abort the host: every entry returns a status and leaves a message in
// b200_last_error() (the reference's guard_ffi_status, lib.rs:53-92, maps panics the same way).
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "b200_kernels.h"
#include "b200_paged.h"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

void count_launches(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(B200_ERR_CUDA, std::string("PagedAttention: CUDA error in ") + what + ": " + cudaGetErrorString(e));
}

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

bool is_act(int dt) { return dt == B200_DTYPE_FLOAT16 || dt == B200_DTYPE_BFLOAT16; }

int device_sm_count(const B200PagedAttentionParams* p) {
  if (p->num_sms > 0) return p->num_sms;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

struct Layout {
  size_t status = 0;
  size_t owner_keys = 0, owner_vals = 0;
  uint32_t owner_cap = 0;
  size_t q_proc = 0, k_proc = 0;
  size_t total_tiles = 0, seq_tile_off = 0, done = 0, part_o = 0, part_ml = 0;
  size_t route = 0, pf_tile_off = 0, pf_total = 0, pf_next = 0;
  size_t v_shadow = 0;  // bf16 prefill: fp16 copy of the new V rows [nt, KV, d] (0 = none)
  int min_tiles_per_warp = 0;
  bool fast_decode = false;
  bool fast_prefill = false;
  bool process = false;
  size_t total = 0;
};

// LATENT layouts (values are key-row prefixes) run on the generic kernel.
bool fast_decode_enabled(const B200PagedAttentionParams* p) {
  return !p->force_generic && !p->kv_cache_latent &&
         b200::decode_supported(p->head_size, p->block_size, p->act_dtype, p->cache_dtype);
}

bool fast_prefill_enabled(const B200PagedAttentionParams* p) {
  return !p->force_generic && !p->kv_cache_latent && p->kv_num_heads > 0 &&
         b200::prefill_supported(p->head_size, p->block_size, p->num_heads / p->kv_num_heads, p->act_dtype,
                                 p->cache_dtype);
}

Layout make_layout(const B200PagedAttentionParams* p) {
  Layout L;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  const size_t nt = (size_t)std::max(p->num_tokens, 0);
  const size_t d = (size_t)p->head_size;
  L.status = take(256);
  uint32_t cap = 64;
  while (cap < 2 * nt) cap <<= 1;
  L.owner_cap = cap;
  L.owner_keys = take(sizeof(int) * cap);
  L.owner_vals = take(sizeof(int) * cap);
  L.process = p->do_rotary || p->q_norm_weight != nullptr;
  if (L.process) {
    L.q_proc = take(2 * nt * p->num_heads * d);
    L.k_proc = take(2 * nt * p->kv_num_heads * d);
  }
  L.fast_decode = fast_decode_enabled(p);
  L.fast_prefill = fast_prefill_enabled(p);
  if (L.fast_decode || L.fast_prefill) {
    L.route = take(sizeof(int) * (size_t)p->batch);
    L.pf_tile_off = take(sizeof(int) * ((size_t)p->batch + 1));
    L.pf_total = take(sizeof(int64_t));
    L.pf_next = take(sizeof(unsigned long long));
  }
  if (L.fast_decode || L.fast_prefill) {
    // Stream-K decode: at most 2 partial slots of 8 rows per warp of the persistent grid, whose
    // size is SMs x resident decode CTAs per SM (the prefill kernel keeps no partials).
    const int ctas = L.fast_decode ? b200::decode_ctas_per_sm(p->head_size, p->act_dtype, p->cache_dtype) : 1;
    const size_t max_warps = (size_t)device_sm_count(p) * ctas * b200::kDecodeWarpsPerCta;
    const size_t part_rows = max_warps * 2 * b200::kDecodeRows;
    L.min_tiles_per_warp = p->decode_min_tiles_per_warp > 0 ? p->decode_min_tiles_per_warp : 4;
    L.total_tiles = take(sizeof(int64_t));
    L.seq_tile_off = take(sizeof(int) * ((size_t)p->batch + 1));
    L.done = take(sizeof(int) * (size_t)p->batch * p->kv_num_heads);
    L.part_o = take(sizeof(float) * part_rows * d);
    L.part_ml = take(sizeof(float) * part_rows * 2);
  }
  if (L.fast_prefill && p->act_dtype == B200_DTYPE_BFLOAT16 && nt > 0)
    L.v_shadow = take(2 * nt * p->kv_num_heads * d);
  L.total = off;
  return L;
}

// Attribute / geometry / pointer checks that do not need metadata values.
int check_params(const B200PagedAttentionParams* p, bool kv_only) {
  if (!p) return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: null params");
  if (p->num_heads <= 0 || p->kv_num_heads <= 0 || p->num_heads % p->kv_num_heads != 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: bad num_heads/kv_num_heads");
  if (p->head_size <= 0) return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: head_size must be positive");
  if (p->head_size > B200_MAX_HEAD_SIZE)
    return fail(B200_ERR_UNSUPPORTED, "PagedAttention: head_size above 640 is not implemented");
  if (p->num_blocks <= 0 || p->block_size <= 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: caches require matching positive block geometry");
  if (!is_act(p->act_dtype))
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention is only supported for fp16/bf16 (T)");
  const int cd = p->cache_dtype;
  if (!(cd == p->act_dtype || cd == B200_DTYPE_INT8 || cd == B200_DTYPE_UINT8 || cd == B200_DTYPE_FLOAT8E4M3FN))
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: cache dtype must be T, int8, int4 (uint8) or fp8e4m3");
  if (cd != p->act_dtype && (!p->k_scale || !p->v_scale))
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: quantized caches require k_scale and v_scale");
  if (p->batch < 1)
    return fail(B200_ERR_FAIL, "PagedAttention: cumulative_sequence_length must have length batch+1");
  if (p->num_tokens < 0 || p->max_blocks_per_seq < 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: negative token or block-table size");
  if ((int64_t)p->num_blocks * p->block_size > INT32_MAX)
    return fail(B200_ERR_UNSUPPORTED, "PagedAttention: cache slot count exceeds int32");
  const bool latent = p->kv_cache_latent != 0;
  if (latent) {  // attention.rs:4426-4535
    if (p->kv_num_heads != 1) return fail(B200_ERR_INVALID_ARGUMENT, "LATENT layout requires kv_num_heads=1");
    if (cd != p->act_dtype)
      return fail(B200_ERR_INVALID_ARGUMENT, "quantized LATENT cache contract is not supported");
    if (p->value || p->value_cache)
      return fail(B200_ERR_INVALID_ARGUMENT,
                  "LATENT layout aliases value to key and requires absent value/value_cache");
    if (p->v_head_size < 0 || p->v_head_size > p->head_size)
      return fail(B200_ERR_INVALID_ARGUMENT, "LATENT v_head_size must not exceed head_size");
  }
  if (!p->key || (!latent && !p->value) || !p->key_cache || (!latent && !p->value_cache) ||
      !p->cumulative_sequence_length || !p->past_seqlens || !p->block_table)
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: missing required input");
  // rows the append prologue stages in shared memory (rotary / norm, or an encoded cache)
  if (p->do_rotary || p->q_norm_weight || cd != p->act_dtype) {
    const size_t rows = (size_t)((p->do_rotary || p->q_norm_weight) ? p->num_heads : 0) + 2 * (size_t)p->kv_num_heads;
    if (sizeof(float) * (size_t)p->head_size * rows > B200_MAX_PROLOGUE_STAGE_BYTES)
      return fail(B200_ERR_UNSUPPORTED,
                  "PagedAttention: rotary / norm / encoded rows of one token exceed the prologue's shared memory");
  }
  if (!kv_only && (!p->query || !p->output))
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: missing query or output");
  if (p->do_rotary) {
    if (!p->cos_cache || !p->sin_cache)
      return fail(B200_ERR_INVALID_ARGUMENT, "do_rotary=1 requires cos_cache and sin_cache inputs");
    if (p->rotary_dim <= 0 || p->rotary_dim % 2 || p->rotary_offset < 0 ||
        p->rotary_offset + p->rotary_dim > p->head_size)
      return fail(B200_ERR_INVALID_ARGUMENT, "rotary_offset + rotary_dim must not exceed head_size");
  }
  if ((p->q_norm_weight == nullptr) != (p->k_norm_weight == nullptr))
    return fail(B200_ERR_INVALID_ARGUMENT, "q_norm_weight and k_norm_weight must be provided together");
  if (p->local_window_size < -1)
    return fail(B200_ERR_INVALID_ARGUMENT, "local_window_size must be -1 or positive");
  if (!(p->softcap >= 0.f) || std::isinf(p->softcap))
    return fail(B200_ERR_INVALID_ARGUMENT, "softcap must be finite and non-negative");
  return B200_OK;
}

int64_t q_stride(const B200PagedAttentionParams* p) {
  return p->query_row_stride ? p->query_row_stride : (int64_t)p->num_heads * p->head_size;
}
int64_t k_stride(const B200PagedAttentionParams* p) {
  return p->key_row_stride ? p->key_row_stride : (int64_t)p->kv_num_heads * p->head_size;
}
int64_t v_stride(const B200PagedAttentionParams* p) {
  return p->value_row_stride ? p->value_row_stride : (int64_t)p->kv_num_heads * p->head_size;
}

// Host metadata checks, attention.rs:3934-3990.  Also reports whether two tokens share a slot.
int validate_host(const B200PagedAttentionParams* p, bool* duplicates) {
  const int32_t* cum = p->host_cumulative_sequence_length;
  const int32_t* past = p->host_past_seqlens;
  const int32_t* bt = p->host_block_table;
  if (!cum || !past || !bt)
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: host metadata copies are required for host validation");
  const int B = p->batch;
  if (B < 1) return fail(B200_ERR_FAIL, "PagedAttention: cumulative_sequence_length must have length batch+1");
  bool bad = cum[0] != 0 || cum[B] != p->num_tokens;
  for (int b = 0; b < B && !bad; ++b) bad = cum[b] < 0 || cum[b] > cum[b + 1] || past[b] < 0;
  if (bad)
    return fail(B200_ERR_FAIL, "PagedAttention: inconsistent cumulative lengths, past lengths or block table");
  const int64_t slots = (int64_t)p->num_blocks * p->block_size;
  if (p->host_slot_mapping) {
    for (int t = 0; t < p->num_tokens; ++t) {
      int64_t s = p->host_slot_mapping[t];
      if (s < -1 || s >= slots)
        return fail(B200_ERR_FAIL, "PagedAttention: slot_mapping must contain -1 or valid physical cache slots");
    }
  }
  const int64_t maxb = p->max_blocks_per_seq;
  const uint32_t nblocks = (uint32_t)std::max(p->num_blocks, 0);
  for (int b = 0; b < B; ++b) {
    int64_t total = (int64_t)past[b] + cum[b + 1] - cum[b];
    if (total > INT32_MAX || total > maxb * p->block_size)
      return fail(B200_ERR_FAIL, "PagedAttention: sequence exceeds block table capacity");
    const int64_t needed = (total + p->block_size - 1) / p->block_size;
    // Branch-free over the row (vectorised): a negative entry is a large unsigned value.
    const int32_t* row = bt + b * maxb;
    uint32_t bad_row = 0;
    for (int64_t j = 0; j < needed; ++j) bad_row |= (uint32_t)((uint32_t)row[j] >= nblocks);
    if (bad_row)
      return fail(B200_ERR_FAIL, "PagedAttention: block table contains an invalid physical block");
    if (p->do_rotary && total > p->rotary_positions)
      return fail(B200_ERR_FAIL, "PagedAttention: rotary position exceeds the cos/sin cache");
  }
  if (duplicates) {
    // Open-addressing set of the written slots (reused across calls on this thread).
    thread_local std::vector<int64_t> table;
    size_t cap = 16;
    while (cap < (size_t)p->num_tokens * 2) cap <<= 1;
    if (table.size() < cap) table.resize(cap);
    std::fill(table.begin(), table.begin() + cap, (int64_t)-1);
    const size_t mask = cap - 1;
    *duplicates = false;
    for (int b = 0; b < B && !*duplicates; ++b) {
      for (int t = cum[b]; t < cum[b + 1]; ++t) {
        int64_t slot;
        if (p->host_slot_mapping) {
          slot = p->host_slot_mapping[t];
        } else {
          int64_t logical = (int64_t)past[b] + (t - cum[b]);
          slot = (int64_t)bt[b * maxb + logical / p->block_size] * p->block_size + logical % p->block_size;
        }
        if (slot < 0) continue;
        size_t h = (size_t)((uint64_t)slot * 0x9e3779b97f4a7c15ull >> 17) & mask;
        while (table[h] != -1 && table[h] != slot) h = (h + 1) & mask;
        if (table[h] == slot) {
          *duplicates = true;
          break;
        }
        table[h] = slot;
      }
    }
  }
  return B200_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// [NB*bs, KV, d] view of a cache: box {64 channels, 1 head, 16 slots}, 128-byte swizzle.
int encode_cache_map(CUtensorMap* map, const void* base, const B200PagedAttentionParams* p) {
  // [NB*bs, KV, d] view of a cache; a box is 16 slots of one kv head x 128 bytes of channels
  // (64 16-bit or 128 fp8 elements)
  const bool fp8 = p->cache_dtype == B200_DTYPE_FLOAT8E4M3FN;
  const uint64_t esz = fp8 ? 1 : 2;
  const uint64_t dims[3] = {(uint64_t)p->head_size, (uint64_t)p->kv_num_heads,
                            (uint64_t)p->num_blocks * (uint64_t)p->block_size};
  const uint64_t strides[2] = {(uint64_t)p->head_size * esz, (uint64_t)p->kv_num_heads * p->head_size * esz};
  const uint32_t box[3] = {fp8 ? 128u : 64u, 1, (uint32_t)b200::kTile};
  int r = fp8 ? b200::encode_tensor_map_u8(map, 3, base, dims, strides, box)
              : b200::encode_tensor_map(map, p->act_dtype == B200_DTYPE_BFLOAT16, 3, base, dims, strides, box);
  if (r != CUDA_SUCCESS)
    return fail(B200_ERR_CUDA, "PagedAttention: cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return B200_OK;
}

b200::PrologueArgs prologue_args(const B200PagedAttentionParams* p, const Layout& L, char* ws, int* status,
                                 bool dedup, bool kv_only, int* route) {
  b200::PrologueArgs a{};
  a.num_heads = p->num_heads;
  a.kv_heads = p->kv_num_heads;
  a.head_size = p->head_size;
  a.num_tokens = p->num_tokens;
  a.batch = p->batch;
  a.num_blocks = p->num_blocks;
  a.block_size = p->block_size;
  a.max_blocks = p->max_blocks_per_seq;
  a.act_dtype = p->act_dtype;
  a.cache_dtype = p->cache_dtype;
  a.k_per_channel = p->k_quant_per_channel;
  a.v_per_channel = p->v_quant_per_channel;
  a.do_norm = p->q_norm_weight != nullptr;
  a.do_rotary = p->do_rotary;
  a.rotary_interleaved = p->rotary_interleaved;
  a.rotary_offset = p->rotary_offset;
  a.rotary_dim = p->rotary_dim;
  a.rotary_positions = p->do_rotary ? p->rotary_positions : 0;
  a.kv_only = kv_only;
  a.latent = p->kv_cache_latent != 0;
  a.norm_eps = p->q_norm_weight ? p->qk_norm_epsilon : 0.f;
  a.query_stride = q_stride(p);
  a.key_stride = k_stride(p);
  a.value_stride = v_stride(p);
  a.query = p->query;
  a.key = p->key;
  a.value = p->value;
  a.key_cache = p->key_cache;
  a.value_cache = p->value_cache;
  a.cum = p->cumulative_sequence_length;
  a.past = p->past_seqlens;
  a.block_table = p->block_table;
  a.slot_mapping = p->slot_mapping;
  a.cos_cache = p->cos_cache;
  a.sin_cache = p->sin_cache;
  a.q_norm = p->q_norm_weight;
  a.k_norm = p->k_norm_weight;
  a.k_scale = p->k_scale;
  a.v_scale = p->v_scale;
  if (L.process && !kv_only) {
    a.q_proc = ws + L.q_proc;
    a.k_proc = ws + L.k_proc;
  }
  if (dedup) {
    a.owner_keys = reinterpret_cast<int*>(ws + L.owner_keys);
    a.owner_vals = reinterpret_cast<int*>(ws + L.owner_vals);
    a.owner_capacity = L.owner_cap;
  }
  a.status = status;
  a.route = route;
  return a;
}

// Shared front half of append and attention: checks, status, dedup table, prologue kernel.
int run_prologue(const B200PagedAttentionParams* p, const Layout& L, cudaStream_t stream, bool kv_only,
                 bool status_cleared, int* route, bool* duplicates_out) {
  char* ws = static_cast<char*>(p->workspace);
  int* status = p->device_status ? p->device_status : reinterpret_cast<int*>(ws + L.status);
  const bool host_meta = p->host_cumulative_sequence_length && p->host_past_seqlens && p->host_block_table;
  bool dedup = true;
  if (host_meta) {
    int rc = validate_host(p, &dedup);
    if (rc) return rc;
  }
  cudaError_t e;
  if (!status_cleared) {
    e = cudaMemsetAsync(status, 0, sizeof(int), stream);
    if (e != cudaSuccess) return cuda_fail(e, "status reset");
    count_launches(1);
  }
  if (duplicates_out) *duplicates_out = dedup;
  b200::PrologueArgs a = prologue_args(p, L, ws, status, dedup, kv_only, route);
  if ((dedup || !host_meta) && b200::append_fused_eligible(a)) {
    e = b200::launch_append_fused(a, stream);
    if (e != cudaSuccess) return cuda_fail(e, "kv_append_fused_kernel");
    count_launches(1);
    return B200_OK;
  }
  if (dedup) {
    e = cudaMemsetAsync(ws + L.owner_keys, 0xff, sizeof(int) * 2 * (size_t)L.owner_cap, stream);
    if (e != cudaSuccess) return cuda_fail(e, "slot table reset");
    count_launches(1);
  }
  if (dedup || !host_meta) {
    b200::launch_meta_check(a, stream);
    count_launches(1);
  }
  e = b200::launch_prologue(a, stream);
  if (e != cudaSuccess) return cuda_fail(e, "kv_prologue_kernel");
  count_launches(1);
  return B200_OK;
}

}  // namespace

namespace b200 {
int set_error(int code, const std::string& msg) { return fail(code, msg); }
void add_launches(uint64_t n) { count_launches(n); }

int encode_tensor_map(CUtensorMap* map, bool bf16, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides, const uint32_t* box) {
  auto enc = tensor_map_encoder();
  if (!enc) return CUDA_ERROR_NOT_SUPPORTED;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i > 0) st[i - 1] = strides[i - 1];
  }
  return (int)enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank,
                  const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}
int encode_tensor_map_u8(CUtensorMap* map, int rank, const void* base, const uint64_t* dims,
                         const uint64_t* strides, const uint32_t* box) {
  auto enc = tensor_map_encoder();
  if (!enc) return CUDA_ERROR_NOT_SUPPORTED;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i > 0) st[i - 1] = strides[i - 1];
  }
  return (int)enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}
}  // namespace b200

extern "C" {

int b200_version(void) { return 100; }

size_t b200_params_size(void) { return sizeof(B200PagedAttentionParams); }

uint64_t b200_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

size_t b200_node_info_size(void) { return sizeof(B200NodeInfo); }

const char* b200_last_error(void) { return g_last_error.c_str(); }

int b200_paged_attention_workspace_size(const B200PagedAttentionParams* p, size_t* bytes) {
  // Sizing depends on shapes only, so an append-only caller (no query / output) may ask too.
  int rc = check_params(p, true);
  if (rc) return rc;
  if (!bytes) return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: null bytes pointer");
  *bytes = make_layout(p).total;
  return B200_OK;
}

int b200_paged_attention_validate_host(const B200PagedAttentionParams* p) {
  int rc = check_params(p, false);
  if (rc) return rc;
  return validate_host(p, nullptr);
}

int b200_kv_append(const B200PagedAttentionParams* p, void* stream_ptr) {
  try {
    int rc = check_params(p, true);
    if (rc) return rc;
    Layout L = make_layout(p);
    if (!p->workspace || p->workspace_bytes < L.total)
      return fail(B200_ERR_WORKSPACE, "PagedAttention: workspace missing or smaller than b200_paged_attention_workspace_size()");
    return run_prologue(p, L, static_cast<cudaStream_t>(stream_ptr), true, false, nullptr, nullptr);
  } catch (const std::exception& ex) {
    return fail(B200_ERR_FAIL, std::string("PagedAttention: ") + ex.what());
  } catch (...) {
    return fail(B200_ERR_FAIL, "PagedAttention: unknown failure");
  }
}

int b200_paged_attention(const B200PagedAttentionParams* p, void* stream_ptr) {
  try {
    int rc = check_params(p, false);
    if (rc) return rc;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    Layout L = make_layout(p);
    if (!p->workspace || p->workspace_bytes < L.total)
      return fail(B200_ERR_WORKSPACE, "PagedAttention: workspace missing or smaller than b200_paged_attention_workspace_size()");
    char* ws = static_cast<char*>(p->workspace);
    int* status = p->device_status ? p->device_status : reinterpret_cast<int*>(ws + L.status);
    if (p->num_tokens == 0) {
      cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), stream);
      count_launches(1);
      return e == cudaSuccess ? B200_OK : cuda_fail(e, "status reset");
    }

    b200::AttnArgs a{};
    a.num_heads = p->num_heads;
    a.kv_heads = p->kv_num_heads;
    a.head_size = p->head_size;
    a.group = p->num_heads / p->kv_num_heads;
    a.num_tokens = p->num_tokens;
    a.batch = p->batch;
    a.num_blocks = p->num_blocks;
    a.block_size = p->block_size;
    a.max_blocks = p->max_blocks_per_seq;
    a.act_dtype = p->act_dtype;
    a.cache_dtype = p->cache_dtype;
    a.k_per_channel = p->k_quant_per_channel;
    a.v_per_channel = p->v_quant_per_channel;
    a.is_causal = p->is_causal;
    a.window = p->local_window_size;
    a.scale = p->scale != 0.f ? p->scale : 1.0f / std::sqrt((float)p->head_size);
    a.softcap = p->softcap;
    a.key_cache = p->key_cache;
    a.value_cache = p->value_cache;
    a.k_scale = p->k_scale;
    a.v_scale = p->v_scale;
    a.cum = p->cumulative_sequence_length;
    a.past = p->past_seqlens;
    a.block_table = p->block_table;
    a.head_sink = p->head_sink;
    a.out = p->output;
    a.status = status;
    if (L.process) {
      a.q = ws + L.q_proc;
      a.q_stride = (int64_t)p->num_heads * p->head_size;
      a.k_new = ws + L.k_proc;
      a.k_stride = (int64_t)p->kv_num_heads * p->head_size;
    } else {
      a.q = p->query;
      a.q_stride = q_stride(p);
      a.k_new = p->key;
      a.k_stride = k_stride(p);
    }
    if (p->kv_cache_latent) {  // values are the first v_head channels of the key rows
      a.v_head = p->v_head_size > 0 ? p->v_head_size : p->head_size;
      a.value_cache = p->key_cache;
      a.v_new = a.k_new;
      a.v_stride = a.k_stride;
    } else {
      a.v_head = p->head_size;
      a.v_new = p->value;
      a.v_stride = v_stride(p);
    }

    b200::DecodePlan plan{};
    b200::DecodeMaps maps;
    b200::PrefillMaps pmaps;
    const bool planned = L.fast_decode || L.fast_prefill;
    const int group = p->num_heads / p->kv_num_heads;
    if (planned) {
      plan.total_tiles = reinterpret_cast<int64_t*>(ws + L.total_tiles);
      plan.seq_tile_off = reinterpret_cast<int*>(ws + L.seq_tile_off);
      plan.done = reinterpret_cast<int*>(ws + L.done);
      plan.part_o = reinterpret_cast<float*>(ws + L.part_o);
      plan.part_ml = reinterpret_cast<float*>(ws + L.part_ml);
      plan.min_tiles_per_warp = L.min_tiles_per_warp;
      plan.pf_tile_off = reinterpret_cast<int*>(ws + L.pf_tile_off);
      plan.pf_total = reinterpret_cast<int64_t*>(ws + L.pf_total);
      plan.pf_next = reinterpret_cast<unsigned long long*>(ws + L.pf_next);
      a.route = reinterpret_cast<int*>(ws + L.route);
      a.decode_on = L.fast_decode;
      a.decode_tile = p->cache_dtype == B200_DTYPE_FLOAT8E4M3FN ? b200::kFp8HalfTiles * b200::kTile : b200::kTile;
      a.prefill_tq = L.fast_prefill ? b200::prefill_tokens_per_item(group) : 0;
      // the status block's second word: the shadow-V range flag (cleared by the plan kernel)
      a.v_shadow_wide = L.v_shadow ? reinterpret_cast<int*>(ws + L.status + 64) : nullptr;
      if ((rc = encode_cache_map(&maps.k_map, p->key_cache, p))) return rc;
      if ((rc = encode_cache_map(&maps.v_map, p->value_cache, p))) return rc;
      if (L.fast_prefill) {
        pmaps.k_map = maps.k_map;
        pmaps.v_map = maps.v_map;
        // [nt, H, d] view of the (processed) queries: box {64 channels, g heads, 128/g tokens}
        const uint64_t dims[3] = {(uint64_t)p->head_size, (uint64_t)p->num_heads, (uint64_t)p->num_tokens};
        const uint64_t strides[2] = {(uint64_t)p->head_size * 2, (uint64_t)a.q_stride * 2};
        const uint32_t box[3] = {64, (uint32_t)group, (uint32_t)(128 / group)};
        int r = b200::encode_tensor_map(&pmaps.q_map, p->act_dtype == B200_DTYPE_BFLOAT16, 3, a.q, dims, strides, box);
        if (r) return fail(B200_ERR_CUDA, "PagedAttention: cuTensorMapEncodeTiled (queries) failed (" + std::to_string(r) + ")");
      }
      // First launch of the call: clears the status word, routes sequences, plans the work.
      cudaError_t e = b200::launch_decode_plan(a, plan, stream);
      if (e != cudaSuccess) return cuda_fail(e, "decode_plan_kernel");
      count_launches(1);
    }
    bool duplicates = true;
    rc = run_prologue(p, L, stream, false, planned, a.route, &duplicates);
    if (rc) return rc;

    // Which kernels can have work.  With host metadata the host knows the routes (a prefill
    // sequence may still move to the generic kernel when slots are remapped or duplicated);
    // without it every enabled kernel is launched and each skips what is not its own.
    const bool host_meta = p->host_cumulative_sequence_length && p->host_past_seqlens;
    bool any_decode = L.fast_decode, any_prefill = L.fast_prefill, any_generic = true;
    if (host_meta) {
      const int32_t* cum = p->host_cumulative_sequence_length;
      any_decode = any_prefill = any_generic = false;
      for (int b = 0; b < p->batch; ++b) {
        const int nq = cum[b + 1] - cum[b];
        if (nq <= 0) continue;
        if (L.fast_decode && nq * group <= b200::kDecodeRows) any_decode = true;
        else if (L.fast_prefill) any_prefill = true;
        else any_generic = true;
      }
      if (any_prefill && (p->host_slot_mapping || p->slot_mapping || duplicates)) any_generic = true;
    }
    // bf16 prefill over an fp16 copy of the new V rows when no prefill sequence has a cached
    // prefix (every key it reads is a new row of this call); known only with host metadata.
    bool shadow_v = false;
    if (any_prefill && host_meta && L.v_shadow && a.v_shadow_wide &&
        ((reinterpret_cast<uintptr_t>(a.v_new) | (uintptr_t)(a.v_stride * 2)) & 15) == 0) {
      const int32_t* cum = p->host_cumulative_sequence_length;
      shadow_v = true;
      for (int b = 0; b < p->batch && shadow_v; ++b) {
        const int nq = cum[b + 1] - cum[b];
        const bool prefill = nq > 0 && !(L.fast_decode && nq * group <= b200::kDecodeRows);
        if (prefill && p->host_past_seqlens[b] != 0) shadow_v = false;
      }
    }
    if (shadow_v) {
      void* shadow = ws + L.v_shadow;
      const uint64_t dims[3] = {(uint64_t)p->head_size, (uint64_t)p->kv_num_heads, (uint64_t)p->num_tokens};
      const uint64_t strides[2] = {(uint64_t)p->head_size * 2, (uint64_t)p->kv_num_heads * p->head_size * 2};
      const uint32_t box[3] = {64, 1, (uint32_t)b200::kTile};
      int r = b200::encode_tensor_map(&pmaps.vs_map, false, 3, shadow, dims, strides, box);
      if (r) return fail(B200_ERR_CUDA, "PagedAttention: cuTensorMapEncodeTiled (V copy) failed (" + std::to_string(r) + ")");
      cudaError_t e = b200::launch_v_shadow(a, shadow, stream);
      if (e != cudaSuccess) return cuda_fail(e, "v_shadow_kernel");
      count_launches(1);
    }
    if (p->attention_event_begin) {
      cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(p->attention_event_begin), stream);
      if (e != cudaSuccess) return cuda_fail(e, "event record");
    }
    if (any_decode) {
      cudaError_t e = b200::launch_decode(a, plan, maps, device_sm_count(p), stream);
      if (e != cudaSuccess) return cuda_fail(e, "paged_decode_kernel");
      count_launches(1);
    }
    if (any_prefill) {
      cudaError_t e = b200::launch_prefill(a, plan, pmaps, device_sm_count(p), stream, shadow_v);
      if (e != cudaSuccess) return cuda_fail(e, "paged_prefill_kernel");
      count_launches(shadow_v ? 2 : 1);
    }
    if (any_generic) {
      cudaError_t e = b200::launch_generic(a, stream);
      if (e != cudaSuccess) return cuda_fail(e, "generic_attention_kernel");
      count_launches(1);
    }
    if (p->attention_event_end) {
      cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(p->attention_event_end), stream);
      if (e != cudaSuccess) return cuda_fail(e, "event record");
    }
    return B200_OK;
  } catch (const std::exception& ex) {
    return fail(B200_ERR_FAIL, std::string("PagedAttention: ") + ex.what());
  } catch (...) {
    return fail(B200_ERR_FAIL, "PagedAttention: unknown failure");
  }
}

int b200_selftest_tcgen05(int32_t dtype, const void* a, const void* b, const void* v, float* c_qk, float* c_pv,
                          float* c_ts, int32_t* device_status, void* stream) {
  if (!a || !b || !v || !c_qk || !c_pv || !device_status)
    return fail(B200_ERR_INVALID_ARGUMENT, "selftest: null pointer");
  if (dtype != B200_DTYPE_FLOAT16 && dtype != B200_DTYPE_BFLOAT16)
    return fail(B200_ERR_INVALID_ARGUMENT, "selftest: dtype must be FLOAT16 or BFLOAT16");
  int cu = 0;
  cudaError_t e = b200::launch_tc_selftest(dtype == B200_DTYPE_BFLOAT16, a, b, v, c_qk, c_pv, c_ts, device_status,
                                           static_cast<cudaStream_t>(stream), &cu);
  if (cu) return fail(B200_ERR_CUDA, "selftest: cuTensorMapEncodeTiled failed (" + std::to_string(cu) + ")");
  if (e != cudaSuccess) return cuda_fail(e, "tc_selftest_kernel");
  count_launches(1);
  return B200_OK;
}

int b200_read_status(const B200PagedAttentionParams* p, void* stream_ptr) {
  if (!p || (!p->workspace && !p->device_status))
    return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: no status word");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  Layout L = make_layout(p);
  int* status = p->device_status ? p->device_status
                                 : reinterpret_cast<int*>(static_cast<char*>(p->workspace) + L.status);
  int bits = 0;
  cudaError_t e = cudaMemcpyAsync(&bits, status, sizeof(int), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_fail(e, "status read");
  if (bits == 0) return B200_OK;
  if (bits & b200::kStatusBadCumulative || bits & b200::kStatusBadPast)
    return fail(B200_ERR_FAIL, "PagedAttention: inconsistent cumulative lengths, past lengths or block table");
  if (bits & b200::kStatusBadSlot)
    return fail(B200_ERR_FAIL, "PagedAttention: slot_mapping must contain -1 or valid physical cache slots");
  if (bits & b200::kStatusBadCapacity)
    return fail(B200_ERR_FAIL, "PagedAttention: sequence exceeds block table capacity");
  if (bits & b200::kStatusBadBlock)
    return fail(B200_ERR_FAIL, "PagedAttention: block table contains an invalid physical block");
  if (bits & b200::kStatusBadPosition)
    return fail(B200_ERR_FAIL, "PagedAttention: rotary position exceeds the cos/sin cache");
  if (bits & b200::kStatusTimeout)
    return fail(B200_ERR_DEVICE, "PagedAttention: a device wait timed out (TMA copy did not complete)");
  return fail(B200_ERR_DEVICE, "PagedAttention: device status " + std::to_string(bits));
}

}  // extern "C"
