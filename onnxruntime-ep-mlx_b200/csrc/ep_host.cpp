// Host layer of the execution provider below ONNX Runtime's own types: session options, error
// classes, the KV block pool and the compiled-node launcher (include/b200_ep.h).
//
//  * options     rust/src/config.rs:18-64 (strict booleans), rust/src/memory.rs:10-98 (strict
//                byte counts, session value before the environment)
//  * errors      rust/src/lib.rs:53-92 (failures become an ORT_EP_FAIL status, bad arguments
//                ORT_INVALID_ARGUMENT)
//  * KV pool     the device allocator and budgets of rust/src/device.rs:409-493 and
//                rust/src/memory.rs:26-98, re-cut for paged caches: one budgeted allocation of
//                both caches, handed out as block ids
//  * launcher    rust/src/runtime.rs:93-331: per-node state, a run gate, inputs to kernel
//                parameters, the device status turned into an error
#include <cuda_runtime.h>

#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "b200_ep.h"
#include "b200_kernels.h"

namespace {

int fail(int code, const std::string& msg) { return b200::set_error(code, msg); }

// ---------------------------------------------------------------------------------------------
// session options
// ---------------------------------------------------------------------------------------------
struct OptionKey {
  const char* session;
  const char* env;
};

constexpr OptionKey kPoolBytes{"ep.b200.kv_pool_bytes", "ONNXRUNTIME_EP_B200_KV_POOL_BYTES"};
constexpr OptionKey kNumGpus{"ep.b200.num_gpus", "ONNXRUNTIME_EP_B200_NUM_GPUS"};
constexpr OptionKey kDeviceId{"ep.b200.device_id", "ONNXRUNTIME_EP_B200_DEVICE_ID"};
constexpr OptionKey kMinTiles{"ep.b200.decode_min_tiles_per_warp", "ONNXRUNTIME_EP_B200_DECODE_MIN_TILES"};
constexpr OptionKey kForceGeneric{"ep.b200.force_generic", "ONNXRUNTIME_EP_B200_FORCE_GENERIC"};
constexpr OptionKey kCheckStatus{"ep.b200.check_status", "ONNXRUNTIME_EP_B200_CHECK_STATUS"};

// Non-empty ASCII decimal digits that fit in 64 bits (memory.rs:10-17).
bool parse_u64(const char* s, uint64_t* out) {
  if (!s || !*s) return false;
  uint64_t v = 0;
  for (const char* c = s; *c; ++c) {
    if (*c < '0' || *c > '9') return false;
    const uint64_t digit = (uint64_t)(*c - '0');
    if (v > (UINT64_MAX - digit) / 10) return false;
    v = v * 10 + digit;
  }
  *out = v;
  return true;
}

// Exactly "0" or "1" (config.rs:46-52).
bool parse_bool(const char* s, int32_t* out) {
  if (s && s[0] == '0' && s[1] == 0) return *out = 0, true;
  if (s && s[0] == '1' && s[1] == 0) return *out = 1, true;
  return false;
}

// The value of `key`: the session entry when present, else the environment variable.
const char* lookup(const OptionKey& key, const char* const* keys, const char* const* values, size_t count,
                   bool* from_session) {
  for (size_t i = 0; i < count; ++i) {
    if (keys && keys[i] && std::strcmp(keys[i], key.session) == 0) {
      *from_session = true;
      return values ? values[i] : nullptr;
    }
  }
  *from_session = false;
  return std::getenv(key.env);
}

std::string where(const OptionKey& key, bool from_session) {
  return from_session ? std::string(key.session) : std::string(key.env) + " (environment)";
}

int parse_int_option(const OptionKey& key, const char* const* keys, const char* const* values, size_t count,
                     int64_t lo, int32_t* out) {
  bool sess = false;
  const char* v = lookup(key, keys, values, count, &sess);
  if (!v) return B200_OK;
  uint64_t x = 0;
  if (!parse_u64(v, &x) || (int64_t)x < lo || x > (uint64_t)INT32_MAX)
    return fail(B200_ERR_INVALID_ARGUMENT, "B200 session option " + where(key, sess) + ": expected a decimal integer >= " +
                                              std::to_string(lo) + ", got \"" + v + "\"");
  *out = (int32_t)x;
  return B200_OK;
}

int parse_bool_option(const OptionKey& key, const char* const* keys, const char* const* values, size_t count,
                      int32_t* out) {
  bool sess = false;
  const char* v = lookup(key, keys, values, count, &sess);
  if (!v) return B200_OK;
  if (!parse_bool(v, out))
    return fail(B200_ERR_INVALID_ARGUMENT, "B200 session option " + where(key, sess) + ": expected 0 or 1, got \"" +
                                              std::string(v) + "\"");
  return B200_OK;
}

// ---------------------------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------------------------
// Makes `device` current for the scope and restores the caller's device.
struct DeviceScope {
  int previous = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceScope(int device) {
    if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
    if (device != previous) err = cudaSetDevice(device);
  }
  ~DeviceScope() {
    if (previous >= 0) cudaSetDevice(previous);
  }
};

int cuda_fail(cudaError_t e, const std::string& what) {
  return fail(B200_ERR_CUDA, what + ": " + cudaGetErrorString(e));
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// KV block pool
// ---------------------------------------------------------------------------------------------
struct B200KvPool {
  std::mutex mu;
  B200KvPoolDesc desc{};
  void* key_cache = nullptr;
  void* value_cache = nullptr;
  float* k_scale = nullptr;
  float* v_scale = nullptr;
  bool owns = false;
  uint64_t block_bytes = 0;
  uint64_t allocated = 0;
  int32_t num_blocks = 0;
  std::vector<int32_t> free_stack;  // back() is handed out next
  std::vector<uint8_t> in_use;
};

namespace {

int cache_row_bytes(const B200KvPoolDesc* d, uint64_t* row) {
  const uint64_t kv = (uint64_t)d->kv_num_heads, hs = (uint64_t)d->head_size;
  switch (d->cache_dtype) {
    case B200_DTYPE_FLOAT16:
    case B200_DTYPE_BFLOAT16: *row = kv * hs * 2; return B200_OK;
    case B200_DTYPE_INT8:
    case B200_DTYPE_FLOAT8E4M3FN: *row = kv * hs; return B200_OK;
    case B200_DTYPE_UINT8: *row = kv * ((hs + 1) / 2); return B200_OK;
    default: return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: cache dtype must be float16, bfloat16, int8, int4 (uint8) or float8e4m3fn");
  }
}

}  // namespace

extern "C" {

int b200_ep_options_parse(const char* const* keys, const char* const* values, size_t count, B200EpOptions* out) {
  if (!out) return fail(B200_ERR_INVALID_ARGUMENT, "B200 session options: null output");
  if (count && (!keys || !values)) return fail(B200_ERR_INVALID_ARGUMENT, "B200 session options: null key/value arrays");
  B200EpOptions o{};
  o.num_gpus = 1;
  o.check_status = 1;
  bool sess = false;
  if (const char* v = lookup(kPoolBytes, keys, values, count, &sess)) {
    uint64_t bytes = 0;
    if (!parse_u64(v, &bytes))
      return fail(B200_ERR_INVALID_ARGUMENT, "B200 KV pool budget: " + where(kPoolBytes, sess) +
                                                 " must be a nonnegative decimal byte count that fits in 64 bits, got \"" +
                                                 std::string(v) + "\"");
    o.kv_pool_bytes = bytes;
    o.has_kv_pool_bytes = 1;
  }
  int rc;
  if ((rc = parse_int_option(kNumGpus, keys, values, count, 1, &o.num_gpus))) return rc;
  if ((rc = parse_int_option(kDeviceId, keys, values, count, 0, &o.device_id))) return rc;
  if ((rc = parse_int_option(kMinTiles, keys, values, count, 1, &o.decode_min_tiles_per_warp))) return rc;
  if ((rc = parse_bool_option(kForceGeneric, keys, values, count, &o.force_generic))) return rc;
  if ((rc = parse_bool_option(kCheckStatus, keys, values, count, &o.check_status))) return rc;
  *out = o;
  return B200_OK;
}

size_t b200_ep_struct_size(int32_t which) {
  switch (which) {
    case 0: return sizeof(B200EpOptions);
    case 1: return sizeof(B200KvPoolDesc);
    case 2: return sizeof(B200KvPoolInfo);
    case 3: return sizeof(B200PagedTensors);
    default: return 0;
  }
}

int b200_ort_error_class(int status) {
  if (status == B200_OK) return B200_ORT_OK;
  if (status == B200_ERR_INVALID_ARGUMENT) return B200_ORT_INVALID_ARGUMENT;
  return B200_ORT_EP_FAIL;
}

int b200_kv_pool_block_bytes(const B200KvPoolDesc* d, uint64_t* bytes) {
  if (!d || !bytes) return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: null argument");
  if (d->block_size <= 0 || d->kv_num_heads <= 0 || d->head_size <= 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: block_size, kv_num_heads and head_size must be positive");
  uint64_t row = 0;
  int rc = cache_row_bytes(d, &row);
  if (rc) return rc;
  *bytes = row * (uint64_t)d->block_size;
  return B200_OK;
}

int b200_kv_pool_create(const B200KvPoolDesc* d, B200KvPool** out) {
  if (!out) return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: null output");
  *out = nullptr;
  uint64_t block = 0;
  int rc = b200_kv_pool_block_bytes(d, &block);
  if (rc) return rc;
  const bool fp8 = d->cache_dtype == B200_DTYPE_FLOAT8E4M3FN;
  const bool external = d->key_cache || d->value_cache;
  if (external && (!d->key_cache || !d->value_cache))
    return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: caller-owned caches need both key_cache and value_cache");
  if (external && fp8 && (!d->k_scale || !d->v_scale))
    return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: caller-owned fp8 caches need k_scale and v_scale");
  // bytes one block costs everything the pool allocates: K and V rows, and fp8 scales
  const uint64_t per_block = 2 * block + (fp8 ? 2ull * (uint64_t)d->kv_num_heads * sizeof(float) : 0);
  int64_t nb = d->num_blocks;
  if (nb < 0) return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: num_blocks must be non-negative");
  if (nb == 0) {
    if (external) return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: caller-owned caches need num_blocks");
    if (d->budget_bytes == 0)
      return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: set num_blocks or a byte budget (ep.b200.kv_pool_bytes)");
    nb = (int64_t)(d->budget_bytes / per_block);
    const int64_t slot_cap = (int64_t)INT32_MAX / d->block_size;  // slot ids are int32
    if (nb > slot_cap) nb = slot_cap;
    if (nb < 1)
      return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: the budget of " + std::to_string(d->budget_bytes) +
                                                 " bytes holds no block of " + std::to_string(per_block) + " bytes");
  } else {
    if ((int64_t)nb * d->block_size > INT32_MAX)
      return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: num_blocks * block_size exceeds int32 slot ids");
    if (!external && d->budget_bytes && (uint64_t)nb * per_block > d->budget_bytes)
      return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: " + std::to_string(nb) + " blocks need " +
                                                 std::to_string((uint64_t)nb * per_block) + " bytes, over the budget of " +
                                                 std::to_string(d->budget_bytes));
  }
  B200KvPool* p = new (std::nothrow) B200KvPool;
  if (!p) return fail(B200_ERR_FAIL, "KV pool: out of host memory");
  p->desc = *d;
  p->num_blocks = (int32_t)nb;
  p->block_bytes = block;
  if (external) {
    p->key_cache = d->key_cache;
    p->value_cache = d->value_cache;
    p->k_scale = d->k_scale;
    p->v_scale = d->v_scale;
  } else {
    DeviceScope scope(d->device);
    if (scope.err != cudaSuccess) {
      delete p;
      return cuda_fail(scope.err, "KV pool: cudaSetDevice");
    }
    const uint64_t cache_bytes = block * (uint64_t)nb;
    cudaError_t e = cudaMalloc(&p->key_cache, cache_bytes);
    if (e == cudaSuccess) e = cudaMalloc(&p->value_cache, cache_bytes);
    if (e == cudaSuccess) e = cudaMemset(p->key_cache, 0, cache_bytes);
    if (e == cudaSuccess) e = cudaMemset(p->value_cache, 0, cache_bytes);
    if (e == cudaSuccess && fp8) {
      const size_t n = (size_t)nb * d->kv_num_heads;
      e = cudaMalloc(reinterpret_cast<void**>(&p->k_scale), n * sizeof(float));
      if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&p->v_scale), n * sizeof(float));
      if (e == cudaSuccess) {  // unit scales until the owner of a block sets its own
        std::vector<float> ones(n, 1.0f);
        e = cudaMemcpy(p->k_scale, ones.data(), n * sizeof(float), cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(p->v_scale, ones.data(), n * sizeof(float), cudaMemcpyHostToDevice);
      }
    }
    if (e != cudaSuccess) {
      cudaFree(p->key_cache);
      cudaFree(p->value_cache);
      cudaFree(p->k_scale);
      cudaFree(p->v_scale);
      delete p;
      return cuda_fail(e, "KV pool: allocating " + std::to_string(nb) + " blocks on device " + std::to_string(d->device));
    }
    p->owns = true;
    p->allocated = 2 * cache_bytes + (fp8 ? 2ull * (uint64_t)nb * d->kv_num_heads * sizeof(float) : 0);
  }
  p->free_stack.resize((size_t)nb);
  for (int64_t i = 0; i < nb; ++i) p->free_stack[(size_t)i] = (int32_t)(nb - 1 - i);
  p->in_use.assign((size_t)nb, 0);
  *out = p;
  return B200_OK;
}

int b200_kv_pool_destroy(B200KvPool* p) {
  if (!p) return B200_OK;
  cudaError_t e = cudaSuccess;
  if (p->owns) {
    DeviceScope scope(p->desc.device);
    for (void* ptr : {p->key_cache, p->value_cache, static_cast<void*>(p->k_scale), static_cast<void*>(p->v_scale)}) {
      if (!ptr) continue;
      cudaError_t r = cudaFree(ptr);
      if (e == cudaSuccess) e = r;
    }
  }
  delete p;
  return e == cudaSuccess ? B200_OK : cuda_fail(e, "KV pool: cudaFree");
}

int b200_kv_pool_info(const B200KvPool* p, B200KvPoolInfo* info) {
  if (!p || !info) return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: null argument");
  B200KvPool* m = const_cast<B200KvPool*>(p);
  std::lock_guard<std::mutex> lock(m->mu);
  info->key_cache = p->key_cache;
  info->value_cache = p->value_cache;
  info->k_scale = p->k_scale;
  info->v_scale = p->v_scale;
  info->num_blocks = p->num_blocks;
  info->free_blocks = (int32_t)p->free_stack.size();
  info->block_size = p->desc.block_size;
  info->owns_memory = p->owns ? 1 : 0;
  info->block_bytes = p->block_bytes;
  info->allocated_bytes = p->allocated;
  return B200_OK;
}

int b200_kv_pool_alloc(B200KvPool* p, int32_t count, int32_t* ids) {
  if (!p || count < 0 || (count && !ids)) return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: bad alloc arguments");
  std::lock_guard<std::mutex> lock(p->mu);
  if ((size_t)count > p->free_stack.size())
    return fail(B200_ERR_FAIL, "KV pool: out of KV cache blocks (" + std::to_string(count) + " requested, " +
                                   std::to_string(p->free_stack.size()) + " of " + std::to_string(p->num_blocks) +
                                   " free); raise ep.b200.kv_pool_bytes or free finished sequences");
  for (int32_t i = 0; i < count; ++i) {
    const int32_t id = p->free_stack.back();
    p->free_stack.pop_back();
    p->in_use[(size_t)id] = 1;
    ids[i] = id;
  }
  return B200_OK;
}

int b200_kv_pool_free(B200KvPool* p, const int32_t* ids, int32_t count) {
  if (!p || count < 0 || (count && !ids)) return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: bad free arguments");
  std::lock_guard<std::mutex> lock(p->mu);
  // validate everything first so a bad call changes nothing
  std::vector<uint8_t> seen;
  for (int32_t i = 0; i < count; ++i) {
    const int32_t id = ids[i];
    if (id < 0 || id >= p->num_blocks)
      return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: block id " + std::to_string(id) + " is outside [0, " +
                                                 std::to_string(p->num_blocks) + ")");
    if (!p->in_use[(size_t)id])
      return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: block " + std::to_string(id) + " is not allocated (double free?)");
    if (seen.empty()) seen.assign((size_t)p->num_blocks, 0);
    if (seen[(size_t)id]) return fail(B200_ERR_INVALID_ARGUMENT, "KV pool: block " + std::to_string(id) + " freed twice in one call");
    seen[(size_t)id] = 1;
  }
  for (int32_t i = 0; i < count; ++i) {
    p->in_use[(size_t)ids[i]] = 0;
    p->free_stack.push_back(ids[i]);
  }
  return B200_OK;
}

int32_t b200_kv_pool_blocks_for(const B200KvPool* p, int64_t tokens) {
  if (!p || tokens <= 0) return 0;
  const int64_t bs = p->desc.block_size;
  const int64_t n = (tokens + bs - 1) / bs;
  return n > INT32_MAX ? INT32_MAX : (int32_t)n;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// compiled-node launcher
// ---------------------------------------------------------------------------------------------
struct B200EpNode {
  enum Kind { kPaged, kGqa } kind;
  std::mutex gate;  // one compute at a time per node
  B200EpOptions options{};
  B200NodeInfo paged{};
  B200GqaNodeInfo gqa{};
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  uint64_t computes = 0;
};

namespace {

std::string fixed_str(const char* s, size_t n) { return std::string(s, strnlen(s, n)); }

// Grow the node's workspace to `need` bytes (the old buffer is released first; cudaFree waits
// for the device, so no earlier kernel still uses it).
int ensure_workspace(B200EpNode* n, size_t need) {
  if (n->workspace && n->workspace_bytes >= need) return B200_OK;
  if (n->workspace) {
    cudaError_t e = cudaFree(n->workspace);
    n->workspace = nullptr;
    n->workspace_bytes = 0;
    if (e != cudaSuccess) return cuda_fail(e, "EP node: freeing the workspace");
  }
  const size_t bytes = need < ((size_t)1 << 20) ? ((size_t)1 << 20) : need;
  cudaError_t e = cudaMalloc(&n->workspace, bytes);
  if (e != cudaSuccess) {
    n->workspace = nullptr;
    return cuda_fail(e, "EP node: allocating a " + std::to_string(bytes) + "-byte workspace");
  }
  n->workspace_bytes = bytes;
  return B200_OK;
}

int make_node(B200EpNode::Kind kind, const B200EpOptions* options, B200EpNode** out) {
  B200EpNode* n = new (std::nothrow) B200EpNode;
  if (!n) return fail(B200_ERR_FAIL, "EP node: out of host memory");
  n->kind = kind;
  if (options) {
    n->options = *options;
  } else {
    int rc = b200_ep_options_parse(nullptr, nullptr, 0, &n->options);
    if (rc) {
      delete n;
      return rc;
    }
  }
  *out = n;
  return B200_OK;
}

}  // namespace

extern "C" {

int b200_ep_node_create_paged(const B200NodeInfo* node, const B200EpOptions* options, B200EpNode** out) {
  if (!node || !out) return fail(B200_ERR_INVALID_ARGUMENT, "EP node: null argument");
  *out = nullptr;
  char reason[512];
  if (!b200_paged_attention_claim(node, reason, sizeof reason))
    return fail(B200_ERR_UNSUPPORTED, std::string("PagedAttention not claimed: ") + reason);
  B200EpNode* n = nullptr;
  int rc = make_node(B200EpNode::kPaged, options, &n);
  if (rc) return rc;
  n->paged = *node;
  *out = n;
  return B200_OK;
}

int b200_ep_node_create_gqa(const B200GqaNodeInfo* node, const B200EpOptions* options, B200EpNode** out) {
  if (!node || !out) return fail(B200_ERR_INVALID_ARGUMENT, "EP node: null argument");
  *out = nullptr;
  char reason[512];
  if (!b200_group_query_attention_claim(node, reason, sizeof reason))
    return fail(B200_ERR_UNSUPPORTED, std::string("GroupQueryAttention not claimed: ") + reason);
  B200EpNode* n = nullptr;
  int rc = make_node(B200EpNode::kGqa, options, &n);
  if (rc) return rc;
  n->gqa = *node;
  *out = n;
  return B200_OK;
}

int b200_ep_node_destroy(B200EpNode* n) {
  if (!n) return B200_OK;
  cudaError_t e = cudaSuccess;
  if (n->workspace) {
    DeviceScope scope(n->options.device_id);
    e = cudaFree(n->workspace);
  }
  delete n;
  return e == cudaSuccess ? B200_OK : cuda_fail(e, "EP node: freeing the workspace");
}

int b200_ep_node_stats(const B200EpNode* n, uint64_t* workspace_bytes, uint64_t* computes) {
  if (!n) return fail(B200_ERR_INVALID_ARGUMENT, "EP node: null node");
  B200EpNode* m = const_cast<B200EpNode*>(n);
  std::lock_guard<std::mutex> lock(m->gate);
  if (workspace_bytes) *workspace_bytes = n->workspace_bytes;
  if (computes) *computes = n->computes;
  return B200_OK;
}

int b200_ep_node_compute_paged(B200EpNode* n, const B200PagedTensors* t, void* stream) {
  if (!n || !t) return fail(B200_ERR_INVALID_ARGUMENT, "EP node: null argument");
  if (n->kind != B200EpNode::kPaged) return fail(B200_ERR_INVALID_ARGUMENT, "EP node: not a PagedAttention node");
  std::lock_guard<std::mutex> lock(n->gate);
  try {
    DeviceScope scope(n->options.device_id);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "EP node: cudaSetDevice");
    const B200NodeInfo& a = n->paged;
    B200PagedAttentionParams p{};
    const int H = (int)a.num_heads, KV = (int)a.kv_num_heads;
    const bool latent = fixed_str(a.kv_cache_layout, sizeof a.kv_cache_layout) == "LATENT";
    const bool packed = !latent && !t->key && !t->value;
    p.kv_cache_latent = latent;
    p.v_head_size = latent ? (int32_t)a.v_head_size : 0;
    p.num_heads = H;
    p.kv_num_heads = KV;
    const int heads_in_query = packed ? H + 2 * KV : H;
    if (t->query_hidden <= 0 || t->query_hidden % heads_in_query)
      return fail(B200_ERR_INVALID_ARGUMENT, "PagedAttention: query hidden size does not match the head count");
    p.head_size = t->query_hidden / heads_in_query;
    p.scale = a.has_scale ? a.scale : 0.f;
    p.is_causal = (int32_t)a.is_causal;
    p.local_window_size = (int32_t)a.local_window_size;
    p.softcap = a.softcap;
    p.do_rotary = (int32_t)a.do_rotary;
    p.rotary_interleaved = (int32_t)a.rotary_interleaved;
    p.rotary_offset = (int32_t)a.rotary_offset;
    p.rotary_dim = 2 * t->rotary_half_dim;
    p.rotary_positions = t->rotary_positions;
    p.qk_norm_epsilon = a.qk_norm_epsilon > 0.f ? a.qk_norm_epsilon : 1e-6f;
    p.act_dtype = t->act_dtype;
    p.cache_dtype = t->cache_dtype;
    p.k_quant_per_channel = fixed_str(a.k_quant_type, sizeof a.k_quant_type) == "PER_CHANNEL";
    p.v_quant_per_channel = fixed_str(a.v_quant_type, sizeof a.v_quant_type) == "PER_CHANNEL";
    p.num_tokens = t->num_tokens;
    p.batch = t->batch;
    p.num_blocks = t->num_blocks;
    p.block_size = t->block_size;
    p.max_blocks_per_seq = t->max_blocks_per_seq;
    p.query = t->query;
    if (packed) {  // K and V columns of the packed rows (attention.rs:3877-3890)
      const size_t esz = 2;
      p.query_row_stride = p.key_row_stride = p.value_row_stride = t->query_hidden;
      p.key = static_cast<const char*>(t->query) + (size_t)H * p.head_size * esz;
      p.value = static_cast<const char*>(t->query) + (size_t)(H + KV) * p.head_size * esz;
    } else {
      p.key = t->key;
      p.value = t->value;
    }
    p.key_cache = t->key_cache;
    p.value_cache = t->value_cache;
    p.cumulative_sequence_length = t->cumulative_sequence_length;
    p.past_seqlens = t->past_seqlens;
    p.block_table = t->block_table;
    p.cos_cache = t->cos_cache;
    p.sin_cache = t->sin_cache;
    p.slot_mapping = t->slot_mapping;
    p.head_sink = t->head_sink;
    p.q_norm_weight = t->q_norm_weight;
    p.k_norm_weight = t->k_norm_weight;
    p.k_scale = t->k_scale;
    p.v_scale = t->v_scale;
    p.output = t->output;
    p.host_cumulative_sequence_length = t->host_cumulative_sequence_length;
    p.host_past_seqlens = t->host_past_seqlens;
    p.host_block_table = t->host_block_table;
    p.host_slot_mapping = t->host_slot_mapping;
    p.decode_min_tiles_per_warp = n->options.decode_min_tiles_per_warp;
    p.force_generic = n->options.force_generic;
    size_t need = 0;
    int rc = b200_paged_attention_workspace_size(&p, &need);
    if (rc) return rc;
    if ((rc = ensure_workspace(n, need))) return rc;
    p.workspace = n->workspace;
    p.workspace_bytes = n->workspace_bytes;
    rc = b200_paged_attention(&p, stream);
    if (rc) return rc;
    ++n->computes;
    if (n->options.check_status) return b200_read_status(&p, stream);
    return B200_OK;
  } catch (const std::exception& ex) {
    return fail(B200_ERR_FAIL, std::string("EP node: ") + ex.what());
  } catch (...) {
    return fail(B200_ERR_FAIL, "EP node: unknown failure");
  }
}

int b200_ep_node_compute_gqa(B200EpNode* n, const B200GqaParams* t, void* stream) {
  if (!n || !t) return fail(B200_ERR_INVALID_ARGUMENT, "EP node: null argument");
  if (n->kind != B200EpNode::kGqa) return fail(B200_ERR_INVALID_ARGUMENT, "EP node: not a GroupQueryAttention node");
  std::lock_guard<std::mutex> lock(n->gate);
  try {
    DeviceScope scope(n->options.device_id);
    if (scope.err != cudaSuccess) return cuda_fail(scope.err, "EP node: cudaSetDevice");
    const B200GqaNodeInfo& a = n->gqa;
    B200GqaParams p = *t;
    p.num_heads = (int32_t)a.num_heads;
    p.kv_num_heads = (int32_t)a.kv_num_heads;
    p.scale = a.has_scale ? a.scale : 0.f;
    p.is_causal = a.has_causal ? (int32_t)a.causal : 1;
    p.local_window_size = a.has_local_window_size ? (int32_t)a.local_window_size : -1;
    p.softcap = a.softcap;
    p.smooth_softmax = (a.has_smooth_softmax && a.smooth_softmax == 1) ? 1 : 0;
    p.do_rotary = a.do_rotary != 0;  // the tensors carry cos / sin / position_ids and their sizes
    p.rotary_interleaved = a.rotary_interleaved != 0;
    p.qk_norm_epsilon = a.has_qk_norm_epsilon ? a.qk_norm_epsilon : 1e-6f;  // the tensors carry the weights
    p.qk_output = (int32_t)a.qk_output;  // the tensors carry output_qk
    p.k_quant_per_channel = fixed_str(a.k_quant_type, sizeof a.k_quant_type) == "PER_CHANNEL";
    p.v_quant_per_channel = fixed_str(a.v_quant_type, sizeof a.v_quant_type) == "PER_CHANNEL";
    p.sliding_window_cache = a.sliding_window_cache != 0;
    size_t need = 0;
    int rc = b200_group_query_attention_workspace_size(&p, &need);
    if (rc) return rc;
    if ((rc = ensure_workspace(n, need))) return rc;
    p.workspace = n->workspace;
    p.workspace_bytes = n->workspace_bytes;
    rc = b200_group_query_attention(&p, stream);
    if (rc) return rc;
    ++n->computes;
    if (n->options.check_status) return b200_group_query_attention_read_status(&p, stream);
    return B200_OK;
  } catch (const std::exception& ex) {
    return fail(B200_ERR_FAIL, std::string("EP node: ") + ex.what());
  } catch (...) {
    return fail(B200_ERR_FAIL, "EP node: unknown failure");
  }
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// device memory, copies and streams for the ORT glue
// ---------------------------------------------------------------------------------------------
extern "C" {

int b200_ep_device_alloc(int32_t device, size_t bytes, void** out) {
  if (!out) return fail(B200_ERR_INVALID_ARGUMENT, "B200 allocator: null output");
  *out = nullptr;
  DeviceScope scope(device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "B200 allocator: cudaSetDevice");
  if (bytes == 0) return B200_OK;
  cudaError_t e = cudaMalloc(out, bytes);
  if (e != cudaSuccess) {
    *out = nullptr;
    return cuda_fail(e, "B200 allocator: cudaMalloc of " + std::to_string(bytes) + " bytes");
  }
  return B200_OK;
}

int b200_ep_device_free(int32_t device, void* ptr) {
  if (!ptr) return B200_OK;
  DeviceScope scope(device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "B200 allocator: cudaSetDevice");
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? B200_OK : cuda_fail(e, "B200 allocator: cudaFree");
}

int b200_ep_copy(int32_t device, void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return B200_OK;
  if (!dst || !src) return fail(B200_ERR_INVALID_ARGUMENT, "B200 copy: null pointer");
  DeviceScope scope(device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "B200 copy: cudaSetDevice");
  cudaError_t e = stream ? cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream))
                         : cudaMemcpy(dst, src, bytes, cudaMemcpyDefault);
  return e == cudaSuccess ? B200_OK : cuda_fail(e, "B200 copy of " + std::to_string(bytes) + " bytes");
}

int b200_ep_is_device_pointer(const void* ptr, int32_t* out) {
  if (!out) return fail(B200_ERR_INVALID_ARGUMENT, "B200: null output");
  *out = 0;
  if (!ptr) return B200_OK;
  cudaPointerAttributes attr{};
  cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();  // plain host memory on old runtimes; not sticky
    return B200_OK;
  }
  *out = attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
  return B200_OK;
}

int b200_ep_stream_create(int32_t device, void** stream) {
  if (!stream) return fail(B200_ERR_INVALID_ARGUMENT, "B200: null output");
  *stream = nullptr;
  DeviceScope scope(device);
  if (scope.err != cudaSuccess) return cuda_fail(scope.err, "B200 stream: cudaSetDevice");
  cudaStream_t s = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return cuda_fail(e, "B200 stream: cudaStreamCreateWithFlags");
  *stream = s;
  return B200_OK;
}

int b200_ep_stream_sync(void* stream) {
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? B200_OK : cuda_fail(e, "B200 stream: cudaStreamSynchronize");
}

int b200_ep_stream_destroy(int32_t device, void* stream) {
  if (!stream) return B200_OK;
  DeviceScope scope(device);
  cudaError_t e = cudaStreamDestroy(static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? B200_OK : cuda_fail(e, "B200 stream: cudaStreamDestroy");
}

}  // extern "C"
