/*
 * b200_ep.h - host layer of the B200 plugin execution provider, below ONNX Runtime's own types.
 *
 * The reference EP (onnxruntime-ep-mlx, rust/src) has three host pieces around its kernels:
 *   - strict ep.* session options, session value first, then the environment
 *     (rust/src/config.rs:18-64, rust/src/memory.rs:10-98);
 *   - a compiled-node launcher: one state per fused node, a run gate that serialises calls,
 *     inputs read from the kernel context, failures turned into an OrtStatus
 *     (rust/src/runtime.rs:93-331, rust/src/lib.rs:53-92);
 *   - device memory for the EP's tensors, bounded by budgets (rust/src/device.rs:409-493 for the
 *     allocator, rust/src/memory.rs:26-98 for the MLX cache budgets).
 * This header restates them on plain C types, so everything except the thin OrtEpFactory / OrtEp
 * glue (which needs ONNX Runtime's headers) builds and is tested without ONNX Runtime.  All entry
 * points return a B200_* status (b200_paged.h) and leave a message in b200_last_error().
 */
#ifndef B200_EP_H
#define B200_EP_H

#include <stddef.h>
#include <stdint.h>

#include "b200_paged.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- session options ---------------------------------------------------------------------
 * Keys (session config entry, then environment variable; a session value wins):
 *   ep.b200.kv_pool_bytes             ONNXRUNTIME_EP_B200_KV_POOL_BYTES   decimal byte count
 *   ep.b200.num_gpus                  ONNXRUNTIME_EP_B200_NUM_GPUS        decimal, >= 1
 *   ep.b200.device_id                 ONNXRUNTIME_EP_B200_DEVICE_ID       decimal, >= 0
 *   ep.b200.decode_min_tiles_per_warp ONNXRUNTIME_EP_B200_DECODE_MIN_TILES decimal, >= 1
 *   ep.b200.force_generic             ONNXRUNTIME_EP_B200_FORCE_GENERIC   "0" or "1"
 *   ep.b200.check_status              ONNXRUNTIME_EP_B200_CHECK_STATUS    "0" or "1" (default 1:
 *                                     each compute synchronises and reports device-side errors,
 *                                     as the reference reports them on the host)
 * Values are parsed strictly (config.rs:46-52: booleans are exactly "0" or "1"; memory.rs:10-17:
 * byte counts are non-empty ASCII digits that fit in 64 bits).  Other keys are ignored, as ORT
 * keeps unrelated entries in the same table. */
typedef struct B200EpOptions {
  uint64_t kv_pool_bytes;            /* 0 = no pool budget set                                */
  int32_t has_kv_pool_bytes;
  int32_t num_gpus;                  /* default 1                                             */
  int32_t device_id;                 /* default 0                                             */
  int32_t decode_min_tiles_per_warp; /* 0 = kernel default                                    */
  int32_t force_generic;             /* default 0                                             */
  int32_t check_status;              /* default 1                                             */
} B200EpOptions;

/* Parse `count` session entries (keys[i] = values[i]; either array may be NULL when count is 0),
 * then fill what the session left unset from the environment.  B200_ERR_INVALID_ARGUMENT with a
 * message naming the key on a malformed value. */
B200_API int b200_ep_options_parse(const char* const* keys, const char* const* values, size_t count,
                                   B200EpOptions* out);

/* ---- error classes for the ORT glue --------------------------------------------------------
 * ORT distinguishes bad arguments (ORT_INVALID_ARGUMENT) from EP failures (ORT_EP_FAIL)
 * (rust/src/config.rs:14, rust/src/runtime.rs:316-327).  The glue maps these classes onto the
 * OrtErrorCode values of the ONNX Runtime headers it is compiled against. */
#define B200_ORT_OK 0
#define B200_ORT_INVALID_ARGUMENT 1
#define B200_ORT_EP_FAIL 2
B200_API int b200_ort_error_class(int b200_status);

/* ---- KV block pool ---------------------------------------------------------------------------
 * Paged K and V caches [num_blocks, block_size, kv_num_heads, head_size] on one device, and the
 * free list of their block ids.  Created from a byte budget (the pool allocates both caches, and
 * the per-(block, kv head) scales of an fp8 pool, once, with cudaMalloc on `device`), or over
 * caches the caller already owns (no allocation; e.g. the key_cache / value_cache tensors ORT
 * binds to a session).  Block ids go straight into block tables.  Thread-safe. */
typedef struct B200KvPoolDesc {
  int32_t device;          /* CUDA device of the caches                                       */
  int32_t block_size;      /* slots per block                                                 */
  int32_t kv_num_heads;
  int32_t head_size;
  int32_t cache_dtype;     /* B200_DTYPE_FLOAT16 / BFLOAT16 / INT8 / UINT8 (int4) / FLOAT8E4M3FN */
  int32_t num_blocks;      /* 0 = as many as budget_bytes holds                               */
  uint64_t budget_bytes;   /* byte budget of everything the pool allocates                    */
  void* key_cache;         /* caller-owned caches (both or neither); NULL = allocate          */
  void* value_cache;
  float* k_scale;          /* caller-owned fp8 scales [num_blocks, kv_num_heads] (fp8 only)    */
  float* v_scale;
} B200KvPoolDesc;

typedef struct B200KvPoolInfo {
  void* key_cache;
  void* value_cache;
  float* k_scale;          /* fp8 pools: [num_blocks, kv_num_heads] fp32, else NULL           */
  float* v_scale;
  int32_t num_blocks;
  int32_t free_blocks;
  int32_t block_size;
  int32_t owns_memory;     /* 1 when the pool allocated the caches                            */
  uint64_t block_bytes;    /* bytes of one block of one cache (scales not included)           */
  uint64_t allocated_bytes;/* device bytes the pool allocated                                 */
} B200KvPoolInfo;

typedef struct B200KvPool B200KvPool;

/* Bytes of one block of one cache for this geometry (int4: ceil(head_size / 2) per row). */
B200_API int b200_kv_pool_block_bytes(const B200KvPoolDesc* desc, uint64_t* bytes);
B200_API int b200_kv_pool_create(const B200KvPoolDesc* desc, B200KvPool** out);
/* Frees what the pool allocated (nothing for caller-owned caches).  NULL is a no-op. */
B200_API int b200_kv_pool_destroy(B200KvPool* pool);
B200_API int b200_kv_pool_info(const B200KvPool* pool, B200KvPoolInfo* info);
/* Take `count` free blocks, all or nothing, lowest ids first after a reset; ids are written to
 * block_ids[0..count).  B200_ERR_FAIL ("out of KV cache blocks") when fewer are free. */
B200_API int b200_kv_pool_alloc(B200KvPool* pool, int32_t count, int32_t* block_ids);
/* Return blocks.  Checks every id first (range, currently allocated, no repeats) and frees none
 * on an error, so a bad call leaves the pool unchanged. */
B200_API int b200_kv_pool_free(B200KvPool* pool, const int32_t* block_ids, int32_t count);
/* Blocks needed to hold `tokens` slots. */
B200_API int32_t b200_kv_pool_blocks_for(const B200KvPool* pool, int64_t tokens);

/* ---- compiled-node launcher ------------------------------------------------------------------
 * One state per claimed node: the node's attributes, the session options, a device workspace
 * kept across calls (grown on demand, freed with the node), and a run gate.  Compute takes only
 * the node's tensors (pointers and the runtime sizes ORT reports), fills the kernel parameters,
 * runs the kernels and, with check_status, synchronises the stream and reports device-side
 * errors.  Calls on one node are serialised by its gate; any thread may call (CUDA work is not
 * thread-affine, unlike the MLX evaluation behind the reference's single-owner gate,
 * runtime.rs:126-169). */
typedef struct B200EpNode B200EpNode;

/* Create the state of a PagedAttention node.  Declined forms (the claim predicate's reasons)
 * return B200_ERR_UNSUPPORTED with the reason in b200_last_error(). */
B200_API int b200_ep_node_create_paged(const B200NodeInfo* node, const B200EpOptions* options, B200EpNode** out);
/* Create the state of a GroupQueryAttention node (claim: b200_group_query_attention_claim). */
B200_API int b200_ep_node_create_gqa(const B200GqaNodeInfo* node, const B200EpOptions* options, B200EpNode** out);
B200_API int b200_ep_node_destroy(B200EpNode* node);

/* The tensors of one PagedAttention Compute, in the node's input order (absent optional inputs
 * are NULL) with the sizes ORT reports for them.  Host copies of the int32 metadata enable the
 * reference's host validation (the reference reads these inputs on the host). */
typedef struct B200PagedTensors {
  const void* query;            /* [num_tokens, query_hidden]                                  */
  const void* key;              /* [num_tokens, kv_num_heads * head_size] or NULL (packed QKV) */
  const void* value;
  void* key_cache;              /* [num_blocks, block_size, kv_num_heads, head_size']          */
  void* value_cache;
  const int32_t* cumulative_sequence_length; /* [batch + 1]                                    */
  const int32_t* past_seqlens;  /* [batch]                                                     */
  const int32_t* block_table;   /* [batch, max_blocks_per_seq]                                 */
  const void* cos_cache;        /* [rotary_positions, rotary_dim / 2]                          */
  const void* sin_cache;
  const int32_t* slot_mapping;  /* [num_tokens] or NULL                                        */
  const void* head_sink;
  const void* q_norm_weight;
  const void* k_norm_weight;
  const float* k_scale;
  const float* v_scale;
  void* output;                 /* [num_tokens, num_heads * head_size]                         */
  const int32_t* host_cumulative_sequence_length;
  const int32_t* host_past_seqlens;
  const int32_t* host_block_table;
  const int32_t* host_slot_mapping;
  int32_t num_tokens;
  int32_t query_hidden;         /* query.shape[1]                                              */
  int32_t batch;
  int32_t num_blocks;
  int32_t block_size;
  int32_t max_blocks_per_seq;
  int32_t rotary_positions;     /* cos_cache.shape[0]                                          */
  int32_t rotary_half_dim;      /* cos_cache.shape[1]                                          */
  int32_t act_dtype;            /* query element type                                          */
  int32_t cache_dtype;          /* key_cache element type                                      */
} B200PagedTensors;

B200_API int b200_ep_node_compute_paged(B200EpNode* node, const B200PagedTensors* tensors, void* stream);

/* The tensors of one GroupQueryAttention Compute: B200GqaParams with the node's attribute fields
 * (heads, scale, causal, window, softcap, smooth_softmax, do_rotary, rotary_interleaved) ignored,
 * as the node supplies them, and the workspace fields ignored (the node owns one). */
B200_API int b200_ep_node_compute_gqa(B200EpNode* node, const B200GqaParams* tensors, void* stream);

/* sizeof the structs above as compiled into the library, for binding layout checks:
 * 0 B200EpOptions, 1 B200KvPoolDesc, 2 B200KvPoolInfo, 3 B200PagedTensors (0 otherwise). */
B200_API size_t b200_ep_struct_size(int32_t which);

/* Bytes of device workspace the node currently holds, and computes run so far. */
B200_API int b200_ep_node_stats(const B200EpNode* node, uint64_t* workspace_bytes, uint64_t* computes);

/* ---- device memory, copies and streams for the ORT glue ---------------------------------------
 * What the EP's OrtAllocator, OrtDataTransferImpl and Compute need from CUDA, so the glue itself
 * is compiled against ONNX Runtime's headers alone (the reference's allocator and transfer are
 * rust/src/device.rs:409-640).  `device` is the CUDA ordinal. */
B200_API int b200_ep_device_alloc(int32_t device, size_t bytes, void** out);
B200_API int b200_ep_device_free(int32_t device, void* ptr);
/* Copy `bytes` between any two of host and device memory (the direction is read from the
 * pointers).  stream NULL: synchronous; otherwise ordered on `stream`. */
B200_API int b200_ep_copy(int32_t device, void* dst, const void* src, size_t bytes, void* stream);
/* *out = 1 when the kernels can read `ptr` directly (device or managed memory), else 0. */
B200_API int b200_ep_is_device_pointer(const void* ptr, int32_t* out);
/* A non-blocking stream on `device`; synchronise; destroy (NULL is a no-op). */
B200_API int b200_ep_stream_create(int32_t device, void** stream);
B200_API int b200_ep_stream_sync(void* stream);
B200_API int b200_ep_stream_destroy(int32_t device, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_EP_H */
