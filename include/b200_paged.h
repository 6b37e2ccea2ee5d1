/*
 * b200_paged.h - C ABI of the B200-native paged-KV attention path.
 *
 * This library replaces the KV-cache attention hot path of the onnxruntime-ep-mlx plugin
 * execution provider (reference: rust/src/ops/attention.rs, rust/src/ops/paged_attention.rs,
 * rust/src/ops/kv_cache.rs) with hand-written sm_100a CUDA kernels.  Every entry point takes
 * plain pointers and sizes, returns a B200_* status code and never throws; a failing call
 * leaves a human-readable message in b200_last_error() (thread local).
 *
 * Device pointers are CUDA device addresses on the current device; `stream` is a
 * cudaStream_t passed as void*.  Host pointers are marked host_*.
 */
#ifndef B200_PAGED_H
#define B200_PAGED_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define B200_API __attribute__((visibility("default")))
#else
#define B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (map to OrtErrorCode in the EP shell) ---------------------------- */
#define B200_OK 0
#define B200_ERR_INVALID_ARGUMENT 1 /* bad attributes / shapes: ORT_INVALID_ARGUMENT */
#define B200_ERR_FAIL 2             /* invalid runtime metadata: ORT_EP_FAIL          */
#define B200_ERR_CUDA 3             /* a CUDA runtime call failed                     */
#define B200_ERR_UNSUPPORTED 4      /* form the kernels do not implement              */
#define B200_ERR_WORKSPACE 5        /* workspace missing or too small                 */
#define B200_ERR_DEVICE 6           /* device-side check failed (see message)         */

/* ---- element types: ONNX TensorProto.DataType values -------------------------------- */
#define B200_DTYPE_FLOAT 1
#define B200_DTYPE_UINT8 2 /* int4 cache: two +8-biased nibbles per byte */
#define B200_DTYPE_INT8 3
#define B200_DTYPE_INT32 6
#define B200_DTYPE_INT64 7
#define B200_DTYPE_FLOAT16 10
#define B200_DTYPE_BFLOAT16 16
#define B200_DTYPE_FLOAT8E4M3FN 17

/*
 * One com.microsoft.PagedAttention call.  Field meanings follow the operator's inputs,
 * outputs and attributes (reference claim rust/src/ops/attention.rs:4384-4645, op
 * :3857-4382).  Zero-initialise and fill what is present.
 */
/* Largest head_size the kernels take (head sizes above 256 and LATENT layouts run on the generic
 * kernel; the fast decode and prefill kernels cover 64 / 128 / 256 and 128). */
#define B200_MAX_HEAD_SIZE 640
/* Shared memory the append prologue may stage per token when it rotates / normalises rows or
 * encodes an integer or fp8 cache: 4 bytes x head_size x (num_heads + 2 kv_num_heads). */
#define B200_MAX_PROLOGUE_STAGE_BYTES (227 * 1024)

typedef struct B200PagedAttentionParams {
  /* attributes */
  int32_t num_heads;          /* H                                                        */
  int32_t kv_num_heads;       /* KV, H % KV == 0                                          */
  int32_t head_size;          /* d (query hidden / H, or packed hidden / (H + 2 KV))      */
  float scale;                /* 0 -> 1/sqrt(d) (attention.rs:448-453)                    */
  int32_t is_causal;          /* operator default is 1: callers set it from the attribute */
  int32_t local_window_size;  /* -1 or 0 = no window, > 0 = left window                   */
  float softcap;              /* 0 = off                                                  */
  int32_t do_rotary;          /* RoPE on new Q/K at positions [past, past + n)            */
  int32_t rotary_interleaved;
  int32_t rotary_offset;      /* first rotated channel, multiple of 8                     */
  int32_t rotary_dim;         /* 2 * cos_cache.shape[1]                                   */
  int32_t rotary_positions;   /* cos_cache.shape[0]                                       */
  float qk_norm_epsilon;      /* used when q_norm_weight is set (1e-6 default)            */
  int32_t act_dtype;          /* FLOAT16 or BFLOAT16 (T)                                  */
  int32_t cache_dtype;        /* T, INT8, UINT8 (int4) or FLOAT8E4M3FN                    */
  int32_t k_quant_per_channel;/* int caches: 0 PER_TENSOR, 1 PER_CHANNEL                  */
  int32_t v_quant_per_channel;

  /* geometry */
  int32_t num_tokens;         /* nt: packed new tokens                                    */
  int32_t batch;              /* B: sequences, cumulative_sequence_length has B + 1       */
  int32_t num_blocks;         /* NB                                                       */
  int32_t block_size;         /* bs                                                       */
  int32_t max_blocks_per_seq; /* block_table is [B, max_blocks_per_seq]                   */
  int64_t query_row_stride;   /* elements between tokens; 0 -> H*d (packed: (H+2KV)*d)   */
  int64_t key_row_stride;     /* 0 -> KV*d                                                */
  int64_t value_row_stride;   /* 0 -> KV*d                                                */

  /* device tensors (inputs 0-15, output 0; caches are updated in place) */
  const void* query;          /* [nt, H*d] (packed: [nt, (H+2KV)*d])                      */
  const void* key;            /* [nt, KV*d]; packed: query + H*d                          */
  const void* value;          /* [nt, KV*d]; packed: query + (H+KV)*d                     */
  void* key_cache;            /* [NB, bs, KV, d] (int4: ceil(d/2) bytes)                  */
  void* value_cache;          /* [NB, bs, KV, d]                                          */
  const int32_t* cumulative_sequence_length; /* [B + 1]                                   */
  const int32_t* past_seqlens;               /* [B]                                       */
  const int32_t* block_table;                /* [B, max_blocks_per_seq]                   */
  const void* cos_cache;      /* [rotary_positions, rotary_dim/2] in T                    */
  const void* sin_cache;
  const int32_t* slot_mapping;/* [nt] or NULL; -1 skips the write                         */
  const void* head_sink;      /* [H] in T or NULL                                         */
  const void* q_norm_weight;  /* [d] in T or NULL (k_norm_weight set together)            */
  const void* k_norm_weight;
  const float* k_scale;       /* int caches: [1] or [KV*d]; fp8: [NB, KV] per block/head  */
  const float* v_scale;
  void* output;               /* [nt, H*d] in T                                           */

  /* optional host copies of the metadata: enable the reference's host validation
   * (attention.rs:3934-3990) before any launch, and skip device-side duplicate-slot work
   * when the host proves slots unique */
  const int32_t* host_cumulative_sequence_length;
  const int32_t* host_past_seqlens;
  const int32_t* host_block_table;
  const int32_t* host_slot_mapping;

  /* scratch */
  void* workspace;            /* device, >= b200_paged_attention_workspace_size()         */
  size_t workspace_bytes;
  int32_t* device_status;     /* optional device int32; NULL -> a word in the workspace   */

  /* tuning (session options ep.b200.*) */
  int32_t decode_min_tiles_per_warp; /* decode stream-K: smallest 16-token tile range a warp
                                      * of the persistent grid takes (0 -> 4)              */
  int32_t force_generic;          /* 1 -> run the generic kernel for every sequence       */
  int32_t num_sms;                /* 0 -> query the device                                */

  /* optional cudaEvent_t handles recorded on `stream` right before the first and right after
   * the last attention kernel of the call (decode + combine + prefill), for live timing */
  void* attention_event_begin;
  void* attention_event_end;

  /* kv_cache_layout LATENT (attention.rs:3862-3867, :4058-4062, :4210-4212): one kv head; value,
   * value_cache (and their outputs) are absent; every value row is the first v_head_size
   * channels of the key row (after RoPE / norm), read from the key cache; the output is
   * [nt, H*v_head_size].  16-bit caches only; such calls run on the generic kernel. */
  int32_t kv_cache_latent;
  int32_t v_head_size;        /* LATENT: value channels (0 -> head_size), <= head_size     */
} B200PagedAttentionParams;

/* Library version (major * 10000 + minor * 100 + patch). */
B200_API int b200_version(void);

/* sizeof(B200PagedAttentionParams) and sizeof(B200NodeInfo) as compiled into the library, so a
 * binding (ctypes, cgo) can check its struct layout at load time. */
B200_API size_t b200_params_size(void);
B200_API size_t b200_node_info_size(void);

/* Number of kernels (and device memsets) this library has enqueued since load. */
B200_API uint64_t b200_launch_count(void);

/* Message of the last failing call on this thread ("" if none). */
B200_API const char* b200_last_error(void);

/* Bytes of device workspace the call needs (depends on shapes only, not on metadata).  The
 * call's kernels read their plan from the workspace while they run, so calls that may overlap
 * on the GPU (different streams, unordered threads) each need their own workspace. */
B200_API int b200_paged_attention_workspace_size(const B200PagedAttentionParams* p, size_t* bytes);

/* Host-side metadata validation, restating attention.rs:3934-3990.  Needs the host_*
 * metadata copies.  Returns B200_OK or B200_ERR_FAIL with the reference's message. */
B200_API int b200_paged_attention_validate_host(const B200PagedAttentionParams* p);

/* Whole PagedAttention node on `stream`: KV append (+ RoPE / q-k norm / integer or fp8
 * encode), paged decode (split-K), ragged prefill, output packing.  Replaces
 * paged_attention_op (rust/src/ops/attention.rs:3857-4382) and the direct Metal decode
 * (rust/src/ops/paged_attention.rs:229-334).  Asynchronous: device-side metadata checks
 * land in the status word, read by b200_read_status(). */
B200_API int b200_paged_attention(const B200PagedAttentionParams* p, void* stream);

/* KV append alone (reshape-and-cache): the scatter of attention.rs:4064-4120 plus the
 * in-place write-back of engine.rs:1212-1364, without attention.  Uses the same params. */
B200_API int b200_kv_append(const B200PagedAttentionParams* p, void* stream);

/* PagedAttention with library-owned scratch, for callers that cannot allocate device memory
 * (a host runtime that passes only the tensors it already owns, a serving loop that forbids
 * device allocations after start-up, a cgo/JNI binding without a CUDA allocator).  No
 * counterpart in the reference.  Same inputs, outputs and semantics as b200_paged_attention,
 * but `workspace` / `workspace_bytes` are ignored: scratch comes from a 32 MiB static device
 * array that every GPU loading the library keeps until exit.  Calls needing more scratch than
 * 32 MiB (see b200_paged_attention_workspace_size) fail with B200_ERR_WORKSPACE.  All calls on
 * a device share the array (each call re-initialises what must start at zero), so calls that
 * overlap on the GPU race and must be serialised by the caller.  The first call on a device
 * resolves the array's address (cudaGetSymbolAddress) and should come before any stream
 * capture; the address is kept until exit, so cudaDeviceReset is not supported alongside this
 * entry point.  The scratch need grows with the token count (RoPE / q-k norm rows, and for
 * bf16 prefill an fp16 copy of the new V rows, 2 x tokens x kv heads x head_size bytes), the
 * batch and the SM count (decode partial rows: SMs x resident decode CTAs x 4 warps x 16 rows x
 * head_size x 4 bytes, about 9.7 MB at head_size 256 on 148 SMs), so a num_sms override far
 * above the device's count can push a call past the limit.  Without device_status the status
 * word lives in the static array too: read it with b200_read_status_static_scratch.  The call
 * allocates nothing. */
B200_API int b200_paged_attention_static_scratch(const B200PagedAttentionParams* p, void* stream);

/* b200_read_status for calls made through b200_paged_attention_static_scratch: reads
 * p->device_status when set, otherwise the status word inside the current device's static
 * scratch (so device-side metadata errors and timed-out waits reach callers that pass no
 * status word).  Reads the last call's word, so calls that overlap on the GPU race here too.
 * No counterpart in the reference; allocates nothing. */
B200_API int b200_read_status_static_scratch(const B200PagedAttentionParams* p, void* stream);

/* Synchronise `stream`, read and clear the device status word of the last call with these
 * params, and turn set bits into B200_ERR_FAIL / B200_ERR_DEVICE with the reference's
 * messages. */
B200_API int b200_read_status(const B200PagedAttentionParams* p, void* stream);

/*
 * Claim predicate, restating paged_attention_claim (rust/src/ops/attention.rs:4384-4645)
 * and the integer-cache claim (rust/src/ops/kv_cache.rs:16-108) over a plain description of
 * the node.  Returns 1 (claim) or 0 (decline, reason written to `reason`).
 */
#define B200_MAX_RANK 8
typedef struct B200TensorInfo {
  int32_t present;              /* 0 = absent optional input/output                     */
  int32_t dtype;                /* B200_DTYPE_* (ONNX enum)                             */
  int32_t rank;                 /* -1 = unknown rank                                    */
  int64_t shape[B200_MAX_RANK]; /* -1 = symbolic dimension                              */
} B200TensorInfo;

typedef struct B200NodeInfo {
  int32_t num_inputs;
  int32_t num_outputs;
  B200TensorInfo inputs[17];
  B200TensorInfo outputs[3];
  /* integer attributes (value used when has_* is 0 is the operator default) */
  int64_t num_heads, kv_num_heads, is_causal, local_window_size, do_rotary, rotary_interleaved,
      rotary_offset, v_head_size;
  int32_t has_scale;
  float scale;
  float softcap;
  float qk_norm_epsilon;
  char kv_cache_layout[16]; /* "SEPARATE" (default) or "LATENT"                       */
  char k_quant_type[16];    /* "NONE" (default), "PER_TENSOR", "PER_CHANNEL"          */
  char v_quant_type[16];
  char k_cache_dtype[16];   /* "" (default), "int8", "int4", "float16", "bfloat16"    */
  char v_cache_dtype[16];
} B200NodeInfo;

B200_API int b200_paged_attention_claim(const B200NodeInfo* node, char* reason, size_t reason_len);

/* ---- com.microsoft.GroupQueryAttention over a contiguous BNSH cache -------------------- */

/*
 * One GroupQueryAttention node, replacing group_query_attention_op
 * (rust/src/ops/attention.rs:932-1454) and its per-batch form gqa_batched (:586-848) for the
 * forms b200_group_query_attention_claim accepts.  Per batch row b, with
 * length = seqlens_k[b] + 1, query_past = max(length - seq, 0),
 * past = new_seq ? query_past : length and new_rows = new_seq ? length - past : 0 (:662-667):
 *   present[b, :, :past]       = past_kv[b, :, :past]
 *   present[b, :, past:length] = the first new_rows rows of key/value[b]
 *   present[b, :, length:]     = past_kv[b, :, length:cap] (if length < cap), then zeros
 * and query row i of batch b (absolute position query_past + i) attends over keys
 * [start, end) with end = min(query_past + i + 1, length) when causal (else length) and
 * start = max(0, end - local_window_size) when local_window_size > 0 (:704-711).  present has
 * present_cap = max(cap, total_sequence_length) rows; when present_key == past_key the call
 * writes only the new rows, in place (shared-buffer contract, :1365-1375).
 */
typedef struct B200GqaParams {
  int32_t num_heads, kv_num_heads, head_size;
  float scale;               /* 0 = 1/sqrt(head_size)                                   */
  int32_t is_causal;         /* op attribute `causal` (default 1)                        */
  int32_t local_window_size; /* -1 (or 0) = none                                         */
  float softcap;             /* 0 = none                                                 */
  int32_t smooth_softmax;    /* 1 = a zero sink in every head's denominator              */
  int32_t dtype;             /* activations and caches: FLOAT, FLOAT16 or BFLOAT16       */
  int32_t batch, seq;        /* query [batch, seq, num_heads*head_size]                  */
  int32_t new_seq;           /* key/value rows per batch: seq, or 0 (past only)          */
  int32_t cap;               /* past axis-2 capacity (0 when past is absent)             */
  int32_t present_cap;       /* present axis-2 length: max(cap, total_sequence_length)   */
  int32_t total_sequence_length; /* host value of input 6                                */
  int64_t query_row_stride, key_row_stride, value_row_stride; /* elements per token; 0 = dense
                                                                 (packed QKV: (H+2KV)*D)  */
  const void* query;
  const void* key;             /* may be NULL when new_seq == 0                          */
  const void* value;
  const void* past_key;        /* [batch, KV, cap, D] or NULL                            */
  const void* past_value;
  void* present_key;           /* [batch, KV, present_cap, D]; may equal past_key        */
  void* present_value;
  const int32_t* seqlens_k;      /* device [batch]                                       */
  const int32_t* host_seqlens_k; /* host [batch] (the reference reads it on the host)    */
  const void* head_sink;         /* [num_heads] in dtype, or NULL                        */
  void* output;                  /* [batch, seq, num_heads*head_size]                    */
  void* workspace;
  size_t workspace_bytes;
  int32_t num_sms;               /* 0 = query the device                                 */
  /* rotary embedding of the new query and key rows (attribute do_rotary, inputs 7-9,
   * attention.rs:538-585, :668-681): the first rotary_dim channels of every head, rotate-half
   * or interleaved pairs, in fp32, rounded once to dtype.  Row s of batch b sits at position
   * query_past(b) + s without position_ids; with them, at position_ids[0] + s on a first prompt
   * (total_sequence_length == seq) and at the flattened id b * seq + s otherwise. */
  int32_t do_rotary;
  int32_t rotary_interleaved;
  int32_t rotary_dim;            /* 2 * cos_cache.shape[1], <= head_size                 */
  int32_t rotary_positions;      /* cos_cache.shape[0]                                   */
  const void* cos_cache;         /* [rotary_positions, rotary_dim / 2] in dtype          */
  const void* sin_cache;
  const int64_t* position_ids;   /* device int64 [batch, position_ids_width] or NULL     */
  const int64_t* host_position_ids; /* host copy, required with position_ids (validation) */
  int32_t position_ids_width;
  /* attention_bias (input 10, attention.rs:637-652, :746-755): added to the (soft-capped)
   * scores of the visible keys, element [bias_batch == 1 ? 0 : b, bias_heads == 1 ? 0 : h, s,
   * key], in dtype; NULL = none.  Shape [bias_batch (1 or batch), bias_heads (1 or num_heads),
   * bias_seq (== seq), bias_total (== total_sequence_length)], row-major. */
  const void* attention_bias;
  int32_t bias_batch, bias_heads, bias_seq, bias_total;
  /* q/k RMS norm (inputs 14 / 15, attention.rs:1070-1078): every query head and every new key
   * head is x / sqrt(mean(x^2) + qk_norm_epsilon) * weight, rounded to dtype, before the rotary
   * embedding; weights [head_size] in dtype, both or neither. */
  const void* q_norm_weight;
  const void* k_norm_weight;
  float qk_norm_epsilon;      /* 0 -> 1e-6                                               */
  /* qk_output diagnostics (attribute qk_output, output 3, attention.rs:771-787): 1 = the
   * logits (scale * q.k, soft-capped, plus attention_bias) of the visible keys and 0
   * elsewhere, 2 = the softmax probabilities (sink included); [batch, num_heads, seq,
   * total_sequence_length] in dtype, columns from each row's length on are 0. */
  int32_t qk_output;
  void* output_qk;
  /* integer caches (kv_cache_bit_width 8 / 4, inputs 12 / 13, kv_cache.rs:16-108,
   * test_quantized_kv.py:22-195): past and present hold int8 codes, or +8-biased int4 nibbles
   * (two channels per byte, the even channel in the low nibble; rows of head_size / 2 bytes).
   * New rows are encoded as rint(x * (1 / scale)) clipped to the code range (scale 0 -> 1) and
   * the attention reads every key and value decoded (code * scale), new rows included; scales
   * are PER_TENSOR [1] or PER_CHANNEL [kv_num_heads, head_size] fp32. */
  int32_t cache_dtype;        /* 0 or dtype: float caches; B200_DTYPE_INT8 or _UINT8 (int4) */
  const float* k_scale;
  const float* v_scale;
  int32_t k_quant_per_channel, v_quant_per_channel;
  /* sliding_window_cache=1 (attention.rs:1139-1379): a cache of capacity `cap` keeps
   * resident(n) rows of a length-n sequence, n up to cap, otherwise n - gap * ceil((n - cap) /
   * gap) with gap = cap - local_window_size + 1.  Batch row b (length = seqlens_k[b] + 1, past =
   * length - seq) attends over its resident(past) past rows, which hold absolute positions
   * past - resident(past) .., and its seq new rows, with the local window on absolute positions
   * and attention_bias columns absolute; present (present_cap == cap, may equal past) then
   * holds the last resident(length) rows of the sequence and zero rows (zero codes) after them.
   * Requires new_seq == seq, 0 < local_window_size <= cap, present, qk_output 0. */
  int32_t sliding_window_cache;
} B200GqaParams;

B200_API int b200_gqa_params_size(void);
/* Bytes of device workspace (shapes only). */
B200_API int b200_group_query_attention_workspace_size(const B200GqaParams* p, size_t* bytes);
/* Validate (reference messages, attention.rs:989-1030, :613-630, :663-667), then append and
 * attend.  B200_ERR_FAIL for invalid lengths, B200_ERR_UNSUPPORTED for unclaimed forms. */
B200_API int b200_group_query_attention(const B200GqaParams* p, void* stream);
/* Synchronise `stream` and report the device status word of the last call that used this
 * workspace: B200_ERR_DEVICE when a bounded device wait ran out.  The reference runs the node
 * on the host and has no device status; this plays the role of its error return for the
 * device side (lib.rs:53-92 turns failures into an OrtStatus). */
B200_API int b200_group_query_attention_read_status(const B200GqaParams* p, void* stream);

/* Claim predicate, restating group_query_attention_claim (attention.rs:2407-2754) over a
 * plain node description, plus this build's own decline (head size).  Returns 1 (claim) or 0
 * (decline, reason written to `reason`). */
typedef struct B200GqaNodeInfo {
  int32_t num_inputs;
  int32_t num_outputs;
  B200TensorInfo inputs[16];
  B200TensorInfo outputs[4];
  int64_t num_heads, kv_num_heads, causal, local_window_size, do_rotary, rotary_interleaved,
      sliding_window_cache, smooth_softmax, qk_output, kv_cache_bit_width;
  int32_t has_causal, has_local_window_size, has_smooth_softmax; /* 0 = operator default   */
  float softcap;
  int32_t has_scale;         /* 0 = attribute absent: 1/sqrt(head_size)                      */
  float scale;
  int32_t has_qk_norm_epsilon; /* 0 = attribute absent: 1e-6                                 */
  float qk_norm_epsilon;
  char k_quant_type[16];     /* "NONE" (default), "PER_TENSOR", "PER_CHANNEL"                */
  char v_quant_type[16];
} B200GqaNodeInfo;

B200_API int b200_group_query_attention_claim(const B200GqaNodeInfo* node, char* reason, size_t reason_len);
/* sizeof(B200GqaNodeInfo), for binding layout checks. */
B200_API int b200_gqa_node_info_size(void);

/* ---- diagnostics (no counterpart in the reference) ------------------------------------ */

/* Known-answer test of the tcgen05 tensor-core path: one CTA computes, for 128x128 fp16/bf16
 * row-major device matrices a, b, v, the fp32 products c_qk = a . b^T and c_pv = a . v through
 * TMA, shared-memory matrix descriptors, tcgen05.mma into tensor memory and tcgen05.ld, and
 * (when c_ts is not NULL) c_ts = a . v again with a held in tensor memory. */
B200_API int b200_selftest_tcgen05(int32_t dtype, const void* a, const void* b, const void* v, float* c_qk,
                                   float* c_pv, float* c_ts, int32_t* device_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_PAGED_H */
