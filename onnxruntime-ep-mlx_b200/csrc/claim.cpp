// Claim predicates for com.microsoft.PagedAttention and com.microsoft.GroupQueryAttention over
// plain node descriptions.
//
// Restates paged_attention_claim (rust/src/ops/attention.rs:4384-4645) and the integer cache
// claim it calls (rust/src/ops/kv_cache.rs:16-108), decline messages included, so an EP shell
// can decide in GetCapability exactly as the reference does.  Two additions: forms this build
// does not implement (head size above B200_MAX_HEAD_SIZE, rows the append prologue cannot stage,
// an fp8 LATENT cache) are declined with a reason, and an fp8 e4m3 cache (extension:
// per-block, per-kv-head fp32 scales [NB, KV]) is accepted when k/v_cache_dtype say
// "float8e4m3".
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <string>
#include <vector>

#include "b200_paged.h"

namespace {

struct Decline {
  std::string reason;
};

[[noreturn]] void deny(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  throw Decline{buf};
}

#define REQUIRE(cond, ...) \
  do {                     \
    if (!(cond)) deny(__VA_ARGS__); \
  } while (0)

const char* dtype_name(int dt) {
  switch (dt) {
    case B200_DTYPE_FLOAT: return "float32";
    case B200_DTYPE_UINT8: return "uint8";
    case B200_DTYPE_INT8: return "int8";
    case B200_DTYPE_INT32: return "int32";
    case B200_DTYPE_INT64: return "int64";
    case B200_DTYPE_FLOAT16: return "float16";
    case B200_DTYPE_BFLOAT16: return "bfloat16";
    case B200_DTYPE_FLOAT8E4M3FN: return "float8e4m3fn";
    default: return "unsupported";
  }
}

struct View {
  const B200NodeInfo* n;
  bool in_present(int i) const { return i < n->num_inputs && n->inputs[i].present; }
  bool out_present(int i) const { return i < n->num_outputs && n->outputs[i].present; }
  const B200TensorInfo* in(int i) const { return in_present(i) ? &n->inputs[i] : nullptr; }
  const B200TensorInfo* out(int i) const { return out_present(i) ? &n->outputs[i] : nullptr; }
  int dtype_of(int i) const { return in_present(i) ? n->inputs[i].dtype : 0; }
  std::string str(const char* s, const char* def) const { return s[0] ? std::string(s, strnlen(s, 16)) : def; }
};

bool shape_is(const B200TensorInfo* t, std::initializer_list<int64_t> dims) {
  if (!t || t->rank != (int)dims.size()) return false;
  int i = 0;
  for (int64_t d : dims) {
    if (t->shape[i++] != d) return false;
  }
  return true;
}

bool integer_cache(int dt) { return dt == B200_DTYPE_INT8 || dt == B200_DTYPE_UINT8; }

// kv_cache.rs:16-108 (paged = true).
void kv_cache_claim(const View& v, int activation, int64_t heads, int64_t head) {
  const int cache_type = v.in(3) ? v.in(3)->dtype : activation;
  const bool quantized = integer_cache(cache_type);
  const bool fp8 = cache_type == B200_DTYPE_FLOAT8E4M3FN;
  struct Side { int cache, scale; const char* name; const char* quant; const char* logical; };
  const Side sides[2] = {{3, 14, "k", v.n->k_quant_type, v.n->k_cache_dtype},
                         {4, 15, "v", v.n->v_quant_type, v.n->v_cache_dtype}};
  for (const Side& s : sides) {
    const int dtype = v.in(s.cache) ? v.in(s.cache)->dtype : activation;
    REQUIRE(dtype == cache_type, "key/value caches must share one storage dtype");
    const std::string mode = v.str(s.quant, "NONE");
    if (quantized) {
      REQUIRE(mode == "PER_TENSOR" || mode == "PER_CHANNEL",
              "integer %s cache requires PER_TENSOR or PER_CHANNEL quantization", s.name);
      const B200TensorInfo* info = v.in(s.scale);
      if (!info) deny("quantized %s cache requires a scale tensor", s.name);
      REQUIRE(info->dtype == B200_DTYPE_FLOAT, "%s_scale must be float32", s.name);
      bool known = info->rank >= 0;
      int64_t count = 1;
      for (int i = 0; i < info->rank && known; ++i) {
        if (info->shape[i] < 0) known = false; else count *= info->shape[i];
      }
      const int64_t expected = mode == "PER_TENSOR" ? 1 : heads * head;
      REQUIRE(!known || count == expected, "%s_scale must contain %lld elements", s.name, (long long)expected);
      if (mode == "PER_CHANNEL") {
        const int64_t last = info->rank > 0 ? info->shape[info->rank - 1] : 0;
        REQUIRE(info->rank > 0 && (last < 0 || last == head), "PagedAttention per-channel scales must end in head_size");
      }
    } else if (fp8) {
      const B200TensorInfo* info = v.in(s.scale);
      if (!info) deny("fp8 %s cache requires a per-block, per-head scale tensor", s.name);
      REQUIRE(info->dtype == B200_DTYPE_FLOAT, "%s_scale must be float32", s.name);
      REQUIRE(info->rank == 2 && (info->shape[1] < 0 || info->shape[1] == heads),
              "fp8 %s_scale must be [num_blocks, kv_num_heads]", s.name);
    } else {
      REQUIRE(dtype == activation && mode == "NONE" && !v.in_present(s.scale),
              "floating %s cache requires activation dtype, NONE quantization and no scale", s.name);
    }
    const std::string logical = v.str(s.logical, "");
    const char* expected = dtype == B200_DTYPE_INT8       ? "int8"
                           : dtype == B200_DTYPE_UINT8    ? "int4"
                           : dtype == B200_DTYPE_FLOAT16  ? "float16"
                           : dtype == B200_DTYPE_BFLOAT16 ? "bfloat16"
                           : dtype == B200_DTYPE_FLOAT8E4M3FN ? "float8e4m3"
                                                              : "";
    REQUIRE(logical == expected || (logical.empty() && std::strcmp(expected, "int4") != 0 &&
                                    std::strcmp(expected, "float8e4m3") != 0),
            "%s_cache_dtype must agree with cache storage; uint8 requires explicit int4", s.name);
    if (v.out_present(s.cache - 2)) {
      REQUIRE(v.out(s.cache - 2)->dtype == dtype, "present %s cache must retain its input storage dtype", s.name);
    }
  }
}

// attention.rs:4384-4645.
void paged_claim(const View& v) {
  const B200NodeInfo* n = v.n;
  REQUIRE(n->is_causal == 0 || n->is_causal == 1, "is_causal must be 0 or 1");
  REQUIRE(n->num_outputs >= 1 && n->num_outputs <= 3, "PagedAttention requires 1 to 3 outputs");
  REQUIRE(n->v_head_size >= 0, "v_head_size must be non-negative");
  REQUIRE(n->rotary_offset >= 0, "rotary_offset must be non-negative");
  const B200TensorInfo* o0 = v.out(0);
  if (!o0) deny("output lacks tensor type/shape info");
  const int out_dt = o0->dtype;
  REQUIRE(out_dt == B200_DTYPE_FLOAT || out_dt == B200_DTYPE_FLOAT16 || out_dt == B200_DTYPE_BFLOAT16,
          "output must be an MLX float dtype, got %s", dtype_name(out_dt));
  REQUIRE(out_dt == B200_DTYPE_FLOAT16 || out_dt == B200_DTYPE_BFLOAT16,
          "PagedAttention is only supported for fp16/bf16 (T)");
  REQUIRE(n->num_inputs >= 8 && n->num_inputs <= 17,
          "expects 8 required inputs plus optional rotary, scheduling, normalization, and scale inputs, got %d",
          n->num_inputs);
  const std::string layout = v.str(n->kv_cache_layout, "SEPARATE");
  REQUIRE(layout == "SEPARATE" || layout == "LATENT", "kv_cache_layout must be SEPARATE or LATENT");
  const bool latent = layout == "LATENT";
  const bool quantized = v.in(3) && integer_cache(v.in(3)->dtype);
  REQUIRE(!latent || !quantized, "quantized LATENT cache contract is not supported");
  const bool packed = !latent && !v.in_present(1) && !v.in_present(2);
  for (int idx : {0, 1}) {
    if (packed && idx == 1) break;
    if (!v.in_present(idx)) deny("input %d (Q/K/V/cache) must be present with a float dtype", idx);
    REQUIRE(v.dtype_of(idx) == out_dt, "input %d must share the output float dtype", idx);
  }
  if (latent) {
    REQUIRE(!v.in_present(2) && !v.in_present(4),
            "LATENT layout aliases value to key and requires absent value/value_cache");
  } else if (!packed) {
    REQUIRE(v.in_present(2) && v.dtype_of(2) == out_dt, "input 2 must be present and share the output float dtype");
  }
  for (int idx : {5, 6, 7}) {
    if (!v.in_present(idx)) deny("input %d (positional) must be present", idx);
    REQUIRE(v.dtype_of(idx) == B200_DTYPE_INT32, "input %d must be int32", idx);
  }
  const int64_t num_heads = n->num_heads, kv_heads = n->kv_num_heads;
  REQUIRE(num_heads > 0 && kv_heads > 0 && num_heads % kv_heads == 0,
          "num_heads (%lld) must be a positive multiple of kv_num_heads (%lld)", (long long)num_heads,
          (long long)kv_heads);
  REQUIRE(!latent || kv_heads == 1, "LATENT layout requires kv_num_heads=1");
  const B200TensorInfo* query = v.in(0);
  const int64_t query_heads = packed ? num_heads + 2 * kv_heads : num_heads;
  REQUIRE(query->rank == 2 && query->shape[1] > 0 && query->shape[1] % query_heads == 0,
          "query must have rank 2 and a hidden size divisible by its separate or packed head count");
  const int64_t head = query->shape[1] / query_heads;
  kv_cache_claim(v, out_dt, kv_heads, head);
  const int64_t cache_head = v.dtype_of(3) == B200_DTYPE_UINT8 ? (head + 1) / 2 : head;
  const int64_t v_head = n->v_head_size == 0 ? head : n->v_head_size;
  REQUIRE(v_head > 0, "effective v_head_size must be positive");
  if (!packed) {
    const B200TensorInfo* k = v.in(1);
    REQUIRE(k && k->rank == 2 && k->shape[1] == kv_heads * head, "key must be [num_tokens,kv_num_heads*head_size]");
    if (!latent) {
      const B200TensorInfo* val = v.in(2);
      REQUIRE(val && val->rank == 2 && val->shape[1] == kv_heads * v_head,
              "value must be [num_tokens,kv_num_heads*v_head_size]");
    }
  }
  if (!latent) {
    REQUIRE(v_head == head, "SEPARATE layout requires equal key and value head sizes");
  } else {
    REQUIRE(v_head <= head, "LATENT v_head_size must not exceed head_size");
    if (v_head != head) REQUIRE(n->has_scale, "LATENT layout with asymmetric value heads requires an explicit scale");
  }
  const B200TensorInfo* kc = v.in(3);
  REQUIRE(kc && kc->rank == 4 && kc->shape[2] == kv_heads && kc->shape[3] == cache_head,
          "key_cache must be [num_blocks,block_size,kv_num_heads,head_size]");
  if (!latent) {
    const B200TensorInfo* vc = v.in(4);
    REQUIRE(vc && vc->rank == 4 && vc->shape[2] == kv_heads && vc->shape[3] == cache_head,
            "value_cache must be [num_blocks,block_size,kv_num_heads,v_head_size]");
  }
  REQUIRE(o0->rank == 2 && (o0->shape[1] < 0 || o0->shape[1] == num_heads * v_head),
          "output must be [num_tokens,num_heads*v_head_size]");
  REQUIRE(n->local_window_size == -1 || n->local_window_size > 0, "local_window_size must be -1 or positive");
  REQUIRE(std::isfinite(n->softcap) && n->softcap >= 0.f, "softcap must be finite and non-negative");
  if (n->do_rotary) {
    REQUIRE(v.in_present(8) && v.in_present(9), "do_rotary=1 requires cos_cache and sin_cache inputs");
    REQUIRE(v.dtype_of(8) == out_dt && v.dtype_of(9) == out_dt, "cos_cache/sin_cache must share the output float dtype");
    const B200TensorInfo* cos = v.in(8);
    const B200TensorInfo* sin = v.in(9);
    bool same = cos->rank == 2 && sin->rank == 2 && cos->shape[0] == sin->shape[0] && cos->shape[1] == sin->shape[1];
    REQUIRE(same && cos->shape[1] > 0, "cos/sin caches must have matching [positions,rotary_dim/2] shapes");
    const int64_t rotary_dim = cos->shape[1] * 2;
    REQUIRE(n->rotary_offset + rotary_dim <= head, "rotary_offset + rotary_dim must not exceed head_size");
    REQUIRE(n->rotary_offset % 8 == 0, "rotary_offset must be a multiple of 8");
  }
  if (v.in_present(10)) {
    const B200TensorInfo* s = v.in(10);
    REQUIRE(s->dtype == B200_DTYPE_INT32 && s->rank == 1 &&
                (s->shape[0] < 0 || query->shape[0] < 0 || s->shape[0] == query->shape[0]),
            "slot_mapping must be int32 [num_tokens]");
  }
  if (v.in_present(11)) {
    REQUIRE(v.in(11)->dtype == out_dt && shape_is(v.in(11), {num_heads}),
            "head_sink must be [num_heads] in activation dtype");
  }
  REQUIRE(v.in_present(12) == v.in_present(13), "q_norm_weight and k_norm_weight must be provided together");
  if (v.in_present(12)) {
    for (int idx : {12, 13})
      REQUIRE(v.in(idx)->dtype == out_dt && shape_is(v.in(idx), {head}),
              "Q/K norm weight %d must be [head_size] in activation dtype", idx);
  }
  if (v.in_present(16)) {
    const B200TensorInfo* m = v.in(16);
    REQUIRE(m->dtype == B200_DTYPE_INT32 && (shape_is(m, {2}) || shape_is(m, {3})),
            "attention_metadata must be int32 [2] or [3]");
  }
  if (latent) REQUIRE(!v.out_present(2), "LATENT layout has no separate value cache output");
  for (int idx = 1; idx < (n->num_outputs < 3 ? n->num_outputs : 3); ++idx) {
    if (v.out_present(idx))
      REQUIRE(v.out(idx)->dtype == v.dtype_of(idx + 2), "cache output %d must retain cache storage dtype", idx);
  }
  // Forms the reference accepts that this build does not implement.
  REQUIRE(head <= B200_MAX_HEAD_SIZE, "head_size above %d is not implemented by the B200 kernels", B200_MAX_HEAD_SIZE);
  REQUIRE(!latent || !v.in(3) || v.in(3)->dtype == out_dt, "fp8 LATENT caches are not implemented by the B200 kernels");
  const bool process = n->do_rotary || v.in_present(12);
  const bool encoded = v.in(3) && v.in(3)->dtype != out_dt;
  if (process || encoded) {
    const int64_t rows = (process ? num_heads : 0) + 2 * kv_heads;
    REQUIRE(4 * head * rows <= B200_MAX_PROLOGUE_STAGE_BYTES,
            "rotary / norm / encoded rows of one token (%lld heads of %lld channels) exceed the B200 append "
            "prologue's shared memory", (long long)rows, (long long)head);
  }
}

// ---------------------------------------------------------------------------------------
// GroupQueryAttention: group_query_attention_claim (attention.rs:2407-2754), then the forms
// this build does not implement.
struct GView {
  const B200GqaNodeInfo* n;
  bool in_present(int i) const { return i < n->num_inputs && n->inputs[i].present; }
  bool out_present(int i) const { return i < n->num_outputs && n->outputs[i].present; }
  const B200TensorInfo* in(int i) const { return in_present(i) ? &n->inputs[i] : nullptr; }
  const B200TensorInfo* out(int i) const { return out_present(i) ? &n->outputs[i] : nullptr; }
};

// kv_cache.rs:16-108 with paged = false: inputs 12 / 13 are the scales, kv_cache_bit_width
// states the storage.
void gqa_kv_cache_claim(const GView& v, int activation, int64_t heads, int64_t head) {
  const B200GqaNodeInfo& n = *v.n;
  const int cache_type = v.in(3) ? v.in(3)->dtype : activation;
  const bool quantized = integer_cache(cache_type);
  struct Side { int cache, scale; const char* name; const char* quant; };
  const Side sides[2] = {{3, 12, "k", n.k_quant_type}, {4, 13, "v", n.v_quant_type}};
  for (const Side& s : sides) {
    const int dtype = v.in(s.cache) ? v.in(s.cache)->dtype : activation;
    REQUIRE(dtype == cache_type, "key/value caches must share one storage dtype");
    const std::string mode = s.quant[0] ? std::string(s.quant, strnlen(s.quant, 16)) : "NONE";
    if (quantized) {
      REQUIRE(mode == "PER_TENSOR" || mode == "PER_CHANNEL",
              "integer %s cache requires PER_TENSOR or PER_CHANNEL quantization", s.name);
      const B200TensorInfo* info = v.in(s.scale);
      if (!info) deny("quantized %s cache requires a scale tensor", s.name);
      REQUIRE(info->dtype == B200_DTYPE_FLOAT, "%s_scale must be float32", s.name);
      bool known = info->rank >= 0;
      int64_t count = 1;
      for (int i = 0; i < info->rank && known; ++i) {
        if (info->shape[i] < 0) known = false; else count *= info->shape[i];
      }
      const int64_t expected = mode == "PER_TENSOR" ? 1 : heads * head;
      REQUIRE(!known || count == expected, "%s_scale must contain %lld elements", s.name, (long long)expected);
    } else {
      REQUIRE(dtype == activation && mode == "NONE" && !v.in_present(s.scale),
              "floating %s cache requires activation dtype, NONE quantization and no scale", s.name);
    }
    if (v.out_present(s.cache - 2))
      REQUIRE(v.out(s.cache - 2)->dtype == dtype, "present %s cache must retain its input storage dtype", s.name);
  }
  const int64_t expected_bits = cache_type == B200_DTYPE_INT8 ? 8 : cache_type == B200_DTYPE_UINT8 ? 4 : 0;
  REQUIRE(n.kv_cache_bit_width == expected_bits, "kv_cache_bit_width must agree with cache storage");
}

bool same_shape(const B200TensorInfo* a, const B200TensorInfo* b) {
  if (!a || !b || a->rank != b->rank) return false;
  for (int i = 0; i < a->rank && i < B200_MAX_RANK; ++i)
    if (a->shape[i] != b->shape[i]) return false;
  return true;
}

void gqa_claim(const GView& v) {
  const B200GqaNodeInfo& n = *v.n;
  const int64_t causal = n.has_causal ? n.causal : 1;
  const int64_t window = n.has_local_window_size ? n.local_window_size : -1;
  const int64_t smooth = n.has_smooth_softmax ? n.smooth_softmax : -1;
  REQUIRE(n.num_outputs >= 1 && n.num_outputs <= 4, "requires 1 to 4 outputs");
  REQUIRE(v.out_present(1) == v.out_present(2), "present_key and present_value must both be provided or both omitted");
  const bool sliding = n.sliding_window_cache != 0;
  REQUIRE(causal == 0 || causal == 1, "causal must be 0 or 1");
  REQUIRE(window == -1 || window > 0, "local_window_size must be -1 or positive");
  REQUIRE(causal != 0 || window == -1, "bidirectional GroupQueryAttention requires local_window_size=-1");
  REQUIRE(v.in_present(3) == v.in_present(4), "past_key and past_value must be provided together");
  const B200TensorInfo* out0 = v.out(0);
  if (!out0) deny("output lacks tensor type/shape info");
  const int out_type = out0->dtype;
  REQUIRE(out_type == B200_DTYPE_FLOAT || out_type == B200_DTYPE_FLOAT16 || out_type == B200_DTYPE_BFLOAT16,
          "output must have an MLX float dtype, got %s", dtype_name(out_type));
  const int ninputs = n.num_inputs;
  REQUIRE(ninputs >= 7 && ninputs <= 16, "expects 7 required inputs plus optional rotary/bias/QK-norm inputs, got %d", ninputs);
  const bool has_bias = v.in_present(10);
  const bool do_rotary = n.do_rotary != 0;
  REQUIRE(ninputs != 7 || !do_rotary, "7-input GroupQueryAttention requires do_rotary=0 because cos/sin caches are absent");
  if (sliding) {
    REQUIRE(window > 0, "sliding_window_cache=1 requires local_window_size > 0");
    REQUIRE(v.out_present(1) && v.out_present(2), "sliding_window_cache requires present key/value outputs");
    const B200TensorInfo* pk = v.in(3);
    const B200TensorInfo* pv = v.in(4);
    REQUIRE(pk && pk->rank == 4 && pk->shape[2] >= window,
            "sliding-window key cache capacity must be at least local_window_size");
    REQUIRE(pv && pv->rank == 4 && pv->shape[2] >= window,
            "sliding-window value cache capacity must be at least local_window_size");
  }
  const bool packed = v.in_present(0) && !v.in_present(1) && !v.in_present(2);
  REQUIRE(packed || (v.in_present(0) && v.in_present(1) && v.in_present(2)),
          "Q/K/V must be either all separate or packed in input 0 with inputs 1 and 2 absent");
  const bool quantized = v.in(3) && integer_cache(v.in(3)->dtype);
  std::vector<int> float_idx = packed ? std::vector<int>{0} : std::vector<int>{0, 1, 2};
  if (v.in_present(3) && !quantized) { float_idx.push_back(3); float_idx.push_back(4); }
  if (do_rotary) { float_idx.push_back(7); float_idx.push_back(8); }
  if (has_bias) float_idx.push_back(10);
  if (v.in_present(14)) { float_idx.push_back(14); float_idx.push_back(15); }
  for (int idx : float_idx) {
    const B200TensorInfo* t = v.in(idx);
    if (!t) deny("input %d lacks tensor type/shape info", idx);
    REQUIRE(t->dtype == out_type, "input %d must have output dtype %s, got %s", idx, dtype_name(out_type), dtype_name(t->dtype));
  }
  if (has_bias)  // attention.rs:2546-2560
    REQUIRE(v.in(10)->rank == 4, "attention_bias (input 10) must have rank 4, got rank %d", v.in(10)->rank);
  for (int idx = 1; idx < std::min(n.num_outputs, 3); ++idx) {
    if (!v.out_present(idx)) continue;
    const int want = v.in(idx + 2) ? v.in(idx + 2)->dtype : out_type;
    REQUIRE(v.out(idx)->dtype == want, "output %d must retain its cache dtype (activation dtype %s), got %s", idx,
            dtype_name(out_type), dtype_name(v.out(idx)->dtype));
  }
  for (int idx : {5, 6}) {
    const B200TensorInfo* t = v.in(idx);
    if (!t) deny("input %d lacks tensor type/shape info", idx);
    REQUIRE(t->dtype == B200_DTYPE_INT32, "input %d must have int32 dtype, got %s", idx, dtype_name(t->dtype));
  }
  const int64_t nh = n.num_heads, kvh = n.kv_num_heads;
  REQUIRE(nh > 0 && kvh > 0 && nh % kvh == 0, "num_heads (%lld) must be a positive multiple of kv_num_heads (%lld)",
          (long long)nh, (long long)kvh);
  const B200TensorInfo* q = v.in(0);
  REQUIRE(q->rank == 3 && q->shape[2] > 0, "query must have rank 3 and a positive static hidden size");
  const int64_t total_heads = packed ? nh + 2 * kvh : nh;
  REQUIRE(q->shape[2] % total_heads == 0, "query hidden size must match head count");
  const int64_t head = q->shape[2] / total_heads;
  gqa_kv_cache_claim(v, out_type, kvh, head);
  const int64_t bits = n.kv_cache_bit_width;
  REQUIRE(bits != 4 || head % 2 == 0,
          "GQA packed INT4 requires an even logical head size (pinned CheckPast byte geometry)");
  REQUIRE(!sliding || bits == 0 || head % (bits == 4 ? 32 : 16) == 0,
          "sliding integer cache rows must satisfy pinned 16-byte alignment");
  const int64_t cache_head = bits == 4 ? (head + 1) / 2 : head;
  if (has_bias) {
    const B200TensorInfo* bias = v.in(10);
    REQUIRE((bias->shape[0] < 0 || bias->shape[0] == 1 || q->shape[0] < 0 || bias->shape[0] == q->shape[0]) &&
                (bias->shape[1] < 0 || bias->shape[1] == 1 || bias->shape[1] == nh) &&
                (bias->shape[2] < 0 || q->shape[1] < 0 || bias->shape[2] == q->shape[1]),
            "attention_bias must broadcast to [batch,num_heads,sequence_length,total_sequence_length]");
  }
  if (!packed) {
    for (int idx : {1, 2}) {
      const B200TensorInfo* kv = v.in(idx);
      REQUIRE(kv->rank == 3 && kv->shape[2] == kvh * head &&
                  (kv->shape[0] < 0 || q->shape[0] < 0 || kv->shape[0] == q->shape[0]) &&
                  (kv->shape[1] < 0 || q->shape[1] < 0 || kv->shape[1] == q->shape[1] ||
                   (kv->shape[1] == 0 && v.in_present(3) && !sliding)),
              "key/value must match query batch, sequence length and KV head geometry");
    }
    REQUIRE(same_shape(v.in(1), v.in(2)), "key/value shapes must match");
  }
  for (int idx : {3, 4}) {
    const B200TensorInfo* c = v.in(idx);
    if (!c) continue;
    REQUIRE(c->rank == 4 && c->shape[1] == kvh && c->shape[3] == cache_head &&
                (c->shape[0] < 0 || q->shape[0] < 0 || c->shape[0] == q->shape[0]),
            "past cache must be [batch,kv_num_heads,capacity,stored_head_size]");
  }
  if (v.in_present(3)) REQUIRE(same_shape(v.in(3), v.in(4)), "past key/value cache shapes must match");
  const B200TensorInfo* lens = v.in(5);
  REQUIRE(lens && lens->rank == 1 && (lens->shape[0] < 0 || q->shape[0] < 0 || lens->shape[0] == q->shape[0]),
          "seqlens_k must be [batch]");
  const B200TensorInfo* tot = v.in(6);
  REQUIRE(tot && (tot->rank == 0 || (tot->rank == 1 && tot->shape[0] == 1)), "total_sequence_length must be scalar or [1]");
  if (do_rotary) {
    const B200TensorInfo* cos = v.in(7);
    const B200TensorInfo* sin = v.in(8);
    REQUIRE(cos && sin && cos->rank == 2 && same_shape(cos, sin) && cos->shape[1] > 0 && 2 * cos->shape[1] <= head,
            "rotary caches must have matching [positions,rotary_dim/2] shapes within the head");
  }
  if (v.in_present(9) && do_rotary) {
    const B200TensorInfo* pos = v.in(9);
    REQUIRE(pos->dtype == B200_DTYPE_INT64 && pos->rank == 2 &&
                (pos->shape[0] < 0 || q->shape[0] < 0 || pos->shape[0] == q->shape[0]) &&
                (pos->shape[1] < 0 || q->shape[1] < 0 || pos->shape[1] >= q->shape[1]),
            "position_ids must be int64 [batch,>=sequence_length]");
  }
  if (v.in_present(11)) {
    const B200TensorInfo* s = v.in(11);
    REQUIRE(s->dtype == out_type && s->rank == 1 && s->shape[0] == nh, "head_sink must be [num_heads] in activation dtype");
  }
  REQUIRE(v.in_present(14) == v.in_present(15), "q_norm_weight and k_norm_weight must be provided together");
  if (v.in_present(14)) {  // attention.rs:2703-2725
    for (int idx : {14, 15})
      REQUIRE(shape_is(v.in(idx), {head}), "Q/K norm weight %d must have shape [head_size=%lld]", idx, (long long)head);
  }
  REQUIRE(smooth >= -1 && smooth <= 1, "smooth_softmax must be -1 (schema default), 0 or 1");
  REQUIRE(n.qk_output >= 0 && n.qk_output <= 2 && (n.qk_output != 0) == v.out_present(3),
          "qk_output must be 0, 1 or 2 and enabled exactly when output_qk is present");
  REQUIRE(!sliding || n.qk_output == 0, "sliding_window_cache with QK diagnostics is unsupported");
  REQUIRE(std::isfinite(n.softcap) && n.softcap >= 0.f, "softcap must be finite and non-negative");
  // Forms the reference accepts that this build does not implement (the node stays on ORT).
  REQUIRE(head % 8 == 0 && head <= 256, "head_size must be a multiple of 8 up to 256 on B200, got %lld", (long long)head);
}

}  // namespace

extern "C" int b200_gqa_node_info_size(void) { return (int)sizeof(B200GqaNodeInfo); }

extern "C" int b200_group_query_attention_claim(const B200GqaNodeInfo* node, char* reason, size_t reason_len) {
  std::string why;
  try {
    if (!node) deny("null node");
    gqa_claim(GView{node});
    if (reason && reason_len) reason[0] = 0;
    return 1;
  } catch (const Decline& d) {
    why = d.reason;
  } catch (...) {
    why = "claim predicate failed";
  }
  if (reason && reason_len) std::snprintf(reason, reason_len, "%s", why.c_str());
  return 0;
}

extern "C" int b200_paged_attention_claim(const B200NodeInfo* node, char* reason, size_t reason_len) {
  std::string why;
  try {
    if (!node) deny("null node");
    paged_claim(View{node});
    if (reason && reason_len) reason[0] = 0;
    return 1;
  } catch (const Decline& d) {
    why = d.reason;
  } catch (...) {
    why = "claim predicate failed";
  }
  if (reason && reason_len) {
    std::snprintf(reason, reason_len, "%s", why.c_str());
  }
  return 0;
}
