// ONNX Runtime plugin-EP glue of the B200 execution provider.
//
// The ORT-facing half of the EP:
//   - CreateEpFactories / ReleaseEpFactory (reference rust/src/lib.rs:100-178);
//   - the OrtEpFactory table: names, device selection, EP creation, allocator, data transfer
//     (rust/src/factory.rs:20-317);
//   - the OrtEp table: GetCapability, Compile, ReleaseNodeComputeInfos, GetDefaultMemoryDevice
//     (rust/src/ep.rs:15-150, rust/src/capability.rs:361);
//   - the OrtNodeComputeInfo callbacks of each compiled node (rust/src/runtime.rs:93-331);
//   - the device OrtAllocator and OrtDataTransferImpl (rust/src/device.rs:85-640).
// Everything below ORT's types - claim predicates, option parsing, node states, kernels, CUDA
// memory, copies and streams - is in libb200_paged.so behind include/b200_ep.h; this file only
// moves values between ORT's objects and those plain structs, and compiles against ONNX
// Runtime's own headers (ORT_INCLUDE_DIR, ONNX Runtime >= 1.31) with no CUDA headers.
//
// Scope: each claimed com.microsoft.PagedAttention or GroupQueryAttention node becomes its own
// single-node fusion.  Its tensors live in the EP's device memory ("B200", vendor 0x10DE), which
// ORT fills through the data transfer; tensors that arrive in host memory anyway are staged
// through device buffers, so results do not depend on where ORT put them.  Each Compute runs on
// the EP's own stream and synchronises before returning (the EP is not stream-aware), so ORT may
// read the outputs as soon as Compute returns.
#include "onnxruntime_c_api.h"

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <stdexcept>
#include <string>
#include <vector>

#include "b200_ep.h"

#define B200_SHELL_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr uint32_t kNvidiaVendorId = 0x10DE;
constexpr const char* kMemoryName = "B200";
constexpr const char* kDefaultName = "B200ExecutionProvider";
constexpr const char* kVendor = "onnxruntime-ep-b200";
// 0.<ORT_API_VERSION>.<patch>, the reference's scheme (factory.rs:62-67).
constexpr const char* kVersion = "0.31.0";
constexpr const char* kMsDomain = "com.microsoft";

// ---------------------------------------------------------------------------------------------
// errors: ORT statuses, kernel-library statuses and exceptions meet here
// ---------------------------------------------------------------------------------------------
struct OrtError {
  OrtErrorCode code;
  std::string msg;
};
struct B200Failure {
  int rc;
};

[[noreturn]] void raise(OrtErrorCode code, const std::string& msg) { throw OrtError{code, msg}; }

// A failing kernel-library call: its message stays in b200_last_error() until converted.
void check_b200(int rc) {
  if (rc != B200_OK) throw B200Failure{rc};
}

OrtStatus* b200_status(const OrtApi* api, int rc) {
  if (rc == B200_OK) return nullptr;
  const OrtErrorCode code = b200_ort_error_class(rc) == B200_ORT_INVALID_ARGUMENT ? ORT_INVALID_ARGUMENT : ORT_EP_FAIL;
  const char* msg = b200_last_error();
  return api->CreateStatus(code, msg && *msg ? msg : "B200 execution provider failure");
}

// An OrtStatus returned by ORT to the glue: released here and re-raised with its message.
void check_ort(const OrtApi* api, OrtStatus* st, const char* what) {
  if (!st) return;
  const char* m = api->GetErrorMessage(st);
  std::string msg = std::string("B200 EP: ") + what + " failed: " + (m ? m : "");
  api->ReleaseStatus(st);
  raise(ORT_EP_FAIL, msg);
}

// Every callback body runs inside this: nothing throws across the C ABI (the reference's
// guard_ffi_status, lib.rs:53-92).
template <class F>
OrtStatus* guarded(const OrtApi* api, const char* where, F&& body) noexcept {
  try {
    return body();
  } catch (const OrtError& e) {
    return api->CreateStatus(e.code, e.msg.c_str());
  } catch (const B200Failure& e) {
    return b200_status(api, e.rc);
  } catch (const std::bad_alloc&) {
    return api->CreateStatus(ORT_EP_FAIL, (std::string("B200 EP: ") + where + ": out of host memory").c_str());
  } catch (const std::exception& e) {
    return api->CreateStatus(ORT_EP_FAIL, (std::string("B200 EP: ") + where + ": " + e.what()).c_str());
  } catch (...) {
    return api->CreateStatus(ORT_EP_FAIL, (std::string("B200 EP: ") + where + ": unknown failure").c_str());
  }
}

// ---------------------------------------------------------------------------------------------
// reading ORT graphs into the plain node descriptions of b200_paged.h
// ---------------------------------------------------------------------------------------------
struct GraphReader {
  const OrtApi* api;

  std::vector<const OrtNode*> nodes(const OrtGraph* graph) const {
    size_t count = 0;
    check_ort(api, api->Graph_GetNumNodes(graph, &count), "Graph_GetNumNodes");
    std::vector<const OrtNode*> out(count);
    if (count) check_ort(api, api->Graph_GetNodes(graph, out.data(), count), "Graph_GetNodes");
    return out;
  }

  using StringGetter = OrtStatus*(ORT_API_CALL*)(const OrtNode*, const char**) NO_EXCEPTION;
  std::string node_string(const OrtNode* node, StringGetter get, const char* what) const {
    const char* s = nullptr;
    check_ort(api, get(node, &s), what);
    return s ? s : "";
  }
  std::string op_type(const OrtNode* n) const { return node_string(n, api->Node_GetOperatorType, "Node_GetOperatorType"); }
  std::string domain(const OrtNode* n) const { return node_string(n, api->Node_GetDomain, "Node_GetDomain"); }
  std::string name(const OrtNode* n) const { return node_string(n, api->Node_GetName, "Node_GetName"); }

  std::vector<const OrtValueInfo*> inputs(const OrtNode* node) const {
    size_t count = 0;
    check_ort(api, api->Node_GetNumInputs(node, &count), "Node_GetNumInputs");
    std::vector<const OrtValueInfo*> out(count);
    if (count) check_ort(api, api->Node_GetInputs(node, out.data(), count), "Node_GetInputs");
    return out;
  }
  std::vector<const OrtValueInfo*> outputs(const OrtNode* node) const {
    size_t count = 0;
    check_ort(api, api->Node_GetNumOutputs(node, &count), "Node_GetNumOutputs");
    std::vector<const OrtValueInfo*> out(count);
    if (count) check_ort(api, api->Node_GetOutputs(node, out.data(), count), "Node_GetOutputs");
    return out;
  }

  std::string value_name(const OrtValueInfo* vi) const {
    if (!vi) return "";
    const char* s = nullptr;
    check_ort(api, api->GetValueInfoName(vi, &s), "GetValueInfoName");
    return s ? s : "";
  }

  // An absent optional input or output (null value info or empty name) stays present = 0; a
  // value without tensor type information gets dtype 0 and rank -1 (the claim declines it).
  void tensor_info(const OrtValueInfo* vi, B200TensorInfo* t) const {
    std::memset(t, 0, sizeof *t);
    if (!vi || value_name(vi).empty()) return;
    t->present = 1;
    t->rank = -1;
    const OrtTypeInfo* type = nullptr;
    OrtStatus* st = api->GetValueInfoTypeInfo(vi, &type);
    if (st || !type) {
      if (st) api->ReleaseStatus(st);
      return;
    }
    ONNXType kind = ONNX_TYPE_UNKNOWN;
    check_ort(api, api->GetOnnxTypeFromTypeInfo(type, &kind), "GetOnnxTypeFromTypeInfo");
    if (kind != ONNX_TYPE_TENSOR) return;
    const OrtTensorTypeAndShapeInfo* info = nullptr;
    check_ort(api, api->CastTypeInfoToTensorInfo(type, &info), "CastTypeInfoToTensorInfo");
    if (!info) return;
    ONNXTensorElementDataType dt = ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED;
    check_ort(api, api->GetTensorElementType(info, &dt), "GetTensorElementType");
    t->dtype = static_cast<int32_t>(dt);  // ORT's element types are ONNX's numbering, as B200_DTYPE_*
    size_t rank = 0;
    check_ort(api, api->GetDimensionsCount(info, &rank), "GetDimensionsCount");
    std::vector<int64_t> dims(rank);
    if (rank) check_ort(api, api->GetDimensions(info, dims.data(), rank), "GetDimensions");
    t->rank = static_cast<int32_t>(rank);
    for (size_t i = 0; i < rank && i < B200_MAX_RANK; ++i) t->shape[i] = dims[i] < 0 ? -1 : dims[i];
  }

  // Attributes: absent (or of another type) leaves the default, like the reference's readers
  // (registry.rs:780-1060).
  const OrtOpAttr* attr(const OrtNode* node, const char* key, OrtOpAttrType want) const {
    const OrtOpAttr* a = nullptr;
    OrtStatus* st = api->Node_GetAttributeByName(node, key, &a);
    if (st) {
      api->ReleaseStatus(st);
      return nullptr;
    }
    if (!a) return nullptr;
    OrtOpAttrType type = ORT_OP_ATTR_UNDEFINED;
    st = api->OpAttr_GetType(a, &type);
    if (st) {
      api->ReleaseStatus(st);
      return nullptr;
    }
    return type == want ? a : nullptr;
  }
  bool int_attr(const OrtNode* node, const char* key, int64_t* value) const {
    const OrtOpAttr* a = attr(node, key, ORT_OP_ATTR_INT);
    if (!a) return false;
    int64_t v = 0;
    size_t got = 0;
    OrtStatus* st = api->ReadOpAttr(a, ORT_OP_ATTR_INT, &v, sizeof v, &got);
    if (st) {
      api->ReleaseStatus(st);
      return false;
    }
    *value = v;
    return true;
  }
  int64_t int_or(const OrtNode* node, const char* key, int64_t fallback) const {
    int64_t v = fallback;
    return int_attr(node, key, &v) ? v : fallback;
  }
  bool float_attr(const OrtNode* node, const char* key, float* value) const {
    const OrtOpAttr* a = attr(node, key, ORT_OP_ATTR_FLOAT);
    if (!a) return false;
    float v = 0.f;
    size_t got = 0;
    OrtStatus* st = api->ReadOpAttr(a, ORT_OP_ATTR_FLOAT, &v, sizeof v, &got);
    if (st) {
      api->ReleaseStatus(st);
      return false;
    }
    *value = v;
    return true;
  }
  // A STRING attribute into a fixed field (truncated to the field; the claim compares the
  // known values, all shorter than the field).
  void string_attr(const OrtNode* node, const char* key, char* field, size_t field_len) const {
    std::memset(field, 0, field_len);
    const OrtOpAttr* a = attr(node, key, ORT_OP_ATTR_STRING);
    if (!a) return;
    size_t need = 0;
    OrtStatus* st = api->ReadOpAttr(a, ORT_OP_ATTR_STRING, nullptr, 0, &need);
    if (st) api->ReleaseStatus(st);  // the size query reports the size through `need`
    if (need == 0) return;
    std::string buf(need, '\0');
    size_t got = 0;
    st = api->ReadOpAttr(a, ORT_OP_ATTR_STRING, &buf[0], need, &got);
    if (st) {
      api->ReleaseStatus(st);
      return;
    }
    buf.resize(std::min(got, need));
    while (!buf.empty() && buf.back() == '\0') buf.pop_back();
    std::memcpy(field, buf.data(), std::min(buf.size(), field_len - 1));
  }
};

enum class OpKind { kNone, kPaged, kGqa };

OpKind op_kind(const GraphReader& g, const OrtNode* node) {
  if (g.domain(node) != kMsDomain) return OpKind::kNone;
  const std::string op = g.op_type(node);
  if (op == "PagedAttention") return OpKind::kPaged;
  if (op == "GroupQueryAttention") return OpKind::kGqa;
  return OpKind::kNone;
}

// com.microsoft.PagedAttention: 17 inputs, 3 outputs; attribute defaults as the reference reads
// them (attention.rs:3857-3935, :4384-4645).
void describe_paged(const GraphReader& g, const OrtNode* node, B200NodeInfo* n) {
  std::memset(n, 0, sizeof *n);
  const auto ins = g.inputs(node), outs = g.outputs(node);
  n->num_inputs = static_cast<int32_t>(ins.size());
  n->num_outputs = static_cast<int32_t>(outs.size());
  for (size_t i = 0; i < ins.size() && i < 17; ++i) g.tensor_info(ins[i], &n->inputs[i]);
  for (size_t i = 0; i < outs.size() && i < 3; ++i) g.tensor_info(outs[i], &n->outputs[i]);
  n->num_heads = g.int_or(node, "num_heads", 0);
  n->kv_num_heads = g.int_or(node, "kv_num_heads", 0);
  n->is_causal = g.int_or(node, "is_causal", 1);
  n->local_window_size = g.int_or(node, "local_window_size", -1);
  n->do_rotary = g.int_or(node, "do_rotary", 0);
  n->rotary_interleaved = g.int_or(node, "rotary_interleaved", 0);
  n->rotary_offset = g.int_or(node, "rotary_offset", 0);
  n->v_head_size = g.int_or(node, "v_head_size", 0);
  n->has_scale = g.float_attr(node, "scale", &n->scale) ? 1 : 0;
  if (!g.float_attr(node, "softcap", &n->softcap)) n->softcap = 0.f;
  if (!g.float_attr(node, "qk_norm_epsilon", &n->qk_norm_epsilon)) n->qk_norm_epsilon = 0.f;
  g.string_attr(node, "kv_cache_layout", n->kv_cache_layout, sizeof n->kv_cache_layout);
  g.string_attr(node, "k_quant_type", n->k_quant_type, sizeof n->k_quant_type);
  g.string_attr(node, "v_quant_type", n->v_quant_type, sizeof n->v_quant_type);
  g.string_attr(node, "k_cache_dtype", n->k_cache_dtype, sizeof n->k_cache_dtype);
  g.string_attr(node, "v_cache_dtype", n->v_cache_dtype, sizeof n->v_cache_dtype);
}

// com.microsoft.GroupQueryAttention: 16 inputs, 4 outputs (attention.rs:2407-2754).
void describe_gqa(const GraphReader& g, const OrtNode* node, B200GqaNodeInfo* n) {
  std::memset(n, 0, sizeof *n);
  const auto ins = g.inputs(node), outs = g.outputs(node);
  n->num_inputs = static_cast<int32_t>(ins.size());
  n->num_outputs = static_cast<int32_t>(outs.size());
  for (size_t i = 0; i < ins.size() && i < 16; ++i) g.tensor_info(ins[i], &n->inputs[i]);
  for (size_t i = 0; i < outs.size() && i < 4; ++i) g.tensor_info(outs[i], &n->outputs[i]);
  n->num_heads = g.int_or(node, "num_heads", 0);
  n->kv_num_heads = g.int_or(node, "kv_num_heads", 0);
  n->has_causal = g.int_attr(node, "causal", &n->causal) ? 1 : 0;
  if (!n->has_causal) n->causal = 1;
  n->has_local_window_size = g.int_attr(node, "local_window_size", &n->local_window_size) ? 1 : 0;
  if (!n->has_local_window_size) n->local_window_size = -1;
  n->has_smooth_softmax = g.int_attr(node, "smooth_softmax", &n->smooth_softmax) ? 1 : 0;
  if (!n->has_smooth_softmax) n->smooth_softmax = -1;
  n->do_rotary = g.int_or(node, "do_rotary", 0);
  n->rotary_interleaved = g.int_or(node, "rotary_interleaved", 0);
  n->sliding_window_cache = g.int_or(node, "sliding_window_cache", 0);
  n->qk_output = g.int_or(node, "qk_output", 0);
  n->kv_cache_bit_width = g.int_or(node, "kv_cache_bit_width", 0);
  if (!g.float_attr(node, "softcap", &n->softcap)) n->softcap = 0.f;
  n->has_scale = g.float_attr(node, "scale", &n->scale) ? 1 : 0;
  n->has_qk_norm_epsilon = g.float_attr(node, "qk_norm_epsilon", &n->qk_norm_epsilon) ? 1 : 0;
  g.string_attr(node, "k_quant_type", n->k_quant_type, sizeof n->k_quant_type);
  g.string_attr(node, "v_quant_type", n->v_quant_type, sizeof n->v_quant_type);
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// factory, EP, allocator and data transfer state
// ---------------------------------------------------------------------------------------------
namespace {

struct B200Factory {
  OrtEpFactory base;  // first member: ORT's pointer is this object's pointer
  const OrtApi* api = nullptr;
  const OrtEpApi* ep_api = nullptr;
  std::string name;
  int32_t device = 0;  // CUDA ordinal (ONNXRUNTIME_EP_B200_DEVICE_ID, default 0)
  std::mutex mu;
  std::vector<OrtMemoryInfo*> infos;  // registered with EP devices, released with the factory
};

struct B200Ep {
  OrtEp base;
  B200Factory* factory = nullptr;
  const OrtApi* api = nullptr;
  const OrtEpApi* ep_api = nullptr;
  std::string name;
  B200EpOptions options{};
  OrtMemoryInfo* memory_info = nullptr;
  std::mutex mu;
  void* stream = nullptr;  // created by the first Compute (EP creation needs no GPU)
  std::string report;      // one line per attention node seen by the last GetCapability

  void* compute_stream() {
    std::lock_guard<std::mutex> lock(mu);
    if (!stream) check_b200(b200_ep_stream_create(options.device_id, &stream));
    return stream;
  }
};

struct B200Allocator {
  OrtAllocator base;
  const OrtApi* api = nullptr;
  OrtMemoryInfo* info = nullptr;
  int32_t device = 0;
};

struct B200Transfer {
  OrtDataTransferImpl base;
  const OrtApi* api = nullptr;
  const OrtEpApi* ep_api = nullptr;
  OrtMemoryInfo* info = nullptr;
  const OrtMemoryDevice* memory_device = nullptr;
  int32_t device = 0;
};

OrtMemoryInfo* create_memory_info(const OrtApi* api, int32_t device) {
  OrtMemoryInfo* info = nullptr;
  check_ort(api,
            api->CreateMemoryInfo_V2(kMemoryName, OrtMemoryInfoDeviceType_GPU, kNvidiaVendorId, device,
                                     OrtDeviceMemoryType_DEFAULT, 256, OrtDeviceAllocator, &info),
            "CreateMemoryInfo_V2");
  return info;
}

// ---- tensors of one Compute ----------------------------------------------------------------
struct Bound {
  bool present = false;
  void* data = nullptr;  // where ORT holds the tensor
  void* dev = nullptr;   // what the kernels read and write (data, or a staging slot)
  std::vector<int64_t> shape;
  int32_t dtype = 0;
  size_t bytes = 0;
  bool on_device = false;
  int64_t dim(size_t i) const { return i < shape.size() ? shape[i] : 0; }
  int32_t dim32(size_t i) const {
    const int64_t d = dim(i);
    if (d < 0 || d > INT32_MAX) raise(ORT_INVALID_ARGUMENT, "B200 EP: tensor dimension out of the int32 range");
    return static_cast<int32_t>(d);
  }
};

void read_value(const OrtApi* api, const OrtValue* v, Bound* b) {
  OrtTensorTypeAndShapeInfo* info = nullptr;
  check_ort(api, api->GetTensorTypeAndShape(v, &info), "GetTensorTypeAndShape");
  try {
    size_t rank = 0;
    check_ort(api, api->GetDimensionsCount(info, &rank), "GetDimensionsCount");
    b->shape.assign(rank, 0);
    if (rank) check_ort(api, api->GetDimensions(info, b->shape.data(), rank), "GetDimensions");
    ONNXTensorElementDataType dt = ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED;
    check_ort(api, api->GetTensorElementType(info, &dt), "GetTensorElementType");
    b->dtype = static_cast<int32_t>(dt);
  } catch (...) {
    api->ReleaseTensorTypeAndShapeInfo(info);
    throw;
  }
  api->ReleaseTensorTypeAndShapeInfo(info);
  check_ort(api, api->GetTensorSizeInBytes(v, &b->bytes), "GetTensorSizeInBytes");
  const void* data = nullptr;
  check_ort(api, api->GetTensorData(v, &data), "GetTensorData");
  b->data = const_cast<void*>(data);  // caches are updated in place, as the reference does
  int32_t dev = 0;
  check_b200(b200_ep_is_device_pointer(b->data, &dev));
  b->on_device = dev != 0 || b->bytes == 0;
  b->dev = b->on_device ? b->data : nullptr;
  b->present = true;
}

// Device staging for tensors ORT handed over in host memory: one buffer per compiled node, grown
// on demand.  Every Compute ends synchronised, so a new Compute finds it idle.
struct Staging {
  int32_t device = 0;
  void* base = nullptr;
  size_t capacity = 0;
  size_t used = 0;
  std::vector<Bound*> to_host;  // staged tensors copied back after the kernels

  ~Staging() { b200_ep_device_free(device, base); }
  static size_t round_up(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }
  void plan(std::initializer_list<Bound*> tensors) {
    size_t need = 0;
    for (Bound* b : tensors)
      if (b && b->present && !b->on_device) need += round_up(b->bytes);
    used = 0;
    to_host.clear();
    if (need <= capacity) return;
    check_b200(b200_ep_device_free(device, base));
    base = nullptr;
    capacity = 0;
    check_b200(b200_ep_device_alloc(device, need, &base));
    capacity = need;
  }
  // Give a host tensor its device slot; inputs are copied in, `write_back` ones out again.
  void place(Bound* b, bool copy_in, bool write_back, void* stream) {
    if (!b->present || b->on_device) return;
    b->dev = static_cast<char*>(base) + used;
    used += round_up(b->bytes);
    if (copy_in) check_b200(b200_ep_copy(device, b->dev, b->data, b->bytes, stream));
    if (write_back) to_host.push_back(b);
  }
  void finish(void* stream) {
    for (Bound* b : to_host) check_b200(b200_ep_copy(device, b->data, b->dev, b->bytes, stream));
  }
};

struct ComputeInfo {
  OrtNodeComputeInfo base;
  B200Ep* ep = nullptr;
  OpKind kind = OpKind::kNone;
  B200EpNode* node = nullptr;
  B200NodeInfo paged{};
  B200GqaNodeInfo gqa{};
  std::vector<int> in_index;   // node input slot -> fused-node input index, -1 when absent
  std::vector<int> out_index;  // node output slot -> fused-node output index, -1 when absent
  std::mutex mu;
  Staging staging;

  ~ComputeInfo() {
    if (node) b200_ep_node_destroy(node);
  }

  // Input `slot` of the node, or an absent Bound.
  Bound input(OrtKernelContext* kctx, size_t slot) {
    Bound b;
    if (slot >= in_index.size() || in_index[slot] < 0) return b;
    const OrtValue* v = nullptr;
    check_ort(ep->api, ep->api->KernelContext_GetInput(kctx, static_cast<size_t>(in_index[slot]), &v),
              "KernelContext_GetInput");
    if (v) read_value(ep->api, v, &b);
    return b;
  }
  // Output `slot` with `shape`, or an absent Bound when the node does not produce it.
  Bound output(OrtKernelContext* kctx, size_t slot, const std::vector<int64_t>& shape) {
    Bound b;
    if (slot >= out_index.size() || out_index[slot] < 0) return b;
    OrtValue* v = nullptr;
    check_ort(ep->api,
              ep->api->KernelContext_GetOutput(kctx, static_cast<size_t>(out_index[slot]), shape.data(), shape.size(),
                                               &v),
              "KernelContext_GetOutput");
    if (!v) raise(ORT_EP_FAIL, "B200 EP: ORT returned no tensor for a requested output");
    read_value(ep->api, v, &b);
    return b;
  }

  void run(OrtKernelContext* kctx);
  void run_paged(OrtKernelContext* kctx, void* stream);
  void run_gqa(OrtKernelContext* kctx, void* stream);
};

}  // namespace

// ---------------------------------------------------------------------------------------------
// Compute
// ---------------------------------------------------------------------------------------------
namespace {

void ComputeInfo::run(OrtKernelContext* kctx) {
  std::lock_guard<std::mutex> lock(mu);
  void* stream = ep->compute_stream();
  staging.device = ep->options.device_id;
  if (kind == OpKind::kPaged)
    run_paged(kctx, stream);
  else
    run_gqa(kctx, stream);
  check_b200(b200_ep_stream_sync(stream));
}

// PagedAttention (attention.rs:3857-4382): inputs 0-16 as in B200NodeInfo; outputs 0 (attention,
// [num_tokens, num_heads * head_size]) and 1 / 2 (the updated caches).  The caches are updated in
// place in the input buffers, as the reference writes its patches back into the inputs
// (engine.rs:1212-1364); a cache output that ORT did not alias to its input gets a copy of the
// whole updated cache.
void ComputeInfo::run_paged(OrtKernelContext* kctx, void* stream) {
  Bound in[17];
  for (size_t i = 0; i < 17; ++i) in[i] = input(kctx, i);
  const Bound &q = in[0], &kc = in[3], &vc = in[4];
  // LATENT (attention.rs:3862-3867): one kv head, no value / value cache; values are key prefixes
  const bool latent = std::strncmp(paged.kv_cache_layout, "LATENT", sizeof paged.kv_cache_layout) == 0;
  if (!q.present || !kc.present || (!latent && !vc.present) || !in[5].present || !in[6].present || !in[7].present)
    raise(ORT_INVALID_ARGUMENT, "PagedAttention: query, caches and positional inputs 5-7 must be present");
  if (q.shape.size() != 2 || kc.shape.size() != 4 || in[6].shape.size() != 1 || in[7].shape.size() != 2)
    raise(ORT_INVALID_ARGUMENT, "PagedAttention: query must be rank 2, caches rank 4, past_seqlens rank 1 and "
                                "block_table rank 2");
  const int64_t H = paged.num_heads, KV = paged.kv_num_heads;
  const bool packed = !latent && !in[1].present && !in[2].present;
  const int64_t heads_in_query = packed ? H + 2 * KV : H;
  if (heads_in_query <= 0 || q.dim(1) % heads_in_query)
    raise(ORT_INVALID_ARGUMENT, "PagedAttention: query hidden size does not match the head count");
  const int64_t D = q.dim(1) / heads_in_query;
  const int64_t DV = latent && paged.v_head_size > 0 ? paged.v_head_size : D;

  Bound out0 = output(kctx, 0, {q.dim(0), H * DV});
  Bound out1 = output(kctx, 1, kc.shape);
  Bound out2 = output(kctx, 2, vc.shape);

  staging.plan({&in[0], &in[1], &in[2], &in[3], &in[4], &in[5], &in[6], &in[7], &in[8], &in[9], &in[10], &in[11],
                &in[12], &in[13], &in[14], &in[15], &out0, &out1, &out2});
  for (int i = 0; i < 17; ++i) staging.place(&in[i], true, /*write_back=*/i == 3 || i == 4, stream);
  staging.place(&out0, false, true, stream);
  staging.place(&out1, false, true, stream);
  staging.place(&out2, false, true, stream);

  B200PagedTensors t{};
  t.query = in[0].dev;
  t.key = in[1].dev;
  t.value = in[2].dev;
  t.key_cache = in[3].dev;
  t.value_cache = in[4].dev;
  t.cumulative_sequence_length = static_cast<const int32_t*>(in[5].dev);
  t.past_seqlens = static_cast<const int32_t*>(in[6].dev);
  t.block_table = static_cast<const int32_t*>(in[7].dev);
  t.cos_cache = in[8].dev;
  t.sin_cache = in[9].dev;
  t.slot_mapping = static_cast<const int32_t*>(in[10].dev);
  t.head_sink = in[11].dev;
  t.q_norm_weight = in[12].dev;
  t.k_norm_weight = in[13].dev;
  t.k_scale = static_cast<const float*>(in[14].dev);
  t.v_scale = static_cast<const float*>(in[15].dev);
  t.output = out0.dev;
  // metadata that ORT handed over in host memory also feeds the host-side validation
  auto host = [](const Bound& b) { return b.present && !b.on_device ? static_cast<const int32_t*>(b.data) : nullptr; };
  t.host_cumulative_sequence_length = host(in[5]);
  t.host_past_seqlens = host(in[6]);
  t.host_block_table = host(in[7]);
  t.host_slot_mapping = host(in[10]);
  t.num_tokens = q.dim32(0);
  t.query_hidden = q.dim32(1);
  t.batch = in[6].dim32(0);
  t.num_blocks = kc.dim32(0);
  t.block_size = kc.dim32(1);
  t.max_blocks_per_seq = in[7].dim32(1);
  if (in[8].present) {
    t.rotary_positions = in[8].dim32(0);
    t.rotary_half_dim = in[8].dim32(1);
  }
  t.act_dtype = q.dtype;
  t.cache_dtype = kc.dtype;
  check_b200(b200_ep_node_compute_paged(node, &t, stream));

  // cache outputs ORT did not alias to the inputs receive the updated caches
  const Bound* cache_in[2] = {&in[3], &in[4]};
  const Bound* cache_out[2] = {&out1, &out2};
  for (int c = 0; c < 2; ++c) {
    const Bound& o = *cache_out[c];
    if (o.present && o.data != cache_in[c]->data)
      check_b200(b200_ep_copy(ep->options.device_id, o.dev, cache_in[c]->dev, o.bytes, stream));
  }
  staging.finish(stream);  // staged outputs and caches back to host memory
}

// Host copy of a small int tensor (GroupQueryAttention reads lengths and position ids on the
// host, as the reference does).
template <class T>
std::vector<T> host_values(const Bound& b, int32_t device) {
  std::vector<T> out(b.bytes / sizeof(T));
  if (out.empty()) return out;
  if (b.on_device)
    check_b200(b200_ep_copy(device, out.data(), b.data, out.size() * sizeof(T), nullptr));
  else
    std::memcpy(out.data(), b.data, out.size() * sizeof(T));
  return out;
}

// GroupQueryAttention (attention.rs:932-1454): inputs 0-15 as in B200GqaNodeInfo; outputs 0
// ([batch, seq, num_heads * head_size]) and 1 / 2 (present caches [batch, kv_heads,
// max(past capacity, total_sequence_length), head_size]; the past capacity for a sliding cache).
void ComputeInfo::run_gqa(OrtKernelContext* kctx, void* stream) {
  Bound in[16];
  for (size_t i = 0; i < 16; ++i) in[i] = input(kctx, i);
  const Bound& q = in[0];
  if (!q.present || !in[5].present || !in[6].present)
    raise(ORT_INVALID_ARGUMENT, "GroupQueryAttention: query, seqlens_k and total_sequence_length must be present");
  if (q.shape.size() != 3)
    raise(ORT_INVALID_ARGUMENT, "GroupQueryAttention: query must have rank 3");
  const int32_t device = ep->options.device_id;
  const int64_t H = gqa.num_heads, KV = gqa.kv_num_heads;
  const bool packed = !in[1].present && !in[2].present;
  const int64_t heads_in_query = packed ? H + 2 * KV : H;
  if (heads_in_query <= 0 || q.dim(2) % heads_in_query)
    raise(ORT_INVALID_ARGUMENT, "GroupQueryAttention: query hidden size does not match the head count");
  const int64_t B = q.dim(0), S = q.dim(1), D = q.dim(2) / heads_in_query;
  const std::vector<int32_t> seqlens = host_values<int32_t>(in[5], device);
  const std::vector<int32_t> total = host_values<int32_t>(in[6], device);
  if (total.empty()) raise(ORT_INVALID_ARGUMENT, "GroupQueryAttention: total_sequence_length must hold one value");
  std::vector<int64_t> ids;
  if (in[9].present) ids = host_values<int64_t>(in[9], device);
  const int64_t cap = in[3].present ? in[3].dim(2) : 0;
  // present: the past's capacity for a sliding cache (its rows move down), else room for total
  const int64_t pcap = gqa.sliding_window_cache ? cap : std::max<int64_t>(cap, total[0]);
  // integer caches (kv_cache_bit_width): present rows keep the past's stored width
  const bool int_cache = in[3].present && (in[3].dtype == B200_DTYPE_INT8 || in[3].dtype == B200_DTYPE_UINT8);
  const int64_t width = int_cache ? in[3].dim(3) : D;

  Bound out0 = output(kctx, 0, {B, S, H * D});
  Bound out1 = output(kctx, 1, {B, KV, pcap, width});
  Bound out2 = output(kctx, 2, {B, KV, pcap, width});
  Bound out3 = output(kctx, 3, {B, H, S, total[0]});  // qk_output diagnostics

  staging.plan({&in[0], &in[1], &in[2], &in[3], &in[4], &in[5], &in[7], &in[8], &in[9], &in[10], &in[11], &in[12],
                &in[13], &in[14], &in[15], &out0, &out1, &out2, &out3});
  for (int i : {0, 1, 2, 3, 4, 5, 7, 8, 9, 10, 11, 12, 13, 14, 15}) staging.place(&in[i], true, false, stream);
  staging.place(&out0, false, true, stream);
  staging.place(&out1, false, true, stream);
  staging.place(&out2, false, true, stream);
  staging.place(&out3, false, true, stream);

  B200GqaParams p{};
  p.head_size = static_cast<int32_t>(D);
  p.dtype = q.dtype;
  p.batch = q.dim32(0);
  p.seq = q.dim32(1);
  p.new_seq = packed ? p.seq : (in[1].present ? in[1].dim32(1) : 0);
  p.cap = static_cast<int32_t>(cap);
  p.present_cap = out1.present ? static_cast<int32_t>(pcap) : 0;
  p.total_sequence_length = total[0];
  p.query = in[0].dev;
  const size_t esz = q.dtype == B200_DTYPE_FLOAT ? 4 : 2;
  if (packed) {  // K and V columns of the packed rows
    p.query_row_stride = p.key_row_stride = p.value_row_stride = q.dim(2);
    p.key = static_cast<const char*>(in[0].dev) + static_cast<size_t>(H * D) * esz;
    p.value = static_cast<const char*>(in[0].dev) + static_cast<size_t>((H + KV) * D) * esz;
  } else {
    p.key = in[1].dev;
    p.value = in[2].dev;
  }
  p.past_key = in[3].dev;
  p.past_value = in[4].dev;
  p.present_key = out1.dev;
  p.present_value = out2.dev;
  p.seqlens_k = static_cast<const int32_t*>(in[5].dev);
  p.host_seqlens_k = seqlens.data();
  if (static_cast<int64_t>(seqlens.size()) < B)
    raise(ORT_INVALID_ARGUMENT, "GroupQueryAttention: seqlens_k must hold batch_size values");
  p.head_sink = in[11].dev;
  p.output_qk = out3.dev;        // with the node's qk_output mode
  if (int_cache) {               // with the node's k / v quant types
    p.cache_dtype = in[3].dtype;
    p.k_scale = static_cast<const float*>(in[12].dev);
    p.v_scale = static_cast<const float*>(in[13].dev);
  }
  p.q_norm_weight = in[14].dev;  // with k_norm_weight; epsilon from the node's attribute
  p.k_norm_weight = in[15].dev;
  if (in[10].present) {  // attention_bias [1|B, 1|H, S, total]
    if (in[10].shape.size() != 4)
      raise(ORT_EP_FAIL, "GroupQueryAttention: attention_bias must broadcast to [batch,heads,sequence,total]");
    p.attention_bias = in[10].dev;
    p.bias_batch = in[10].dim32(0);
    p.bias_heads = in[10].dim32(1);
    p.bias_seq = in[10].dim32(2);
    p.bias_total = in[10].dim32(3);
  }
  p.output = out0.dev;
  if (gqa.do_rotary && in[7].present) {
    p.rotary_dim = 2 * in[7].dim32(1);
    p.rotary_positions = in[7].dim32(0);
    p.cos_cache = in[7].dev;
    p.sin_cache = in[8].dev;
    if (in[9].present) {
      p.position_ids = static_cast<const int64_t*>(in[9].dev);
      p.host_position_ids = ids.data();
      p.position_ids_width = in[9].shape.size() == 2 ? in[9].dim32(1) : static_cast<int32_t>(ids.size());
    }
  }
  check_b200(b200_ep_node_compute_gqa(node, &p, stream));
  staging.finish(stream);
}

// ---------------------------------------------------------------------------------------------
// OrtNodeComputeInfo callbacks (runtime.rs:171-331)
// ---------------------------------------------------------------------------------------------
OrtStatus* ORT_API_CALL create_state(OrtNodeComputeInfo* self, OrtNodeComputeContext*, void** state) noexcept {
  *state = self;
  return nullptr;
}

OrtStatus* ORT_API_CALL compute(OrtNodeComputeInfo* self, void* state, OrtKernelContext* kctx) noexcept {
  ComputeInfo* info = static_cast<ComputeInfo*>(state ? state : static_cast<void*>(self));
  return guarded(info->ep->api, "Compute", [&]() -> OrtStatus* {
    info->run(kctx);
    return nullptr;
  });
}

void ORT_API_CALL release_state(OrtNodeComputeInfo*, void*) noexcept {}

// ---------------------------------------------------------------------------------------------
// allocator and data transfer (device.rs:409-640)
// ---------------------------------------------------------------------------------------------
void* ORT_API_CALL alloc_device(OrtAllocator* self, size_t size) noexcept {
  B200Allocator* a = reinterpret_cast<B200Allocator*>(self);
  void* p = nullptr;
  return b200_ep_device_alloc(a->device, size, &p) == B200_OK ? p : nullptr;
}

void ORT_API_CALL free_device(OrtAllocator* self, void* p) noexcept {
  B200Allocator* a = reinterpret_cast<B200Allocator*>(self);
  b200_ep_device_free(a->device, p);
}

const OrtMemoryInfo* ORT_API_CALL allocator_info(const OrtAllocator* self) noexcept {
  return reinterpret_cast<const B200Allocator*>(self)->info;
}

void ORT_API_CALL release_transfer(OrtDataTransferImpl* self) noexcept {
  B200Transfer* t = reinterpret_cast<B200Transfer*>(self);
  if (t->info) t->api->ReleaseMemoryInfo(t->info);
  delete t;
}

// Host <-> the EP's device and device <-> device (device.rs:509-527).
bool ORT_API_CALL can_copy(const OrtDataTransferImpl* self, const OrtMemoryDevice* src,
                           const OrtMemoryDevice* dst) noexcept {
  const B200Transfer* t = reinterpret_cast<const B200Transfer*>(self);
  auto ours = [&](const OrtMemoryDevice* d) { return t->ep_api->MemoryDevice_AreEqual(d, t->memory_device); };
  auto cpu = [&](const OrtMemoryDevice* d) {
    return t->ep_api->MemoryDevice_GetDeviceType(d) == OrtMemoryInfoDeviceType_CPU;
  };
  return (ours(src) && (cpu(dst) || ours(dst))) || (ours(dst) && cpu(src));
}

// One synchronous copy per tensor pair; shapes, element types and sizes must match.
OrtStatus* ORT_API_CALL copy_tensors(OrtDataTransferImpl* self, const OrtValue** src, OrtValue** dst, OrtSyncStream**,
                                     size_t count) noexcept {
  B200Transfer* t = reinterpret_cast<B200Transfer*>(self);
  return guarded(t->api, "data transfer", [&]() -> OrtStatus* {
    for (size_t i = 0; i < count; ++i) {
      Bound s, d;
      read_value(t->api, src[i], &s);
      read_value(t->api, dst[i], &d);
      if (s.shape != d.shape || s.dtype != d.dtype || s.bytes != d.bytes)
        raise(ORT_INVALID_ARGUMENT, "B200 device transfer requires matching shapes and dtypes");
      void* out = nullptr;
      check_ort(t->api, t->api->GetTensorMutableData(dst[i], &out), "GetTensorMutableData");
      check_b200(b200_ep_copy(t->device, out, s.data, s.bytes, nullptr));
    }
    return nullptr;
  });
}

// ---------------------------------------------------------------------------------------------
// OrtEp callbacks (ep.rs:76-150)
// ---------------------------------------------------------------------------------------------
B200Ep* ep_of(const OrtEp* p) { return reinterpret_cast<B200Ep*>(const_cast<OrtEp*>(p)); }

const char* ORT_API_CALL ep_get_name(const OrtEp* self) noexcept { return ep_of(self)->name.c_str(); }

OrtStatus* ORT_API_CALL ep_default_memory_device(const OrtEp* self, const OrtMemoryDevice** device) noexcept {
  B200Ep* ep = ep_of(self);
  *device = ep->memory_info ? ep->ep_api->MemoryInfo_GetMemoryDevice(ep->memory_info) : nullptr;
  return nullptr;
}

// Claim each PagedAttention / GroupQueryAttention node the predicates accept, as a fusion of its
// own (the reference fuses whole partitions, capability.rs:361-377; this EP accelerates only
// these nodes).  Constant initializers stay inputs of the fused node, so Compute sees every
// input in the node's order.
OrtStatus* ORT_API_CALL ep_get_capability(OrtEp* self, const OrtGraph* graph, OrtEpGraphSupportInfo* support) noexcept {
  B200Ep* ep = ep_of(self);
  return guarded(ep->api, "GetCapability", [&]() -> OrtStatus* {
    const GraphReader g{ep->api};
    std::string report;
    for (const OrtNode* node : g.nodes(graph)) {
      const OpKind kind = op_kind(g, node);
      if (kind == OpKind::kNone) continue;
      char reason[512] = {0};
      int claimed = 0;
      if (kind == OpKind::kPaged) {
        B200NodeInfo info;
        describe_paged(g, node, &info);
        claimed = b200_paged_attention_claim(&info, reason, sizeof reason);
      } else {
        B200GqaNodeInfo info;
        describe_gqa(g, node, &info);
        claimed = b200_group_query_attention_claim(&info, reason, sizeof reason);
      }
      report += g.name(node) + (claimed ? ": claimed\n" : std::string(": declined: ") + reason + "\n");
      if (!claimed) continue;
      OrtNodeFusionOptions options;
      std::memset(&options, 0, sizeof options);
      options.ort_version_supported = ORT_API_VERSION;
      options.drop_constant_initializers = false;
      const OrtNode* group[1] = {node};
      OrtStatus* st = ep->ep_api->EpGraphSupportInfo_AddNodesToFuse(support, group, 1, &options);
      if (st) return st;
    }
    std::lock_guard<std::mutex> lock(ep->mu);
    ep->report = report;
    return nullptr;
  });
}

// Node input / output slot -> index among the fused node's inputs / outputs, matched by value
// name (the fused node lists the values that cross its boundary, without absent optional ones).
std::vector<int> slot_map(const GraphReader& g, const std::vector<const OrtValueInfo*>& node_values,
                          const std::vector<const OrtValueInfo*>& fused_values, const char* what) {
  std::vector<std::string> fused_names;
  for (const OrtValueInfo* v : fused_values) fused_names.push_back(g.value_name(v));
  std::vector<int> map(node_values.size(), -1);
  for (size_t i = 0; i < node_values.size(); ++i) {
    const std::string name = g.value_name(node_values[i]);
    if (name.empty()) continue;
    auto it = std::find(fused_names.begin(), fused_names.end(), name);
    if (it == fused_names.end())
      raise(ORT_EP_FAIL, std::string("B200 EP: ") + what + " '" + name + "' is not on the fused node's boundary");
    map[i] = static_cast<int>(it - fused_names.begin());
  }
  return map;
}

ComputeInfo* compile_one(B200Ep* ep, const OrtGraph* graph, const OrtNode* fused) {
  const GraphReader g{ep->api};
  const std::vector<const OrtNode*> nodes = g.nodes(graph);
  if (nodes.size() != 1) raise(ORT_EP_FAIL, "B200 EP: a fused subgraph must hold exactly one attention node");
  const OrtNode* node = nodes[0];
  const OpKind kind = op_kind(g, node);
  if (kind == OpKind::kNone) raise(ORT_EP_FAIL, "B200 EP: the fused node is not an attention node this EP claims");
  ComputeInfo* info = new ComputeInfo;
  try {
    std::memset(&info->base, 0, sizeof info->base);
    info->base.ort_version_supported = ORT_API_VERSION;
    info->base.CreateState = create_state;
    info->base.Compute = compute;
    info->base.ReleaseState = release_state;
    info->ep = ep;
    info->kind = kind;
    info->staging.device = ep->options.device_id;
    if (kind == OpKind::kPaged) {
      describe_paged(g, node, &info->paged);
      check_b200(b200_ep_node_create_paged(&info->paged, &ep->options, &info->node));
    } else {
      describe_gqa(g, node, &info->gqa);
      check_b200(b200_ep_node_create_gqa(&info->gqa, &ep->options, &info->node));
    }
    info->in_index = slot_map(g, g.inputs(node), g.inputs(fused), "input");
    info->out_index = slot_map(g, g.outputs(node), g.outputs(fused), "output");
  } catch (...) {
    delete info;
    throw;
  }
  return info;
}

OrtStatus* ORT_API_CALL ep_compile(OrtEp* self, const OrtGraph** graphs, const OrtNode** fused_nodes, size_t count,
                                   OrtNodeComputeInfo** infos, OrtNode** /*ep_context_nodes*/) noexcept {
  B200Ep* ep = ep_of(self);
  for (size_t i = 0; i < count; ++i) infos[i] = nullptr;
  OrtStatus* st = guarded(ep->api, "Compile", [&]() -> OrtStatus* {
    for (size_t i = 0; i < count; ++i) infos[i] = &compile_one(ep, graphs[i], fused_nodes[i])->base;
    return nullptr;
  });
  if (st) {  // a failed Compile owns nothing afterwards
    for (size_t i = 0; i < count; ++i) {
      delete reinterpret_cast<ComputeInfo*>(infos[i]);
      infos[i] = nullptr;
    }
  }
  return st;
}

void ORT_API_CALL ep_release_infos(OrtEp*, OrtNodeComputeInfo** infos, size_t count) noexcept {
  for (size_t i = 0; i < count; ++i) delete reinterpret_cast<ComputeInfo*>(infos[i]);
}

// ---------------------------------------------------------------------------------------------
// OrtEpFactory callbacks (factory.rs:80-317)
// ---------------------------------------------------------------------------------------------
B200Factory* factory_of(const OrtEpFactory* p) {
  return reinterpret_cast<B200Factory*>(const_cast<OrtEpFactory*>(p));
}

const char* ORT_API_CALL f_get_name(const OrtEpFactory* self) noexcept { return factory_of(self)->name.c_str(); }
const char* ORT_API_CALL f_get_vendor(const OrtEpFactory*) noexcept { return kVendor; }
uint32_t ORT_API_CALL f_get_vendor_id(const OrtEpFactory*) noexcept { return kNvidiaVendorId; }
const char* ORT_API_CALL f_get_version(const OrtEpFactory*) noexcept { return kVersion; }
bool ORT_API_CALL f_is_stream_aware(const OrtEpFactory*) noexcept { return false; }

// One EP device on the first NVIDIA GPU ORT offers, with the EP's device memory registered as
// its allocator (factory.rs:123-197; the reference falls back to the CPU device because MLX
// runs there too - these kernels need the GPU, so no GPU means no EP device).
OrtStatus* ORT_API_CALL f_get_supported_devices(OrtEpFactory* self, const OrtHardwareDevice* const* devices,
                                                size_t num_devices, OrtEpDevice** ep_devices, size_t max_ep_devices,
                                                size_t* num_ep_devices) noexcept {
  B200Factory* f = factory_of(self);
  return guarded(f->api, "GetSupportedDevices", [&]() -> OrtStatus* {
    *num_ep_devices = 0;
    const OrtHardwareDevice* gpu = nullptr;
    for (size_t i = 0; i < num_devices && !gpu; ++i) {
      if (f->api->HardwareDevice_Type(devices[i]) == OrtHardwareDeviceType_GPU &&
          f->api->HardwareDevice_VendorId(devices[i]) == kNvidiaVendorId)
        gpu = devices[i];
    }
    if (!gpu || max_ep_devices < 1) return nullptr;
    OrtEpDevice* dev = nullptr;
    OrtStatus* st = f->ep_api->CreateEpDevice(self, gpu, nullptr, nullptr, &dev);
    if (st) return st;
    OrtMemoryInfo* info = create_memory_info(f->api, f->device);
    st = f->ep_api->EpDevice_AddAllocatorInfo(dev, info);
    if (st) {
      f->api->ReleaseMemoryInfo(info);
      return st;
    }
    {
      std::lock_guard<std::mutex> lock(f->mu);
      f->infos.push_back(info);
    }
    ep_devices[0] = dev;
    *num_ep_devices = 1;
    return nullptr;
  });
}

// The ep.b200.* entries of the session (config.rs:18-54), then the environment, strictly parsed.
B200EpOptions session_options(const OrtApi* api, const OrtSessionOptions* options) {
  static const char* const kKeys[] = {"ep.b200.kv_pool_bytes", "ep.b200.num_gpus", "ep.b200.device_id",
                                      "ep.b200.decode_min_tiles_per_warp", "ep.b200.force_generic",
                                      "ep.b200.check_status"};
  std::vector<std::string> keys, values;
  for (const char* key : kKeys) {
    if (!options) break;
    int present = 0;
    check_ort(api, api->HasSessionConfigEntry(options, key, &present), "HasSessionConfigEntry");
    if (!present) continue;
    size_t size = 0;
    check_ort(api, api->GetSessionConfigEntry(options, key, nullptr, &size), "GetSessionConfigEntry");
    std::string value(size, '\0');
    if (size) check_ort(api, api->GetSessionConfigEntry(options, key, &value[0], &size), "GetSessionConfigEntry");
    value.resize(strnlen(value.c_str(), value.size()));
    keys.push_back(key);
    values.push_back(value);
  }
  std::vector<const char*> k, v;
  for (size_t i = 0; i < keys.size(); ++i) {
    k.push_back(keys[i].c_str());
    v.push_back(values[i].c_str());
  }
  B200EpOptions out{};
  check_b200(b200_ep_options_parse(k.data(), v.data(), k.size(), &out));
  return out;
}

OrtStatus* ORT_API_CALL f_create_ep(OrtEpFactory* self, const OrtHardwareDevice* const*,
                                    const OrtKeyValuePairs* const*, size_t num_devices,
                                    const OrtSessionOptions* options, const OrtLogger*, OrtEp** out) noexcept {
  B200Factory* f = factory_of(self);
  *out = nullptr;
  return guarded(f->api, "CreateEp", [&]() -> OrtStatus* {
    if (num_devices != 1) raise(ORT_INVALID_ARGUMENT, f->name + " expects exactly one device");
    const B200EpOptions opts = session_options(f->api, options);
    if (opts.device_id != f->device)
      raise(ORT_INVALID_ARGUMENT, "B200 session option ep.b200.device_id: " + std::to_string(opts.device_id) +
                                      " differs from the device the EP registered its memory on (" +
                                      std::to_string(f->device) + ", ONNXRUNTIME_EP_B200_DEVICE_ID)");
    B200Ep* ep = new B200Ep;
    std::memset(&ep->base, 0, sizeof ep->base);
    ep->base.ort_version_supported = ORT_API_VERSION;
    ep->base.GetName = ep_get_name;
    ep->base.GetCapability = ep_get_capability;
    ep->base.Compile = ep_compile;
    ep->base.ReleaseNodeComputeInfos = ep_release_infos;
    ep->base.GetDefaultMemoryDevice = ep_default_memory_device;
    ep->factory = f;
    ep->api = f->api;
    ep->ep_api = f->ep_api;
    ep->name = f->name;
    ep->options = opts;
    try {
      ep->memory_info = create_memory_info(f->api, f->device);
    } catch (...) {
      delete ep;
      throw;
    }
    *out = &ep->base;
    return nullptr;
  });
}

void ORT_API_CALL f_release_ep(OrtEpFactory*, OrtEp* p) noexcept {
  if (!p) return;
  B200Ep* ep = ep_of(p);
  if (ep->stream) b200_ep_stream_destroy(ep->options.device_id, ep->stream);
  if (ep->memory_info) ep->api->ReleaseMemoryInfo(ep->memory_info);
  delete ep;
}

// The device allocator for memory infos named "B200"; ORT's default for anything else
// (factory.rs:267-288).
OrtStatus* ORT_API_CALL f_create_allocator(OrtEpFactory* self, const OrtMemoryInfo* memory_info,
                                           const OrtKeyValuePairs*, OrtAllocator** allocator) noexcept {
  B200Factory* f = factory_of(self);
  *allocator = nullptr;
  return guarded(f->api, "CreateAllocator", [&]() -> OrtStatus* {
    const char* name = nullptr;
    OrtStatus* st = f->api->MemoryInfoGetName(memory_info, &name);
    if (st) return st;
    if (!name || std::strcmp(name, kMemoryName) != 0) return nullptr;
    B200Allocator* a = new B200Allocator;
    std::memset(&a->base, 0, sizeof a->base);
    a->base.version = ORT_API_VERSION;
    a->base.Alloc = alloc_device;
    a->base.Reserve = alloc_device;
    a->base.Free = free_device;
    a->base.Info = allocator_info;
    a->api = f->api;
    a->device = f->device;
    try {
      a->info = create_memory_info(f->api, f->device);
    } catch (...) {
      delete a;
      throw;
    }
    *allocator = &a->base;
    return nullptr;
  });
}

void ORT_API_CALL f_release_allocator(OrtEpFactory*, OrtAllocator* allocator) noexcept {
  if (!allocator) return;
  B200Allocator* a = reinterpret_cast<B200Allocator*>(allocator);
  if (a->info) a->api->ReleaseMemoryInfo(a->info);
  delete a;
}

OrtStatus* ORT_API_CALL f_create_data_transfer(OrtEpFactory* self, OrtDataTransferImpl** out) noexcept {
  B200Factory* f = factory_of(self);
  *out = nullptr;
  return guarded(f->api, "CreateDataTransfer", [&]() -> OrtStatus* {
    B200Transfer* t = new B200Transfer;
    std::memset(&t->base, 0, sizeof t->base);
    t->base.ort_version_supported = ORT_API_VERSION;
    t->base.Release = release_transfer;
    t->base.CanCopy = can_copy;
    t->base.CopyTensors = copy_tensors;
    t->api = f->api;
    t->ep_api = f->ep_api;
    t->device = f->device;
    try {
      t->info = create_memory_info(f->api, f->device);
    } catch (...) {
      delete t;
      throw;
    }
    t->memory_device = f->ep_api->MemoryInfo_GetMemoryDevice(t->info);
    if (!t->memory_device) {
      release_transfer(&t->base);
      raise(ORT_EP_FAIL, "B200 device transfer could not obtain its memory-device identity; use ONNX Runtime "
                         "1.31 or newer");
    }
    *out = &t->base;
    return nullptr;
  });
}

OrtStatus* ORT_API_CALL f_create_sync_stream(OrtEpFactory*, const OrtMemoryDevice*, const OrtKeyValuePairs*,
                                             OrtSyncStreamImpl** stream) noexcept {
  *stream = nullptr;
  return nullptr;
}

}  // namespace

// ---------------------------------------------------------------------------------------------
// library entry points (lib.rs:100-178)
// ---------------------------------------------------------------------------------------------
B200_SHELL_API OrtStatus* CreateEpFactories(const char* registration_name, const OrtApiBase* ort_api_base,
                                            const OrtLogger* /*default_logger*/, OrtEpFactory** factories,
                                            size_t max_factories, size_t* num_factories) {
  const OrtApi* api = ort_api_base->GetApi(ORT_API_VERSION);
  if (!api) {
    // an older runtime: report through its version-1 table, whose CreateStatus every version has
    const OrtApi* legacy = ort_api_base->GetApi(1);
    return legacy->CreateStatus(ORT_INVALID_ARGUMENT,
                                "B200ExecutionProvider requires ONNX Runtime 1.31 or newer (ORT_API_VERSION >= 31)");
  }
  return guarded(api, "CreateEpFactories", [&]() -> OrtStatus* {
    *num_factories = 0;
    if (max_factories < 1) raise(ORT_INVALID_ARGUMENT, "B200ExecutionProvider needs room for one OrtEpFactory");
    B200EpOptions env{};
    check_b200(b200_ep_options_parse(nullptr, nullptr, 0, &env));  // environment only
    B200Factory* f = new B200Factory;
    std::memset(&f->base, 0, sizeof f->base);
    f->base.ort_version_supported = ORT_API_VERSION;
    f->base.GetName = f_get_name;
    f->base.GetVendor = f_get_vendor;
    f->base.GetVendorId = f_get_vendor_id;
    f->base.GetVersion = f_get_version;
    f->base.GetSupportedDevices = f_get_supported_devices;
    f->base.CreateEp = f_create_ep;
    f->base.ReleaseEp = f_release_ep;
    f->base.CreateAllocator = f_create_allocator;
    f->base.ReleaseAllocator = f_release_allocator;
    f->base.CreateDataTransfer = f_create_data_transfer;
    f->base.IsStreamAware = f_is_stream_aware;
    f->base.CreateSyncStreamForDevice = f_create_sync_stream;
    f->api = api;
    f->ep_api = api->GetEpApi();
    f->name = registration_name && *registration_name ? registration_name : kDefaultName;
    f->device = env.device_id;
    factories[0] = &f->base;
    *num_factories = 1;
    return nullptr;
  });
}

B200_SHELL_API OrtStatus* ReleaseEpFactory(OrtEpFactory* factory) {
  if (!factory) return nullptr;
  B200Factory* f = factory_of(factory);
  for (OrtMemoryInfo* info : f->infos) f->api->ReleaseMemoryInfo(info);
  delete f;
  return nullptr;
}

// Diagnostics (no counterpart in ORT's API): the last GetCapability's verdict per attention node,
// "<node name>: claimed" or "<node name>: declined: <reason>", one per line.  The string stays
// valid until the next GetCapability of this EP or its release.
B200_SHELL_API const char* b200_ep_shell_capability_report(const OrtEp* ep) {
  if (!ep) return "";
  B200Ep* e = ep_of(ep);
  std::lock_guard<std::mutex> lock(e->mu);
  return e->report.c_str();
}
