// Fake ONNX Runtime host for testing the B200 EP glue (onnxruntime-ep-mlx_b200/csrc/ep_shell.cpp)
// without ONNX Runtime.
//
// Implements the OrtApi / OrtEpApi members that onnxruntime_c_api.h in this folder declares over
// plain C++ objects (graphs, nodes, value infos, attributes, tensors, session options, memory
// infos), loads the glue library with dlopen and drives it the way ORT's plugin-EP host does:
// CreateEpFactories, GetSupportedDevices, CreateEp, GetCapability, Compile (building the fused
// node from the claimed node), CreateState / Compute / ReleaseState, CreateAllocator,
// CreateDataTransfer, ReleaseEp, ReleaseEpFactory.  The fake_* functions at the end are the
// test-facing C API (driven from tests/test_ep_shell_*.py through ctypes).
#include "onnxruntime_c_api.h"

#include <dlfcn.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#define FAKE_API extern "C" __attribute__((visibility("default")))

struct OrtStatus {
  OrtErrorCode code;
  std::string msg;
};
struct OrtTensorTypeAndShapeInfo {
  ONNXTensorElementDataType dtype = ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED;
  std::vector<int64_t> shape;
};
struct OrtTypeInfo {
  OrtTensorTypeAndShapeInfo tensor;
};
struct OrtValueInfo {
  std::string name;
  bool typed = true;
  OrtTypeInfo type;
};
struct OrtOpAttr {
  OrtOpAttrType type = ORT_OP_ATTR_UNDEFINED;
  int64_t i = 0;
  float f = 0.f;
  std::string s;
};
struct OrtNode {
  std::string op, domain, name;
  std::vector<OrtValueInfo*> inputs, outputs;  // nullptr = absent optional value
  std::map<std::string, OrtOpAttr> attrs;
  ~OrtNode() {
    for (auto* v : inputs) delete v;
    for (auto* v : outputs) delete v;
  }
};
struct OrtGraph {
  std::vector<OrtNode*> nodes;
  bool owns = true;
  ~OrtGraph() {
    if (owns)
      for (auto* n : nodes) delete n;
  }
};
struct OrtValue {
  OrtTensorTypeAndShapeInfo info;
  void* data = nullptr;
  size_t bytes = 0;
};
struct OrtSessionOptions {
  std::map<std::string, std::string> entries;
};
struct OrtHardwareDevice {
  OrtHardwareDeviceType type;
  uint32_t vendor;
};
struct OrtMemoryDevice {
  OrtMemoryInfoDeviceType type;
  uint32_t vendor;
  int32_t id;
  OrtDeviceMemoryType mem;
};
struct OrtMemoryInfo {
  std::string name;
  OrtMemoryDevice device;
  size_t alignment;
  OrtAllocatorType allocator;
};
struct OrtEpDevice {
  const OrtHardwareDevice* hw;
  std::vector<const OrtMemoryInfo*> allocator_infos;
};
struct OrtEpGraphSupportInfo {
  std::vector<std::vector<const OrtNode*>> groups;
  std::vector<OrtNodeFusionOptions> options;
};
struct OrtKernelContext {
  const OrtNode* fused = nullptr;
  std::map<std::string, OrtValue> inputs;   // by value name
  std::map<std::string, OrtValue> outputs;  // pre-bound, by value name
  std::map<std::string, std::vector<int64_t>> requested;  // output shapes the glue asked for
};

namespace {

uint32_t g_max_api_version = ORT_API_VERSION;
int g_live_memory_infos = 0;
int g_live_statuses = 0;

OrtStatus* make_status(OrtErrorCode code, const std::string& msg) {
  ++g_live_statuses;
  return new OrtStatus{code, msg};
}
#define FAIL(code, msg) return make_status(code, msg)

// ---- OrtApi ----------------------------------------------------------------------------------
OrtStatus* CreateStatus(OrtErrorCode code, const char* msg) noexcept { return make_status(code, msg ? msg : ""); }
OrtErrorCode GetErrorCode(const OrtStatus* s) noexcept { return s->code; }
const char* GetErrorMessage(const OrtStatus* s) noexcept { return s->msg.c_str(); }
void ReleaseStatus(OrtStatus* s) noexcept {
  if (s) --g_live_statuses;
  delete s;
}

OrtHardwareDeviceType HardwareDevice_Type(const OrtHardwareDevice* d) noexcept { return d->type; }
uint32_t HardwareDevice_VendorId(const OrtHardwareDevice* d) noexcept { return d->vendor; }

OrtStatus* HasSessionConfigEntry(const OrtSessionOptions* o, const char* key, int* out) noexcept {
  *out = o->entries.count(key) ? 1 : 0;
  return nullptr;
}
// As ORT: a null buffer asks for the size (terminator included); a short buffer is an error.
OrtStatus* GetSessionConfigEntry(const OrtSessionOptions* o, const char* key, char* value, size_t* size) noexcept {
  auto it = o->entries.find(key);
  if (it == o->entries.end()) FAIL(ORT_INVALID_ARGUMENT, std::string("no session config entry ") + key);
  const size_t need = it->second.size() + 1;
  if (!value) {
    *size = need;
    return nullptr;
  }
  if (*size < need) {
    *size = need;
    FAIL(ORT_INVALID_ARGUMENT, "session config buffer too small");
  }
  std::memcpy(value, it->second.c_str(), need);
  *size = need;
  return nullptr;
}

OrtStatus* Graph_GetNumNodes(const OrtGraph* g, size_t* n) noexcept {
  *n = g->nodes.size();
  return nullptr;
}
OrtStatus* Graph_GetNodes(const OrtGraph* g, const OrtNode** nodes, size_t n) noexcept {
  if (n != g->nodes.size()) FAIL(ORT_INVALID_ARGUMENT, "node count mismatch");
  for (size_t i = 0; i < n; ++i) nodes[i] = g->nodes[i];
  return nullptr;
}
OrtStatus* Node_GetName(const OrtNode* n, const char** out) noexcept {
  *out = n->name.c_str();
  return nullptr;
}
OrtStatus* Node_GetOperatorType(const OrtNode* n, const char** out) noexcept {
  *out = n->op.c_str();
  return nullptr;
}
OrtStatus* Node_GetDomain(const OrtNode* n, const char** out) noexcept {
  *out = n->domain.c_str();
  return nullptr;
}
OrtStatus* Node_GetNumInputs(const OrtNode* n, size_t* out) noexcept {
  *out = n->inputs.size();
  return nullptr;
}
OrtStatus* Node_GetInputs(const OrtNode* n, const OrtValueInfo** out, size_t count) noexcept {
  if (count != n->inputs.size()) FAIL(ORT_INVALID_ARGUMENT, "input count mismatch");
  for (size_t i = 0; i < count; ++i) out[i] = n->inputs[i];
  return nullptr;
}
OrtStatus* Node_GetNumOutputs(const OrtNode* n, size_t* out) noexcept {
  *out = n->outputs.size();
  return nullptr;
}
OrtStatus* Node_GetOutputs(const OrtNode* n, const OrtValueInfo** out, size_t count) noexcept {
  if (count != n->outputs.size()) FAIL(ORT_INVALID_ARGUMENT, "output count mismatch");
  for (size_t i = 0; i < count; ++i) out[i] = n->outputs[i];
  return nullptr;
}
OrtStatus* Node_GetAttributeByName(const OrtNode* n, const char* key, const OrtOpAttr** out) noexcept {
  auto it = n->attrs.find(key);
  *out = nullptr;
  if (it == n->attrs.end()) FAIL(ORT_FAIL, std::string("attribute ") + key + " not found");
  *out = &it->second;
  return nullptr;
}
OrtStatus* OpAttr_GetType(const OrtOpAttr* a, OrtOpAttrType* t) noexcept {
  *t = a->type;
  return nullptr;
}
OrtStatus* ReadOpAttr(const OrtOpAttr* a, OrtOpAttrType type, void* data, size_t len, size_t* out) noexcept {
  if (type != a->type) FAIL(ORT_INVALID_ARGUMENT, "attribute type mismatch");
  size_t need = 0;
  const void* src = nullptr;
  switch (type) {
    case ORT_OP_ATTR_INT: need = sizeof(int64_t); src = &a->i; break;
    case ORT_OP_ATTR_FLOAT: need = sizeof(float); src = &a->f; break;
    case ORT_OP_ATTR_STRING: need = a->s.size(); src = a->s.data(); break;
    default: FAIL(ORT_NOT_IMPLEMENTED, "attribute type not supported by the fake host");
  }
  *out = need;
  if (!data || len < need) FAIL(ORT_INVALID_ARGUMENT, "attribute buffer too small");
  std::memcpy(data, src, need);
  return nullptr;
}
OrtStatus* GetValueInfoName(const OrtValueInfo* v, const char** out) noexcept {
  *out = v->name.c_str();
  return nullptr;
}
OrtStatus* GetValueInfoTypeInfo(const OrtValueInfo* v, const OrtTypeInfo** out) noexcept {
  *out = v->typed ? &v->type : nullptr;
  if (!v->typed) FAIL(ORT_FAIL, "value has no type information");
  return nullptr;
}
OrtStatus* GetOnnxTypeFromTypeInfo(const OrtTypeInfo*, ONNXType* out) noexcept {
  *out = ONNX_TYPE_TENSOR;
  return nullptr;
}
OrtStatus* CastTypeInfoToTensorInfo(const OrtTypeInfo* t, const OrtTensorTypeAndShapeInfo** out) noexcept {
  *out = &t->tensor;
  return nullptr;
}
OrtStatus* GetTensorElementType(const OrtTensorTypeAndShapeInfo* i, ONNXTensorElementDataType* out) noexcept {
  *out = i->dtype;
  return nullptr;
}
OrtStatus* GetDimensionsCount(const OrtTensorTypeAndShapeInfo* i, size_t* out) noexcept {
  *out = i->shape.size();
  return nullptr;
}
OrtStatus* GetDimensions(const OrtTensorTypeAndShapeInfo* i, int64_t* dims, size_t n) noexcept {
  if (n != i->shape.size()) FAIL(ORT_INVALID_ARGUMENT, "rank mismatch");
  for (size_t k = 0; k < n; ++k) dims[k] = i->shape[k];
  return nullptr;
}

const OrtValue* find_input(const OrtKernelContext* c, size_t index) {
  if (!c->fused || index >= c->fused->inputs.size()) return nullptr;
  auto it = c->inputs.find(c->fused->inputs[index]->name);
  return it == c->inputs.end() ? nullptr : &it->second;
}
OrtStatus* KernelContext_GetInputCount(const OrtKernelContext* c, size_t* out) noexcept {
  *out = c->fused ? c->fused->inputs.size() : 0;
  return nullptr;
}
OrtStatus* KernelContext_GetInput(const OrtKernelContext* c, size_t index, const OrtValue** out) noexcept {
  if (!c->fused || index >= c->fused->inputs.size()) FAIL(ORT_INVALID_ARGUMENT, "input index out of range");
  *out = find_input(c, index);
  return nullptr;
}
// As ORT binds outputs: the glue names the shape; the pre-bound tensor must have it.
OrtStatus* KernelContext_GetOutput(OrtKernelContext* c, size_t index, const int64_t* dims, size_t n,
                                   OrtValue** out) noexcept {
  *out = nullptr;
  if (!c->fused || index >= c->fused->outputs.size()) FAIL(ORT_INVALID_ARGUMENT, "output index out of range");
  const std::string& name = c->fused->outputs[index]->name;
  std::vector<int64_t> shape(dims, dims + n);
  c->requested[name] = shape;
  auto it = c->outputs.find(name);
  if (it == c->outputs.end()) FAIL(ORT_FAIL, "output " + name + " is not bound");
  if (it->second.info.shape != shape) FAIL(ORT_INVALID_ARGUMENT, "output " + name + " requested with another shape");
  *out = &it->second;
  return nullptr;
}
OrtStatus* GetTensorTypeAndShape(const OrtValue* v, OrtTensorTypeAndShapeInfo** out) noexcept {
  *out = new OrtTensorTypeAndShapeInfo(v->info);
  return nullptr;
}
void ReleaseTensorTypeAndShapeInfo(OrtTensorTypeAndShapeInfo* i) noexcept { delete i; }
OrtStatus* GetTensorData(const OrtValue* v, const void** out) noexcept {
  *out = v->data;
  return nullptr;
}
OrtStatus* GetTensorMutableData(OrtValue* v, void** out) noexcept {
  *out = v->data;
  return nullptr;
}
OrtStatus* GetTensorSizeInBytes(const OrtValue* v, size_t* out) noexcept {
  *out = v->bytes;
  return nullptr;
}
OrtStatus* CreateMemoryInfo_V2(const char* name, OrtMemoryInfoDeviceType type, uint32_t vendor, int32_t id,
                               OrtDeviceMemoryType mem, size_t alignment, OrtAllocatorType alloc,
                               OrtMemoryInfo** out) noexcept {
  ++g_live_memory_infos;
  *out = new OrtMemoryInfo{name, {type, vendor, id, mem}, alignment, alloc};
  return nullptr;
}
void ReleaseMemoryInfo(OrtMemoryInfo* i) noexcept {
  if (i) --g_live_memory_infos;
  delete i;
}
OrtStatus* MemoryInfoGetName(const OrtMemoryInfo* i, const char** out) noexcept {
  *out = i->name.c_str();
  return nullptr;
}

// ---- OrtEpApi --------------------------------------------------------------------------------
OrtStatus* CreateEpDevice(OrtEpFactory*, const OrtHardwareDevice* hw, const OrtKeyValuePairs*, const OrtKeyValuePairs*,
                          OrtEpDevice** out) noexcept {
  *out = new OrtEpDevice{hw, {}};
  return nullptr;
}
OrtStatus* EpGraphSupportInfo_AddNodesToFuse(OrtEpGraphSupportInfo* s, const OrtNode* const* nodes, size_t n,
                                             const OrtNodeFusionOptions* o) noexcept {
  s->groups.emplace_back(nodes, nodes + n);
  s->options.push_back(*o);
  return nullptr;
}
OrtStatus* EpDevice_AddAllocatorInfo(OrtEpDevice* d, const OrtMemoryInfo* i) noexcept {
  d->allocator_infos.push_back(i);
  return nullptr;
}
const OrtMemoryDevice* MemoryInfo_GetMemoryDevice(const OrtMemoryInfo* i) noexcept { return &i->device; }
bool MemoryDevice_AreEqual(const OrtMemoryDevice* a, const OrtMemoryDevice* b) noexcept {
  return a->type == b->type && a->vendor == b->vendor && a->id == b->id && a->mem == b->mem;
}
OrtMemoryInfoDeviceType MemoryDevice_GetDeviceType(const OrtMemoryDevice* d) noexcept { return d->type; }

OrtEpApi g_ep_api = {CreateEpDevice, EpGraphSupportInfo_AddNodesToFuse, EpDevice_AddAllocatorInfo,
                     MemoryInfo_GetMemoryDevice, MemoryDevice_AreEqual, MemoryDevice_GetDeviceType};
const OrtEpApi* GetEpApi() noexcept { return &g_ep_api; }

OrtApi g_api = {CreateStatus,
                GetErrorCode,
                GetErrorMessage,
                ReleaseStatus,
                GetEpApi,
                HardwareDevice_Type,
                HardwareDevice_VendorId,
                HasSessionConfigEntry,
                GetSessionConfigEntry,
                Graph_GetNumNodes,
                Graph_GetNodes,
                Node_GetName,
                Node_GetOperatorType,
                Node_GetDomain,
                Node_GetNumInputs,
                Node_GetInputs,
                Node_GetNumOutputs,
                Node_GetOutputs,
                Node_GetAttributeByName,
                OpAttr_GetType,
                ReadOpAttr,
                GetValueInfoName,
                GetValueInfoTypeInfo,
                GetOnnxTypeFromTypeInfo,
                CastTypeInfoToTensorInfo,
                GetTensorElementType,
                GetDimensionsCount,
                GetDimensions,
                KernelContext_GetInputCount,
                KernelContext_GetInput,
                KernelContext_GetOutput,
                GetTensorTypeAndShape,
                ReleaseTensorTypeAndShapeInfo,
                GetTensorData,
                GetTensorMutableData,
                GetTensorSizeInBytes,
                CreateMemoryInfo_V2,
                ReleaseMemoryInfo,
                MemoryInfoGetName};

const OrtApi* GetApi(uint32_t version) noexcept { return version <= g_max_api_version ? &g_api : nullptr; }
const char* GetVersionString() noexcept { return "fake-1.31"; }
OrtApiBase g_api_base = {GetApi, GetVersionString};

}  // namespace

// =============================================================================================
// test-facing C API
// =============================================================================================
namespace {

int g_last_code = 0;
std::string g_last_msg;

// Record and release a status the glue returned; returns its code (0 for none).
int take(OrtStatus* st) {
  if (!st) {
    g_last_code = 0;
    g_last_msg.clear();
    return 0;
  }
  g_last_code = st->code;
  g_last_msg = st->msg;
  ReleaseStatus(st);
  return g_last_code;
}

OrtValueInfo* value_info(const char* name, int dtype, int rank, const int64_t* shape) {
  if (!name || !*name) return nullptr;
  auto* v = new OrtValueInfo;
  v->name = name;
  v->type.tensor.dtype = static_cast<ONNXTensorElementDataType>(dtype);
  v->type.tensor.shape.assign(shape, shape + rank);
  return v;
}

OrtValue make_value(int dtype, int rank, const int64_t* shape, void* data, size_t bytes) {
  OrtValue v;
  v.info.dtype = static_cast<ONNXTensorElementDataType>(dtype);
  v.info.shape.assign(shape, shape + rank);
  v.data = data;
  v.bytes = bytes;
  return v;
}

}  // namespace

struct FakeCompiled {
  std::unique_ptr<OrtGraph> sub;
  std::unique_ptr<OrtNode> fused;
  OrtNodeComputeInfo* info = nullptr;
  void* state = nullptr;
};

struct FakeHost {
  void* lib = nullptr;
  OrtStatus* (*release_factory)(OrtEpFactory*) = nullptr;
  const char* (*report)(const OrtEp*) = nullptr;
  OrtEpFactory* factory = nullptr;
  std::vector<OrtHardwareDevice> hw;
  std::vector<OrtEpDevice*> ep_devices;
  OrtEp* ep = nullptr;
  OrtSessionOptions session;
  std::vector<FakeCompiled> compiled;
  OrtAllocator* allocator = nullptr;
  OrtDataTransferImpl* transfer = nullptr;
};

FAKE_API int fake_last_code() { return g_last_code; }
FAKE_API const char* fake_last_error() { return g_last_msg.c_str(); }
FAKE_API void fake_live_counts(int* memory_infos, int* statuses) {
  *memory_infos = g_live_memory_infos;
  *statuses = g_live_statuses;
}
FAKE_API int fake_ort_api_version() { return ORT_API_VERSION; }

// ---- graphs ------------------------------------------------------------------------------------
FAKE_API OrtGraph* fake_graph_new() { return new OrtGraph; }
FAKE_API void fake_graph_free(OrtGraph* g) { delete g; }
FAKE_API OrtNode* fake_node_new(OrtGraph* g, const char* op, const char* domain, const char* name) {
  auto* n = new OrtNode;
  n->op = op;
  n->domain = domain;
  n->name = name;
  g->nodes.push_back(n);
  return n;
}
// name NULL or "" = an absent optional input / output
FAKE_API void fake_node_input(OrtNode* n, const char* name, int dtype, int rank, const int64_t* shape) {
  n->inputs.push_back(value_info(name, dtype, rank, shape));
}
FAKE_API void fake_node_input_untyped(OrtNode* n, const char* name) {
  OrtValueInfo* v = value_info(name, 0, 0, nullptr);
  if (v) v->typed = false;
  n->inputs.push_back(v);
}
FAKE_API void fake_node_output(OrtNode* n, const char* name, int dtype, int rank, const int64_t* shape) {
  n->outputs.push_back(value_info(name, dtype, rank, shape));
}
FAKE_API void fake_node_attr_int(OrtNode* n, const char* key, int64_t v) {
  OrtOpAttr& a = n->attrs[key];
  a.type = ORT_OP_ATTR_INT;
  a.i = v;
}
FAKE_API void fake_node_attr_float(OrtNode* n, const char* key, float v) {
  OrtOpAttr& a = n->attrs[key];
  a.type = ORT_OP_ATTR_FLOAT;
  a.f = v;
}
FAKE_API void fake_node_attr_string(OrtNode* n, const char* key, const char* v) {
  OrtOpAttr& a = n->attrs[key];
  a.type = ORT_OP_ATTR_STRING;
  a.s = v;
}

// ---- kernel contexts -----------------------------------------------------------------------------
FAKE_API OrtKernelContext* fake_kctx_new() { return new OrtKernelContext; }
FAKE_API void fake_kctx_free(OrtKernelContext* c) { delete c; }
FAKE_API void fake_kctx_input(OrtKernelContext* c, const char* name, int dtype, int rank, const int64_t* shape,
                              void* data, size_t bytes) {
  c->inputs[name] = make_value(dtype, rank, shape, data, bytes);
}
FAKE_API void fake_kctx_output(OrtKernelContext* c, const char* name, int dtype, int rank, const int64_t* shape,
                               void* data, size_t bytes) {
  c->outputs[name] = make_value(dtype, rank, shape, data, bytes);
}
// The shape the glue asked for output `name` (-1 when it did not ask).
FAKE_API int fake_kctx_requested(const OrtKernelContext* c, const char* name, int64_t* shape, int max_rank) {
  auto it = c->requested.find(name);
  if (it == c->requested.end()) return -1;
  const int rank = static_cast<int>(it->second.size());
  for (int i = 0; i < rank && i < max_rank; ++i) shape[i] = it->second[i];
  return rank;
}

// ---- the plugin-EP host flow -------------------------------------------------------------------
FAKE_API FakeHost* fake_host_open(const char* shell_path, uint32_t max_api_version, const char* registration_name) {
  g_max_api_version = max_api_version;
  void* lib = dlopen(shell_path, RTLD_NOW | RTLD_LOCAL);
  if (!lib) {
    g_last_code = -1;
    g_last_msg = dlerror();
    return nullptr;
  }
  using CreateFn = OrtStatus* (*)(const char*, const OrtApiBase*, const OrtLogger*, OrtEpFactory**, size_t, size_t*);
  auto create = reinterpret_cast<CreateFn>(dlsym(lib, "CreateEpFactories"));
  auto host = std::make_unique<FakeHost>();
  host->lib = lib;
  host->release_factory = reinterpret_cast<OrtStatus* (*)(OrtEpFactory*)>(dlsym(lib, "ReleaseEpFactory"));
  host->report = reinterpret_cast<const char* (*)(const OrtEp*)>(dlsym(lib, "b200_ep_shell_capability_report"));
  if (!create || !host->release_factory) {
    g_last_code = -1;
    g_last_msg = "CreateEpFactories / ReleaseEpFactory not exported";
    dlclose(lib);
    return nullptr;
  }
  OrtEpFactory* factories[2] = {nullptr, nullptr};
  size_t n = 0;
  if (take(create(registration_name, &g_api_base, nullptr, factories, 2, &n)) || n != 1) {
    if (n != 1 && g_last_code == 0) {
      g_last_code = -1;
      g_last_msg = "CreateEpFactories returned no factory";
    }
    dlclose(lib);
    return nullptr;
  }
  host->factory = factories[0];
  return host.release();
}

// CreateEpFactories with room for `max_factories` (0 exercises its argument check).
FAKE_API int fake_create_factories_raw(const char* shell_path, size_t max_factories) {
  g_max_api_version = ORT_API_VERSION;
  void* lib = dlopen(shell_path, RTLD_NOW | RTLD_LOCAL);
  if (!lib) return -1;
  using CreateFn = OrtStatus* (*)(const char*, const OrtApiBase*, const OrtLogger*, OrtEpFactory**, size_t, size_t*);
  auto create = reinterpret_cast<CreateFn>(dlsym(lib, "CreateEpFactories"));
  auto release = reinterpret_cast<OrtStatus* (*)(OrtEpFactory*)>(dlsym(lib, "ReleaseEpFactory"));
  OrtEpFactory* f[1] = {nullptr};
  size_t n = 0;
  int rc = take(create(nullptr, &g_api_base, nullptr, f, max_factories, &n));
  if (n == 1) release(f[0]);
  dlclose(lib);
  return rc;
}

FAKE_API const char* fake_host_string(FakeHost* h, int which) {
  switch (which) {
    case 0: return h->factory->GetName(h->factory);
    case 1: return h->factory->GetVendor(h->factory);
    case 2: return h->factory->GetVersion(h->factory);
    default: return "";
  }
}
FAKE_API uint32_t fake_host_vendor_id(FakeHost* h) { return h->factory->GetVendorId(h->factory); }
FAKE_API int fake_host_stream_aware(FakeHost* h) { return h->factory->IsStreamAware(h->factory) ? 1 : 0; }

// GetSupportedDevices over hardware devices (types: 0 CPU, 1 GPU, 2 NPU; vendor ids).  Returns the
// status code; *num_ep_devices and the registered allocator infos of the first EP device.
FAKE_API int fake_host_devices(FakeHost* h, const int* types, const uint32_t* vendors, size_t n,
                               size_t* num_ep_devices, int* allocator_infos) {
  h->hw.clear();
  for (size_t i = 0; i < n; ++i) h->hw.push_back({static_cast<OrtHardwareDeviceType>(types[i]), vendors[i]});
  std::vector<const OrtHardwareDevice*> ptrs;
  for (auto& d : h->hw) ptrs.push_back(&d);
  OrtEpDevice* out[4] = {nullptr, nullptr, nullptr, nullptr};
  *num_ep_devices = 0;
  const int rc = take(h->factory->GetSupportedDevices(h->factory, ptrs.data(), ptrs.size(), out, 4, num_ep_devices));
  for (size_t i = 0; i < *num_ep_devices; ++i) h->ep_devices.push_back(out[i]);
  *allocator_infos = *num_ep_devices ? static_cast<int>(out[0]->allocator_infos.size()) : 0;
  return rc;
}
// The first allocator info of the first EP device: name, device type, vendor, id.
FAKE_API int fake_host_device_memory(FakeHost* h, char* name, size_t len, int* type, uint32_t* vendor, int* id) {
  if (h->ep_devices.empty() || h->ep_devices[0]->allocator_infos.empty()) return -1;
  const OrtMemoryInfo* i = h->ep_devices[0]->allocator_infos[0];
  std::snprintf(name, len, "%s", i->name.c_str());
  *type = i->device.type;
  *vendor = i->device.vendor;
  *id = i->device.id;
  return 0;
}

FAKE_API int fake_host_create_ep(FakeHost* h, const char* const* keys, const char* const* values, size_t n,
                                 size_t num_devices) {
  h->session.entries.clear();
  for (size_t i = 0; i < n; ++i) h->session.entries[keys[i]] = values[i];
  std::vector<const OrtHardwareDevice*> ptrs;
  for (size_t i = 0; i < num_devices && i < h->hw.size(); ++i) ptrs.push_back(&h->hw[i]);
  OrtEp* ep = nullptr;
  const int rc = take(h->factory->CreateEp(h->factory, ptrs.data(), nullptr, num_devices, &h->session, nullptr, &ep));
  if (rc == 0) h->ep = ep;
  return rc;
}
FAKE_API const char* fake_host_ep_name(FakeHost* h) { return h->ep->GetName(h->ep); }
FAKE_API int fake_host_default_memory(FakeHost* h, int* type, uint32_t* vendor, int* id) {
  const OrtMemoryDevice* d = nullptr;
  const int rc = take(h->ep->GetDefaultMemoryDevice(h->ep, &d));
  if (rc || !d) return rc ? rc : -1;
  *type = d->type;
  *vendor = d->vendor;
  *id = d->id;
  return 0;
}

// GetCapability: indices (in graph order) of the claimed nodes, each expected as its own group.
FAKE_API int fake_host_capability(FakeHost* h, OrtGraph* g, int* claimed, size_t max, size_t* n, int* drop_const) {
  OrtEpGraphSupportInfo s;
  const int rc = take(h->ep->GetCapability(h->ep, g, &s));
  *n = 0;
  *drop_const = -1;
  for (size_t k = 0; k < s.groups.size() && *n < max; ++k) {
    if (s.groups[k].size() != 1) return -2;
    for (size_t i = 0; i < g->nodes.size(); ++i)
      if (g->nodes[i] == s.groups[k][0]) claimed[(*n)++] = static_cast<int>(i);
    *drop_const = s.options[k].drop_constant_initializers ? 1 : 0;
  }
  return rc;
}
FAKE_API const char* fake_host_report(FakeHost* h) { return h->report ? h->report(h->ep) : ""; }

// Compile node `index` of `g` as ORT does for a single-node fusion: a subgraph holding the node
// and a fused node whose inputs / outputs are the node's present values (each name once),
// reversed when `reverse` is set (the glue must map by name, not by position).  Returns the
// compiled index, or -1 with the status in fake_last_*.
FAKE_API int fake_host_compile(FakeHost* h, OrtGraph* g, int index, int reverse) {
  FakeCompiled c;
  c.sub.reset(new OrtGraph);
  c.sub->owns = false;
  c.sub->nodes.push_back(g->nodes[index]);
  c.fused.reset(new OrtNode);
  c.fused->op = "B200Fused";
  c.fused->domain = "com.b200";
  c.fused->name = "fused_" + g->nodes[index]->name;
  auto boundary = [](const std::vector<OrtValueInfo*>& values, std::vector<OrtValueInfo*>* out) {
    for (OrtValueInfo* v : values) {
      if (!v || v->name.empty()) continue;
      bool seen = false;
      for (OrtValueInfo* o : *out) seen = seen || o->name == v->name;
      if (!seen) out->push_back(new OrtValueInfo(*v));
    }
  };
  boundary(g->nodes[index]->inputs, &c.fused->inputs);
  boundary(g->nodes[index]->outputs, &c.fused->outputs);
  if (reverse) {
    std::vector<OrtValueInfo*> r(c.fused->inputs.rbegin(), c.fused->inputs.rend());
    c.fused->inputs = r;
  }
  const OrtGraph* graphs[1] = {c.sub.get()};
  const OrtNode* fused[1] = {c.fused.get()};
  OrtNodeComputeInfo* infos[1] = {nullptr};
  if (take(h->ep->Compile(h->ep, graphs, fused, 1, infos, nullptr))) return -1;
  c.info = infos[0];
  if (take(c.info->CreateState(c.info, nullptr, &c.state))) {
    h->ep->ReleaseNodeComputeInfos(h->ep, infos, 1);
    return -1;
  }
  h->compiled.push_back(std::move(c));
  return static_cast<int>(h->compiled.size()) - 1;
}

FAKE_API int fake_host_compute(FakeHost* h, int compiled, OrtKernelContext* ctx) {
  FakeCompiled& c = h->compiled[compiled];
  ctx->fused = c.fused.get();
  ctx->requested.clear();
  return take(c.info->Compute(c.info, c.state, ctx));
}

// CreateAllocator for a memory info named `name` (GPU, NVIDIA, device `id`): 1 = the glue
// returned an allocator, 0 = none (ORT's default applies), else the status code.
FAKE_API int fake_host_allocator(FakeHost* h, const char* name, int id) {
  OrtMemoryInfo* info = nullptr;
  CreateMemoryInfo_V2(name, OrtMemoryInfoDeviceType_GPU, 0x10DE, id, OrtDeviceMemoryType_DEFAULT, 256,
                      OrtDeviceAllocator, &info);
  OrtAllocator* a = nullptr;
  const int rc = take(h->factory->CreateAllocator(h->factory, info, nullptr, &a));
  ReleaseMemoryInfo(info);
  if (rc) return rc;
  if (!a) return 0;
  if (h->allocator) h->factory->ReleaseAllocator(h->factory, h->allocator);
  h->allocator = a;
  return 1;
}
FAKE_API void* fake_host_alloc(FakeHost* h, size_t bytes) { return h->allocator->Alloc(h->allocator, bytes); }
FAKE_API void fake_host_free(FakeHost* h, void* p) { h->allocator->Free(h->allocator, p); }
FAKE_API const char* fake_host_allocator_name(FakeHost* h) { return h->allocator->Info(h->allocator)->name.c_str(); }

FAKE_API int fake_host_transfer(FakeHost* h) {
  if (h->transfer) return 0;
  OrtDataTransferImpl* t = nullptr;
  const int rc = take(h->factory->CreateDataTransfer(h->factory, &t));
  h->transfer = t;
  return rc;
}
// CanCopy between memory devices of kind 0 = CPU, 1 = the EP's ("B200", NVIDIA, device `id`),
// 2 = another vendor's GPU.
FAKE_API int fake_host_can_copy(FakeHost* h, int src, int dst, int id) {
  auto dev = [&](int kind) {
    switch (kind) {
      case 0: return OrtMemoryDevice{OrtMemoryInfoDeviceType_CPU, 0, 0, OrtDeviceMemoryType_DEFAULT};
      case 1: return OrtMemoryDevice{OrtMemoryInfoDeviceType_GPU, 0x10DE, id, OrtDeviceMemoryType_DEFAULT};
      default: return OrtMemoryDevice{OrtMemoryInfoDeviceType_GPU, 0x1002, 0, OrtDeviceMemoryType_DEFAULT};
    }
  };
  const OrtMemoryDevice a = dev(src), b = dev(dst);
  return h->transfer->CanCopy(h->transfer, &a, &b) ? 1 : 0;
}
FAKE_API int fake_host_copy(FakeHost* h, int dtype, int rank, const int64_t* shape, void* src, size_t src_bytes,
                            int dst_rank, const int64_t* dst_shape, void* dst, size_t dst_bytes) {
  OrtValue s = make_value(dtype, rank, shape, src, src_bytes);
  OrtValue d = make_value(dtype, dst_rank, dst_shape, dst, dst_bytes);
  const OrtValue* sp[1] = {&s};
  OrtValue* dp[1] = {&d};
  return take(h->transfer->CopyTensors(h->transfer, sp, dp, nullptr, 1));
}

FAKE_API void fake_host_close(FakeHost* h) {
  if (!h) return;
  for (auto& c : h->compiled) {
    c.info->ReleaseState(c.info, c.state);
    OrtNodeComputeInfo* infos[1] = {c.info};
    h->ep->ReleaseNodeComputeInfos(h->ep, infos, 1);
  }
  h->compiled.clear();
  if (h->transfer) h->transfer->Release(h->transfer);
  if (h->allocator) h->factory->ReleaseAllocator(h->factory, h->allocator);
  if (h->ep) h->factory->ReleaseEp(h->factory, h->ep);
  take(h->release_factory(h->factory));
  for (auto* d : h->ep_devices) delete d;
  dlclose(h->lib);
  delete h;
}
