/*
 * TEST DOUBLE - not ONNX Runtime's header.
 *
 * Declares only the ONNX Runtime C API members that the B200 EP glue
 * (onnxruntime-ep-mlx_b200/csrc/ep_shell.cpp) names, under their ONNX Runtime 1.31 names and
 * parameter types, so that the glue compiles and runs here against the fake host in
 * fake_ort.cpp.  Struct member ORDER, enum VALUES (other than the ONNX tensor element types,
 * which are ONNX's own numbering) and everything the glue does not name are this stub's own:
 * a glue library that ONNX Runtime loads must be compiled against ONNX Runtime's headers
 * (`make -C onnxruntime-ep-mlx_b200/csrc shell ORT_INCLUDE_DIR=...`).
 */
#ifndef B200_TEST_ORT_STUB_H
#define B200_TEST_ORT_STUB_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#define ORT_API_VERSION 31
#define ORT_API_CALL
#ifdef __cplusplus
#define NO_EXCEPTION noexcept
extern "C" {
#else
#define NO_EXCEPTION
#endif

typedef struct OrtStatus OrtStatus;
typedef struct OrtSessionOptions OrtSessionOptions;
typedef struct OrtLogger OrtLogger;
typedef struct OrtHardwareDevice OrtHardwareDevice;
typedef struct OrtEpDevice OrtEpDevice;
typedef struct OrtKeyValuePairs OrtKeyValuePairs;
typedef struct OrtGraph OrtGraph;
typedef struct OrtNode OrtNode;
typedef struct OrtValueInfo OrtValueInfo;
typedef struct OrtTypeInfo OrtTypeInfo;
typedef struct OrtTensorTypeAndShapeInfo OrtTensorTypeAndShapeInfo;
typedef struct OrtOpAttr OrtOpAttr;
typedef struct OrtValue OrtValue;
typedef struct OrtKernelContext OrtKernelContext;
typedef struct OrtMemoryInfo OrtMemoryInfo;
typedef struct OrtMemoryDevice OrtMemoryDevice;
typedef struct OrtEpGraphSupportInfo OrtEpGraphSupportInfo;
typedef struct OrtNodeComputeContext OrtNodeComputeContext;
typedef struct OrtSyncStream OrtSyncStream;
typedef struct OrtSyncStreamImpl OrtSyncStreamImpl;

typedef enum OrtErrorCode {
  ORT_OK = 0,
  ORT_FAIL = 1,
  ORT_INVALID_ARGUMENT = 2,
  ORT_NOT_IMPLEMENTED = 9,
  ORT_EP_FAIL = 11
} OrtErrorCode;

typedef enum ONNXTensorElementDataType {
  ONNX_TENSOR_ELEMENT_DATA_TYPE_UNDEFINED = 0,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT = 1,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_UINT8 = 2,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_INT8 = 3,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_INT32 = 6,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_INT64 = 7,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT16 = 10,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_BFLOAT16 = 16,
  ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT8E4M3FN = 17
} ONNXTensorElementDataType;

typedef enum ONNXType { ONNX_TYPE_UNKNOWN = 0, ONNX_TYPE_TENSOR = 1 } ONNXType;

typedef enum OrtOpAttrType {
  ORT_OP_ATTR_UNDEFINED = 0,
  ORT_OP_ATTR_INT,
  ORT_OP_ATTR_INTS,
  ORT_OP_ATTR_FLOAT,
  ORT_OP_ATTR_FLOATS,
  ORT_OP_ATTR_STRING,
  ORT_OP_ATTR_STRINGS
} OrtOpAttrType;

typedef enum OrtHardwareDeviceType {
  OrtHardwareDeviceType_CPU,
  OrtHardwareDeviceType_GPU,
  OrtHardwareDeviceType_NPU
} OrtHardwareDeviceType;

typedef enum OrtMemoryInfoDeviceType {
  OrtMemoryInfoDeviceType_CPU = 0,
  OrtMemoryInfoDeviceType_GPU = 1
} OrtMemoryInfoDeviceType;

typedef enum OrtDeviceMemoryType {
  OrtDeviceMemoryType_DEFAULT = 0,
  OrtDeviceMemoryType_HOST_ACCESSIBLE = 5
} OrtDeviceMemoryType;

typedef enum OrtAllocatorType { OrtInvalidAllocator = -1, OrtDeviceAllocator = 0, OrtArenaAllocator = 1 } OrtAllocatorType;

typedef struct OrtAllocator {
  uint32_t version;
  void*(ORT_API_CALL* Alloc)(struct OrtAllocator* this_, size_t size) NO_EXCEPTION;
  void(ORT_API_CALL* Free)(struct OrtAllocator* this_, void* p) NO_EXCEPTION;
  const OrtMemoryInfo*(ORT_API_CALL* Info)(const struct OrtAllocator* this_) NO_EXCEPTION;
  void*(ORT_API_CALL* Reserve)(struct OrtAllocator* this_, size_t size) NO_EXCEPTION;
} OrtAllocator;

typedef struct OrtDataTransferImpl {
  uint32_t ort_version_supported;
  void(ORT_API_CALL* Release)(struct OrtDataTransferImpl* this_ptr) NO_EXCEPTION;
  bool(ORT_API_CALL* CanCopy)(const struct OrtDataTransferImpl* this_ptr, const OrtMemoryDevice* src_memory_device,
                              const OrtMemoryDevice* dst_memory_device) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* CopyTensors)(struct OrtDataTransferImpl* this_ptr, const OrtValue** src_tensors,
                                        OrtValue** dst_tensors, OrtSyncStream** streams,
                                        size_t num_tensors) NO_EXCEPTION;
} OrtDataTransferImpl;

typedef struct OrtNodeFusionOptions {
  uint32_t ort_version_supported;
  bool drop_constant_initializers;
} OrtNodeFusionOptions;

typedef struct OrtNodeComputeInfo {
  uint32_t ort_version_supported;
  OrtStatus*(ORT_API_CALL* CreateState)(struct OrtNodeComputeInfo* this_ptr, OrtNodeComputeContext* compute_context,
                                        void** compute_state) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Compute)(struct OrtNodeComputeInfo* this_ptr, void* compute_state,
                                    OrtKernelContext* kernel_context) NO_EXCEPTION;
  void(ORT_API_CALL* ReleaseState)(struct OrtNodeComputeInfo* this_ptr, void* compute_state) NO_EXCEPTION;
} OrtNodeComputeInfo;

typedef struct OrtEp {
  uint32_t ort_version_supported;
  const char*(ORT_API_CALL* GetName)(const struct OrtEp* this_ptr) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetCapability)(struct OrtEp* this_ptr, const OrtGraph* graph,
                                          OrtEpGraphSupportInfo* graph_support_info) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Compile)(struct OrtEp* this_ptr, const OrtGraph** graphs, const OrtNode** fused_nodes,
                                    size_t count, OrtNodeComputeInfo** node_compute_infos,
                                    OrtNode** ep_context_nodes) NO_EXCEPTION;
  void(ORT_API_CALL* ReleaseNodeComputeInfos)(struct OrtEp* this_ptr, OrtNodeComputeInfo** node_compute_infos,
                                              size_t num_node_compute_infos) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetDefaultMemoryDevice)(const struct OrtEp* this_ptr,
                                                   const OrtMemoryDevice** device) NO_EXCEPTION;
} OrtEp;

typedef struct OrtEpFactory {
  uint32_t ort_version_supported;
  const char*(ORT_API_CALL* GetName)(const struct OrtEpFactory* this_ptr) NO_EXCEPTION;
  const char*(ORT_API_CALL* GetVendor)(const struct OrtEpFactory* this_ptr) NO_EXCEPTION;
  uint32_t(ORT_API_CALL* GetVendorId)(const struct OrtEpFactory* this_ptr) NO_EXCEPTION;
  const char*(ORT_API_CALL* GetVersion)(const struct OrtEpFactory* this_ptr) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetSupportedDevices)(struct OrtEpFactory* this_ptr, const OrtHardwareDevice* const* devices,
                                                size_t num_devices, OrtEpDevice** ep_devices, size_t max_ep_devices,
                                                size_t* num_ep_devices) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* CreateEp)(struct OrtEpFactory* this_ptr, const OrtHardwareDevice* const* devices,
                                     const OrtKeyValuePairs* const* ep_metadata_pairs, size_t num_devices,
                                     const OrtSessionOptions* session_options, const OrtLogger* logger,
                                     OrtEp** ep) NO_EXCEPTION;
  void(ORT_API_CALL* ReleaseEp)(struct OrtEpFactory* this_ptr, OrtEp* ep) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* CreateAllocator)(struct OrtEpFactory* this_ptr, const OrtMemoryInfo* memory_info,
                                            const OrtKeyValuePairs* allocator_options,
                                            OrtAllocator** allocator) NO_EXCEPTION;
  void(ORT_API_CALL* ReleaseAllocator)(struct OrtEpFactory* this_ptr, OrtAllocator* allocator) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* CreateDataTransfer)(struct OrtEpFactory* this_ptr,
                                               OrtDataTransferImpl** data_transfer) NO_EXCEPTION;
  bool(ORT_API_CALL* IsStreamAware)(const struct OrtEpFactory* this_ptr) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* CreateSyncStreamForDevice)(struct OrtEpFactory* this_ptr,
                                                      const OrtMemoryDevice* memory_device,
                                                      const OrtKeyValuePairs* stream_options,
                                                      OrtSyncStreamImpl** stream) NO_EXCEPTION;
} OrtEpFactory;

typedef struct OrtEpApi {
  OrtStatus*(ORT_API_CALL* CreateEpDevice)(OrtEpFactory* ep_factory, const OrtHardwareDevice* hardware_device,
                                           const OrtKeyValuePairs* ep_metadata, const OrtKeyValuePairs* ep_options,
                                           OrtEpDevice** ep_device) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* EpGraphSupportInfo_AddNodesToFuse)(OrtEpGraphSupportInfo* graph_support_info,
                                                              const OrtNode* const* nodes, size_t num_nodes,
                                                              const OrtNodeFusionOptions* node_fusion_options)
      NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* EpDevice_AddAllocatorInfo)(OrtEpDevice* ep_device,
                                                      const OrtMemoryInfo* allocator_memory_info) NO_EXCEPTION;
  const OrtMemoryDevice*(ORT_API_CALL* MemoryInfo_GetMemoryDevice)(const OrtMemoryInfo* memory_info) NO_EXCEPTION;
  bool(ORT_API_CALL* MemoryDevice_AreEqual)(const OrtMemoryDevice* a, const OrtMemoryDevice* b) NO_EXCEPTION;
  OrtMemoryInfoDeviceType(ORT_API_CALL* MemoryDevice_GetDeviceType)(const OrtMemoryDevice* memory_device) NO_EXCEPTION;
} OrtEpApi;

typedef struct OrtApi {
  OrtStatus*(ORT_API_CALL* CreateStatus)(OrtErrorCode code, const char* msg) NO_EXCEPTION;
  OrtErrorCode(ORT_API_CALL* GetErrorCode)(const OrtStatus* status) NO_EXCEPTION;
  const char*(ORT_API_CALL* GetErrorMessage)(const OrtStatus* status) NO_EXCEPTION;
  void(ORT_API_CALL* ReleaseStatus)(OrtStatus* input) NO_EXCEPTION;
  const OrtEpApi*(ORT_API_CALL* GetEpApi)(void) NO_EXCEPTION;
  OrtHardwareDeviceType(ORT_API_CALL* HardwareDevice_Type)(const OrtHardwareDevice* device) NO_EXCEPTION;
  uint32_t(ORT_API_CALL* HardwareDevice_VendorId)(const OrtHardwareDevice* device) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* HasSessionConfigEntry)(const OrtSessionOptions* options, const char* config_key,
                                                  int* out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetSessionConfigEntry)(const OrtSessionOptions* options, const char* config_key,
                                                  char* config_value, size_t* size) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Graph_GetNumNodes)(const OrtGraph* graph, size_t* num_nodes) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Graph_GetNodes)(const OrtGraph* graph, const OrtNode** nodes, size_t num_nodes) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Node_GetName)(const OrtNode* node, const char** node_name) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Node_GetOperatorType)(const OrtNode* node, const char** operator_type) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Node_GetDomain)(const OrtNode* node, const char** domain_name) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Node_GetNumInputs)(const OrtNode* node, size_t* num_inputs) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Node_GetInputs)(const OrtNode* node, const OrtValueInfo** inputs,
                                           size_t num_inputs) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Node_GetNumOutputs)(const OrtNode* node, size_t* num_outputs) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Node_GetOutputs)(const OrtNode* node, const OrtValueInfo** outputs,
                                            size_t num_outputs) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* Node_GetAttributeByName)(const OrtNode* node, const char* attribute_name,
                                                    const OrtOpAttr** attribute) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* OpAttr_GetType)(const OrtOpAttr* attribute, OrtOpAttrType* type) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* ReadOpAttr)(const OrtOpAttr* op_attr, OrtOpAttrType type, void* data, size_t len,
                                       size_t* out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetValueInfoName)(const OrtValueInfo* value_info, const char** name) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetValueInfoTypeInfo)(const OrtValueInfo* value_info,
                                                 const OrtTypeInfo** type_info) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetOnnxTypeFromTypeInfo)(const OrtTypeInfo* type_info, ONNXType* out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* CastTypeInfoToTensorInfo)(const OrtTypeInfo* type_info,
                                                     const OrtTensorTypeAndShapeInfo** out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetTensorElementType)(const OrtTensorTypeAndShapeInfo* info,
                                                 ONNXTensorElementDataType* out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetDimensionsCount)(const OrtTensorTypeAndShapeInfo* info, size_t* out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetDimensions)(const OrtTensorTypeAndShapeInfo* info, int64_t* dim_values,
                                          size_t dim_values_length) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* KernelContext_GetInputCount)(const OrtKernelContext* context, size_t* out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* KernelContext_GetInput)(const OrtKernelContext* context, size_t index,
                                                   const OrtValue** out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* KernelContext_GetOutput)(OrtKernelContext* context, size_t index, const int64_t* dim_values,
                                                    size_t dim_count, OrtValue** out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetTensorTypeAndShape)(const OrtValue* value, OrtTensorTypeAndShapeInfo** out) NO_EXCEPTION;
  void(ORT_API_CALL* ReleaseTensorTypeAndShapeInfo)(OrtTensorTypeAndShapeInfo* input) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetTensorData)(const OrtValue* value, const void** out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetTensorMutableData)(OrtValue* value, void** out) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* GetTensorSizeInBytes)(const OrtValue* ort_value, size_t* size) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* CreateMemoryInfo_V2)(const char* name, OrtMemoryInfoDeviceType device_type,
                                                uint32_t vendor_id, int32_t device_id, OrtDeviceMemoryType mem_type,
                                                size_t alignment, OrtAllocatorType allocator_type,
                                                OrtMemoryInfo** out) NO_EXCEPTION;
  void(ORT_API_CALL* ReleaseMemoryInfo)(OrtMemoryInfo* input) NO_EXCEPTION;
  OrtStatus*(ORT_API_CALL* MemoryInfoGetName)(const OrtMemoryInfo* ptr, const char** out) NO_EXCEPTION;
} OrtApi;

typedef struct OrtApiBase {
  const OrtApi*(ORT_API_CALL* GetApi)(uint32_t version) NO_EXCEPTION;
  const char*(ORT_API_CALL* GetVersionString)(void) NO_EXCEPTION;
} OrtApiBase;

#ifdef __cplusplus
}
#endif

#endif /* B200_TEST_ORT_STUB_H */
