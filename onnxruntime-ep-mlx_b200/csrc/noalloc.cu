// PagedAttention with library-owned static scratch, for callers that cannot allocate device
// memory.
//
// Some callers cannot call cudaMalloc at the moment they run attention: a host runtime that hands
// the kernel library only the tensors it already owns, a serving loop that forbids device
// allocations after start-up, or a foreign-language binding (cgo, JNI) with no CUDA allocator of
// its own.  b200_paged_attention_static_scratch serves them: the caller still passes every input
// and output, but the scratch that b200_paged_attention takes from the caller's workspace (decode
// partials, tile-stream plan, duplicate-slot table, status word) lives in a file-scope
// `static __device__` array of kStaticScratchBytes instead.
//
// Consequences a caller must know:
//  * every GPU on which the library's module is loaded holds the array until the process exits;
//  * calls whose scratch need exceeds kStaticScratchBytes are rejected (B200_ERR_WORKSPACE);
//  * all calls on a device share the array and it keeps the last call's contents: each call
//    re-initialises what must start from zero (status word, slot table, completion counters)
//    in its own stream order, so calls that overlap on the GPU (different streams, or threads
//    without ordering) race on it and must be serialised by the caller;
//  * the first call on a device resolves the array's device address with cudaGetSymbolAddress,
//    which may load the module onto that device; make that first call before any stream capture.
//    The address is kept for the life of the process, so cudaDeviceReset (which unloads the
//    module and frees the array) is not supported while this entry point is in use;
//  * without a caller-provided device_status the status word also lives in the array: read it
//    with b200_read_status_static_scratch (b200_read_status sees no workspace and refuses).
// The call itself allocates nothing: no cudaMalloc/cudaFree and no allocating library routine.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "b200_kernels.h"
#include "b200_paged.h"

namespace {

constexpr size_t kStaticScratchBytes = 32ull << 20;  // 32 MiB per device

// Device-side scratch.  In host code this name is only a stand-in for the symbol: its device
// address comes from cudaGetSymbolAddress below and is what the kernels receive.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mutex;

// Device address of this device's static scratch; resolved once per device, with that device
// current (the set-up step of the first call on it).
int static_scratch_address(const char* who, void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return b200::set_error(B200_ERR_CUDA, std::string(who) + ": no current CUDA device");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess || !ptr)
      return b200::set_error(B200_ERR_CUDA, std::string(who) + ": cudaGetSymbolAddress failed: " + cudaGetErrorString(e));
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return B200_OK;
}

}  // namespace

extern "C" int b200_paged_attention_static_scratch(const B200PagedAttentionParams* p, void* stream) {
  if (!p) return b200::set_error(B200_ERR_INVALID_ARGUMENT, "PagedAttention (static scratch): null params");
  void* scratch = nullptr;
  int rc0 = static_scratch_address("PagedAttention (static scratch)", &scratch);
  if (rc0 != B200_OK) return rc0;

  B200PagedAttentionParams q = *p;
  q.workspace = scratch;
  q.workspace_bytes = kStaticScratchBytes;
  // Host metadata: keep the reference's host validation (no allocation), then hand only the
  // device copies on, so duplicate slots are resolved on the device (the host-side duplicate
  // check of b200_paged_attention uses a heap-allocated set).
  if (q.host_cumulative_sequence_length && q.host_past_seqlens && q.host_block_table) {
    int rc = b200_paged_attention_validate_host(&q);
    if (rc != B200_OK) return rc;
  }
  q.host_cumulative_sequence_length = nullptr;
  q.host_past_seqlens = nullptr;
  q.host_block_table = nullptr;
  q.host_slot_mapping = nullptr;

  size_t need = 0;
  int rc = b200_paged_attention_workspace_size(&q, &need);
  if (rc != B200_OK) return rc;
  if (need > kStaticScratchBytes) {
    return b200::set_error(B200_ERR_WORKSPACE,
                           "PagedAttention (static scratch): the call needs " + std::to_string(need) +
                               " bytes of scratch but the static scratch holds " +
                               std::to_string(kStaticScratchBytes) +
                               " (32 MiB); use b200_paged_attention with a caller workspace");
  }
  return b200_paged_attention(&q, stream);
}

extern "C" int b200_read_status_static_scratch(const B200PagedAttentionParams* p, void* stream) {
  if (!p) return b200::set_error(B200_ERR_INVALID_ARGUMENT, "PagedAttention (static scratch): null params");
  if (p->device_status) return b200_read_status(p, stream);
  void* scratch = nullptr;
  int rc = static_scratch_address("PagedAttention (static scratch)", &scratch);
  if (rc != B200_OK) return rc;
  // The status word sits where b200_paged_attention_static_scratch put it: at the workspace
  // layout's status offset inside this device's static array.
  B200PagedAttentionParams q = *p;
  q.workspace = scratch;
  q.workspace_bytes = kStaticScratchBytes;
  return b200_read_status(&q, stream);
}
