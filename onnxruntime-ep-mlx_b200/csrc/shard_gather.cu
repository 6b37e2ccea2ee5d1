// Gather of kv-head-sharded attention outputs across the GPUs of one node: every rank stores its
// [rows, slice] output into every rank's [rows, world * slice] output at its own column offset
// (all-gather and head permute in one pass), with plain 16-byte peer stores over NVLink between
// an entry and an exit barrier on flag words in peer memory.  No multicast, no NVLS.
//
// Flags of rank t: words [0, world) are entry slots, [world, 2 world) exit slots; slot s holds
// the number of the last call that rank s announced.  Calls are numbered per rank on the device
// (state[0]), so a CUDA graph replaying the call needs no host input; all ranks make the same
// calls in the same order, so the numbers agree.  Ordering: a rank's slice stores are fenced at
// system scope before its exit flags are released, and the waiting side reads flags with
// acquire loads, so every slice has landed once all exit flags show the call.
#include <cuda_runtime.h>

#include <algorithm>
#include <string>

#include "b200_common.cuh"
#include "b200_shard.h"

namespace b200 {
namespace {

constexpr int kGatherThreads = 256;

struct GatherArgs {
  int world, rank, rows, vecs;  // vecs: 16-byte pieces of one row slice
  int64_t slice_bytes;
  const uint4* local;
  char* outputs[B200_SHARD_MAX_RANKS];
  uint32_t* flags[B200_SHARD_MAX_RANKS];
  uint32_t* state;
  int* status;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Until words[t] has reached call `e` for every rank t (wrap-safe), at most kWaitLimitNs.
__device__ bool wait_all(const uint32_t* words, int world, uint32_t e) {
  const uint64_t start = globaltimer_ns();
  for (int t = 0; t < world; ++t) {
    while ((int32_t)(ld_acquire_sys(words + t) - e) < 0) {
      if (globaltimer_ns() - start > kWaitLimitNs) return false;
    }
  }
  return true;
}

__global__ void __launch_bounds__(kGatherThreads) shard_gather_kernel(const __grid_constant__ GatherArgs g) {
  __shared__ int entered, last;
  const uint32_t e = g.state[0] + 1;  // this call; the last CTA advances state[0] after every CTA read it

  // entry: announce the call to every rank, then wait until every rank has announced it
  if (blockIdx.x == 0 && (int)threadIdx.x < g.world) st_release_sys(g.flags[threadIdx.x] + g.rank, e);
  if (threadIdx.x == 0) {
    entered = wait_all(g.flags[g.rank], g.world, e);
    if (!entered) set_status(g.status, kStatusTimeout);
  }
  __syncthreads();

  if (entered) {
    // piece i: destination rank t = i / per_rank, then row, then 16-byte piece of the slice
    const int64_t per_rank = (int64_t)g.rows * g.vecs;
    const int64_t total = per_rank * g.world;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
      const int t = (int)(i / per_rank);
      const int64_t j = i - (int64_t)t * per_rank;
      const int64_t row = j / g.vecs;
      const int c = (int)(j - row * g.vecs);
      const uint4 v = g.local[j];
      reinterpret_cast<uint4*>(g.outputs[t] + (row * g.world + g.rank) * g.slice_bytes)[c] = v;
    }
  }
  // The CTA's peer stores before its arrival: the block barrier orders every thread's stores
  // before thread 0's system-scope fence (the grid-barrier pattern), so one fence per CTA.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    last = atomicAdd(&g.state[1], 1u) == gridDim.x - 1;
    if (last) __threadfence_system();  // every CTA's arrival (and so its stores) before the exit flags
  }
  __syncthreads();
  if (!last) return;

  // exit (last CTA): release the exit flags, then wait for every rank's
  if ((int)threadIdx.x < g.world) st_release_sys(g.flags[threadIdx.x] + g.world + g.rank, e);
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!wait_all(g.flags[g.rank] + g.world, g.world, e)) set_status(g.status, kStatusTimeout);
    g.state[1] = 0;
    g.state[0] = e;
  }
}

int gfail(int code, const std::string& msg) { return set_error(code, msg); }

}  // namespace
}  // namespace b200

extern "C" {

int b200_shard_gather_params_size(void) { return (int)sizeof(B200ShardGatherParams); }

int b200_shard_gather(const B200ShardGatherParams* p, void* stream_ptr) {
  using namespace b200;
  if (!p) return gfail(B200_ERR_INVALID_ARGUMENT, "shard gather: null params");
  if (p->world < 1 || p->world > B200_SHARD_MAX_RANKS || p->rank < 0 || p->rank >= p->world)
    return gfail(B200_ERR_INVALID_ARGUMENT, "shard gather: world must be 1..8 and rank in [0, world)");
  if (p->rows < 0 || p->slice_bytes <= 0 || p->slice_bytes % 16)
    return gfail(B200_ERR_INVALID_ARGUMENT, "shard gather: rows >= 0 and slice_bytes a positive multiple of 16");
  if (!p->local || !p->state || reinterpret_cast<uintptr_t>(p->local) % 16)
    return gfail(B200_ERR_INVALID_ARGUMENT, "shard gather: local (16-byte aligned) and state are required");
  GatherArgs g{};
  for (int t = 0; t < p->world; ++t) {
    if (!p->outputs[t] || !p->flags[t] || reinterpret_cast<uintptr_t>(p->outputs[t]) % 16)
      return gfail(B200_ERR_INVALID_ARGUMENT, "shard gather: every rank's output (16-byte aligned) and flags are required");
    g.outputs[t] = static_cast<char*>(p->outputs[t]);
    g.flags[t] = p->flags[t];
  }
  g.world = p->world;
  g.rank = p->rank;
  g.rows = p->rows;
  g.vecs = p->slice_bytes / 16;
  g.slice_bytes = p->slice_bytes;
  g.local = static_cast<const uint4*>(p->local);
  g.state = p->state;
  g.status = p->status;
  int sms = p->num_sms;
  if (sms <= 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
  }
  // one wave (every CTA resident), at most one thread per 16-byte piece
  const int64_t pieces = (int64_t)p->rows * g.vecs * p->world;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(sms, (pieces + kGatherThreads - 1) / kGatherThreads));
  shard_gather_kernel<<<grid, kGatherThreads, 0, static_cast<cudaStream_t>(stream_ptr)>>>(g);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return gfail(B200_ERR_CUDA, std::string("shard gather: CUDA error: ") + cudaGetErrorString(e));
  add_launches(1);
  return B200_OK;
}

int b200_ipc_handle_size(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int b200_ipc_get_handle(const void* base, void* handle) {
  using namespace b200;
  if (!base || !handle) return gfail(B200_ERR_INVALID_ARGUMENT, "ipc: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(base));
  if (e != cudaSuccess) return gfail(B200_ERR_CUDA, std::string("ipc: cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  memcpy(handle, &h, sizeof(h));
  return B200_OK;
}

int b200_ipc_open_handle(int32_t device, const void* handle, void** ptr) {
  using namespace b200;
  if (!handle || !ptr) return gfail(B200_ERR_INVALID_ARGUMENT, "ipc: null pointer");
  *ptr = nullptr;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) {
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) return gfail(B200_ERR_CUDA, std::string("ipc: cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  return B200_OK;
}

int b200_ipc_close_handle(int32_t device, void* ptr) {
  using namespace b200;
  if (!ptr) return B200_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaIpcCloseMemHandle(ptr);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return gfail(B200_ERR_CUDA, std::string("ipc: cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
  return B200_OK;
}

}  // extern "C"
