// Shared device helpers for the B200 paged-KV attention kernels (sm_100a).
//
// Element access for every cache storage type, the device status word, and thin inline-PTX
// wrappers for mbarrier, TMA (cp.async.bulk.tensor, single-CTA destination), ldmatrix / movmatrix and
// the m16n8k16 tensor-core MMA.  Every spin-wait is bounded by %globaltimer and reports a
// timeout through the status word instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "b200_kernels.h"
#include "b200_paged.h"

namespace b200 {

__device__ __forceinline__ void set_status(int* status, int bits) {
  if (status) atomicOr(status, bits);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound for any single wait on an mbarrier (TMA completion).  A TMA of a few KB
// completes in microseconds; one second means the hardware is not answering.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

// ---------------------------------------------------------------------------------------
// Scalar conversions.  Activations are fp16 or bf16; caches add int8, int4 (uint8 pairs)
// and fp8 e4m3.
// ---------------------------------------------------------------------------------------
template <typename T> struct act;
template <> struct act<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct act<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

__device__ __forceinline__ float load_act(const void* p, int64_t i, int dtype) {
  if (dtype == B200_DTYPE_BFLOAT16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(reinterpret_cast<const __half*>(p)[i]);
}
__device__ __forceinline__ float round_act(float x, int dtype) {
  if (dtype == B200_DTYPE_BFLOAT16) return __bfloat162float(__float2bfloat16_rn(x));
  return __half2float(__float2half_rn(x));
}
__device__ __forceinline__ void store_act(void* p, int64_t i, float x, int dtype) {
  if (dtype == B200_DTYPE_BFLOAT16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(x);
  else reinterpret_cast<__half*>(p)[i] = __float2half_rn(x);
}

// Integer KV encode, PagedAttention variant (kv_cache.rs:170-220): IEEE divide by the scale,
// zero scale -> code 0, round half to even, clip to the signed range.
__device__ __forceinline__ int quant_code(float x, float scale, int bits) {
  float scaled = (scale == 0.0f) ? 0.0f : __fdiv_rn(x, scale);
  float lo = bits == 8 ? -128.0f : -8.0f, hi = bits == 8 ? 127.0f : 7.0f;
  scaled = fminf(fmaxf(scaled, lo), hi);
  return __float2int_rn(scaled);  // round-half-even on an in-range value
}

// fp8 e4m3 (fn) with saturation to +-448, round to nearest even.
__device__ __forceinline__ uint8_t fp8_code(float x, float scale) {
  float y = __fdiv_rn(x, scale);
  return (uint8_t)__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float fp8_value(uint8_t c) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)c, __NV_E4M3);
  return __half2float(__half(h));
}

// Cache element description used by the generic kernels.
struct CacheView {
  const void* data;     // [NB, bs, KV, width]
  int dtype;            // B200_DTYPE_*
  int width;            // stored elements per (slot, head): d, or ceil(d/2) for int4
  const float* scale;   // int8/int4: [1] or [KV*d]; fp8: [NB*KV] per block and head
  int per_channel;      // int8/int4 only
};

__device__ __forceinline__ float cache_value(const CacheView& c, int64_t slot, int kv_heads, int head,
                                             int d, int head_size, int block_size) {
  int64_t row = (slot * kv_heads + head) * (int64_t)c.width;
  switch (c.dtype) {
    case B200_DTYPE_FLOAT16: return __half2float(reinterpret_cast<const __half*>(c.data)[row + d]);
    case B200_DTYPE_BFLOAT16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(c.data)[row + d]);
    case B200_DTYPE_INT8: {
      float s = c.per_channel ? c.scale[head * head_size + d] : c.scale[0];
      return (float)reinterpret_cast<const int8_t*>(c.data)[row + d] * s;
    }
    case B200_DTYPE_UINT8: {
      uint8_t byte = reinterpret_cast<const uint8_t*>(c.data)[row + d / 2];
      int code = (d & 1) ? (byte >> 4) : (byte & 15);
      float s = c.per_channel ? c.scale[head * head_size + d] : c.scale[0];
      return (float)(code - 8) * s;
    }
    case B200_DTYPE_FLOAT8E4M3FN: {
      float s = c.scale[(slot / block_size) * kv_heads + head];
      return fp8_value(reinterpret_cast<const uint8_t*>(c.data)[row + d]) * s;
    }
    default: return 0.0f;
  }
}

// ---------------------------------------------------------------------------------------
// Inline PTX: shared-memory addresses, mbarrier, TMA, ldmatrix, movmatrix, mma.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on a phase of an mbarrier; false once kWaitLimitNs has passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - start > kWaitLimitNs) return false;
  }
}

// Non-blocking probe of a phase (mbarrier.test_wait never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait that spins on test_wait instead of letting try_wait suspend the thread: for a
// waiter on the critical path that must react to the phase change within a few cycles.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity) {
  if (mbar_test_wait(bar, parity)) return true;
  uint64_t start = globaltimer_ns();
  while (true) {
    for (int i = 0; i < 256; ++i)
      if (mbar_test_wait(bar, parity)) return true;
    if (globaltimer_ns() - start > kWaitLimitNs) return false;
  }
}

// 3-D tiled TMA load global -> this CTA's shared memory, completion counted on an mbarrier.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory (both addresses 16-byte aligned, bytes a
// multiple of 16), completion counted on an mbarrier.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy this CTA's shared memory -> global (both addresses 16-byte aligned, bytes a
// multiple of 16), tracked by the issuing thread's bulk groups: bulk_commit() closes a group and
// bulk_wait_read() waits until every committed copy has read its shared-memory source.  Shared
// memory written by threads (generic proxy) needs fence_proxy_async_smem() by each writer and a
// barrier before the copy is issued.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T> struct mma_op;
template <> struct mma_op<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t v) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v));
  }
};
template <> struct mma_op<__half> {
  static __device__ __forceinline__ void run(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t v) {
    return __half22float2(*reinterpret_cast<__half2*>(&v));
  }
};

// Sequence owning a packed token: largest b with cum[b] <= t (binary search over B+1 entries).
__device__ __forceinline__ int seq_of_token(const int32_t* cum, int batch, int t) {
  int lo = 0, hi = batch - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (cum[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

}  // namespace b200
