// Known-answer self-test of the tcgen05 building blocks the prefill kernel is made of.
//
// One CTA computes, for 128x128x128 tiles of fp16/bf16:
//   C_qk = A . B^T   A written into swizzled shared memory by threads (as P is), B by TMA
//                    (both K-major, 128B swizzle)
//   C_pv = A . V     V by TMA as [K rows][N contiguous] (MN-major B operand)
//   C_ts = A . V     the same product with A held in tensor memory (lane = row, two 16-bit
//                    elements per column), written there by the threads with tcgen05.st
// with tcgen05.mma accumulating in tensor memory, tcgen05.commit on an mbarrier and 32x32b
// tensor-memory loads.  The test compares against torch.matmul; a wrong descriptor bit shows
// up as a wrong product, not as a fault.
#include "b200_common.cuh"
#include "b200_kernels.h"
#include "b200_tcgen05.cuh"

namespace b200 {

struct SelfTestMaps {
  CUtensorMap b_map;  // [128 rows][128] box {64, 128}
  CUtensorMap v_map;  // [128 K rows][128 N] box {64, 128}
};

template <bool BF16>
__global__ void __launch_bounds__(128) tc_selftest_kernel(const __grid_constant__ SelfTestMaps maps, const void* a,
                                                           float* c_qk, float* c_pv, float* c_ts, int* status) {
  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) uint64_t tma_bar, mma_bar;
  __shared__ uint32_t tmem_slot;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;            // A: 2 x [128][64] swizzled, 32 KB
  uint8_t* sb = smem + 32768;    // B: 2 x [128][64]
  uint8_t* sv = smem + 65536;    // V: 2 x [128 K][64 N]
  const int tid = threadIdx.x, warp = tid >> 5;

  if (warp == 0) tc::alloc(&tmem_slot, 512);
  if (tid == 0) {
    mbar_init(&tma_bar, 1);
    mbar_init(&mma_bar, 1);
    fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tmem_slot;

  if (tid == 0) {
    mbar_arrive_expect_tx(&tma_bar, 65536);
    for (int h = 0; h < 2; ++h) {
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
          ::"r"(smem_u32(sb + h * 16384)), "l"(reinterpret_cast<uint64_t>(&maps.b_map)), "r"(h * 64), "r"(0),
          "r"(smem_u32(&tma_bar)) : "memory");
      asm volatile(
          "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
          ::"r"(smem_u32(sv + h * 16384)), "l"(reinterpret_cast<uint64_t>(&maps.v_map)), "r"(h * 64), "r"(0),
          "r"(smem_u32(&tma_bar)) : "memory");
    }
  }
  // Thread r writes row r of A (128 elements = 16 chunks of 16 B) in the swizzled K-major layout.
  {
    const uint4* src = reinterpret_cast<const uint4*>(a) + tid * 16;
    for (int c = 0; c < 16; ++c) {
      uint4 v = src[c];
      *reinterpret_cast<uint4*>(sa + (c >> 3) * 16384 + tc::sw128(tid, c & 7)) = v;
    }
  }
  {
    // A row tid -> tensor memory columns [256, 320): 64 columns of two 16-bit elements
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a) + tid * 64;
    const uint32_t row_addr = tmem_slot + ((uint32_t)((warp & 3) * 32) << 16) + 256;
    for (int c = 0; c < 4; ++c) {
      uint32_t w[16];
      for (int i = 0; i < 16; ++i) w[i] = src[c * 16 + i];
      tc::st16u(row_addr + c * 16, w);
    }
    tc::wait_st();
  }
  fence_proxy_async_smem();
  tc::fence_before_sync();
  __syncthreads();
  if (!mbar_wait(&tma_bar, 0)) {
    if (tid == 0) set_status(status, kStatusTimeout);
  }
  tc::fence_after_sync();
  if (tid == 0) {
    constexpr uint32_t id_kk = tc::idesc_f16(128, 128, BF16, false, false);
    constexpr uint32_t id_kn = tc::idesc_f16(128, 128, BF16, false, true);
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t koff = (kk >> 2) * 16384 + (kk & 3) * 32;
      tc::mma_ss(tmem, tc::smem_desc(smem_u32(sa) + koff, 16, 1024), tc::smem_desc(smem_u32(sb) + koff, 16, 1024),
                 id_kk, kk > 0);
    }
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
      const uint32_t voff = kk * 2048;  // 16 K rows further
      tc::mma_ss(tmem + 128, tc::smem_desc(smem_u32(sa) + aoff, 16, 1024),
                 tc::smem_desc(smem_u32(sv) + voff, 16384, 1024), id_kn, kk > 0);
    }
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t voff = kk * 2048;
      tc::mma_ts(tmem + 384, tmem + 256 + kk * 8, tc::smem_desc(smem_u32(sv) + voff, 16384, 1024), id_kn, kk > 0);
    }
    tc::commit(&mma_bar);
  }
  __syncwarp();
  if (!mbar_wait(&mma_bar, 0)) {
    if (tid == 0) set_status(status, kStatusTimeout);
  }
  tc::fence_after_sync();
  const int row = (warp & 3) * 32 + (tid & 31);
  const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  for (int j = 0; j < 8; ++j) {
    float r[16];
    tc::ld16(lane_addr + j * 16, r);
    tc::wait_ld();
    for (int i = 0; i < 16; ++i) c_qk[row * 128 + j * 16 + i] = r[i];
    tc::ld16(lane_addr + 128 + j * 16, r);
    tc::wait_ld();
    for (int i = 0; i < 16; ++i) c_pv[row * 128 + j * 16 + i] = r[i];
    if (c_ts) {
      tc::ld16(lane_addr + 384 + j * 16, r);
      tc::wait_ld();
      for (int i = 0; i < 16; ++i) c_ts[row * 128 + j * 16 + i] = r[i];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::dealloc(tmem, 512);
}

cudaError_t launch_tc_selftest(bool bf16, const void* a, const void* b, const void* v, float* c_qk, float* c_pv,
                               float* c_ts, int* status, cudaStream_t stream, int* cu_result) {
  SelfTestMaps maps;
  const uint64_t dims[2] = {128, 128};
  const uint64_t strides[1] = {256};
  const uint32_t box[2] = {64, 128};
  *cu_result = encode_tensor_map(&maps.b_map, bf16, 2, b, dims, strides, box);
  if (*cu_result) return cudaErrorInvalidValue;
  *cu_result = encode_tensor_map(&maps.v_map, bf16, 2, v, dims, strides, box);
  if (*cu_result) return cudaErrorInvalidValue;
  const int smem = 3 * 32768 + 1024;
  if (bf16) {
    cudaFuncSetAttribute(tc_selftest_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    tc_selftest_kernel<true><<<1, 128, smem, stream>>>(maps, a, c_qk, c_pv, c_ts, status);
  } else {
    cudaFuncSetAttribute(tc_selftest_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    tc_selftest_kernel<false><<<1, 128, smem, stream>>>(maps, a, c_qk, c_pv, c_ts, status);
  }
  return cudaGetLastError();
}

}  // namespace b200
