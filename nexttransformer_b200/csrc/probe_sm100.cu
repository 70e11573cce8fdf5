// tcgen05.mma issue-rate probe (microbenchmark, not on any training path): one CTA per SM, one
// thread issues `groups` groups of eight MMAs of K = 16 into one accumulator, then commits and waits.
// Each CTA reports the clocks its issue loop took and the clocks until the last MMA completed.
// Operands are zeroed shared memory and tensor memory; only the rate matters.
//   variant 0: k-step loop rolled, descriptors computed each step (issue-bound form)
//           1: k-steps unrolled (SS, 128 x 128 x 16)
//           2: as 1 with N = 256
//           3: as 1 with A read from tensor memory (the P V form)
#include "probe_sm100.h"
#include "common.cuh"

namespace nt {
namespace probe {

constexpr int BOX = 128 * 128;  // one [128 rows x 64 bf16] box with 128-byte rows
constexpr int OPERAND_BYTES = 6 * 32768;

__device__ __forceinline__ uint64_t kdesc(uint32_t base, int j) {
  return smem_desc(base + (j >> 2) * BOX + (j & 3) * 32, 16, 1024);
}
__device__ __forceinline__ uint64_t mndesc(uint32_t base, int j) { return smem_desc(base + j * 2048, BOX, 1024); }

template <int V>
__global__ void __launch_bounds__(128, 1) mma_rate_kernel(long long* out, int groups) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OPERAND_BYTES);
  uint32_t* holder = reinterpret_cast<uint32_t*>(bar + 2);
  for (int i = threadIdx.x; i < OPERAND_BYTES / 16; i += blockDim.x) reinterpret_cast<uint4*>(sm)[i] = make_uint4(0, 0, 0, 0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(holder, 512);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = *holder;
  const uint32_t a_addr = smem_u32(sm), b_addr = smem_u32(sm + 2 * 32768);
  constexpr uint32_t id128 = idesc_bf16_f32(128, 128, 0, 0);
  constexpr uint32_t id256 = idesc_bf16_f32(128, 256, 0, 0);
  constexpr uint32_t idpv = idesc_bf16_f32(128, 128, 0, 1);
  if (warp == 0) {
    long long t0 = 0, t1 = 0;
    if (lane == 0) {
      t0 = clock64();
      for (int g = 0; g < groups; ++g) {
        if (V == 0) {
#pragma unroll 1
          for (int q = 0; q < 8; ++q) umma_bf16(tb, kdesc(a_addr, q), kdesc(b_addr, q), id128, g > 0 || q > 0);
        } else if (V == 1) {
#pragma unroll
          for (int q = 0; q < 8; ++q) umma_bf16(tb, kdesc(a_addr, q), kdesc(b_addr, q), id128, g > 0 || q > 0);
        } else if (V == 2) {
#pragma unroll
          for (int q = 0; q < 8; ++q) umma_bf16(tb, kdesc(a_addr, q), kdesc(b_addr, q), id256, g > 0 || q > 0);
        } else {
#pragma unroll
          for (int q = 0; q < 8; ++q) umma_bf16_tmem_a(tb, tb + 256 + q * 8, mndesc(b_addr, q), idpv, g > 0 || q > 0);
        }
      }
      umma_commit(bar);
      t1 = clock64();
    }
    __syncwarp();
    const bool ok = mbar_wait(bar, 0, 0x900u, nullptr);
    const long long t2 = clock64();
    if (lane == 0) {
      out[blockIdx.x * 3 + 0] = t1 - t0;
      out[blockIdx.x * 3 + 1] = t2 - t0;
      out[blockIdx.x * 3 + 2] = ok ? 1 : 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tb, 512);
}

}  // namespace probe
}  // namespace nt

int nt_mma_rate(int variant, int groups, int ctas, long long* out, cudaStream_t s) {
  using namespace nt::probe;
  const int smem = OPERAND_BYTES + 1024 + 64;
  auto run = [&](auto kern) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -1;
    kern<<<ctas, 128, smem, s>>>(out, groups);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  };
  if (groups <= 0 || ctas <= 0) return -1;
  switch (variant) {
    case 0: return run(mma_rate_kernel<0>);
    case 1: return run(mma_rate_kernel<1>);
    case 2: return run(mma_rate_kernel<2>);
    case 3: return run(mma_rate_kernel<3>);
    default: return -1;
  }
}
