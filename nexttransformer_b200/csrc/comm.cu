// K8: data-parallel gradient reduce-scatter over NVLink peer memory (no NCCL on this path).
//
// Every rank's fp32 gradients live in one flat buffer of symmetric memory: the same allocation
// mapped into every rank's address space (peer pointers `peers[w]`).  Each rank owns a list of
// segments of that buffer (whole Muon matrices, row shards of the AdamW tables).  One kernel per
// rank reads its owned segments from every peer's buffer with plain vector loads over NVLink, sums
// them in the fixed order of ranks 0..world-1 (so every rank's result is bitwise reproducible),
// multiplies by `scale` (1 / world for an average) and writes the result in place into its own
// buffer - the segments no other rank reads.
//
// Synchronisation uses per-peer flags in each rank's signal pad (also symmetric memory):
//   entry:  block b stores `epoch` into slot (b, me) of every peer's pad with release semantics at
//           system scope, then waits until slot (b, p) of its own pad holds `epoch` for every peer
//           p: every rank's gradients are final before anyone reads them;
//   exit:   the same on a second slot region: no rank leaves (and lets the next backward overwrite
//           its buffer) before every peer has finished reading it.
// `epoch` grows by one per call on every rank.  Every wait is bounded by `timeout_ns`; on expiry the
// block records an error code, skips its share of the work and returns, and the host raises.
#include <cuda_runtime.h>
#include <stdint.h>

#include "comm.h"
#include "common.cuh"

namespace nt {
namespace comm {

NT_DEVICE void store_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
NT_DEVICE uint32_t load_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Block-level barrier with every peer through slot region `region` of the signal pads.
NT_DEVICE bool peer_barrier(const uint64_t* pads, int rank, int world, int region, uint32_t epoch,
                            uint64_t timeout_ns, uint32_t where) {
  bool ok = true;
  const int slots = gridDim.x * world;
  if (threadIdx.x < world) {
    const int p = threadIdx.x;
    __threadfence_system();  // this rank's earlier writes are visible system-wide before the flag
    uint32_t* remote = reinterpret_cast<uint32_t*>(pads[p]) + region * slots + blockIdx.x * world + rank;
    store_release_sys(remote, epoch);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(pads[rank]) + region * slots + blockIdx.x * world + p;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0;; ++i) {
      if (static_cast<int32_t>(load_acquire_sys(mine) - epoch) >= 0) break;
      if ((i & 63u) == 63u && global_ns() - t0 > timeout_ns) {
        record_error(3u, where + p);
        ok = false;
        break;
      }
    }
  }
  return __syncthreads_and(ok ? 1 : 0) != 0;
}

__global__ void __launch_bounds__(256) p2p_reduce_scatter_kernel(const uint64_t* __restrict__ peers,
                                                                 const uint64_t* __restrict__ pads,
                                                                 const int64_t* __restrict__ seg_off,
                                                                 const int64_t* __restrict__ seg_len, int nseg,
                                                                 int rank, int world, float scale, uint32_t epoch,
                                                                 uint64_t timeout_ns) {
  const bool ok = peer_barrier(pads, rank, world, 0, epoch, timeout_ns, 0x800u);
  if (ok) {
    float* mine = reinterpret_cast<float*>(peers[rank]);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int s = 0; s < nseg; ++s) {
      const int64_t off = seg_off[s], n4 = seg_len[s] >> 2;
      for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < world; ++p) {
          const float4 v = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(peers[p]) + off)[i];
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
        reinterpret_cast<float4*>(mine + off)[i] = acc;
      }
    }
  }
  peer_barrier(pads, rank, world, 1, epoch, timeout_ns, 0x900u);
}

// Parameter all-gather over peer memory: after an entry barrier (every owner has written its
// updated fp32 parameters), every segment owned by another rank is read from the owner's
// buffer with plain peer loads and written here; every segment with a shadow pointer also gets
// its bf16 copy written (the forward reads the shadows).  Its barriers use slot regions 2 and 3,
// the reduce-scatter's 0 and 1, so the two kernels never see each other's flags even when their
// buffers share one allocation (and with it one signal pad).
__global__ void __launch_bounds__(256) p2p_gather_kernel(const uint64_t* __restrict__ peers,
                                                         const uint64_t* __restrict__ pads,
                                                         const int64_t* __restrict__ seg_off,
                                                         const int64_t* __restrict__ seg_len,
                                                         const int* __restrict__ seg_owner,
                                                         const uint64_t* __restrict__ seg_shadow, int nseg, int rank,
                                                         int world, uint32_t epoch, uint64_t timeout_ns) {
  const bool ok = peer_barrier(pads, rank, world, 2, epoch, timeout_ns, 0xB00u);
  if (ok) {
    float* mine = reinterpret_cast<float*>(peers[rank]);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int s = 0; s < nseg; ++s) {
      const int owner = seg_owner[s];
      const int64_t off = seg_off[s], n4 = seg_len[s] >> 2;
      const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(peers[owner]) + off);
      float4* dst = reinterpret_cast<float4*>(mine + off);
      uint2* sh = reinterpret_cast<uint2*>(seg_shadow[s]);
      for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 v = src[i];
        if (owner != rank) dst[i] = v;
        if (sh) sh[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
      }
    }
  }
  // no owner updates its segments again before every peer has finished copying them
  peer_barrier(pads, rank, world, 3, epoch, timeout_ns, 0xC00u);
}

// A standalone barrier with every peer (one block; region 0 of the pads, `world` slots).
__global__ void p2p_barrier_kernel(const uint64_t* __restrict__ pads, int rank, int world, uint32_t epoch,
                                   uint64_t timeout_ns) {
  peer_barrier(pads, rank, world, 0, epoch, timeout_ns, 0xA00u);
}

// Copy n16 16-byte words from src to byte offset dst_off of every peer's buffer (plain peer stores).
__global__ void p2p_put_kernel(const uint64_t* __restrict__ peers, int world, int64_t dst_off,
                               const uint4* __restrict__ src, int64_t n16) {
  for (int p = 0; p < world; ++p) {
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(peers[p]) + dst_off);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
      dst[i] = src[i];
  }
}

}  // namespace comm
}  // namespace nt

int nt_p2p_gather(const uint64_t* peers_dev, const uint64_t* pads_dev, const int64_t* seg_off, const int64_t* seg_len,
                  const int* seg_owner, const uint64_t* seg_shadow, int nseg, int rank, int world, uint32_t epoch,
                  int blocks, uint64_t timeout_ns, cudaStream_t stream) {
  if (world < 1 || world > 64 || blocks < 1 || rank < 0 || rank >= world) return -1;
  nt::comm::p2p_gather_kernel<<<blocks, 256, 0, stream>>>(peers_dev, pads_dev, seg_off, seg_len, seg_owner, seg_shadow,
                                                          nseg, rank, world, epoch, timeout_ns);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int nt_p2p_barrier(const uint64_t* pads_dev, int rank, int world, uint32_t epoch, uint64_t timeout_ns,
                   cudaStream_t stream) {
  if (world < 1 || world > 64 || rank < 0 || rank >= world) return -1;
  nt::comm::p2p_barrier_kernel<<<1, 64, 0, stream>>>(pads_dev, rank, world, epoch, timeout_ns);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int nt_p2p_put(const uint64_t* peers_dev, int world, int64_t dst_off, const void* src, int64_t nbytes,
               cudaStream_t stream) {
  if (world < 1 || nbytes % 16 || dst_off % 16 || reinterpret_cast<uintptr_t>(src) % 16) return -1;
  const int64_t n16 = nbytes / 16;
  if (!n16) return 0;
  const int blocks = static_cast<int>(n16 / 256 + 1 < 64 ? n16 / 256 + 1 : 64);
  nt::comm::p2p_put_kernel<<<blocks, 256, 0, stream>>>(peers_dev, world, dst_off, reinterpret_cast<const uint4*>(src),
                                                       n16);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int nt_p2p_reduce_scatter(const uint64_t* peers_dev, const uint64_t* pads_dev, const int64_t* seg_off,
                          const int64_t* seg_len, int nseg, int rank, int world, float scale, uint32_t epoch,
                          int blocks, uint64_t timeout_ns, cudaStream_t stream) {
  if (world < 1 || world > 64 || blocks < 1 || rank < 0 || rank >= world) return -1;
  nt::comm::p2p_reduce_scatter_kernel<<<blocks, 256, 0, stream>>>(peers_dev, pads_dev, seg_off, seg_len, nseg, rank,
                                                                  world, scale, epoch, timeout_ns);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -2;
}

int nt_comm_read_error(unsigned* where) {
  nt::ErrorWord w{0, 0};
  cudaMemcpyFromSymbol(&w, nt::g_nt_error, sizeof(w));
  if (where) *where = w.where;
  return static_cast<int>(w.code);
}

int nt_comm_clear_error() {
  const nt::ErrorWord zero{0, 0};
  return cudaMemcpyToSymbol(nt::g_nt_error, &zero, sizeof(zero)) == cudaSuccess ? 0 : -2;
}
