// Host interface of the peer-memory collectives (comm.cu).
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

// In-place reduce-scatter over symmetric memory: for every owned segment (element offset, length;
// both multiples of 4) buf_me[seg] = scale * sum_w buf_w[seg].  `peers_dev` / `pads_dev` are device
// arrays of the world's buffer and signal-pad pointers; `epoch` grows by one per call on every rank.
// The signal pads need 2 * blocks * world 32-bit slots.
int nt_p2p_reduce_scatter(const uint64_t* peers_dev, const uint64_t* pads_dev, const int64_t* seg_off,
                          const int64_t* seg_len, int nseg, int rank, int world, float scale, uint32_t epoch,
                          int blocks, uint64_t timeout_ns, cudaStream_t stream);
// Parameter all-gather over symmetric memory: segment s (element offset, length, both multiples of 4)
// is read from rank seg_owner[s]'s buffer into this rank's (skipped when owned here) and, when
// seg_shadow[s] != 0, written as bf16 to that address.  One entry barrier; `blocks * world` slots.
int nt_p2p_gather(const uint64_t* peers_dev, const uint64_t* pads_dev, const int64_t* seg_off, const int64_t* seg_len,
                  const int* seg_owner, const uint64_t* seg_shadow, int nseg, int rank, int world, uint32_t epoch,
                  int blocks, uint64_t timeout_ns, cudaStream_t stream);
// Barrier with every peer (bounded wait; needs `world` 32-bit signal-pad slots; epoch as above).
int nt_p2p_barrier(const uint64_t* pads_dev, int rank, int world, uint32_t epoch, uint64_t timeout_ns,
                   cudaStream_t stream);
// Copy nbytes (multiple of 16) from local src to byte offset dst_off of every peer's buffer.
int nt_p2p_put(const uint64_t* peers_dev, int world, int64_t dst_off, const void* src, int64_t nbytes,
               cudaStream_t stream);
int nt_comm_read_error(unsigned* where);
// Reset the error word after the host has handled a recorded failure (synchronous).
int nt_comm_clear_error();
