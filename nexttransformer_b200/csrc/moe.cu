// Mixture-of-experts data movement on sm_100a: the row permutations around the grouped expert
// GEMMs, the weighted combine and their backward, and the expert-parallel exchange over NVLink
// peer memory.
//
// Layout: the (token, slot) assignments are laid out expert by expert, each expert's segment
// padded to a multiple of 128 rows (so every 128-row GEMM tile belongs to one expert); padding
// rows are zero.  `src_of[row]` names the token a row is copied from (-1: padding) and
// `row_of[t * k + s]` the row holding assignment (t, s).
//
// Expert parallelism: every rank lays its own assignments out in owner order in a send buffer
// (symmetric memory).  The owner of a group of experts PULLS its rows from the peers' send
// buffers with plain peer loads (`moe_pull_rows`), runs the grouped GEMMs on local memory, and
// PUSHES the result rows back into the peers' return buffers with plain peer stores
// (`moe_push_rows`); a flag barrier over the symmetric signal pads (comm.cu) orders the phases.
// No TMA load ever reads another GPU's memory.
#include <stdexcept>

#include "common.cuh"
#include "moe.h"

namespace nt {
namespace {

constexpr int WARPS = 8;  // rows per 256-thread block, one warp per row

NT_DEVICE void add8(float* acc, uint4 v, float w) {
  const uint32_t x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(x[i]);
    acc[2 * i] += w * f.x;
    acc[2 * i + 1] += w * f.y;
  }
}
NT_DEVICE uint4 pack8f(const float* f) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

// out[r] = src[src_of[r]] (zero row when src_of[r] < 0); d % 8 == 0
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ src, const int* __restrict__ src_of,
                                   __nv_bfloat16* __restrict__ out, int64_t rows, int d) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const int s = src_of[r];
  uint4* o = reinterpret_cast<uint4*>(out + r * d);
  if (s < 0) {
    for (int c = lane; c < d / 8; c += 32) o[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* i = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(s) * d);
  for (int c = lane; c < d / 8; c += 32) o[c] = i[c];
}

// out[t] = sum_s w[t, s] rows[row_of[t, s]]  (+ add[t] when given); fp32 accumulation
__global__ void combine_kernel(const __nv_bfloat16* __restrict__ rows, const int* __restrict__ row_of,
                               const float* __restrict__ w, const __nv_bfloat16* __restrict__ add,
                               __nv_bfloat16* __restrict__ out, int T, int k, int d) {
  const int t = blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  for (int c = lane; c < d / 8; c += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (add) add8(acc, reinterpret_cast<const uint4*>(add + static_cast<int64_t>(t) * d)[c], 1.f);
    for (int s = 0; s < k; ++s) {
      const int r = row_of[t * k + s];
      add8(acc, reinterpret_cast<const uint4*>(rows + static_cast<int64_t>(r) * d)[c], w ? w[t * k + s] : 1.f);
    }
    reinterpret_cast<uint4*>(out + static_cast<int64_t>(t) * d)[c] = pack8f(acc);
  }
}

// Backward of combine: d_rows[row_of[t, s]] = w[t, s] dy[t];  dw[t, s] = dy[t] . rows[row_of[t, s]]
__global__ void combine_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ rows,
                                   const int* __restrict__ row_of, const float* __restrict__ w,
                                   __nv_bfloat16* __restrict__ d_rows, float* __restrict__ dw, int T, int k, int d) {
  const int j = blockIdx.x * WARPS + (threadIdx.x >> 5);  // assignment index t * k + s
  if (j >= T * k) return;
  const int lane = threadIdx.x & 31;
  const int t = j / k;
  const int r = row_of[j];
  const float wj = w[j];
  const uint4* g = reinterpret_cast<const uint4*>(dy + static_cast<int64_t>(t) * d);
  const uint4* y = reinterpret_cast<const uint4*>(rows + static_cast<int64_t>(r) * d);
  uint4* o = reinterpret_cast<uint4*>(d_rows + static_cast<int64_t>(r) * d);
  float dot = 0.f;
  for (int c = lane; c < d / 8; c += 32) {
    float gf[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, yf[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    add8(gf, g[c], 1.f);
    add8(yf, y[c], 1.f);
    float sc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      dot += gf[e] * yf[e];
      sc[e] = gf[e] * wj;
    }
    o[c] = pack8f(sc);
  }
  dot = warp_sum(dot);
  if (lane == 0) dw[j] = dot;
}

// Expert parallelism: out[r] = peers[src_rank[r]][src_row[r]] over plain peer loads (zero when
// src_rank[r] < 0).  peers[i] is rank i's send buffer (bf16 rows of d).
__global__ void pull_rows_kernel(const uint64_t* __restrict__ peers, const int* __restrict__ src_rank,
                                 const int* __restrict__ src_row, __nv_bfloat16* __restrict__ out, int64_t rows,
                                 int d) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const int pr = src_rank[r];
  uint4* o = reinterpret_cast<uint4*>(out + r * d);
  if (pr < 0) {
    for (int c = lane; c < d / 8; c += 32) o[c] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* i = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(peers[pr]) +
                                                  static_cast<int64_t>(src_row[r]) * d);
  for (int c = lane; c < d / 8; c += 32) o[c] = i[c];
}

// Expert parallelism: peers[dst_rank[r]][dst_row[r]] = rows[r] over plain peer stores (rows with
// dst_rank < 0 are padding and stay here).
__global__ void push_rows_kernel(const __nv_bfloat16* __restrict__ rows, const uint64_t* __restrict__ peers,
                                 const int* __restrict__ dst_rank, const int* __restrict__ dst_row, int64_t n,
                                 int d) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5);
  if (r >= n) return;
  const int pr = dst_rank[r];
  if (pr < 0) return;
  const int lane = threadIdx.x & 31;
  const uint4* i = reinterpret_cast<const uint4*>(rows + r * d);
  uint4* o = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers[pr]) + static_cast<int64_t>(dst_row[r]) * d);
  for (int c = lane; c < d / 8; c += 32) o[c] = i[c];
}

unsigned blocks_for(int64_t rows) { return static_cast<unsigned>((rows + WARPS - 1) / WARPS); }

}  // namespace
}  // namespace nt

using namespace nt;

int nt_moe_gather_rows(const void* src, const int* src_of, void* out, int64_t rows, int d, cudaStream_t s) {
  if (d % 8 || rows < 0) return -1;
  if (!rows) return 0;
  gather_rows_kernel<<<blocks_for(rows), 32 * WARPS, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(src), src_of,
                                                              reinterpret_cast<__nv_bfloat16*>(out), rows, d);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int nt_moe_combine(const void* rows, const int* row_of, const float* w, const void* add, void* out, int T, int k, int d,
                   cudaStream_t s) {
  if (d % 8 || T < 0 || k <= 0) return -1;
  if (!T) return 0;
  combine_kernel<<<blocks_for(T), 32 * WARPS, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(rows), row_of, w,
                                                       reinterpret_cast<const __nv_bfloat16*>(add),
                                                       reinterpret_cast<__nv_bfloat16*>(out), T, k, d);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int nt_moe_combine_bwd(const void* dy, const void* rows, const int* row_of, const float* w, void* d_rows, float* dw,
                       int T, int k, int d, cudaStream_t s) {
  if (d % 8 || T < 0 || k <= 0) return -1;
  if (!T) return 0;
  combine_bwd_kernel<<<blocks_for(static_cast<int64_t>(T) * k), 32 * WARPS, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy), reinterpret_cast<const __nv_bfloat16*>(rows), row_of, w,
      reinterpret_cast<__nv_bfloat16*>(d_rows), dw, T, k, d);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int nt_moe_pull_rows(const uint64_t* peers, const int* src_rank, const int* src_row, void* out, int64_t rows, int d,
                     cudaStream_t s) {
  if (d % 8 || rows < 0) return -1;
  if (!rows) return 0;
  pull_rows_kernel<<<blocks_for(rows), 32 * WARPS, 0, s>>>(peers, src_rank, src_row,
                                                            reinterpret_cast<__nv_bfloat16*>(out), rows, d);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int nt_moe_push_rows(const void* rows, const uint64_t* peers, const int* dst_rank, const int* dst_row, int64_t n, int d,
                     cudaStream_t s) {
  if (d % 8 || n < 0) return -1;
  if (!n) return 0;
  push_rows_kernel<<<blocks_for(n), 32 * WARPS, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(rows), peers, dst_rank,
                                                         dst_row, n, d);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
