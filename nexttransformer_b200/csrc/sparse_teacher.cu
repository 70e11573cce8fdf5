// Head-mean distillation teacher of the learned sparse indexers (DSA / QSA / Seer) without the
// [B, H, Q, T] score tensor:
//   teacher[b, i, j] = (1/H) sum_h softmax_j(s_hij | domain)   s_hij = scale q_hi . k_hj
// over the domain "key j <= absolute query position, j < T, mask[b, i, j]" (mask null: causal only);
// an empty domain gives zeros.  Two kernels:
//   lse:   one CTA per (64-query tile, batch x head); the 128-feature q tile stays in shared memory,
//          key tiles of 64 stream through it, each warp owns 16 query rows and keeps an online row
//          max / sum; writes the log-sum-exp (+inf for an empty row).
//   mean:  one CTA per (64-query tile, 64-key tile, batch), tiles above the causal diagonal return
//          at once (the output is zero-filled); for every head the q and k tiles come into shared
//          memory and exp(s - lse) accumulates in registers, then the mean is stored.
// Scores come from bf16 tensor-core MMAs (mma.sync m16n8k16, fp32 accumulation): the products of
// bf16 inputs are exact in fp32, as in the fp32 matmul of the reference path
// (nexttransformer/models/sparse_kernels.py:38-116 computes the same two passes in Triton).
#include "sparse_teacher.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace nt {
namespace teacher {

constexpr int TQ = 64, TK = 64, HD = 128;
constexpr int LDS = HD + 8;  // bf16 row stride of the shared tiles (272 B: conflict-free fragment loads)
constexpr int THREADS = 128;

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// rows [r0, r0 + rows) of a [.., 128] bf16 matrix with row stride ld (elements) into a shared tile;
// rows past `valid` are zero
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, int64_t ld, int r0,
                                          int rows, int valid) {
  for (int e = threadIdx.x; e < rows * (HD / 8); e += THREADS) {
    const int r = e / (HD / 8), c = (e % (HD / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r0 + r < valid) v = *reinterpret_cast<const uint4*>(src + (r0 + r) * ld + c);
    *reinterpret_cast<uint4*>(dst + r * LDS + c) = v;
  }
}

// S (16 rows of this warp x 64 keys) = q_tile rows [16w, 16w + 16) . k_tile^T, fp32 fragments:
// acc[n][0..1] row g, keys 8n + 2t, +1; acc[n][2..3] row g + 8
__device__ __forceinline__ void scores(const __nv_bfloat16* sq, const __nv_bfloat16* sk, float (&acc)[8][4]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  const __nv_bfloat16* qa = sq + (16 * warp + g) * LDS + 2 * t;
#pragma unroll
  for (int k0 = 0; k0 < HD; k0 += 16) {
    uint32_t a[4];
    a[0] = *reinterpret_cast<const uint32_t*>(qa + k0);
    a[1] = *reinterpret_cast<const uint32_t*>(qa + 8 * LDS + k0);
    a[2] = *reinterpret_cast<const uint32_t*>(qa + k0 + 8);
    a[3] = *reinterpret_cast<const uint32_t*>(qa + 8 * LDS + k0 + 8);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const __nv_bfloat16* kb = sk + (8 * n + g) * LDS + k0 + 2 * t;
      uint32_t b[2];
      b[0] = *reinterpret_cast<const uint32_t*>(kb);
      b[1] = *reinterpret_cast<const uint32_t*>(kb + 8);
      mma_bf16(acc[n], a, b);
    }
  }
}

__device__ __forceinline__ bool in_domain(const TeacherArgs& a, int b, int qi, int kj) {
  if (qi >= a.Q || kj >= a.T || kj > a.q_start + qi) return false;
  return a.mask == nullptr || a.mask[(static_cast<int64_t>(b) * a.Q + qi) * a.T + kj] != 0;
}

__global__ void __launch_bounds__(THREADS) lse_kernel(const TeacherArgs a) {
  __shared__ __align__(16) __nv_bfloat16 sq[TQ * LDS];
  __shared__ __align__(16) __nv_bfloat16 sk[TK * LDS];
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H, hk = h / (a.H / a.Hk);
  const int q0 = blockIdx.x * TQ;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  const __nv_bfloat16* q = a.q + static_cast<int64_t>(b) * a.sqb + static_cast<int64_t>(h) * a.sqh;
  const __nv_bfloat16* k = a.k + static_cast<int64_t>(b) * a.skb + static_cast<int64_t>(hk) * a.skh;
  load_tile(sq, q, a.sqt, q0, TQ, a.Q);
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int last_key = min(a.T - 1, a.q_start + min(q0 + TQ, a.Q) - 1);
  for (int k0 = 0; k0 <= last_key; k0 += TK) {
    __syncthreads();
    load_tile(sk, k, a.skt, k0, TK, a.T);
    __syncthreads();
    float acc[8][4];
    scores(sq, sk, acc);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int qi = q0 + 16 * warp + g + 8 * half;
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kj = k0 + 8 * n + 2 * t + e;
          float& s = acc[n][2 * half + e];
          s = in_domain(a, b, qi, kj) ? s * a.scale : -INFINITY;
          mx = fmaxf(mx, s);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m[half], mx);
      const float ref = m_new == -INFINITY ? 0.f : m_new;
      float sum = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) sum += expf(acc[n][2 * half + e] - ref);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      l[half] = l[half] * expf(m[half] - ref) + sum;
      m[half] = m_new;
    }
  }
  if (t == 0) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int qi = q0 + 16 * warp + g + 8 * half;
      if (qi < a.Q)
        a.lse[(static_cast<int64_t>(b) * a.H + h) * a.Q + qi] = l[half] > 0.f ? m[half] + logf(l[half]) : INFINITY;
    }
  }
}

__global__ void __launch_bounds__(THREADS) mean_kernel(const TeacherArgs a) {
  __shared__ __align__(16) __nv_bfloat16 sq[TQ * LDS];
  __shared__ __align__(16) __nv_bfloat16 sk[TK * LDS];
  const int q0 = blockIdx.x * TQ, k0 = blockIdx.y * TK, b = blockIdx.z;
  if (k0 > a.q_start + min(q0 + TQ, a.Q) - 1) return;  // entirely above the causal diagonal
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  float out[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) out[n][e] = 0.f;
  bool valid[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      valid[n][e] = in_domain(a, b, q0 + 16 * warp + g + 8 * (e >> 1), k0 + 8 * n + 2 * t + (e & 1));
  for (int h = 0; h < a.H; ++h) {
    const int hk = h / (a.H / a.Hk);
    __syncthreads();
    load_tile(sq, a.q + static_cast<int64_t>(b) * a.sqb + static_cast<int64_t>(h) * a.sqh, a.sqt, q0, TQ, a.Q);
    load_tile(sk, a.k + static_cast<int64_t>(b) * a.skb + static_cast<int64_t>(hk) * a.skh, a.skt, k0, TK, a.T);
    __syncthreads();
    float acc[8][4];
    scores(sq, sk, acc);
    float lz[2];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int qi = q0 + 16 * warp + g + 8 * half;
      lz[half] = qi < a.Q ? a.lse[(static_cast<int64_t>(b) * a.H + h) * a.Q + qi] : INFINITY;
    }
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (valid[n][e]) out[n][e] += expf(acc[n][e] * a.scale - lz[e >> 1]);
  }
  const float inv = 1.f / a.H;
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int qi = q0 + 16 * warp + g + 8 * (e >> 1), kj = k0 + 8 * n + 2 * t + (e & 1);
      if (qi < a.Q && kj < a.T) a.out[(static_cast<int64_t>(b) * a.Q + qi) * a.T + kj] = out[n][e] * inv;
    }
}

}  // namespace teacher
}  // namespace nt

int nt_sparse_teacher(const TeacherArgs& a, cudaStream_t s) {
  using namespace nt::teacher;
  if (a.B <= 0 || a.H <= 0 || a.Hk <= 0 || a.H % a.Hk || a.Q <= 0 || a.T <= 0 || a.D != HD || !a.q || !a.k ||
      !a.lse || !a.out)
    return -1;
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k)) & 15u || a.sqt % 8 || a.skt % 8 ||
      a.sqh % 8 || a.skh % 8 || a.sqb % 8 || a.skb % 8)
    return -1;
  lse_kernel<<<dim3((a.Q + TQ - 1) / TQ, a.B * a.H), THREADS, 0, s>>>(a);
  mean_kernel<<<dim3((a.Q + TQ - 1) / TQ, (a.T + TK - 1) / TK, a.B), THREADS, 0, s>>>(a);
  return 0;
}
