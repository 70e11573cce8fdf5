// Fused mixture-of-experts routing on sm_100a: from fp32 router logits to the grouped-GEMM row plan.
//
//   route   (one CTA per 128 tokens, one warp per token at a time): softmax over the E logits,
//           top-k of (probability + selection bias) by repeated warp arg-max (ties to the lower
//           expert), the chosen probabilities normalised over the k, the log-sum-exp, and the
//           block's per-expert assignment counts, probability sums and sum of lse^2 (fixed-order
//           sums: no atomics anywhere, so the plan is bitwise reproducible);
//   plan    (one CTA): per-expert totals and each block's offset inside the expert's segment
//           (lanes scan blocks, warp shuffles combine them), segments padded to 128 rows, the
//           tile -> expert table, the padding rows of src_of, the load statistic, and the
//           Switch balance loss / z-loss with the balance loss's per-expert gradient;
//   scatter (one CTA per 128 tokens): the row of every (token, choice) in flat order, via
//           match-any within a warp and per-warp counts across the CTA, and src_of.
//   route_bwd: d logits of the normalised weights (w_s = softmax over the chosen logits, so
//           dl_c = w (dw - sum w dw)) and of both losses.
// The unfused form (torch softmax / topk / gather / bincount / stable argsort / searchsorted) is
// the oracle in the tests; the reference routes in Megatron's router
// (nexttransformer/scaling/megatron_moe.py:153-182).
#include "moe_route.h"

#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <stdint.h>

namespace nt {
namespace route {

constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;
constexpr int TOK_PER_WARP = NT_ROUTE_TOKENS / WARPS;

__device__ __forceinline__ float wmax(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float wsum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int wsum_i(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int VPL>
__global__ void __launch_bounds__(THREADS) route_kernel(const MoeRouteArgs a) {
  __shared__ float s_prob[WARPS][256];
  __shared__ int s_cnt[WARPS][256];
  __shared__ float s_z[WARPS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = blockIdx.x;
  float psum[VPL], bias[VPL];
  int cnt[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    psum[i] = 0.f;
    cnt[i] = 0;
    bias[i] = a.bias ? a.bias[lane + 32 * i] : 0.f;
  }
  float zsum = 0.f;
  for (int j = 0; j < TOK_PER_WARP; ++j) {
    const int t = blk * NT_ROUTE_TOKENS + warp * TOK_PER_WARP + j;
    if (t >= a.N) break;
    const float* lg = a.logits + static_cast<int64_t>(t) * a.E;
    float l[VPL], p[VPL], sc[VPL];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      l[i] = lg[lane + 32 * i];
      mx = fmaxf(mx, l[i]);
    }
    mx = wmax(mx);
    float se = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) se += expf(l[i] - mx);
    const float lz = mx + logf(wsum(se));
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      p[i] = expf(l[i] - lz);
      sc[i] = p[i] + bias[i];
      psum[i] += p[i];
    }
    float w_mine = 0.f, wtot = 0.f;
    int c_mine = 0;
    for (int r = 0; r < a.k; ++r) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < VPL; ++i)
        if (sc[i] > bv) {
          bv = sc[i];
          bi = lane + 32 * i;
        }
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      float pw = 0.f;
      if ((bi & 31) == lane) {
#pragma unroll
        for (int i = 0; i < VPL; ++i)
          if (i == (bi >> 5)) {
            pw = p[i];
            sc[i] = -INFINITY;
            ++cnt[i];
          }
      }
      pw = __shfl_sync(0xffffffffu, pw, bi & 31);
      if (lane == r) {
        w_mine = pw;
        c_mine = bi;
      }
      wtot += pw;
    }
    if (lane < a.k) {
      a.choice[static_cast<int64_t>(t) * a.k + lane] = c_mine;
      a.w[static_cast<int64_t>(t) * a.k + lane] = w_mine / wtot;
    }
    if (lane == 0) {
      a.lse[t] = lz;
      zsum += lz * lz;
    }
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    s_prob[warp][lane + 32 * i] = psum[i];
    s_cnt[warp][lane + 32 * i] = cnt[i];
  }
  if (lane == 0) s_z[warp] = zsum;
  __syncthreads();
  for (int e = threadIdx.x; e < a.E; e += THREADS) {
    float ps = 0.f;
    int c = 0;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) {
      ps += s_prob[w][e];
      c += s_cnt[w][e];
    }
    a.blk_probs[static_cast<int64_t>(blk) * a.E + e] = ps;
    a.blk_counts[static_cast<int64_t>(blk) * a.E + e] = c;
  }
  if (threadIdx.x == 0) {
    float z = 0.f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) z += s_z[w];
    a.blk_z[blk] = z;
  }
}

constexpr int PLAN_THREADS = 1024;

__global__ void __launch_bounds__(PLAN_THREADS) plan_kernel(const MoeRouteArgs a) {
  __shared__ int s_count[256], s_seg[256], s_end[256];
  __shared__ float s_prob[256];
  __shared__ int s_total;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = (a.N + NT_ROUTE_TOKENS - 1) / NT_ROUTE_TOKENS;
  const int per = (nblk + 31) / 32;
  // 1. per expert: totals and every block's offset inside the expert's segment
  for (int e = warp; e < a.E; e += PLAN_THREADS / 32) {
    const int b0 = min(nblk, lane * per), b1 = min(nblk, b0 + per);
    int c = 0;
    float ps = 0.f;
    for (int b = b0; b < b1; ++b) {
      c += a.blk_counts[static_cast<int64_t>(b) * a.E + e];
      ps += a.blk_probs[static_cast<int64_t>(b) * a.E + e];
    }
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - c;
    for (int b = b0; b < b1; ++b) {
      a.blk_offset[static_cast<int64_t>(b) * a.E + e] = run;
      run += a.blk_counts[static_cast<int64_t>(b) * a.E + e];
    }
    const int tot = __shfl_sync(0xffffffffu, incl, 31);
    ps = wsum(ps);
    if (lane == 0) {
      s_count[e] = tot;
      s_prob[e] = ps;
    }
  }
  __syncthreads();
  // 2. padded segments (one warp scans the experts)
  if (warp == 0) {
    int carry = 0;
    for (int e0 = 0; e0 < a.E; e0 += 32) {
      const int e = e0 + lane;
      const int padded = (s_count[e] + NT_ROUTE_PAD - 1) / NT_ROUTE_PAD * NT_ROUTE_PAD;
      int incl = padded;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      s_seg[e] = carry + incl - padded;
      s_end[e] = carry + incl;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_total = carry;
  }
  __syncthreads();
  const int total = s_total;
  for (int e = threadIdx.x; e < a.E; e += PLAN_THREADS) {
    a.counts[e] = s_count[e];
    a.seg_start[e] = s_seg[e];
    a.grp_k[e] = s_seg[e];
    if (a.load) a.load[e] += static_cast<float>(s_count[e]);
    if (a.aux_grad) {
      const float frac = static_cast<float>(s_count[e]) / (static_cast<float>(a.N) * a.k);
      a.aux_grad[e] = a.aux_coeff * a.E * frac / a.N;
    }
  }
  if (threadIdx.x == 0) a.grp_k[a.E] = total;
  // 3. tile -> expert (first expert whose segment ends past the tile's first row)
  for (int t = threadIdx.x; t < a.P / NT_ROUTE_PAD; t += PLAN_THREADS) {
    const int row = t * NT_ROUTE_PAD;
    int g = -1;
    if (row < total) {
      int lo = 0, hi = a.E - 1;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (s_end[mid] > row) hi = mid; else lo = mid + 1;
      }
      g = lo;
    }
    a.grp_m[t] = g;
  }
  // 4. padding rows of src_of: the tail of each segment and everything past the last one
  for (int i = threadIdx.x; i < a.E * NT_ROUTE_PAD; i += PLAN_THREADS) {
    const int e = i / NT_ROUTE_PAD, j = i % NT_ROUTE_PAD;
    const int row = s_seg[e] + s_count[e] + j;
    if (row < s_end[e]) a.src_of[row] = -1;
  }
  for (int row = total + threadIdx.x; row < a.P; row += PLAN_THREADS) a.src_of[row] = -1;
  // 5. losses (fixed-order sums)
  if (a.aux && warp == 0) {
    float bal = 0.f;
    for (int e = lane; e < a.E; e += 32)
      bal += (static_cast<float>(s_count[e]) / (static_cast<float>(a.N) * a.k)) * (s_prob[e] / a.N);
    bal = wsum(bal) * a.aux_coeff * a.E;
    float z = 0.f;
    for (int b = lane; b < nblk; b += 32) z += a.blk_z[b];
    z = wsum(z) * a.z_coeff / a.N;
    if (lane == 0) {
      a.aux[0] = bal;
      a.aux[1] = z;
    }
  }
}

__global__ void __launch_bounds__(THREADS) scatter_kernel(const MoeRouteArgs a) {
  __shared__ int s_base[256], s_run[256];
  __shared__ int s_w[WARPS][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = blockIdx.x;
  for (int e = threadIdx.x; e < a.E; e += THREADS) {
    s_base[e] = a.seg_start[e] + a.blk_offset[static_cast<int64_t>(blk) * a.E + e];
    s_run[e] = 0;
  }
  const int tokens = min(NT_ROUTE_TOKENS, a.N - blk * NT_ROUTE_TOKENS);
  const int total = tokens * a.k;
  const int64_t f0 = static_cast<int64_t>(blk) * NT_ROUTE_TOKENS * a.k;
  for (int c0 = 0; c0 < total; c0 += THREADS) {
    for (int i = threadIdx.x; i < WARPS * a.E; i += THREADS) s_w[i / a.E][i % a.E] = 0;
    __syncthreads();
    const int i = c0 + threadIdx.x;
    const bool live = i < total;
    const int e = live ? a.choice[f0 + i] : -1;
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(same & ((1u << lane) - 1u));
    if (live && rank == 0) s_w[warp][e] = __popc(same);
    __syncthreads();
    if (live) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += s_w[w][e];
      const int row = s_base[e] + s_run[e] + before + rank;
      a.row_of[f0 + i] = row;
      a.src_of[row] = static_cast<int>((f0 + i) / a.k);
    }
    __syncthreads();
    for (int x = threadIdx.x; x < a.E; x += THREADS) {
      int s = 0;
#pragma unroll
      for (int w = 0; w < WARPS; ++w) s += s_w[w][x];
      s_run[x] += s;
    }
    __syncthreads();
  }
}

template <int VPL>
__global__ void __launch_bounds__(THREADS) route_bwd_kernel(const float* __restrict__ logits,
                                                            const float* __restrict__ lse, const int* __restrict__ choice,
                                                            const float* __restrict__ w, const float* __restrict__ dw,
                                                            const float* __restrict__ aux_grad,
                                                            const float* __restrict__ daux_p, float z_coeff,
                                                            float* __restrict__ dlogits, int N, int E, int k) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * WARPS;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5); t < N; t += warps) {
    const float* lg = logits + t * E;
    const float lz = lse[t];
    float p[VPL], d[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      p[i] = expf(lg[lane + 32 * i] - lz);
      d[i] = 0.f;
    }
    const float daux = daux_p ? *daux_p : 0.f;
    if (daux != 0.f) {
      if (aux_grad) {
        float pg = 0.f;
#pragma unroll
        for (int i = 0; i < VPL; ++i) pg += p[i] * aux_grad[lane + 32 * i];
        pg = wsum(pg);
#pragma unroll
        for (int i = 0; i < VPL; ++i) d[i] += daux * p[i] * (aux_grad[lane + 32 * i] - pg);
      }
      if (z_coeff != 0.f) {
        const float zg = daux * z_coeff * 2.f * lz / N;
#pragma unroll
        for (int i = 0; i < VPL; ++i) d[i] += zg * p[i];
      }
    }
    const float ws = lane < k ? w[t * k + lane] : 0.f;
    const float dws = lane < k && dw ? dw[t * k + lane] : 0.f;
    const int cs = lane < k ? choice[t * k + lane] : -1;
    const float wd = wsum(ws * dws);
    for (int s = 0; s < k; ++s) {
      const int c = __shfl_sync(0xffffffffu, cs, s);
      const float g = __shfl_sync(0xffffffffu, ws * (dws - wd), s);
      if ((c & 31) == lane) {
#pragma unroll
        for (int i = 0; i < VPL; ++i)
          if (i == (c >> 5)) d[i] += g;
      }
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) dlogits[t * E + lane + 32 * i] = d[i];
  }
}

}  // namespace route
}  // namespace nt

using namespace nt::route;

static bool route_ok(int N, int E, int k) {
  return N > 0 && E >= 32 && E <= 256 && E % 32 == 0 && k >= 1 && k <= 16 && k <= E;
}

int nt_moe_route(const MoeRouteArgs& a, cudaStream_t s) {
  if (!route_ok(a.N, a.E, a.k) || a.P % NT_ROUTE_PAD ||
      static_cast<int64_t>(a.P) < (static_cast<int64_t>(a.N) * a.k + NT_ROUTE_PAD - 1) / NT_ROUTE_PAD * NT_ROUTE_PAD +
                                       static_cast<int64_t>(NT_ROUTE_PAD) * a.E)
    return -1;
  const int nblk = (a.N + NT_ROUTE_TOKENS - 1) / NT_ROUTE_TOKENS;
  switch (a.E / 32) {
    case 1: route_kernel<1><<<nblk, THREADS, 0, s>>>(a); break;
    case 2: route_kernel<2><<<nblk, THREADS, 0, s>>>(a); break;
    case 3: route_kernel<3><<<nblk, THREADS, 0, s>>>(a); break;
    case 4: route_kernel<4><<<nblk, THREADS, 0, s>>>(a); break;
    case 5: route_kernel<5><<<nblk, THREADS, 0, s>>>(a); break;
    case 6: route_kernel<6><<<nblk, THREADS, 0, s>>>(a); break;
    case 7: route_kernel<7><<<nblk, THREADS, 0, s>>>(a); break;
    default: route_kernel<8><<<nblk, THREADS, 0, s>>>(a); break;
  }
  plan_kernel<<<1, PLAN_THREADS, 0, s>>>(a);
  scatter_kernel<<<nblk, THREADS, 0, s>>>(a);
  return 0;
}

int nt_moe_route_bwd(const float* logits, const float* lse, const int* choice, const float* w, const float* dw,
                     const float* aux_grad, const float* daux, float z_coeff, float* dlogits, int N, int E, int k,
                     cudaStream_t s) {
  if (!route_ok(N, E, k)) return -1;
  const int blocks = static_cast<int>(std::min<int64_t>((static_cast<int64_t>(N) + WARPS - 1) / WARPS, 148 * 16));
#define NT_ROUTE_BWD(V)                                                                                          \
  route_bwd_kernel<V><<<blocks, THREADS, 0, s>>>(logits, lse, choice, w, dw, aux_grad, daux, z_coeff, dlogits, N, \
                                                 E, k)
  switch (E / 32) {
    case 1: NT_ROUTE_BWD(1); break;
    case 2: NT_ROUTE_BWD(2); break;
    case 3: NT_ROUTE_BWD(3); break;
    case 4: NT_ROUTE_BWD(4); break;
    case 5: NT_ROUTE_BWD(5); break;
    case 6: NT_ROUTE_BWD(6); break;
    case 7: NT_ROUTE_BWD(7); break;
    default: NT_ROUTE_BWD(8); break;
  }
#undef NT_ROUTE_BWD
  return 0;
}
