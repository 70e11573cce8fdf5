// K6 / K7: optimizer kernels for sm_100a.
//
// AdamW (nanochat/optim.py:23-63 in the reference): decoupled decay, lerp moments, bias
// correction, fp32 math and fp32 moments for fp32 or bf16 parameters, optional bf16 shadow.
//
// Muon (nanochat/optim.py:111-180): the Polar-Express iterations themselves run on the GEMM
// engine; the kernels here are the memory-bound steps around them, operating on a "stack"
// of K same-shape matrices addressed through device pointer tables (the matrices need not
// be contiguous):
//   muon_prep      Nesterov momentum (lerp), bf16 cast into the contiguous workspace X,
//                  per-row sum of squares
//   muon_rowscale  MuonEq row equilibration, writes X' and its sum of squares
//   muon_scale     Frobenius normalisation X'' = X' / (||X'|| * 1.01 + 1e-6)
//   muon_stats     per-row or per-column sums of squares of the orthogonalised X
//   muon_factors   Muon+ renormalisation and NorMuon factored second moment -> per-row or
//                  per-column final scale (one CTA per matrix)
//   muon_update    cautious weight decay + update, fp32 master and bf16 shadow
#include "common.cuh"
#include "optim.h"

namespace nt {
namespace opt {

NT_DEVICE float rbf(float v) { return bf2f(f2bf(v)); }

template <typename P>
__global__ void adamw_kernel(P* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ shadow, int64_t n, AdamWHyper h) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float pv;
    if constexpr (sizeof(P) == 2) pv = bf2f(p[i]);
    else pv = p[i];
    const float gv = g[i];
    pv *= 1.f - h.lr * h.wd;
    float mv = m[i], vv = v[i];
    mv += (1.f - h.beta1) * (gv - mv);
    vv += (1.f - h.beta2) * (gv * gv - vv);
    const float denom = sqrtf(vv / h.bias2) + h.eps;
    pv -= (h.lr / h.bias1) * (mv / denom);
    m[i] = mv;
    v[i] = vv;
    if constexpr (sizeof(P) == 2) p[i] = f2bf(pv);
    else p[i] = pv;
    if (shadow) shadow[i] = f2bf(pv);
  }
}

// One warp per (matrix, row).
__global__ void muon_prep_kernel(float* const* __restrict__ grads, float* const* __restrict__ moms,
                                 __nv_bfloat16* __restrict__ X, float* __restrict__ rowss, int K, int m, int n,
                                 float mu) {
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(K) * m) return;
  const int k = static_cast<int>(gw / m), r = static_cast<int>(gw - static_cast<int64_t>(k) * m);
  float* g = grads[k] + static_cast<int64_t>(r) * n;
  float* mo = moms[k] + static_cast<int64_t>(r) * n;
  __nv_bfloat16* x = X + (static_cast<int64_t>(k) * m + r) * n;
  float ss = 0.f;
  for (int c = lane; c < n; c += 32) {
    float gv = g[c], mv = mo[c];
    mv += (1.f - mu) * (gv - mv);  // momentum_buffer.lerp_(grad, 1 - mu)
    gv += mu * (mv - gv);          // grad.lerp_(momentum_buffer, mu)
    mo[c] = mv;
    const float xv = rbf(gv);
    x[c] = f2bf(xv);
    ss += xv * xv;
  }
  ss = warp_sum(ss);
  if (lane == 0) rowss[static_cast<int64_t>(k) * m + r] = ss;
}

// X[k, r, :] *= bf16(target_k / max(sqrt(rowss), 1e-6)),  target_k = ||X_k|| / sqrt(m)
// tot[k] (fp32) accumulates the sum of squares of the result.
__global__ void muon_rowscale_kernel(__nv_bfloat16* __restrict__ X, const float* __restrict__ rowss,
                                     float* __restrict__ tot, int K, int m, int n) {
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(K) * m) return;
  const int k = static_cast<int>(gw / m), r = static_cast<int>(gw - static_cast<int64_t>(k) * m);
  // total norm of matrix k: sum of its row sums (m is small enough to re-sum per warp)
  float t = 0.f;
  for (int i = lane; i < m; i += 32) t += rowss[static_cast<int64_t>(k) * m + i];
  t = warp_sum(t);
  const float target = sqrtf(t) / sqrtf(static_cast<float>(m));
  const float rn = fmaxf(sqrtf(rowss[static_cast<int64_t>(k) * m + r]), 1e-6f);
  const float s = rbf(target / rn);
  __nv_bfloat16* x = X + (static_cast<int64_t>(k) * m + r) * n;
  float ss = 0.f;
  for (int c = lane; c < n; c += 32) {
    const float xv = rbf(bf2f(x[c]) * s);
    x[c] = f2bf(xv);
    ss += xv * xv;
  }
  ss = warp_sum(ss);
  if (lane == 0) atomicAdd(tot + k, ss);
}

__global__ void muon_scale_kernel(__nv_bfloat16* __restrict__ X, const float* __restrict__ tot, int K,
                                  int64_t per) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= K * per) return;
  const int k = static_cast<int>(i / per);
  const float nrm = rbf(sqrtf(tot[k]));
  const float den = rbf(rbf(nrm * 1.01f) + 1e-6f);
  X[i] = f2bf(bf2f(X[i]) / den);
}

// Sums of squares of the orthogonalised X (fp32 of bf16 values): per row (by_row) or per column.
// tot[k] also receives the total.
__global__ void muon_stats_kernel(const __nv_bfloat16* __restrict__ X, float* __restrict__ red,
                                  float* __restrict__ tot, int K, int m, int n, int by_row) {
  if (by_row) {
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (gw >= static_cast<int64_t>(K) * m) return;
    const int k = static_cast<int>(gw / m);
    const __nv_bfloat16* x = X + gw * n;
    float ss = 0.f;
    for (int c = lane; c < n; c += 32) {
      const float v = bf2f(x[c]);
      ss += v * v;
    }
    ss = warp_sum(ss);
    if (lane == 0) {
      red[gw] = ss;
      atomicAdd(tot + k, ss);
    }
  } else {
    // thread per (matrix, column); rows strided, coalesced across threads
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(K) * n) return;
    const int k = static_cast<int>(i / n), c = static_cast<int>(i - static_cast<int64_t>(k) * n);
    const __nv_bfloat16* x = X + static_cast<int64_t>(k) * m * n + c;
    float ss = 0.f;
    for (int r = 0; r < m; ++r) {
      const float v = bf2f(x[static_cast<int64_t>(r) * n]);
      ss += v * v;
    }
    red[i] = ss;
    atomicAdd(tot + k, ss);
  }
}

// One CTA per matrix.  L = length of the factored dimension (m rows or n columns), red_size the
// reduced extent (n or m).  smb: second-moment buffer [K, L] (fp32); out fscale [K, L] holds
// the per-row/column multiplier of X: (sqrt(min(m,n)) / ||X||) * final_scale.
__global__ void muon_factors_kernel(const float* __restrict__ red, const float* __restrict__ tot,
                                    float* const* __restrict__ smbs, float* __restrict__ fscale, int L,
                                    int red_size, float muon_plus_target, float beta2) {
  __shared__ float scratch[32];
  const int k = blockIdx.x;
  const float cur = fmaxf(sqrtf(tot[k]), 1e-6f);
  const float s = muon_plus_target / cur;
  float* smb = smbs[k];
  const float* rr = red + static_cast<int64_t>(k) * L;
  float a = 0.f, b = 0.f;
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    const float vmean = s * s * rr[i] / red_size;
    float sb = smb[i];
    sb += (1.f - beta2) * (vmean - sb);
    smb[i] = sb;
    const float step = rsqrtf(fmaxf(sb, 1e-10f));
    a += vmean * red_size;
    b += vmean * red_size * step * step;
  }
  const float vnorm = sqrtf(block_sum(a, scratch));
  const float vnorm_new = sqrtf(block_sum(b, scratch));
  const float ratio = vnorm / fmaxf(vnorm_new, 1e-10f);
  for (int i = threadIdx.x; i < L; i += blockDim.x) {
    const float step = rsqrtf(fmaxf(smb[i], 1e-10f));
    fscale[static_cast<int64_t>(k) * L + i] = s * step * ratio;
  }
}

// p -= lr * g + lr * wd * p * (g * p >= 0),  g = X * fscale[row or col]
__global__ void muon_update_kernel(const __nv_bfloat16* __restrict__ X, const float* __restrict__ fscale,
                                   float* const* __restrict__ params, __nv_bfloat16* const* __restrict__ shadows,
                                   int K, int m, int n, int by_row, float lr, float wd) {
  const int64_t per = static_cast<int64_t>(m) * n;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= K * per) return;
  const int k = static_cast<int>(i / per);
  const int64_t e = i - k * per;
  const int r = static_cast<int>(e / n), c = static_cast<int>(e - static_cast<int64_t>(r) * n);
  const float f = by_row ? fscale[static_cast<int64_t>(k) * m + r] : fscale[static_cast<int64_t>(k) * n + c];
  const float g = bf2f(X[i]) * f;
  float* p = params[k];
  float pv = p[e];
  const float mask = (g * pv >= 0.f) ? 1.f : 0.f;
  pv -= lr * g + lr * wd * pv * mask;
  p[e] = pv;
  if (shadows && shadows[k]) shadows[k][e] = f2bf(pv);
}

}  // namespace opt
}  // namespace nt

using namespace nt::opt;

static unsigned blocks_for(int64_t n, int t) { return static_cast<unsigned>((n + t - 1) / t); }

int nt_adamw(void* p, int p_is_bf16, const float* g, float* m, float* v, void* shadow, int64_t n, AdamWHyper h,
             cudaStream_t s) {
  if (n <= 0) return 0;
  const unsigned grid = blocks_for(n, 256) < 4096u ? blocks_for(n, 256) : 4096u;
  if (p_is_bf16) adamw_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>((__nv_bfloat16*)p, g, m, v, (__nv_bfloat16*)shadow, n, h);
  else adamw_kernel<float><<<grid, 256, 0, s>>>((float*)p, g, m, v, (__nv_bfloat16*)shadow, n, h);
  return 0;
}

int nt_muon_prep(float* const* grads, float* const* moms, void* X, float* rowss, int K, int m, int n, float mu,
                 cudaStream_t s) {
  muon_prep_kernel<<<blocks_for(static_cast<int64_t>(K) * m, 8), 256, 0, s>>>(grads, moms, (__nv_bfloat16*)X, rowss,
                                                                              K, m, n, mu);
  return 0;
}

int nt_muon_normalize(void* X, const float* rowss, float* tot, int K, int m, int n, cudaStream_t s) {
  cudaMemsetAsync(tot, 0, sizeof(float) * K, s);
  muon_rowscale_kernel<<<blocks_for(static_cast<int64_t>(K) * m, 8), 256, 0, s>>>((__nv_bfloat16*)X, rowss, tot, K,
                                                                                  m, n);
  const int64_t per = static_cast<int64_t>(m) * n;
  muon_scale_kernel<<<blocks_for(K * per, 256), 256, 0, s>>>((__nv_bfloat16*)X, tot, K, per);
  return 0;
}

int nt_muon_finish(const void* X, float* red, float* tot, float* const* smbs, float* fscale, float* const* params,
                   void* const* shadows, int K, int m, int n, float beta2, float lr, float wd, cudaStream_t s) {
  const int by_row = m >= n ? 1 : 0;
  cudaMemsetAsync(tot, 0, sizeof(float) * K, s);
  if (by_row)
    muon_stats_kernel<<<blocks_for(static_cast<int64_t>(K) * m, 8), 256, 0, s>>>((const __nv_bfloat16*)X, red, tot,
                                                                                 K, m, n, 1);
  else
    muon_stats_kernel<<<blocks_for(static_cast<int64_t>(K) * n, 256), 256, 0, s>>>((const __nv_bfloat16*)X, red,
                                                                                   tot, K, m, n, 0);
  const int L = by_row ? m : n;
  const int red_size = by_row ? n : m;
  const float target = sqrtf(static_cast<float>(m < n ? m : n));
  muon_factors_kernel<<<K, 256, 0, s>>>(red, tot, smbs, fscale, L, red_size, target, beta2);
  const int64_t total = static_cast<int64_t>(K) * m * n;
  muon_update_kernel<<<blocks_for(total, 256), 256, 0, s>>>((const __nv_bfloat16*)X, fscale, params,
                                                            (__nv_bfloat16* const*)shadows, K, m, n, by_row, lr, wd);
  return 0;
}
