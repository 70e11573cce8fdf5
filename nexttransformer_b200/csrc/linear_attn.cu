// K11: elementwise kernels of the linear-attention mixers (DeltaNet / GDN / KDA).
//
//   causal_conv_silu  y[b, t, c] = SiLU( sum_{i<K} w[c, i] x[b, t - K + 1 + i, c] )   (zero history)
//                     and its backward (dx by the transposed filter, dw by per-channel reduction);
//   gated_rmsnorm     y = x / rms(x) * gain * SiLU(gate) over the head dimension (eps: fp32 epsilon)
//                     and its backward.
// One thread per (row, 8 channels): 16-byte bf16 vector loads/stores; the K = 4 history rows of
// a channel group stay in registers while a thread walks a stretch of time steps.
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include "common.cuh"
#include "linear_attn.h"

#include <algorithm>

namespace nt {
namespace lin {

constexpr int KMAX = 8;
constexpr int TSTEP = 32;  // time steps per thread

NT_DEVICE void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
NT_DEVICE void store8(__nv_bfloat16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                            pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}
NT_DEVICE float silu(float z) { return z / (1.f + __expf(-z)); }

// grid: (ceil(C/8 / 32), ceil(T / TSTEP), B); block 32 threads along channel groups
// CANON: y = x + conv(x) (the Canon layer of the AttnRes-Canon plugins) instead of SiLU(conv(x)).
template <int K, bool CANON = false>
__global__ void conv_silu_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ w,
                                     __nv_bfloat16* __restrict__ y, __nv_bfloat16* __restrict__ pre, int T, int C) {
  const int cg = blockIdx.x * blockDim.x + threadIdx.x;
  if (cg * 8 >= C) return;
  const int c0 = cg * 8, t0 = blockIdx.y * TSTEP, b = blockIdx.z;
  float wk[8][K];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < K; ++i) wk[j][i] = w[(c0 + j) * K + i];
  float hist[K - 1][8];
#pragma unroll
  for (int i = 0; i < K - 1; ++i) {
    const int t = t0 - (K - 1) + i;
    if (t >= 0) load8(x + (static_cast<int64_t>(b) * T + t) * C + c0, hist[i]);
    else
#pragma unroll
      for (int j = 0; j < 8; ++j) hist[i][j] = 0.f;
  }
  for (int t = t0; t < min(T, t0 + TSTEP); ++t) {
    float cur[8];
    const int64_t row = (static_cast<int64_t>(b) * T + t) * C + c0;
    load8(x + row, cur);
    float o[8], z[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float s = wk[j][K - 1] * cur[j];
#pragma unroll
      for (int i = 0; i < K - 1; ++i) s += wk[j][i] * hist[i][j];
      z[j] = s;
      o[j] = CANON ? cur[j] + s : silu(s);
    }
    store8(y + row, o);
    if (!CANON && pre) store8(pre + row, z);
#pragma unroll
    for (int i = 0; i < K - 2; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) hist[i][j] = hist[i + 1][j];
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[K - 2][j] = cur[j];
  }
}

// dz = dy * SiLU'(z);  dx[t] = sum_i w[i] dz[t + K - 1 - i];  dw partial sums per block (fp32 atomics)
template <int K, bool CANON = false>
__global__ void conv_silu_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ pre,
                                     const __nv_bfloat16* __restrict__ dy, const float* __restrict__ w,
                                     __nv_bfloat16* __restrict__ dx, float* __restrict__ dw, int T, int C) {
  const int cg = blockIdx.x * blockDim.x + threadIdx.x;
  if (cg * 8 >= C) return;
  const int c0 = cg * 8, t0 = blockIdx.y * TSTEP, b = blockIdx.z;
  float wk[8][K];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < K; ++i) wk[j][i] = w[(c0 + j) * K + i];
  float dwacc[8][K];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < K; ++i) dwacc[j][i] = 0.f;
  auto dz_at = [&](int t, float (&out)[8]) {
    if (t >= T) {
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = 0.f;
      return;
    }
    const int64_t row = (static_cast<int64_t>(b) * T + t) * C + c0;
    float g[8];
    load8(dy + row, g);
    if (CANON) {
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j] = g[j];
      return;
    }
    float z[8];
    load8(pre + row, z);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sg = 1.f / (1.f + __expf(-z[j]));
      out[j] = g[j] * sg * (1.f + z[j] * (1.f - sg));
    }
  };
  // future dz window: dz[t .. t + K - 1]
  float fut[K][8];
#pragma unroll
  for (int i = 0; i < K; ++i) dz_at(t0 + i, fut[i]);
  for (int t = t0; t < min(T, t0 + TSTEP); ++t) {
    const int64_t row = (static_cast<int64_t>(b) * T + t) * C + c0;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float s = CANON ? fut[0][j] : 0.f;  // the residual path of the Canon layer
#pragma unroll
      for (int i = 0; i < K; ++i) s += wk[j][K - 1 - i] * fut[i][j];
      o[j] = s;
    }
    store8(dx + row, o);
    // dw[c, i] += dz[t] * x[t - K + 1 + i]
#pragma unroll
    for (int i = 0; i < K; ++i) {
      const int tx = t - (K - 1) + i;
      if (tx >= 0) {
        float xv[8];
        load8(x + (static_cast<int64_t>(b) * T + tx) * C + c0, xv);
#pragma unroll
        for (int j = 0; j < 8; ++j) dwacc[j][i] += fut[0][j] * xv[j];
      }
    }
#pragma unroll
    for (int i = 0; i < K - 1; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) fut[i][j] = fut[i + 1][j];
    dz_at(t + K, fut[K - 1]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < K; ++i) atomicAdd(&dw[(c0 + j) * K + i], dwacc[j][i]);
}

// One warp per (row, head) of D = 32 * E channels: y = x * rsqrt(mean(x^2) + eps) * gain * SiLU(g)
template <int E>
__global__ void gated_rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ g,
                                         const float* __restrict__ gain, __nv_bfloat16* __restrict__ y,
                                         float* __restrict__ rstd, int64_t rows) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* xr = x + r * 32 * E + lane * E;
  float xv[E], ss = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    xv[e] = bf2f(xr[e]);
    ss += xv[e] * xv[e];
  }
  ss = warp_sum(ss);
  const float rs = rsqrtf(ss / (32 * E) + FLT_EPSILON);
  if (lane == 0) rstd[r] = rs;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float gv = bf2f(g[r * 32 * E + lane * E + e]);
    y[r * 32 * E + lane * E + e] = f2bf(xv[e] * rs * gain[lane * E + e] * silu(gv));
  }
}

// dx and dg of the gated RMSNorm, one warp per row with the warps striding over the rows; each warp
// keeps its dgain terms in registers and every block writes one partial row (fixed order, no
// atomics), summed by gated_rmsnorm_dgain_kernel.
template <int E>
__global__ void __launch_bounds__(256) gated_rmsnorm_bwd_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ g, const float* __restrict__ gain,
    const float* __restrict__ rstd, const __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ dx,
    __nv_bfloat16* __restrict__ dg, float* __restrict__ part, int64_t rows) {
  __shared__ float red[8][32 * E];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float gn[E], acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    gn[e] = gain[lane * E + e];
    acc[e] = 0.f;
  }
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * 8 + warp; r < rows; r += static_cast<int64_t>(gridDim.x) * 8) {
    const int64_t base = r * 32 * E + lane * E;
    const float rs = rstd[r];
    float n[E], a[E], dot = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float xv = bf2f(x[base + e]), gv = bf2f(g[base + e]), d = bf2f(dy[base + e]);
      const float sg = 1.f / (1.f + __expf(-gv));
      const float sl = gv * sg;
      n[e] = xv * rs;
      dg[base + e] = f2bf(d * n[e] * gn[e] * sg * (1.f + gv * (1.f - sg)));
      acc[e] = fmaf(d * n[e], sl, acc[e]);
      a[e] = d * gn[e] * sl;  // dL/dn
      dot += a[e] * n[e];
    }
    dot = warp_sum(dot) / (32 * E);
#pragma unroll
    for (int e = 0; e < E; ++e) dx[base + e] = f2bf(rs * (a[e] - n[e] * dot));
  }
#pragma unroll
  for (int e = 0; e < E; ++e) red[warp][lane * E + e] = acc[e];
  __syncthreads();
  for (int c = threadIdx.x; c < 32 * E; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][c];
    part[static_cast<int64_t>(blockIdx.x) * 32 * E + c] = t;
  }
}

// dgain[c] += sum over the blocks' partial rows, in block order
__global__ void gated_rmsnorm_dgain_kernel(const float* __restrict__ part, float* __restrict__ dgain, int parts, int D) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= D) return;
  float t = 0.f;
  for (int p = 0; p < parts; ++p) t += part[static_cast<int64_t>(p) * D + c];
  dgain[c] += t;
}

}  // namespace lin
}  // namespace nt

using namespace nt::lin;

template <bool CANON>
static int conv_fwd(const void* x, const float* w, void* y, void* pre, int B, int T, int C, int K, cudaStream_t s) {
  if (C % 8 || K < 2 || K > 4) return -1;
  dim3 grid((C / 8 + 31) / 32, (T + TSTEP - 1) / TSTEP, B);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto Y = static_cast<__nv_bfloat16*>(y);
  auto P = static_cast<__nv_bfloat16*>(pre);
  switch (K) {
    case 2: conv_silu_fwd_kernel<2, CANON><<<grid, 32, 0, s>>>(X, w, Y, P, T, C); break;
    case 3: conv_silu_fwd_kernel<3, CANON><<<grid, 32, 0, s>>>(X, w, Y, P, T, C); break;
    case 4: conv_silu_fwd_kernel<4, CANON><<<grid, 32, 0, s>>>(X, w, Y, P, T, C); break;
    default: return -1;
  }
  return 0;
}

template <bool CANON>
static int conv_bwd(const void* x, const void* pre, const void* dy, const float* w, void* dx, float* dw, int B, int T,
                    int C, int K, cudaStream_t s) {
  if (C % 8 || K < 2 || K > 4) return -1;
  dim3 grid((C / 8 + 31) / 32, (T + TSTEP - 1) / TSTEP, B);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto P = static_cast<const __nv_bfloat16*>(pre);
  auto DY = static_cast<const __nv_bfloat16*>(dy);
  auto DX = static_cast<__nv_bfloat16*>(dx);
  switch (K) {
    case 2: conv_silu_bwd_kernel<2, CANON><<<grid, 32, 0, s>>>(X, P, DY, w, DX, dw, T, C); break;
    case 3: conv_silu_bwd_kernel<3, CANON><<<grid, 32, 0, s>>>(X, P, DY, w, DX, dw, T, C); break;
    case 4: conv_silu_bwd_kernel<4, CANON><<<grid, 32, 0, s>>>(X, P, DY, w, DX, dw, T, C); break;
    default: return -1;
  }
  return 0;
}

int nt_causal_conv_silu_fwd(const void* x, const float* w, void* y, void* pre, int B, int T, int C, int K,
                            cudaStream_t s) {
  return conv_fwd<false>(x, w, y, pre, B, T, C, K, s);
}

int nt_causal_conv_silu_bwd(const void* x, const void* pre, const void* dy, const float* w, void* dx, float* dw,
                            int B, int T, int C, int K, cudaStream_t s) {
  return conv_bwd<false>(x, pre, dy, w, dx, dw, B, T, C, K, s);
}

int nt_canon_conv_fwd(const void* x, const float* w, void* y, int B, int T, int C, int K, cudaStream_t s) {
  return conv_fwd<true>(x, w, y, nullptr, B, T, C, K, s);
}

int nt_canon_conv_bwd(const void* x, const void* dy, const float* w, void* dx, float* dw, int B, int T, int C, int K,
                      cudaStream_t s) {
  return conv_bwd<true>(x, nullptr, dy, w, dx, dw, B, T, C, K, s);
}

int nt_gated_rmsnorm_fwd(const void* x, const void* g, const float* gain, void* y, float* rstd, int64_t rows, int D,
                         cudaStream_t s) {
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto G = static_cast<const __nv_bfloat16*>(g);
  auto Y = static_cast<__nv_bfloat16*>(y);
  if (D == 128) gated_rmsnorm_fwd_kernel<4><<<blocks, 256, 0, s>>>(X, G, gain, Y, rstd, rows);
  else if (D == 64) gated_rmsnorm_fwd_kernel<2><<<blocks, 256, 0, s>>>(X, G, gain, Y, rstd, rows);
  else return -1;
  return 0;
}

int nt_gated_rmsnorm_bwd(const void* x, const void* g, const float* gain, const float* rstd, const void* dy, void* dx,
                         void* dg, float* dgain, float* work, int64_t rows, int D, cudaStream_t s) {
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((rows + 7) / 8, NT_GATED_NORM_PARTS));
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto G = static_cast<const __nv_bfloat16*>(g);
  auto DY = static_cast<const __nv_bfloat16*>(dy);
  auto DX = static_cast<__nv_bfloat16*>(dx);
  auto DG = static_cast<__nv_bfloat16*>(dg);
  if (rows <= 0) return 0;
  if (D == 128) gated_rmsnorm_bwd_kernel<4><<<blocks, 256, 0, s>>>(X, G, gain, rstd, DY, DX, DG, work, rows);
  else if (D == 64) gated_rmsnorm_bwd_kernel<2><<<blocks, 256, 0, s>>>(X, G, gain, rstd, DY, DX, DG, work, rows);
  else return -1;
  gated_rmsnorm_dgain_kernel<<<1, 128, 0, s>>>(work, dgain, static_cast<int>(blocks), D);
  return 0;
}
