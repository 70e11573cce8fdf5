// MSAR (multi-stream attention residuals) element kernels on sm_100a.
//
// Temporal augmentation: a source x [B, T, C] becomes four streams [B, T, 4, C]: x itself and three
// causal depthwise convolutions of widths 4, 8 and 12, y_w[t, c] = sum_j tap_w[c, j] x[t - (w - 1) + j, c]
// (zero before the sequence).  Forward: one thread per channel and 64-token run, the last 11 inputs
// in registers.  Backward: dx[t] = dy_0[t] + sum_w sum_m tap_w[c, w - 1 - m] dy_w[t + m] over a
// window of future gradients walked backwards; the tap gradients are per-run partial sums
// (sum_t dy_w[t] x[t - (w - 1) + j]) reduced in a fixed order by a second kernel.
//
// Depth read gate: for streams s [N, 4, C] of one token, flat = s flattened (4C), r = rsqrt(mean flat^2)
// (1 for an all-zero row), z = r (flat P) with P [4C, 4], g = sigmoid(alpha z + bias), out = sum_k g_k s_k.
// Forward: one warp per token.  Backward: one warp per token gives ds, the per-token factors that the
// projection gradient needs (y = r dz), and the alpha / bias partials; dP = flat^T y is a column
// reduction over tokens (one thread per row of P, fixed-order partial sums).
// Behaviour: the torch modules of methods/msar/ops.py (nexttransformer/methods/msar/ops.py:17-100).
#include "msar.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

namespace nt {
namespace msar {

constexpr int RUN = 64;     // tokens per thread in the temporal kernels
constexpr int CH = 128;     // channels per CTA in the temporal kernels
constexpr int NTAPS = 24;   // 4 + 8 + 12

template <typename T>
__device__ __forceinline__ float ld(const T* p);
template <>
__device__ __forceinline__ float ld<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
__device__ __forceinline__ void st(T* p, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void st<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// taps [C, 24]: widths 4, 8, 12 back to back (tap index j of width w at offset base(w) + j)
template <typename T>
__global__ void temporal_fwd_kernel(const T* __restrict__ x, const float* __restrict__ taps, T* __restrict__ y,
                                    int B, int Tn, int C) {
  const int c = blockIdx.x * CH + threadIdx.x, t0 = blockIdx.y * RUN, b = blockIdx.z;
  if (c >= C) return;
  float w[NTAPS];
#pragma unroll
  for (int j = 0; j < NTAPS; ++j) w[j] = taps[c * NTAPS + j];
  float win[12];  // win[11] = x[t], win[11 - d] = x[t - d]
#pragma unroll
  for (int d = 1; d < 12; ++d) {
    const int t = t0 - d;
    win[11 - d] = t >= 0 ? ld(x + (static_cast<int64_t>(b) * Tn + t) * C + c) : 0.f;
  }
  const int t1 = min(t0 + RUN, Tn);
  for (int t = t0; t < t1; ++t) {
    win[11] = ld(x + (static_cast<int64_t>(b) * Tn + t) * C + c);
    float y4 = 0.f, y8 = 0.f, y12 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) y4 = fmaf(w[j], win[8 + j], y4);
#pragma unroll
    for (int j = 0; j < 8; ++j) y8 = fmaf(w[4 + j], win[4 + j], y8);
#pragma unroll
    for (int j = 0; j < 12; ++j) y12 = fmaf(w[12 + j], win[j], y12);
    T* out = y + (static_cast<int64_t>(b) * Tn + t) * 4 * C + c;
    st(out, win[11]);
    st(out + C, y4);
    st(out + 2 * C, y8);
    st(out + 3 * C, y12);
#pragma unroll
    for (int d = 0; d < 11; ++d) win[d] = win[d + 1];
  }
}

template <typename T>
__global__ void temporal_bwd_kernel(const T* __restrict__ x, const float* __restrict__ taps,
                                    const T* __restrict__ dy, T* __restrict__ dx, float* __restrict__ part,
                                    int B, int Tn, int C) {
  const int c = blockIdx.x * CH + threadIdx.x, t0 = blockIdx.y * RUN, b = blockIdx.z;
  if (c >= C) return;
  const int64_t row = static_cast<int64_t>(b) * Tn;
  float w[NTAPS];
#pragma unroll
  for (int j = 0; j < NTAPS; ++j) w[j] = taps[c * NTAPS + j];
  const int t1 = min(t0 + RUN, Tn);
  // tap gradients over this run (ascending, the past inputs in a window)
  float g[NTAPS];
#pragma unroll
  for (int j = 0; j < NTAPS; ++j) g[j] = 0.f;
  {
    float win[12];
#pragma unroll
    for (int d = 1; d < 12; ++d) {
      const int t = t0 - d;
      win[11 - d] = t >= 0 ? ld(x + (row + t) * C + c) : 0.f;
    }
    for (int t = t0; t < t1; ++t) {
      win[11] = ld(x + (row + t) * C + c);
      const T* d = dy + (row + t) * 4 * C + c;
      const float d4 = ld(d + C), d8 = ld(d + 2 * C), d12 = ld(d + 3 * C);
#pragma unroll
      for (int j = 0; j < 4; ++j) g[j] = fmaf(d4, win[8 + j], g[j]);
#pragma unroll
      for (int j = 0; j < 8; ++j) g[4 + j] = fmaf(d8, win[4 + j], g[4 + j]);
#pragma unroll
      for (int j = 0; j < 12; ++j) g[12 + j] = fmaf(d12, win[j], g[12 + j]);
#pragma unroll
      for (int k = 0; k < 11; ++k) win[k] = win[k + 1];
    }
  }
  float* pp = part + ((static_cast<int64_t>(b) * gridDim.y + blockIdx.y) * NTAPS) * C + c;
#pragma unroll
  for (int j = 0; j < NTAPS; ++j) pp[j * C] = g[j];
  // input gradient (descending, the future output gradients in windows f_w[m] = dy_w[t + m])
  float f4[4], f8[8], f12[12];
#pragma unroll
  for (int m = 0; m < 4; ++m) f4[m] = 0.f;
#pragma unroll
  for (int m = 0; m < 8; ++m) f8[m] = 0.f;
#pragma unroll
  for (int m = 0; m < 12; ++m) f12[m] = 0.f;
  // prime the windows with t1 .. t1 + 10
  for (int t = min(t1 + 10, Tn - 1); t >= t1; --t) {
    const T* d = dy + (row + t) * 4 * C + c;
#pragma unroll
    for (int m = 3; m > 0; --m) f4[m] = f4[m - 1];
#pragma unroll
    for (int m = 7; m > 0; --m) f8[m] = f8[m - 1];
#pragma unroll
    for (int m = 11; m > 0; --m) f12[m] = f12[m - 1];
    f4[0] = ld(d + C);
    f8[0] = ld(d + 2 * C);
    f12[0] = ld(d + 3 * C);
  }
  for (int t = t1 - 1; t >= t0; --t) {
    const T* d = dy + (row + t) * 4 * C + c;
#pragma unroll
    for (int m = 3; m > 0; --m) f4[m] = f4[m - 1];
#pragma unroll
    for (int m = 7; m > 0; --m) f8[m] = f8[m - 1];
#pragma unroll
    for (int m = 11; m > 0; --m) f12[m] = f12[m - 1];
    f4[0] = ld(d + C);
    f8[0] = ld(d + 2 * C);
    f12[0] = ld(d + 3 * C);
    float s = ld(d);
#pragma unroll
    for (int m = 0; m < 4; ++m) s = fmaf(w[3 - m], f4[m], s);
#pragma unroll
    for (int m = 0; m < 8; ++m) s = fmaf(w[4 + 7 - m], f8[m], s);
#pragma unroll
    for (int m = 0; m < 12; ++m) s = fmaf(w[12 + 11 - m], f12[m], s);
    st(dx + (row + t) * C + c, s);
  }
}

// fixed-order sum of the per-run tap partials [runs][24][C] -> dtaps [C, 24]
__global__ void tap_reduce_kernel(const float* __restrict__ part, float* __restrict__ dtaps, int runs, int C) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= NTAPS * C) return;
  const int j = i / C, c = i % C;
  float s = 0.f;
  for (int r = 0; r < runs; ++r) s += part[(static_cast<int64_t>(r) * NTAPS + j) * C + c];
  dtaps[c * NTAPS + j] = s;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// forward gate: one warp per token
template <typename T>
__global__ void gate_fwd_kernel(const T* __restrict__ s, const float* __restrict__ P, const float* __restrict__ alpha_p,
                                const float* __restrict__ bias, T* __restrict__ out, float* __restrict__ zr,
                                int N, int C) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N) return;
  const float alpha = *alpha_p;
  const T* x = s + static_cast<int64_t>(warp) * 4 * C;
  float ss = 0.f, u[4] = {0.f, 0.f, 0.f, 0.f};
  for (int i = lane; i < 4 * C; i += 32) {
    const float v = ld(x + i);
    ss = fmaf(v, v, ss);
    const float4 p = *reinterpret_cast<const float4*>(P + 4 * i);
    u[0] = fmaf(v, p.x, u[0]);
    u[1] = fmaf(v, p.y, u[1]);
    u[2] = fmaf(v, p.z, u[2]);
    u[3] = fmaf(v, p.w, u[3]);
  }
  ss = warp_sum(ss);
  const float ms = ss / (4 * C);
  const float r = ms > 0.f ? rsqrtf(ms) : 1.f;
  float gk[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float z = warp_sum(u[k]) * r;
    gk[k] = 1.f / (1.f + expf(-(alpha * z + bias[k])));
    if (lane == 0) zr[warp * 5 + k] = z;
  }
  if (lane == 0) zr[warp * 5 + 4] = ms > 0.f ? r : 0.f;   // 0 marks an all-zero row (r fixed to 1)
  T* o = out + static_cast<int64_t>(warp) * C;
  for (int c = lane; c < C; c += 32)
    st(o + c, gk[0] * ld(x + c) + gk[1] * ld(x + C + c) + gk[2] * ld(x + 2 * C + c) + gk[3] * ld(x + 3 * C + c));
}

// backward gate: ds, y = r dz (for dP = flat^T y) and per-warp alpha / bias partials
template <typename T>
__global__ void gate_bwd_kernel(const T* __restrict__ s, const float* __restrict__ P, const float* __restrict__ alpha_p,
                                const float* __restrict__ bias, const float* __restrict__ zr, const T* __restrict__ dout,
                                T* __restrict__ ds, float* __restrict__ y, float* __restrict__ ab_part, int N, int C) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N) return;
  const float alpha = *alpha_p;
  const T* x = s + static_cast<int64_t>(warp) * 4 * C;
  const T* go = dout + static_cast<int64_t>(warp) * C;
  float dg[4] = {0.f, 0.f, 0.f, 0.f};
  for (int c = lane; c < C; c += 32) {
    const float d = ld(go + c);
#pragma unroll
    for (int k = 0; k < 4; ++k) dg[k] = fmaf(d, ld(x + k * C + c), dg[k]);
  }
  float z[4], gk[4], dz[4];
  float dalpha = 0.f, zdz = 0.f;
  const float rr = zr[warp * 5 + 4];
  const bool zero_row = rr == 0.f;
  const float r = zero_row ? 1.f : rr;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    dg[k] = warp_sum(dg[k]);
    z[k] = zr[warp * 5 + k];
    gk[k] = 1.f / (1.f + expf(-(alpha * z[k] + bias[k])));
    const float dl = dg[k] * gk[k] * (1.f - gk[k]);   // d (alpha z + bias)
    dz[k] = dl * alpha;
    dalpha = fmaf(dl, z[k], dalpha);
    zdz = fmaf(dz[k], z[k], zdz);
    if (lane == 0) {
      y[warp * 4 + k] = r * dz[k];
      ab_part[warp * 5 + 1 + k] = dl;
    }
  }
  if (lane == 0) ab_part[warp * 5] = dalpha;
  // d flat_i = r sum_k dz_k P_ik - (r^2 / 4C) flat_i sum_k dz_k z_k   (the second term vanishes for a zero row)
  const float corr = zero_row ? 0.f : r * r / (4 * C) * zdz;
  T* d = ds + static_cast<int64_t>(warp) * 4 * C;
  for (int i = lane; i < 4 * C; i += 32) {
    const float4 p = *reinterpret_cast<const float4*>(P + 4 * i);
    const float v = ld(x + i);
    const float df = r * (dz[0] * p.x + dz[1] * p.y + dz[2] * p.z + dz[3] * p.w) - corr * v;
    st(d + i, gk[i / C] * ld(go + i % C) + df);
  }
}

// dP [4C, 4] partials: thread per row i of P over a slice of tokens (fixed order), then summed in order
template <typename T>
__global__ void proj_grad_kernel(const T* __restrict__ s, const float* __restrict__ y, float* __restrict__ part,
                                 int N, int C, int slice) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int n0 = blockIdx.y * slice, n1 = min(N, n0 + slice);
  if (i >= 4 * C) return;
  float a[4] = {0.f, 0.f, 0.f, 0.f};
  for (int n = n0; n < n1; ++n) {
    const float v = ld(s + static_cast<int64_t>(n) * 4 * C + i);
    const float4 yy = *reinterpret_cast<const float4*>(y + 4 * n);
    a[0] = fmaf(v, yy.x, a[0]);
    a[1] = fmaf(v, yy.y, a[1]);
    a[2] = fmaf(v, yy.z, a[2]);
    a[3] = fmaf(v, yy.w, a[3]);
  }
  float* o = part + (static_cast<int64_t>(blockIdx.y) * 4 * C + i) * 4;
#pragma unroll
  for (int k = 0; k < 4; ++k) o[k] = a[k];
}

}  // namespace msar
}  // namespace nt

using namespace nt::msar;

template <typename T>
static int temporal_fwd_t(const MsarTemporalArgs& a, cudaStream_t s) {
  temporal_fwd_kernel<T><<<dim3((a.C + CH - 1) / CH, (a.T + RUN - 1) / RUN, a.B), CH, 0, s>>>(
      static_cast<const T*>(a.x), a.taps, static_cast<T*>(a.y), a.B, a.T, a.C);
  return 0;
}

template <typename T>
static int temporal_bwd_t(const MsarTemporalArgs& a, cudaStream_t s) {
  const int runs = (a.T + RUN - 1) / RUN;
  temporal_bwd_kernel<T><<<dim3((a.C + CH - 1) / CH, runs, a.B), CH, 0, s>>>(
      static_cast<const T*>(a.x), a.taps, static_cast<const T*>(a.dy), static_cast<T*>(a.dx), a.part, a.B, a.T, a.C);
  tap_reduce_kernel<<<(NTAPS * a.C + 255) / 256, 256, 0, s>>>(a.part, a.dtaps, a.B * runs, a.C);
  return 0;
}

int nt_msar_temporal_fwd(const MsarTemporalArgs& a, cudaStream_t s) {
  if (a.B <= 0 || a.T <= 0 || a.C <= 0 || !a.x || !a.taps || !a.y) return -1;
  return a.bf16 ? temporal_fwd_t<__nv_bfloat16>(a, s) : temporal_fwd_t<float>(a, s);
}

int nt_msar_temporal_bwd(const MsarTemporalArgs& a, cudaStream_t s) {
  if (a.B <= 0 || a.T <= 0 || a.C <= 0 || !a.x || !a.taps || !a.dy || !a.dx || !a.part || !a.dtaps) return -1;
  return a.bf16 ? temporal_bwd_t<__nv_bfloat16>(a, s) : temporal_bwd_t<float>(a, s);
}

int nt_msar_temporal_part_floats(int B, int T, int C) { return B * ((T + RUN - 1) / RUN) * NTAPS * C; }

int nt_msar_gate_fwd(const MsarGateArgs& a, cudaStream_t s) {
  if (a.N <= 0 || a.C <= 0 || !a.s || !a.P || !a.alpha || !a.bias || !a.out || !a.zr) return -1;
  const int blocks = (a.N * 32 + 255) / 256;
  if (a.bf16)
    gate_fwd_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(a.s), a.P, a.alpha,
                                                          a.bias, static_cast<__nv_bfloat16*>(a.out), a.zr, a.N, a.C);
  else
    gate_fwd_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(a.s), a.P, a.alpha, a.bias,
                                                  static_cast<float*>(a.out), a.zr, a.N, a.C);
  return 0;
}

int nt_msar_gate_bwd(const MsarGateArgs& a, cudaStream_t s) {
  if (a.N <= 0 || a.C <= 0 || !a.s || !a.P || !a.alpha || !a.bias || !a.zr || !a.dout || !a.ds || !a.y || !a.ab_part ||
      !a.p_part)
    return -1;
  const int blocks = (a.N * 32 + 255) / 256;
  const int slice = 256, slices = (a.N + slice - 1) / slice;
  const dim3 pg((4 * a.C + 127) / 128, slices);
  if (a.bf16) {
    gate_bwd_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(a.s), a.P, a.alpha, a.bias, a.zr,
        static_cast<const __nv_bfloat16*>(a.dout), static_cast<__nv_bfloat16*>(a.ds), a.y, a.ab_part, a.N, a.C);
    proj_grad_kernel<__nv_bfloat16><<<pg, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(a.s), a.y, a.p_part,
                                                       a.N, a.C, slice);
  } else {
    gate_bwd_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(a.s), a.P, a.alpha, a.bias, a.zr,
                                                  static_cast<const float*>(a.dout), static_cast<float*>(a.ds), a.y,
                                                  a.ab_part, a.N, a.C);
    proj_grad_kernel<float><<<pg, 128, 0, s>>>(static_cast<const float*>(a.s), a.y, a.p_part, a.N, a.C, slice);
  }
  return 0;
}

int nt_msar_gate_proj_slices(int N) { return (N + 255) / 256; }
