// K19: elementwise heads of the attention plugins, one kernel each way instead of chains of
// PyTorch element-wise kernels, fp32 math on bf16 tensors, heads of 128 channels (4 per lane):
//   gate_mul   z = y sigmoid(g) per head channel (g [.., H, 128]) or per head (g [.., H, 1])
//              (gated attention, nexttransformer/methods/gated_attention/__init__.py:29-67);
//   xsa        z = y - <y, u> u with u = v / max(|v|, 1e-12), v the head's value (GQA: its KV head)
//              (exclusive self attention, nexttransformer/methods/xsa/__init__.py:19-58).
// One warp per (row, head); the XSA backward takes one warp per (row, KV head) and adds the value
// gradient of the KV head's query heads in a fixed order.
#include "plugin_ops.h"
#include "common.cuh"

namespace nt {
namespace plugin {

constexpr int D = 128, E = 4;

NT_DEVICE void ld4(const __nv_bfloat16* p, float (&v)[E]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
NT_DEVICE void st4(__nv_bfloat16* p, const float (&v)[E]) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
}
NT_DEVICE float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

template <bool PER_HEAD>
__global__ void gate_mul_fwd_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ g,
                                    __nv_bfloat16* __restrict__ z, int64_t rows, int H) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows * H) return;
  const int64_t o = w * D + lane * E;
  float yv[E], gv[E], out[E];
  ld4(y + o, yv);
  if (PER_HEAD) {
    const float s = sigm(bf2f(g[w]));
#pragma unroll
    for (int e = 0; e < E; ++e) gv[e] = s;
  } else {
    ld4(g + o, gv);
#pragma unroll
    for (int e = 0; e < E; ++e) gv[e] = sigm(gv[e]);
  }
#pragma unroll
  for (int e = 0; e < E; ++e) out[e] = yv[e] * gv[e];
  st4(z + o, out);
}

template <bool PER_HEAD>
__global__ void gate_mul_bwd_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ g,
                                    const __nv_bfloat16* __restrict__ dz, __nv_bfloat16* __restrict__ dy,
                                    __nv_bfloat16* __restrict__ dg, int64_t rows, int H) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows * H) return;
  const int64_t o = w * D + lane * E;
  float yv[E], dv[E], gv[E], dyo[E], dgo[E];
  ld4(y + o, yv);
  ld4(dz + o, dv);
  if (PER_HEAD) {
    const float s = sigm(bf2f(g[w]));
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      dyo[e] = dv[e] * s;
      acc = fmaf(dv[e], yv[e], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) dg[w] = f2bf(acc * s * (1.f - s));
  } else {
    ld4(g + o, gv);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float s = sigm(gv[e]);
      dyo[e] = dv[e] * s;
      dgo[e] = dv[e] * yv[e] * s * (1.f - s);
    }
    st4(dg + o, dgo);
  }
  st4(dy + o, dyo);
}

// z = y - <y, u> u;  rows of H query heads, v rows of Hk heads (query head h reads KV head h / (H / Hk))
__global__ void xsa_fwd_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ v,
                               __nv_bfloat16* __restrict__ z, int64_t rows, int H, int Hk) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows * H) return;
  const int64_t row = w / H;
  const int h = static_cast<int>(w - row * H), hk = h / (H / Hk);
  float yv[E], vv[E], out[E];
  ld4(y + w * D + lane * E, yv);
  ld4(v + (row * Hk + hk) * D + lane * E, vv);
  float n2 = 0.f, c = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    n2 = fmaf(vv[e], vv[e], n2);
    c = fmaf(yv[e], vv[e], c);
  }
  n2 = warp_sum(n2);
  c = warp_sum(c);
  const float inv = 1.f / fmaxf(sqrtf(n2), 1e-12f);
  c *= inv;  // <y, u>
#pragma unroll
  for (int e = 0; e < E; ++e) out[e] = yv[e] - c * vv[e] * inv;
  st4(z + w * D + lane * E, out);
}

// dy = dz - <dz, u> u;  du = -(<y, u> dz + <dz, u> y) summed over the KV head's query heads;
// dv = (du - <du, u> u) / |v| (|v| > 1e-12), du / 1e-12 otherwise (F.normalize's clamp)
__global__ void xsa_bwd_kernel(const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ v,
                               const __nv_bfloat16* __restrict__ dz, __nv_bfloat16* __restrict__ dy,
                               __nv_bfloat16* __restrict__ dvout, int64_t rows, int H, int Hk) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows * Hk) return;
  const int64_t row = w / Hk;
  const int hk = static_cast<int>(w - row * Hk), group = H / Hk;
  float vv[E], u[E], du[E];
  ld4(v + w * D + lane * E, vv);
  float n2 = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) n2 = fmaf(vv[e], vv[e], n2);
  const float nrm = sqrtf(warp_sum(n2));
  const float inv = 1.f / fmaxf(nrm, 1e-12f);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    u[e] = vv[e] * inv;
    du[e] = 0.f;
  }
  for (int j = 0; j < group; ++j) {
    const int64_t o = (row * H + hk * group + j) * D + lane * E;
    float yv[E], dv[E], out[E];
    ld4(y + o, yv);
    ld4(dz + o, dv);
    float c = 0.f, d = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      c = fmaf(yv[e], u[e], c);
      d = fmaf(dv[e], u[e], d);
    }
    c = warp_sum(c);
    d = warp_sum(d);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      out[e] = dv[e] - d * u[e];
      du[e] -= c * dv[e] + d * yv[e];
    }
    st4(dy + o, out);
  }
  float p = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) p = fmaf(du[e], u[e], p);
  p = warp_sum(p);
  float out[E];
#pragma unroll
  for (int e = 0; e < E; ++e) out[e] = nrm > 1e-12f ? (du[e] - p * u[e]) * inv : du[e] * inv;
  st4(dvout + w * D + lane * E, out);
}

}  // namespace plugin
}  // namespace nt

using namespace nt::plugin;

static unsigned warp_blocks(int64_t warps) { return static_cast<unsigned>((warps + 7) / 8); }

int nt_gate_mul_fwd(const void* y, const void* g, void* z, int64_t rows, int H, int G, cudaStream_t s) {
  if (rows <= 0 || H <= 0) return rows == 0 ? 0 : -1;
  auto Y = static_cast<const __nv_bfloat16*>(y);
  auto Gt = static_cast<const __nv_bfloat16*>(g);
  auto Z = static_cast<__nv_bfloat16*>(z);
  if (G == 1) gate_mul_fwd_kernel<true><<<warp_blocks(rows * H), 256, 0, s>>>(Y, Gt, Z, rows, H);
  else if (G == D) gate_mul_fwd_kernel<false><<<warp_blocks(rows * H), 256, 0, s>>>(Y, Gt, Z, rows, H);
  else return -1;
  return 0;
}

int nt_gate_mul_bwd(const void* y, const void* g, const void* dz, void* dy, void* dg, int64_t rows, int H, int G,
                    cudaStream_t s) {
  if (rows <= 0 || H <= 0) return rows == 0 ? 0 : -1;
  auto Y = static_cast<const __nv_bfloat16*>(y);
  auto Gt = static_cast<const __nv_bfloat16*>(g);
  auto DZ = static_cast<const __nv_bfloat16*>(dz);
  auto DY = static_cast<__nv_bfloat16*>(dy);
  auto DG = static_cast<__nv_bfloat16*>(dg);
  if (G == 1) gate_mul_bwd_kernel<true><<<warp_blocks(rows * H), 256, 0, s>>>(Y, Gt, DZ, DY, DG, rows, H);
  else if (G == D) gate_mul_bwd_kernel<false><<<warp_blocks(rows * H), 256, 0, s>>>(Y, Gt, DZ, DY, DG, rows, H);
  else return -1;
  return 0;
}

int nt_xsa_fwd(const void* y, const void* v, void* z, int64_t rows, int H, int Hk, cudaStream_t s) {
  if (rows <= 0 || H <= 0 || Hk <= 0 || H % Hk) return rows == 0 ? 0 : -1;
  xsa_fwd_kernel<<<warp_blocks(rows * H), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(y),
                                                       static_cast<const __nv_bfloat16*>(v),
                                                       static_cast<__nv_bfloat16*>(z), rows, H, Hk);
  return 0;
}

int nt_xsa_bwd(const void* y, const void* v, const void* dz, void* dy, void* dv, int64_t rows, int H, int Hk,
               cudaStream_t s) {
  if (rows <= 0 || H <= 0 || Hk <= 0 || H % Hk) return rows == 0 ? 0 : -1;
  xsa_bwd_kernel<<<warp_blocks(rows * Hk), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(v), static_cast<const __nv_bfloat16*>(dz),
      static_cast<__nv_bfloat16*>(dy), static_cast<__nv_bfloat16*>(dv), rows, H, Hk);
  return 0;
}
