// K2/K3/K5/K22 elementwise and row-reduction kernels for sm_100a.
//
//  * RMSNorm without weight (eps = FLT_EPSILON, the value torch's rms_norm uses for bf16
//    inputs), optionally fused with the per-layer residual mix  xm = a*x + b*x0
//    (nexttransformer/models/backbone.py:150-153, 500-503 in the reference shell).
//  * Its backward, fused with the residual-gradient add and with the mix's gradients.
//  * RoPE (rotation by -theta, base cached in bf16 tables) + per-head RMSNorm x 1.2 on the
//    packed q|k|v projection, fused with the value-embedding gate  v += 3 sigmoid(W x[:12]) ve
//    (backbone.py:57-65, 92-104), and its backward.
//  * Soft-capped cross entropy  CE(cap * tanh(l / cap))  over one row of logits, writing the
//    per-row loss and the logit gradient in place (lm.py:211-219).
//  * Token-embedding gather + RMSNorm + smear gate (backbone.py:475-484).
//  * fp32 -> bf16 weight shadow cast.
// Rows are handled one warp per row with 16-byte vector accesses; every kernel here is
// memory bound and is written to touch each byte once.
#include "common.cuh"
#include "elementwise.h"

#include <cstdlib>

namespace nt {
namespace ew {

constexpr float kNormEps = 1.1920928955078125e-07f;

NT_DEVICE void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 q = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(q.x), b = unpack_bf16x2(q.y), c = unpack_bf16x2(q.z), d = unpack_bf16x2(q.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
NT_DEVICE void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 q = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                       pack_bf16x2(v[6], v[7]));
  *reinterpret_cast<uint4*>(p) = q;
}
NT_DEVICE float rbf(float v) { return bf2f(f2bf(v)); }

// P consecutive bf16 values (P = 1, 2 or 4) as floats / from floats, vectorised.
template <int P>
NT_DEVICE void ldp(const __nv_bfloat16* p, float (&v)[P]) {
  if constexpr (P == 1) {
    v[0] = bf2f(*p);
  } else if constexpr (P == 2) {
    const float2 f = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(p));
    v[0] = f.x; v[1] = f.y;
  } else {
    const uint2 q = *reinterpret_cast<const uint2*>(p);
    const float2 a = unpack_bf16x2(q.x), b = unpack_bf16x2(q.y);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
}
template <int P>
NT_DEVICE void stp(__nv_bfloat16* p, const float (&v)[P]) {
  if constexpr (P == 1) {
    *p = f2bf(v[0]);
  } else if constexpr (P == 2) {
    *reinterpret_cast<uint32_t*>(p) = pack_bf16x2(v[0], v[1]);
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  }
}

// ------------------------------------------------------------------ mix + norm forward
// xm = bf16(bf16(bf16(a) x) + bf16(bf16(b) x0))  (x0 == nullptr: xm = x, nothing written)
// h = bf16(xm * rsqrt(mean(xm^2) + eps)); rstd saved per row.
template <int NCH>
__global__ void mix_norm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ x0,
                                    const float* __restrict__ ab, __nv_bfloat16* __restrict__ xm,
                                    __nv_bfloat16* __restrict__ h, float* __restrict__ rstd, int M, int d,
                                    float out_scale) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int64_t off = static_cast<int64_t>(row) * d;
  float v[NCH][8];
  float a = 1.f, b = 0.f;
  if (x0) {
    a = rbf(ab[0]);
    b = rbf(ab[1]);
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < d) {
      load8(x + off + col, v[c]);
      if (x0) {
        float w[8];
        load8(x0 + off + col, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[c][i] = rbf(rbf(a * v[c][i]) + rbf(b * w[i]));
        store8(xm + off + col, v[c]);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += v[c][i] * v[c][i];
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / d + kNormEps);
  if (lane == 0 && rstd) rstd[row] = r;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < d) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = out_scale == 1.f ? v[c][i] * r : rbf(v[c][i] * r) * out_scale;
      store8(h + off + col, o);
    }
  }
}

// ------------------------------------------------------------------ norm backward (+ residual)
// dx = dres + rstd * (dy - n * mean(dy * n)),  n = x * rstd   (all fp32, output bf16)
template <int NCH>
__global__ void norm_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ dy,
                                const __nv_bfloat16* __restrict__ dres, __nv_bfloat16* __restrict__ dx, int M,
                                int d) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int64_t off = static_cast<int64_t>(row) * d;
  float xv[NCH][8], gv[NCH][8];
  float ss = 0.f, dot = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < d) {
      load8(x + off + col, xv[c]);
      load8(dy + off + col, gv[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ss += xv[c][i] * xv[c][i];
        dot += gv[c][i] * xv[c][i];
      }
    }
  }
  ss = warp_sum(ss);
  dot = warp_sum(dot);
  const float r = rsqrtf(ss / d + kNormEps);
  const float k = r * r * r * dot / d;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < d) {
      float o[8], rr[8];
      if (dres) load8(dres + off + col, rr);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = r * gv[c][i] - k * xv[c][i] + (dres ? rr[i] : 0.f);
      store8(dx + off + col, o);
    }
  }
}

// ------------------------------------------------------------------ mix + norm backward
// dxm = dres + norm_bwd(xm, dh);  dx = a * dxm;  dx0_acc += b * dxm;
// part[row] = (sum dxm * x, sum dxm * x0)   (reduced to d a, d b by the caller)
template <int NCH>
__global__ void mix_norm_bwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ x0,
                                    const __nv_bfloat16* __restrict__ xm, const __nv_bfloat16* __restrict__ dh,
                                    const __nv_bfloat16* __restrict__ dres, const float* __restrict__ ab,
                                    __nv_bfloat16* __restrict__ dx, float* __restrict__ dx0_acc,
                                    float* __restrict__ part, int M, int d) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int64_t off = static_cast<int64_t>(row) * d;
  const float a = rbf(ab[0]), b = rbf(ab[1]);
  float mv[NCH][8], gv[NCH][8];
  float ss = 0.f, dot = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < d) {
      load8(xm + off + col, mv[c]);
      load8(dh + off + col, gv[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ss += mv[c][i] * mv[c][i];
        dot += gv[c][i] * mv[c][i];
      }
    }
  }
  ss = warp_sum(ss);
  dot = warp_sum(dot);
  const float r = rsqrtf(ss / d + kNormEps);
  const float k = r * r * r * dot / d;
  float pa = 0.f, pb = 0.f;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < d) {
      float rr[8], xv[8], x0v[8], o[8];
      load8(dres + off + col, rr);
      load8(x + off + col, xv);
      load8(x0 + off + col, x0v);
      float4* acc = reinterpret_cast<float4*>(dx0_acc + off + col);
      float4 a0 = acc[0], a1 = acc[1];
      float g[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        g[i] = rr[i] + r * gv[c][i] - k * mv[c][i];
        o[i] = a * g[i];
        pa += g[i] * xv[i];
        pb += g[i] * x0v[i];
      }
      a0.x += b * g[0]; a0.y += b * g[1]; a0.z += b * g[2]; a0.w += b * g[3];
      a1.x += b * g[4]; a1.y += b * g[5]; a1.z += b * g[6]; a1.w += b * g[7];
      acc[0] = a0;
      acc[1] = a1;
      store8(dx + off + col, o);
    }
  }
  pa = warp_sum(pa);
  pb = warp_sum(pb);
  if (lane == 0) {
    part[2 * row] = pa;
    part[2 * row + 1] = pb;
  }
}

// ------------------------------------------------------------------ RoPE + QK norm + VE gate
// qkv row layout: [H q-heads | Hk k-heads | Hk v-heads] x D.  One warp per (row, head).
// q,k:  y = scale * norm(rope(x))  in place; rstd saved in rstd[row * (H + Hk) + head].
// v:    v += gate * ve_table[idx[row]] with gate = 3 sigmoid(dot(h[row, :G], wg[head]));
//       gate saved in gate_out[row * Hk + head].
template <int P>  // P = D / 64 rotation pairs per lane
__global__ void rope_norm_fwd_kernel(__nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ cosb,
                                     const __nv_bfloat16* __restrict__ sinb, float* __restrict__ rstd, int M, int T,
                                     int H, int Hk, float scale, const __nv_bfloat16* __restrict__ ve_table,
                                     const int64_t* __restrict__ idx, const __nv_bfloat16* __restrict__ hrow,
                                     int ldh, const __nv_bfloat16* __restrict__ wg, int G,
                                     float* __restrict__ gate_out, int head0) {
  constexpr int D = P * 64;
  const int nheads = H + 2 * Hk, nsub = nheads - head0;  // heads [head0, nheads) of every row
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(M) * nsub) return;
  const int row = static_cast<int>(gw / nsub);
  const int head = head0 + static_cast<int>(gw - static_cast<int64_t>(row) * nsub);
  const int ld = nheads * D;
  __nv_bfloat16* base = qkv + static_cast<int64_t>(row) * ld + head * D;
  if (head < H + Hk) {
    const int t = row % T;
    float x1[P], x2[P], c[P], sn[P], y1[P], y2[P];
    const int i0 = lane * P;
    ldp<P>(base + i0, x1);
    ldp<P>(base + i0 + D / 2, x2);
    ldp<P>(cosb + static_cast<int64_t>(t) * (D / 2) + i0, c);
    ldp<P>(sinb + static_cast<int64_t>(t) * (D / 2) + i0, sn);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      y1[j] = rbf(rbf(x1[j] * c[j]) + rbf(x2[j] * sn[j]));
      y2[j] = rbf(rbf(x1[j] * -sn[j]) + rbf(x2[j] * c[j]));
      ss += y1[j] * y1[j] + y2[j] * y2[j];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + kNormEps);
    if (lane == 0) rstd[static_cast<int64_t>(row) * (H + Hk) + head] = r;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      y1[j] = rbf(y1[j] * r) * scale;
      y2[j] = rbf(y2[j] * r) * scale;
    }
    stp<P>(base + i0, y1);
    stp<P>(base + i0 + D / 2, y2);
  } else if (ve_table) {
    const int hk = head - H - Hk;
    float z = 0.f;
    if (lane < G) z = bf2f(hrow[static_cast<int64_t>(row) * ldh + lane]) * bf2f(wg[hk * G + lane]);
    z = rbf(warp_sum(z));
    const float gate = rbf(3.f * rbf(1.f / (1.f + __expf(-z))));
    if (lane == 0) gate_out[static_cast<int64_t>(row) * Hk + hk] = gate;
    const __nv_bfloat16* ve = ve_table + idx[row] * static_cast<int64_t>(Hk * D) + hk * D;
    float a[2 * P], e[2 * P];
    const int i0 = lane * 2 * P;
    if constexpr (P == 1) {
      ldp<2>(base + i0, a);
      ldp<2>(ve + i0, e);
    } else {
      ldp<4>(base + i0, *reinterpret_cast<float(*)[4]>(&a[0]));
      ldp<4>(ve + i0, *reinterpret_cast<float(*)[4]>(&e[0]));
      if constexpr (P == 4) {
        ldp<4>(base + i0 + 4, *reinterpret_cast<float(*)[4]>(&a[4]));
        ldp<4>(ve + i0 + 4, *reinterpret_cast<float(*)[4]>(&e[4]));
      }
    }
#pragma unroll
    for (int j = 0; j < 2 * P; ++j) a[j] = rbf(a[j] + rbf(gate * e[j]));
    if constexpr (P == 1) {
      stp<2>(base + i0, a);
    } else {
      stp<4>(base + i0, *reinterpret_cast<float(*)[4]>(&a[0]));
      if constexpr (P == 4) stp<4>(base + i0 + 4, *reinterpret_cast<float(*)[4]>(&a[4]));
    }
  }
}

// Backward, in place on dqkv.  q/k heads: undo scale, norm, rotation.  v heads: dv passes
// through; dz[row, hk] = d(gate logit); ve_grad[idx[row]] += gate * dv (fp32 atomics).
template <int P>
__global__ void rope_norm_bwd_kernel(__nv_bfloat16* __restrict__ dqkv, const __nv_bfloat16* __restrict__ qkv,
                                     const __nv_bfloat16* __restrict__ cosb, const __nv_bfloat16* __restrict__ sinb,
                                     const float* __restrict__ rstd, int M, int T, int H, int Hk, float scale,
                                     const __nv_bfloat16* __restrict__ ve_table, const int64_t* __restrict__ idx,
                                     const float* __restrict__ gate_in, float* __restrict__ dz,
                                     float* __restrict__ ve_grad, int head0) {
  constexpr int D = P * 64;
  const int nheads = H + 2 * Hk, nsub = nheads - head0;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(M) * nsub) return;
  const int row = static_cast<int>(gw / nsub);
  const int head = head0 + static_cast<int>(gw - static_cast<int64_t>(row) * nsub);
  const int ld = nheads * D;
  const int64_t o = static_cast<int64_t>(row) * ld + head * D;
  if (head < H + Hk) {
    const int t = row % T;
    const float r = rstd[static_cast<int64_t>(row) * (H + Hk) + head];
    float n1[P], n2[P], g1[P], g2[P], c[P], sn[P];
    const int i0 = lane * P;
    ldp<P>(qkv + o + i0, n1);
    ldp<P>(qkv + o + i0 + D / 2, n2);
    ldp<P>(dqkv + o + i0, g1);
    ldp<P>(dqkv + o + i0 + D / 2, g2);
    ldp<P>(cosb + static_cast<int64_t>(t) * (D / 2) + i0, c);
    ldp<P>(sinb + static_cast<int64_t>(t) * (D / 2) + i0, sn);
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      n1[j] /= scale;
      n2[j] /= scale;
      g1[j] *= scale;
      g2[j] *= scale;
      dot += g1[j] * n1[j] + g2[j] * n2[j];
    }
    dot = warp_sum(dot) / D;
    float o1[P], o2[P];
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const float d1 = r * (g1[j] - n1[j] * dot), d2 = r * (g2[j] - n2[j] * dot);
      // forward: y1 = x1 c + x2 s ; y2 = -x1 s + x2 c  =>  dx1 = d1 c - d2 s ; dx2 = d1 s + d2 c
      o1[j] = d1 * c[j] - d2 * sn[j];
      o2[j] = d1 * sn[j] + d2 * c[j];
    }
    stp<P>(dqkv + o + i0, o1);
    stp<P>(dqkv + o + i0 + D / 2, o2);
  } else if (ve_table) {
    const int hk = head - H - Hk;
    const float gate = gate_in[static_cast<int64_t>(row) * Hk + hk];
    const int64_t tok = idx[row];
    const __nv_bfloat16* ve = ve_table + tok * static_cast<int64_t>(Hk * D) + hk * D;
    float* vg = ve_grad + tok * static_cast<int64_t>(Hk * D) + hk * D;
    float dg = 0.f;
    const int i0 = lane * 2 * P;
#pragma unroll
    for (int j = 0; j < 2 * P; j += 2) {
      const float2 g = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(dqkv + o + i0 + j));
      const float2 e = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(ve + i0 + j));
      dg += g.x * e.x + g.y * e.y;
      atomicAdd(reinterpret_cast<float2*>(vg + i0 + j), make_float2(g.x * gate, g.y * gate));
    }
    dg = warp_sum(dg);
    // gate = 3 sigmoid(z): dgate/dz = gate * (1 - gate / 3)
    if (lane == 0) dz[static_cast<int64_t>(row) * Hk + hk] = dg * gate * (1.f - gate / 3.f);
  }
}

// rope_norm backward for heads of 128 with 16 lanes each (two half-warps per warp, U heads per
// half-warp, every load issued before the math) and 16-byte accesses: lane l of a head holds elements
// [8 l, 8 l + 8), so lanes l and l ^ 8 hold the two halves of the same rotation pairs and swap them with
// one shuffle.  Same arithmetic as rope_norm_bwd_kernel; q / k heads only (value heads take the
// per-warp kernel when value embeddings are mixed in).  The same layout for the forward measured no
// faster than the per-warp forward (0.257 vs 0.252 ms at 65536 rows), which stays.
// Backward in place on dqkv (q / k heads): undo the scale and the norm, then the rotation with the
// partner lane's half: dx1 = d1 c - d2 s, dx2 = d1 s + d2 c.
template <int U>
__global__ void rope_norm_bwd_wide_kernel(__nv_bfloat16* __restrict__ dqkv, const __nv_bfloat16* __restrict__ qkv,
                                          const __nv_bfloat16* __restrict__ cosb,
                                          const __nv_bfloat16* __restrict__ sinb, const float* __restrict__ rstd,
                                          int M, int T, int H, int Hk, float scale) {
  constexpr int D = 128;
  const int nqk = H + Hk, ld = (H + 2 * Hk) * D;
  const int lane = threadIdx.x & 31, hl = lane & 15, sub = lane >> 4;
  const int units = M * nqk;
  const int g0 = ((blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 2 + sub) * U;
  if (g0 >= units) return;
  const unsigned mask = 0xFFFFu << (16 * sub);
  const int k = 8 * (hl & 7);
  const bool first = hl < 8;
  uint4 nraw[U], graw[U];
  int row[U], head[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int gu = min(g0 + u, units - 1);
    row[u] = gu / nqk;
    head[u] = gu - row[u] * nqk;
    const int64_t o = static_cast<int64_t>(row[u]) * ld + head[u] * D + 8 * hl;
    nraw[u] = *reinterpret_cast<const uint4*>(qkv + o);
    graw[u] = *reinterpret_cast<const uint4*>(dqkv + o);
  }
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (g0 + u >= units) break;
    auto unpack = [](const uint4& q, float (&v)[8]) {
      const float2 a = unpack_bf16x2(q.x), b = unpack_bf16x2(q.y), cc = unpack_bf16x2(q.z), d = unpack_bf16x2(q.w);
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = cc.x; v[5] = cc.y; v[6] = d.x; v[7] = d.y;
    };
    float n[8], g[8], c[8], sn[8];
    unpack(nraw[u], n);
    unpack(graw[u], g);
    const int t = row[u] % T;
    load8(cosb + static_cast<int64_t>(t) * (D / 2) + k, c);
    load8(sinb + static_cast<int64_t>(t) * (D / 2) + k, sn);
    const float r = rstd[static_cast<int64_t>(row[u]) * nqk + head[u]];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      n[j] /= scale;
      g[j] *= scale;
      dot += g[j] * n[j];
    }
#pragma unroll
    for (int of = 8; of > 0; of >>= 1) dot += __shfl_xor_sync(mask, dot, of);
    dot /= D;
    float d[8], dp[8], out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] = r * (g[j] - n[j] * dot);
#pragma unroll
    for (int j = 0; j < 8; ++j) dp[j] = __shfl_xor_sync(mask, d[j], 8);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float d1 = first ? d[j] : dp[j], d2 = first ? dp[j] : d[j];
      out[j] = first ? d1 * c[j] - d2 * sn[j] : d1 * sn[j] + d2 * c[j];
    }
    store8(dqkv + static_cast<int64_t>(row[u]) * ld + head[u] * D + 8 * hl, out);
  }
}

// ------------------------------------------------------------------ soft-capped cross entropy
// One CTA per row.  z = cap tanh(l / cap) over the first V of Vp columns.
// loss[row] = logsumexp(z) - z[target]  (0 for target < 0);
// logits[row, :] <- (softmax(z) - onehot(target)) * (1 - (z / cap)^2)   (0 on padding / ignored rows)
__global__ void softcap_ce_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, const int64_t* __restrict__ tgt,
                                  float* __restrict__ loss, float* __restrict__ lse_out, int V, int Vp, float cap) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  __nv_bfloat16* l = logits + static_cast<int64_t>(row) * ld;
  const int64_t target = tgt[row];
  const float inv = 1.f / cap;
  float mx = -INFINITY, sm = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    float v[8];
    if (c + 8 <= V) {
      load8(l + c, v);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = (c + i < V) ? bf2f(l[c + i]) : -INFINITY;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (c + i < V) {
        const float z = cap * tanhf(v[i] * inv);
        if (z > mx) {
          sm = sm * __expf(mx - z) + 1.f;
          mx = z;
        } else {
          sm += __expf(z - mx);
        }
      }
    }
  }
  // combine (max, sum) pairs across the block
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, o), os = __shfl_xor_sync(0xffffffffu, sm, o);
    const float nm = fmaxf(mx, om);
    sm = (mx == -INFINITY ? 0.f : sm * __expf(mx - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
    mx = nm;
  }
  __shared__ float wm[32], ws[32];
  if (lane == 0) { wm[warp] = mx; ws[warp] = sm; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    mx = lane < nw ? wm[lane] : -INFINITY;
    sm = lane < nw ? ws[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, mx, o), os = __shfl_xor_sync(0xffffffffu, sm, o);
      const float nm = fmaxf(mx, om);
      sm = (mx == -INFINITY ? 0.f : sm * __expf(mx - nm)) + (om == -INFINITY ? 0.f : os * __expf(om - nm));
      mx = nm;
    }
    if (lane == 0) { red[0] = mx; red[1] = sm; }
  }
  __syncthreads();
  const float lse = red[0] + __logf(red[1]);
  if (threadIdx.x == 0) {
    float zt = 0.f;
    if (target >= 0) zt = cap * tanhf(bf2f(l[target]) * inv);
    loss[row] = target >= 0 ? lse - zt : 0.f;
    if (lse_out) lse_out[row] = lse;
  }
  __syncthreads();  // the target logit is read above before any thread overwrites it
  for (int c = threadIdx.x * 8; c < Vp; c += blockDim.x * 8) {
    float v[8], o[8];
    const bool vec = (c + 8 <= Vp);
    if (vec) load8(l + c, v);
    else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = (c + i < Vp) ? bf2f(l[c + i]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int col = c + i;
      float g = 0.f;
      if (target >= 0 && col < V) {
        const float th = tanhf(v[i] * inv);
        const float z = cap * th;
        g = __expf(z - lse) - (col == target ? 1.f : 0.f);
        g *= (1.f - th * th);
      }
      o[i] = g;
    }
    if (vec) store8(l + c, o);
    else {
      for (int i = 0; i < 8 && c + i < Vp; ++i) l[c + i] = f2bf(o[i]);
    }
  }
}

// ------------------------------------------------------------------ embedding + norm + smear
// n[row] = norm(wte[idx[row]]);  x[row] = n[row] + gate[row] * n[row-1]  (t > 0 within a sequence)
// gate = bf16(lambda) * sigmoid(dot(n[row, :24], w_smear)); the sigmoid is saved (0 at t == 0)
template <int NCH>
__global__ void embed_smear_kernel(const __nv_bfloat16* __restrict__ wte, const int64_t* __restrict__ idx,
                                   const __nv_bfloat16* __restrict__ wsm, const float* __restrict__ lam,
                                   __nv_bfloat16* __restrict__ n_out, __nv_bfloat16* __restrict__ x_out,
                                   float* __restrict__ gate_out, int M, int T, int d, int G) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const int t = row % T;
  float cur[NCH][8], prev[NCH][8];
  float ss = 0.f, ssp = 0.f;
  const __nv_bfloat16* e = wte + idx[row] * static_cast<int64_t>(d);
  const __nv_bfloat16* ep = t > 0 ? wte + idx[row - 1] * static_cast<int64_t>(d) : e;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < d) {
      load8(e + col, cur[c]);
      load8(ep + col, prev[c]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ss += cur[c][i] * cur[c][i];
        ssp += prev[c][i] * prev[c][i];
      }
    }
  }
  ss = warp_sum(ss);
  ssp = warp_sum(ssp);
  const float r = rsqrtf(ss / d + kNormEps), rp = rsqrtf(ssp / d + kNormEps);
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      cur[c][i] = rbf(cur[c][i] * r);
      prev[c][i] = rbf(prev[c][i] * rp);
    }
  // gate from the first G (= 24) channels of n[row]: lanes 0..2 own channels 0..23 of chunk 0
  float z = 0.f;
  if (lane * 8 < G) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (lane * 8 + i < G) z += cur[0][i] * bf2f(wsm[lane * 8 + i]);
  }
  z = rbf(warp_sum(z));
  const float sig = rbf(1.f / (1.f + __expf(-z)));
  const float gate = t > 0 ? rbf(rbf(lam[0]) * sig) : 0.f;
  if (lane == 0) gate_out[row] = t > 0 ? sig : 0.f;
  const int64_t off = static_cast<int64_t>(row) * d;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int col = (c * 32 + lane) * 8;
    if (col < d) {
      float o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = t > 0 ? rbf(cur[c][i] + rbf(gate * prev[c][i])) : cur[c][i];
      store8(n_out + off + col, cur[c]);
      store8(x_out + off + col, o);
    }
  }
}

// Embedding-gradient scatter: grad_table[idx[row]] += dy[row]  (fp32 atomics; dy fp32 or bf16)
template <typename TIn>
__global__ void embed_scatter_kernel(const TIn* __restrict__ dy, const int64_t* __restrict__ idx,
                                     float* __restrict__ grad, int M, int d) {
  const int row = blockIdx.x;
  const int64_t tok = idx[row];
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    float v;
    if constexpr (sizeof(TIn) == 2) v = bf2f(dy[static_cast<int64_t>(row) * d + c]);
    else v = dy[static_cast<int64_t>(row) * d + c];
    atomicAdd(grad + tok * d + c, v);
  }
}

__global__ void cast_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, int64_t n,
                                 int vec) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (vec && i + 4 <= n) {
    float4 v = *reinterpret_cast<const float4*>(src + i);
    uint2 o = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
    *reinterpret_cast<uint2*>(dst + i) = o;
  } else {
    for (int64_t j = i; j < n && j < i + 4; ++j) dst[j] = f2bf(src[j]);
  }
}

}  // namespace ew
}  // namespace nt

// ==================================================================== launchers
using namespace nt::ew;

static int rows_per_block(int nch) { return nch <= 2 ? 8 : 4; }

#define NT_DISPATCH_NCH(d, ...)                                  \
  do {                                                                   \
    const int _nch = ((d) + 255) / 256;                                  \
    switch (_nch) {                                                      \
      case 1: { constexpr int NCH = 1; __VA_ARGS__; } break;             \
      case 2: { constexpr int NCH = 2; __VA_ARGS__; } break;             \
      case 3: { constexpr int NCH = 3; __VA_ARGS__; } break;             \
      case 4: { constexpr int NCH = 4; __VA_ARGS__; } break;             \
      case 5: { constexpr int NCH = 5; __VA_ARGS__; } break;             \
      case 6: { constexpr int NCH = 6; __VA_ARGS__; } break;             \
      case 7: { constexpr int NCH = 7; __VA_ARGS__; } break;             \
      case 8: { constexpr int NCH = 8; __VA_ARGS__; } break;             \
      default: return -1;                                                \
    }                                                                    \
  } while (0)

int nt_mix_norm_fwd(const void* x, const void* x0, const float* ab, void* xm, void* h, float* rstd, int M, int d,
                    float out_scale, cudaStream_t s) {
  if (d % 8) return -1;
  NT_DISPATCH_NCH(d, {
    const int rpb = rows_per_block(NCH);
    mix_norm_fwd_kernel<NCH><<<(M + rpb - 1) / rpb, rpb * 32, 0, s>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)x0, ab, (__nv_bfloat16*)xm, (__nv_bfloat16*)h, rstd, M, d,
        out_scale);
  });
  return 0;
}

int nt_norm_bwd(const void* x, const void* dy, const void* dres, void* dx, int M, int d, cudaStream_t s) {
  if (d % 8) return -1;
  NT_DISPATCH_NCH(d, {
    const int rpb = rows_per_block(NCH);
    norm_bwd_kernel<NCH><<<(M + rpb - 1) / rpb, rpb * 32, 0, s>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)dy, (const __nv_bfloat16*)dres, (__nv_bfloat16*)dx, M, d);
  });
  return 0;
}

int nt_mix_norm_bwd(const void* x, const void* x0, const void* xm, const void* dh, const void* dres,
                    const float* ab, void* dx, float* dx0_acc, float* part, int M, int d, cudaStream_t s) {
  if (d % 8) return -1;
  NT_DISPATCH_NCH(d, {
    const int rpb = rows_per_block(NCH);
    mix_norm_bwd_kernel<NCH><<<(M + rpb - 1) / rpb, rpb * 32, 0, s>>>(
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)x0, (const __nv_bfloat16*)xm, (const __nv_bfloat16*)dh,
        (const __nv_bfloat16*)dres, ab, (__nv_bfloat16*)dx, dx0_acc, part, M, d);
  });
  return 0;
}

int nt_rope_norm_fwd(void* qkv, const void* cosb, const void* sinb, float* rstd, int M, int T, int H, int Hk, int D,
                     float scale, const void* ve_table, const int64_t* idx, const void* hrow, int ldh,
                     const void* wg, int G, float* gate_out, cudaStream_t s) {
  const int wpb = 8;
  if (G > 32) return -1;
  const int head0 = 0;
  const int64_t warps = static_cast<int64_t>(M) * (H + 2 * Hk - head0);
  const unsigned blocks = static_cast<unsigned>((warps + wpb - 1) / wpb);
#define NT_RN(P)                                                                                                 \
  rope_norm_fwd_kernel<P><<<blocks, wpb * 32, 0, s>>>((__nv_bfloat16*)qkv, (const __nv_bfloat16*)cosb,          \
                                                      (const __nv_bfloat16*)sinb, rstd, M, T, H, Hk, scale,     \
                                                      (const __nv_bfloat16*)ve_table, idx,                      \
                                                      (const __nv_bfloat16*)hrow, ldh, (const __nv_bfloat16*)wg, \
                                                      G, gate_out, head0)
  switch (D) {
    case 64: NT_RN(1); break;
    case 128: NT_RN(2); break;
    case 256: NT_RN(4); break;
    default: return -1;
  }
#undef NT_RN
  return 0;
}

int nt_rope_norm_bwd(void* dqkv, const void* qkv, const void* cosb, const void* sinb, const float* rstd, int M,
                     int T, int H, int Hk, int D, float scale, const void* ve_table, const int64_t* idx,
                     const float* gate, float* dz, float* ve_grad, cudaStream_t s) {
  const int wpb = 8;
  // heads of 128: q / k heads by the wide kernel, value heads (only with value embeddings) per warp
  int head0 = 0;
  constexpr int U = 2;
  if (D == 128 && static_cast<int64_t>(M) * (H + Hk) < (int64_t(1) << 30)) {
    const int64_t halves = (static_cast<int64_t>(M) * (H + Hk) + U - 1) / U;
    rope_norm_bwd_wide_kernel<U><<<static_cast<unsigned>((halves + 2 * wpb - 1) / (2 * wpb)), wpb * 32, 0, s>>>(
        (__nv_bfloat16*)dqkv, (const __nv_bfloat16*)qkv, (const __nv_bfloat16*)cosb, (const __nv_bfloat16*)sinb, rstd,
        M, T, H, Hk, scale);
    if (!ve_table) return 0;
    head0 = H + Hk;
  }
  const int64_t warps = static_cast<int64_t>(M) * (H + 2 * Hk - head0);
  const unsigned blocks = static_cast<unsigned>((warps + wpb - 1) / wpb);
#define NT_RNB(P)                                                                                                  \
  rope_norm_bwd_kernel<P><<<blocks, wpb * 32, 0, s>>>((__nv_bfloat16*)dqkv, (const __nv_bfloat16*)qkv,            \
                                                      (const __nv_bfloat16*)cosb, (const __nv_bfloat16*)sinb,     \
                                                      rstd, M, T, H, Hk, scale, (const __nv_bfloat16*)ve_table,   \
                                                      idx, gate, dz, ve_grad, head0)
  switch (D) {
    case 64: NT_RNB(1); break;
    case 128: NT_RNB(2); break;
    case 256: NT_RNB(4); break;
    default: return -1;
  }
#undef NT_RNB
  return 0;
}

int nt_softcap_ce(void* logits, int64_t ld, const int64_t* tgt, float* loss, float* lse, int rows, int V, int Vp,
                  float cap, int variant, cudaStream_t s) {
  if (ld % 8 || Vp % 8) return -1;
  if (rows <= 0) return 0;
  (void)variant;
  softcap_ce_kernel<<<rows, 1024, 0, s>>>((__nv_bfloat16*)logits, ld, tgt, loss, lse, V, Vp, cap);
  return 0;
}

int nt_embed_smear(const void* wte, const int64_t* idx, const void* wsm, const float* lam, void* n_out, void* x_out,
                   float* gate_out, int M, int T, int d, int G, cudaStream_t s) {
  if (d % 8 || G > 32) return -1;
  NT_DISPATCH_NCH(d, {
    const int rpb = rows_per_block(NCH);
    embed_smear_kernel<NCH><<<(M + rpb - 1) / rpb, rpb * 32, 0, s>>>(
        (const __nv_bfloat16*)wte, idx, (const __nv_bfloat16*)wsm, lam, (__nv_bfloat16*)n_out,
        (__nv_bfloat16*)x_out, gate_out, M, T, d, G);
  });
  return 0;
}

int nt_embed_scatter(const void* dy, int dy_is_f32, const int64_t* idx, float* grad, int M, int d, cudaStream_t s) {
  if (M <= 0) return 0;
  if (dy_is_f32) embed_scatter_kernel<float><<<M, 256, 0, s>>>((const float*)dy, idx, grad, M, d);
  else embed_scatter_kernel<__nv_bfloat16><<<M, 256, 0, s>>>((const __nv_bfloat16*)dy, idx, grad, M, d);
  return 0;
}

int nt_cast_bf16(const float* src, void* dst, int64_t n, cudaStream_t s) {
  if (n <= 0) return 0;
  const int64_t threads = (n + 3) / 4;
  const int vec = (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (reinterpret_cast<uintptr_t>(dst) % 8 == 0);
  cast_bf16_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, s>>>(src, (__nv_bfloat16*)dst, n, vec);
  return 0;
}
