// Per-chunk terms of the chunked (gated) delta rule on sm_100a: one CTA per (64-token chunk,
// head, batch) computes, entirely on chip, what the inter-chunk scan (delta_scan.cu) consumes, and
// the backward of the same terms.
//
// Inside chunk n with tokens i, j in [0, 64), cumulative log decay b_i (b = cumsum of the gate
// within the chunk; b = 0 without a gate) and the delta-rule strength beta_i:
//   GDN (scalar gate):  q <- s q / |q|, k <- k / |k| (here);  P_ij = e^{b_i - b_j} for j <= i
//                       akk_ij = (k_i . k_j) P_ij,  aqk_ij = (q_i . k_j) P_ij,  kt_i = k_i e^{b_i}
//   KDA (feature gate): kt = k e^{b}, qt = q e^{b}, ki = k e^{-b} (per feature)
//                       akk = kt ki^T,  aqk = qt ki^T
//   DeltaNet:           akk = k k^T, aqk = q k^T, kt = k
//   L = I + strict_tril(beta_i akk_ij);   L [w | u0] = beta [kt | v]   (forward substitution)
//   outputs: w, u0, qt = q e^{b}, kc = k e^{b_last - b}, aqk (lower incl. diagonal), carry = e^{b_last}
// Backward (the forward's products are recomputed from q, k, v, g, beta in the same CTA; the
// solution [w | u0] is read back from the forward's outputs):
//   dR = L^{-T} [dw | du0] (back substitution), dA = -dR [w|u0]^T (strict lower), dv = beta dR_v,
//   dbeta = rowsum(dR * [kt|v]) + rowsum(dA * akk), then the products and exponentials are
//   differentiated in closed form and dg is the reverse cumulative sum of db within the chunk.
// The reference computes these terms with FLA's chunk_kda / chunk_gated_delta_rule Triton kernels
// (nexttransformer/models/linear.py:302-328); this is a design of its own: fp32 CUDA-core math
// with 4 x 4 register tiles on shared memory, one solve column per thread, deterministic
// reductions (warp shuffles and fixed-order sums, no atomics).
#include "delta_prep.h"
#include "common.cuh"

#include <stdexcept>

namespace nt {
namespace dprep {

constexpr int C = 64;      // chunk length
constexpr int D = 128;     // head dimension (keys and values)
constexpr int LDF = 129;   // fp32 row stride of [64 x 128] tiles (odd: conflict-free column walks)
constexpr int LDA = 65;    // fp32 row stride of [64 x 64] tiles
constexpr int NT = 256;    // threads per CTA

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }

// 16 bytes at p (16-byte aligned) as floats: 8 bf16 or 4 fp32 elements.
template <typename TIn>
__device__ __forceinline__ void load_vec(const TIn* p, float (&out)[16 / sizeof(TIn)]);
template <>
__device__ __forceinline__ void load_vec<__nv_bfloat16>(const __nv_bfloat16* p, float (&out)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  // a bf16 is the upper half of the fp32 with the same value: widen by shifting
  out[0] = __uint_as_float(raw.x << 16);
  out[1] = __uint_as_float(raw.x & 0xffff0000u);
  out[2] = __uint_as_float(raw.y << 16);
  out[3] = __uint_as_float(raw.y & 0xffff0000u);
  out[4] = __uint_as_float(raw.z << 16);
  out[5] = __uint_as_float(raw.z & 0xffff0000u);
  out[6] = __uint_as_float(raw.w << 16);
  out[7] = __uint_as_float(raw.w & 0xffff0000u);
}
template <>
__device__ __forceinline__ void load_vec<float>(const float* p, float (&out)[4]) {
  const float4 f = __ldg(reinterpret_cast<const float4*>(p));
  out[0] = f.x;
  out[1] = f.y;
  out[2] = f.z;
  out[3] = f.w;
}

// torch's softplus (beta 1, threshold 20), for the KDA gate
__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }

__device__ __forceinline__ float sum16(float v) {  // sum over 16 consecutive lanes
  v += __shfl_xor_sync(0xffffffffu, v, 8);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v;
}
__device__ __forceinline__ float sum32(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 16);
  return sum16(v);
}

// Shared-memory layout shared by both kernels (fp32 unless noted).
template <int GATE>
struct Smem {
  static constexpr int Q = 0;                                   // [C][LDF] q (GDN: normalised), KDA: qt
  static constexpr int K = Q + C * LDF;                         // [C][LDF] k (GDN: normalised), KDA: kt
  static constexpr int KI = K + C * LDF;                        // [C][LDF] KDA: k e^{-b}
  static constexpr int B = KI + (GATE == DELTA_FEATURE ? C * LDF : 0);   // KDA [C][LDF], else [C]
  static constexpr int A = B + (GATE == DELTA_FEATURE ? C * LDF : C);    // [C][LDA] beta-scaled strict akk
  static constexpr int K2 = A + C * LDA;                        // [C][LDA] akk without the gate factor
  static constexpr int Q2 = K2 + C * LDA;                       // [C][LDA] GDN: q.k dots
  static constexpr int SX = Q2 + (GATE == DELTA_SCALAR ? C * LDA : 0);   // [C][LDA] stage / Gq
  static constexpr int SY = SX + C * LDA;                       // [C][LDA] stage / dP
  static constexpr int BETA = SY + C * LDA;                     // [C]
  static constexpr int NQ = BETA + C;                           // [C] GDN: |q|, |k| before normalisation
  static constexpr int NK = NQ + C;
  static constexpr int DB = NK + C;                             // [C] scalar db / dbeta partials
  static constexpr int DBETA = DB + C;                          // [C]
  static constexpr int V = DBETA + C;                           // bf16 [C][D] v
  static constexpr int FLOATS = V + C * D / 2;
  static constexpr int BYTES = FLOATS * 4;
};

// Loads q, k, v, g, beta of chunk (n, h, b), normalises q / k (GDN), forms the cumulative decay and
// the KDA scaled copies; returns after a __syncthreads.
template <int GATE, typename TIn>
__device__ void load_chunk(const DeltaPrepArgs& a, float* sm, int n, int h, int b) {
  using S = Smem<GATE>;
  float* sq = sm + S::Q;
  float* sk = sm + S::K;
  float* sb = sm + S::B;
  __nv_bfloat16* sv = reinterpret_cast<__nv_bfloat16*>(sm + S::V);
  const int tid = threadIdx.x;
  const int t0 = n * C;
  const int64_t rs = static_cast<int64_t>(a.H) * D;
  const int64_t base = (static_cast<int64_t>(b) * a.T * a.H + h) * D;
  const TIn* q = reinterpret_cast<const TIn*>(a.q) + base;
  const TIn* k = reinterpret_cast<const TIn*>(a.k) + base;
  const TIn* v = reinterpret_cast<const TIn*>(a.v) + base;
  // 16-byte vector loads, every pass's loads issued before any is used (one memory latency, not one
  // per element): VEC elements per load, LPR lanes per 128-feature row, RPP rows per pass
  {
    constexpr int VEC = 16 / static_cast<int>(sizeof(TIn));
    constexpr int LPR = D / VEC, RPP = NT / LPR, PASSES = C / RPP;
    const int d0 = (tid % LPR) * VEC, i0 = tid / LPR;
    float qv[PASSES][VEC], kv[PASSES][VEC], vv[PASSES][VEC];
#pragma unroll
    for (int ps = 0; ps < PASSES; ++ps) {
      const int t = t0 + i0 + ps * RPP;
      if (t < a.T) {
        load_vec<TIn>(q + t * rs + d0, qv[ps]);
        load_vec<TIn>(k + t * rs + d0, kv[ps]);
        load_vec<TIn>(v + t * rs + d0, vv[ps]);
      } else {
#pragma unroll
        for (int u = 0; u < VEC; ++u) qv[ps][u] = kv[ps][u] = vv[ps][u] = 0.f;
      }
    }
#pragma unroll
    for (int ps = 0; ps < PASSES; ++ps) {
      const int i = i0 + ps * RPP;
#pragma unroll
      for (int u = 0; u < VEC; ++u) {
        sq[i * LDF + d0 + u] = qv[ps][u];
        sk[i * LDF + d0 + u] = kv[ps][u];
        sv[i * D + d0 + u] = __float2bfloat16_rn(vv[ps][u]);
      }
    }
  }
  if (GATE == DELTA_FEATURE && a.g_raw) {
    // g = -exp(g_log) softplus(g_raw + g_bias) per feature (0 past the end of the sequence)
    constexpr int LPR = D / 8, RPP = NT / LPR, PASSES = C / RPP;
    const int d0 = (tid % LPR) * 8, i0 = tid / LPR;
    float rv[PASSES][8];
#pragma unroll
    for (int ps = 0; ps < PASSES; ++ps) {
      const int t = t0 + i0 + ps * RPP;
      if (t < a.T) {
        load_vec<__nv_bfloat16>(a.g_raw + ((static_cast<int64_t>(b) * a.T + t) * a.H + h) * D + d0, rv[ps]);
      } else {
#pragma unroll
        for (int u = 0; u < 8; ++u) rv[ps][u] = 0.f;
      }
    }
    float ea[8], bias[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      ea[u] = expf(a.g_log[h * D + d0 + u]);
      bias[u] = a.g_bias[h * D + d0 + u];
    }
#pragma unroll
    for (int ps = 0; ps < PASSES; ++ps) {
      const bool live = t0 + i0 + ps * RPP < a.T;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        sb[(i0 + ps * RPP) * LDF + d0 + u] = live ? -ea[u] * softplus_f(rv[ps][u] + bias[u]) : 0.f;
    }
  } else if (GATE == DELTA_FEATURE) {
    constexpr int LPR = D / 4, RPP = NT / LPR, PASSES = C / RPP;
    const int d0 = (tid % LPR) * 4, i0 = tid / LPR;
    float gv[PASSES][4];
#pragma unroll
    for (int ps = 0; ps < PASSES; ++ps) {
      const int t = t0 + i0 + ps * RPP;
      if (t < a.T) {
        load_vec<float>(a.g + ((static_cast<int64_t>(b) * a.T + t) * a.H + h) * D + d0, gv[ps]);
      } else {
#pragma unroll
        for (int u = 0; u < 4; ++u) gv[ps][u] = 0.f;
      }
    }
#pragma unroll
    for (int ps = 0; ps < PASSES; ++ps)
#pragma unroll
      for (int u = 0; u < 4; ++u) sb[(i0 + ps * RPP) * LDF + d0 + u] = gv[ps][u];
  } else if (GATE == DELTA_SCALAR) {
    if (tid < C) {
      const int t = t0 + tid;
      sb[tid] = t < a.T ? a.g[(static_cast<int64_t>(b) * a.T + t) * a.H + h] : 0.f;
    }
  }
  if (tid < C) {
    const int t = t0 + tid;
    sm[S::BETA + tid] = t < a.T ? a.beta[(static_cast<int64_t>(b) * a.T + t) * a.H + h] : 0.f;
  }
  __syncthreads();
  if (GATE == DELTA_SCALAR || (GATE == DELTA_FEATURE && a.qk_norm)) {
    // L2 normalisation of every q and k row (one warp per row; F.normalize's eps of 1e-12)
    const int warp = tid >> 5, lane = tid & 31;
    for (int i = warp; i < C; i += NT / 32) {
      float s2q = 0.f, s2k = 0.f;
      for (int d = lane; d < D; d += 32) {
        const float x = sq[i * LDF + d], y = sk[i * LDF + d];
        s2q = fmaf(x, x, s2q);
        s2k = fmaf(y, y, s2k);
      }
      const float nq = fmaxf(sqrtf(sum32(s2q)), 1e-12f), nk = fmaxf(sqrtf(sum32(s2k)), 1e-12f);
      const float rq = a.qk_scale / nq, rk = 1.f / nk;
      for (int d = lane; d < D; d += 32) {
        sq[i * LDF + d] *= rq;
        sk[i * LDF + d] *= rk;
      }
      if (lane == 0) {
        sm[S::NQ + i] = nq;
        sm[S::NK + i] = nk;
      }
    }
  }
  if (GATE == DELTA_SCALAR) {
    if (tid == 0) {
      float s = 0.f;
      for (int i = 0; i < C; ++i) {
        s += sb[i];
        sb[i] = s;
      }
    }
  } else if (GATE == DELTA_FEATURE) {
    if (tid < D) {
      float s = 0.f;
      for (int i = 0; i < C; ++i) {
        s += sb[i * LDF + tid];
        sb[i * LDF + tid] = s;
      }
    }
  }
  __syncthreads();
  if (GATE == DELTA_FEATURE) {
    float* ski = sm + S::KI;
    for (int e = tid; e < C * D; e += NT) {
      const int i = e / D, d = e % D;
      const float bi = sb[i * LDF + d], kv = sk[i * LDF + d];
      sq[i * LDF + d] *= __expf(bi);
      sk[i * LDF + d] = kv * __expf(bi);
      ski[i * LDF + d] = kv * __expf(-bi);
    }
    __syncthreads();
  }
}

// Gate factor e^{b_i - b_j} (GDN, j <= i) or 1.
template <int GATE>
__device__ __forceinline__ float pair(const float* sb, int i, int j) {
  if (GATE == DELTA_SCALAR) return j <= i ? __expf(sb[i] - sb[j]) : 0.f;
  return 1.f;
}

// akk / aqk dot products (4 x 4 register tiles; rows 4 ti + r, columns tj + 16 c), the beta-scaled
// strict lower akk into A, the ungated dots into K2 (and Q2 for GDN); aqk (lower, gated) returned
// through the callback.  Ends with a __syncthreads.
template <int GATE, typename F>
__device__ void dots(float* sm, F&& emit_aqk) {
  using S = Smem<GATE>;
  const float* sq = sm + S::Q;
  const float* sk = sm + S::K;
  const float* sy = GATE == DELTA_FEATURE ? sm + S::KI : sm + S::K;
  const float* sb = sm + S::B;
  const int tid = threadIdx.x, ti = tid >> 4, tj = tid & 15;
  float kk[4][4], qk[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) kk[r][c] = qk[r][c] = 0.f;
#pragma unroll 4
  for (int d = 0; d < D; ++d) {
    float x[4], xq[4], y[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      x[r] = sk[(4 * ti + r) * LDF + d];
      xq[r] = sq[(4 * ti + r) * LDF + d];
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) y[c] = sy[(tj + 16 * c) * LDF + d];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        kk[r][c] = fmaf(x[r], y[c], kk[r][c]);
        qk[r][c] = fmaf(xq[r], y[c], qk[r][c]);
      }
  }
  float* sA = sm + S::A;
  float* sK2 = sm + S::K2;
  float* sQ2 = sm + S::Q2;
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = 4 * ti + r, j = tj + 16 * c;
      const float p = pair<GATE>(sb, i, j);
      sA[i * LDA + j] = j < i ? sm[S::BETA + i] * kk[r][c] * p : 0.f;
      sK2[i * LDA + j] = kk[r][c];
      if (GATE == DELTA_SCALAR) sQ2[i * LDA + j] = qk[r][c];
      emit_aqk(i, j, j <= i ? qk[r][c] * p : 0.f);
    }
  __syncthreads();
}

// kt of row i, feature d (the left half of the right-hand side)
template <int GATE>
__device__ __forceinline__ float kt_of(const float* sm, int i, int d) {
  using S = Smem<GATE>;
  const float kv = sm[S::K + i * LDF + d];
  if (GATE == DELTA_SCALAR) return kv * __expf(sm[S::B + i]);
  return kv;  // KDA: K holds kt already; DeltaNet: kt = k
}

// Forward substitution of column c of L X = beta [kt | v] into x[64].
template <int GATE>
__device__ __forceinline__ void solve_column(const float* sm, int c, float (&x)[C]) {
  using S = Smem<GATE>;
  const float* sA = sm + S::A;
  const __nv_bfloat16* sv = reinterpret_cast<const __nv_bfloat16*>(sm + S::V);
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const float rhs = c < D ? kt_of<GATE>(sm, i, c) : __bfloat162float(sv[i * D + (c - D)]);
    float s = sm[S::BETA + i] * rhs;
#pragma unroll
    for (int j = 0; j < i; ++j) s = fmaf(-sA[i * LDA + j], x[j], s);
    x[i] = s;
  }
}

template <int GATE, typename TIn>
__global__ void __launch_bounds__(NT, 1) prep_fwd_kernel(const DeltaPrepArgs a) {
  using S = Smem<GATE>;
  extern __shared__ float sm[];
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z, N = gridDim.x;
  const int tid = threadIdx.x;
  load_chunk<GATE, TIn>(a, sm, n, h, b);
  const int64_t chunk = (static_cast<int64_t>(b) * a.H + h) * N + n;
  const int64_t row0 = chunk * C;
  const float* sb = sm + S::B;
  __nv_bfloat16* aqk = reinterpret_cast<__nv_bfloat16*>(a.aqk) + row0 * C;
  dots<GATE>(sm, [&](int i, int j, float val) { aqk[i * C + j] = __float2bfloat16_rn(val); });
  // w | u0: one column of the solve per thread
  {
    float x[C];
    solve_column<GATE>(sm, tid, x);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(tid < D ? a.w : a.u0) + row0 * D + (tid & (D - 1));
#pragma unroll
    for (int i = 0; i < C; ++i) out[i * D] = __float2bfloat16_rn(x[i]);
  }
  // qt, kc, carry
  __nv_bfloat16* qt = reinterpret_cast<__nv_bfloat16*>(a.qt) + row0 * D;
  __nv_bfloat16* kc = reinterpret_cast<__nv_bfloat16*>(a.kc) + row0 * D;
  for (int e = tid; e < C * D; e += NT) {
    const int i = e / D, d = e % D;
    float qv = sm[S::Q + i * LDF + d], kv;
    if (GATE == DELTA_SCALAR) {
      qv *= __expf(sb[i]);
      kv = sm[S::K + i * LDF + d] * __expf(sb[C - 1] - sb[i]);
    } else if (GATE == DELTA_FEATURE) {
      kv = sm[S::KI + i * LDF + d] * __expf(sb[(C - 1) * LDF + d]);  // k e^{-b} e^{b_last}
    } else {
      kv = sm[S::K + i * LDF + d];
    }
    qt[i * D + d] = __float2bfloat16_rn(qv);
    kc[i * D + d] = __float2bfloat16_rn(kv);
  }
  if (tid < D) {
    float cl = 1.f;
    if (GATE == DELTA_SCALAR) cl = __expf(sb[C - 1]);
    if (GATE == DELTA_FEATURE) cl = __expf(sb[(C - 1) * LDF + tid]);
    a.carry[chunk * D + tid] = cl;
  }
}

template <int GATE, typename TIn>
__global__ void __launch_bounds__(NT, 1) prep_bwd_kernel(const DeltaPrepArgs a) {
  using S = Smem<GATE>;
  extern __shared__ float sm[];
  const int n = blockIdx.x, h = blockIdx.y, b = blockIdx.z, N = gridDim.x;
  const int tid = threadIdx.x, ti = tid >> 4, tj = tid & 15;
  load_chunk<GATE, TIn>(a, sm, n, h, b);
  const int64_t chunk = (static_cast<int64_t>(b) * a.H + h) * N + n;
  const int64_t row0 = chunk * C;
  const float* sb = sm + S::B;
  dots<GATE>(sm, [](int, int, float) {});
  float* sA = sm + S::A;
  float* sX = sm + S::SX;
  float* sY = sm + S::SY;
  const __nv_bfloat16* sv = reinterpret_cast<const __nv_bfloat16*>(sm + S::V);
  const float* dX = (tid < D ? a.dw : a.du0) + row0 * D + (tid & (D - 1));

  // ---- dR = L^{-T} dX (back substitution, one column per thread).  X = [w | u0] is read back
  // from the forward's bf16 outputs in the stages below (the scan consumed the same values).
  float y[C];
#pragma unroll
  for (int i = 0; i < C; ++i) y[i] = __ldg(dX + i * D);  // all 64 loads in flight before the solve
#pragma unroll
  for (int i = C - 1; i >= 0; --i) {
    float s = y[i];
#pragma unroll
    for (int k = C - 1; k > i; --k) s = fmaf(-sA[k * LDA + i], y[k], s);
    y[i] = s;
  }
  __syncthreads();  // every thread is done with A as the solve matrix

  // ---- four stages of 64 columns: dA = -dR X^T accumulated over the stages; the kt / v halves
  // of dR give dk (through kt), dv and the right-hand-side part of dbeta
  float dA[4][4];
  float dK[4][8], dbp[4], dbeta_p[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    dbp[r] = dbeta_p[r] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) dA[r][c] = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) dK[r][c] = 0.f;
  }
  const int64_t tok_base = (static_cast<int64_t>(b) * a.T + n * C) * a.H + h;  // token i: tok_base + i*H
  const __nv_bfloat16* xw = reinterpret_cast<const __nv_bfloat16*>(a.w) + row0 * D;
  const __nv_bfloat16* xu = reinterpret_cast<const __nv_bfloat16*>(a.u0) + row0 * D;
#pragma unroll 1
  for (int st = 0; st < 4; ++st) {
    if (tid >= 64 * st && tid < 64 * st + 64) {
      const int cc = tid - 64 * st;
#pragma unroll
      for (int i = 0; i < C; ++i) sY[i * LDA + cc] = y[i];
    }
    {
      // X columns [c0, c0 + 64) of this stage: two 16-byte loads per thread, both in flight
      const __nv_bfloat16* src = st < 2 ? xw : xu;
      const int c0 = 64 * (st & 1);
      float xv[2][8];
#pragma unroll
      for (int ps = 0; ps < 2; ++ps) {
        const int e = tid + ps * NT, i = e >> 3, cc = (e & 7) * 8;
        load_vec<__nv_bfloat16>(src + i * D + c0 + cc, xv[ps]);
      }
#pragma unroll
      for (int ps = 0; ps < 2; ++ps) {
        const int e = tid + ps * NT, i = e >> 3, cc = (e & 7) * 8;
#pragma unroll
        for (int u = 0; u < 8; ++u) sX[i * LDA + cc + u] = xv[ps][u];
      }
    }
    __syncthreads();
#pragma unroll 4
    for (int cc = 0; cc < 64; ++cc) {
      float yy[4], xx[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) yy[r] = sY[(4 * ti + r) * LDA + cc];
#pragma unroll
      for (int c = 0; c < 4; ++c) xx[c] = sX[(tj + 16 * c) * LDA + cc];
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) dA[r][c] = fmaf(yy[r], xx[c], dA[r][c]);
    }
    // this thread's entries of the stage: rows 4 ti + r, stage columns tj + 16 m
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = 4 * ti + r;
      const float be = sm[S::BETA + i];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int cs = tj + 16 * m;             // column within the stage
        const float yv = sY[i * LDA + cs];
        if (st < 2) {
          const int d = 64 * st + cs;           // kt feature
          const float kt = kt_of<GATE>(sm, i, d);
          const float g = be * yv;              // d loss / d kt
          dbeta_p[r] = fmaf(yv, kt, dbeta_p[r]);
          const int oc = m + 4 * st;            // output column slot: d = tj + 16 oc
          if (GATE == DELTA_SCALAR) {
            dK[r][oc] = fmaf(g, __expf(sb[i]), dK[r][oc]);
            dbp[r] = fmaf(g, kt, dbp[r]);
          } else if (GATE == DELTA_FEATURE) {
            dK[r][oc] += g;                     // d / d kt
          } else {
            dK[r][oc] += g;
          }
        } else {
          const int d = 64 * (st - 2) + cs;     // v feature
          dbeta_p[r] = fmaf(yv, __bfloat162float(sv[i * D + d]), dbeta_p[r]);
          if (n * C + i < a.T) a.dv[(tok_base + static_cast<int64_t>(i) * a.H) * D + d] = be * yv;
        }
      }
    }
    __syncthreads();
  }

  // ---- dA -> d akk (Gk), dbeta; daqk -> Gq; GDN: dP for the decay
  float* sK2 = sm + S::K2;
  float* sQ2 = sm + S::Q2;
  float* sGq = sX;    // stage buffers are free now
  float* sM = sY;
  const float* daqk = a.daqk + row0 * C;
  float dqv[4][4];  // this thread's daqk entries, loaded together
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) dqv[r][c] = __ldg(daqk + (4 * ti + r) * C + tj + 16 * c);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = 4 * ti + r;
    const float be = sm[S::BETA + i];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = tj + 16 * c;
      const float p = pair<GATE>(sb, i, j);
      const float dAij = j < i ? -dA[r][c] : 0.f;
      const float akk_ungated = sK2[i * LDA + j];
      dbeta_p[r] = fmaf(dAij, akk_ungated * p, dbeta_p[r]);
      const float dakk = be * dAij;
      const float dq_ = j <= i ? dqv[r][c] : 0.f;
      sA[i * LDA + j] = dakk * p;       // Gk
      sGq[i * LDA + j] = dq_ * p;       // Gq
      if (GATE == DELTA_SCALAR) sM[i * LDA + j] = (dakk * akk_ungated + dq_ * sQ2[i * LDA + j]) * p;
    }
  }
  __syncthreads();

  // ---- products: rows 4 ti + r, columns d = tj + 16 oc (x and y are dead from here on)
  float dQ[4][8], dKI[4][8], dBt[4][8];  // dBt: KDA db tile
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) dQ[r][c] = dKI[r][c] = dBt[r][c] = 0.f;
  //   GDN / DeltaNet: dK += (Gk + Gk^T) K + Gq^T Q,  dQ += Gq K
  //   KDA: d kt += Gk KI,  d ki += Gk^T Kt + Gq^T Qt,  d qt += Gq KI
  {
    const float* sq = sm + S::Q;
    const float* sk = sm + S::K;
    const float* ski = sm + S::KI;
#pragma unroll 2
    for (int j = 0; j < C; ++j) {
      float gk[4], gkt[4], gq[4], gqt[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = 4 * ti + r;
        gk[r] = sA[i * LDA + j];
        gkt[r] = sA[j * LDA + i];
        gq[r] = sGq[i * LDA + j];
        gqt[r] = sGq[j * LDA + i];
      }
#pragma unroll
      for (int oc = 0; oc < 8; ++oc) {
        const int d = tj + 16 * oc;
        const float kj = sk[j * LDF + d], qj = sq[j * LDF + d];
        if (GATE == DELTA_FEATURE) {
          const float kij = ski[j * LDF + d];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            dK[r][oc] = fmaf(gk[r], kij, dK[r][oc]);
            dKI[r][oc] = fmaf(gkt[r], kj, fmaf(gqt[r], qj, dKI[r][oc]));
            dQ[r][oc] = fmaf(gq[r], kij, dQ[r][oc]);
          }
        } else {
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            dK[r][oc] = fmaf(gk[r] + gkt[r], kj, fmaf(gqt[r], qj, dK[r][oc]));
            dQ[r][oc] = fmaf(gq[r], kj, dQ[r][oc]);
          }
        }
      }
    }
  }

  // ---- direct terms (qt, kc, carry) and the decay gradient db
  const float* dqt = a.dqt + row0 * D;
  const float* dkc = a.dkc + row0 * D;
  const float* dcar = a.dcarry + chunk * D;
  float dlast = 0.f;  // GDN: d b_last from kc and the carry
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = 4 * ti + r;
    float gqv[8], gkv[8];  // the row's incoming gradients, loaded together
#pragma unroll
    for (int oc = 0; oc < 8; ++oc) {
      gqv[oc] = __ldg(dqt + i * D + tj + 16 * oc);
      gkv[oc] = __ldg(dkc + i * D + tj + 16 * oc);
    }
#pragma unroll
    for (int oc = 0; oc < 8; ++oc) {
      const int d = tj + 16 * oc;
      const float gq_in = gqv[oc], gkc = gkv[oc];
      if (GATE == DELTA_SCALAR) {
        const float eb = __expf(sb[i]), el = __expf(sb[C - 1] - sb[i]);
        const float qh = sm[S::Q + i * LDF + d], kh = sm[S::K + i * LDF + d];
        dQ[r][oc] = fmaf(gq_in, eb, dQ[r][oc]);
        dbp[r] = fmaf(gq_in, qh * eb, dbp[r]);
        dK[r][oc] = fmaf(gkc, el, dK[r][oc]);
        const float kcv = kh * el;
        dbp[r] = fmaf(-gkc, kcv, dbp[r]);
        dlast = fmaf(gkc, kcv, dlast);
      } else if (GATE == DELTA_FEATURE) {
        const float bi = sb[i * LDF + d], bl = sb[(C - 1) * LDF + d];
        const float qtv = sm[S::Q + i * LDF + d], ktv = sm[S::K + i * LDF + d], kiv = sm[S::KI + i * LDF + d];
        const float dqt_tot = dQ[r][oc] + gq_in;
        const float kcv = kiv * __expf(bl);
        // dk = d kt e^{b} + d ki e^{-b} + dkc e^{b_last - b};  db = d kt kt - d ki ki + d qt qt - dkc kc
        dBt[r][oc] = dK[r][oc] * ktv - dKI[r][oc] * kiv + dqt_tot * qtv - gkc * kcv;
        dQ[r][oc] = dqt_tot * __expf(bi);
        dK[r][oc] = dK[r][oc] * __expf(bi) + dKI[r][oc] * __expf(-bi) + gkc * __expf(bl - bi);
        dKI[r][oc] = gkc * kcv;  // reused: this entry's contribution to d b_last (summed below)
      } else {
        dQ[r][oc] += gq_in;
        dK[r][oc] += gkc;
      }
    }
  }

  // ---- KDA with the normalisation in this kernel: dQ / dK are gradients of q^ = s q / |q| and
  // k^ = k / |k|.  The raw rows come back with 16-byte loads into the KI and A..SY regions (free once
  // the products and direct terms above are done), then through the normalisation per thread.
  if (GATE == DELTA_FEATURE && a.qk_norm) {
    __syncthreads();  // every thread is done reading KI, A, K2 and the stage buffers
    float* sqr = sm + S::KI;
    float* skr = sm + S::A;  // 64 x LDF floats spill over K2 and SX, both free here
    {
      constexpr int VEC = 16 / static_cast<int>(sizeof(TIn));
      constexpr int LPR = D / VEC, RPP = NT / LPR, PASSES = C / RPP;
      const int d0 = (tid % LPR) * VEC, i0 = tid / LPR;
      const int64_t rs = static_cast<int64_t>(a.H) * D;
      const TIn* qg = reinterpret_cast<const TIn*>(a.q) + (static_cast<int64_t>(b) * a.T * a.H + h) * D;
      const TIn* kg = reinterpret_cast<const TIn*>(a.k) + (static_cast<int64_t>(b) * a.T * a.H + h) * D;
      float qv[PASSES][VEC], kv[PASSES][VEC];
#pragma unroll
      for (int ps = 0; ps < PASSES; ++ps) {
        const int t = n * C + i0 + ps * RPP;
        if (t < a.T) {
          load_vec<TIn>(qg + t * rs + d0, qv[ps]);
          load_vec<TIn>(kg + t * rs + d0, kv[ps]);
        } else {
#pragma unroll
          for (int u = 0; u < VEC; ++u) qv[ps][u] = kv[ps][u] = 0.f;
        }
      }
#pragma unroll
      for (int ps = 0; ps < PASSES; ++ps)
#pragma unroll
        for (int u = 0; u < VEC; ++u) {
          sqr[(i0 + ps * RPP) * LDF + d0 + u] = qv[ps][u];
          skr[(i0 + ps * RPP) * LDF + d0 + u] = kv[ps][u];
        }
    }
    __syncthreads();
    const float s = a.qk_scale;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = 4 * ti + r;
      const float nq = sm[S::NQ + i], nk = sm[S::NK + i];
      float pq = 0.f, pk = 0.f;
#pragma unroll
      for (int oc = 0; oc < 8; ++oc) {
        const int d = tj + 16 * oc;
        pq = fmaf(s * sqr[i * LDF + d] / nq, dQ[r][oc], pq);
        pk = fmaf(skr[i * LDF + d] / nk, dK[r][oc], pk);
      }
      pq = sum16(pq);
      pk = sum16(pk);
      const bool liveq = nq > 1e-12f, livek = nk > 1e-12f;
#pragma unroll
      for (int oc = 0; oc < 8; ++oc) {
        const int d = tj + 16 * oc;
        const float qh = s * sqr[i * LDF + d] / nq, kh = skr[i * LDF + d] / nk;
        dQ[r][oc] = liveq ? (s / nq) * (dQ[r][oc] - qh * pq / (s * s)) : (s / nq) * dQ[r][oc];
        dK[r][oc] = livek ? (dK[r][oc] - kh * pk) / nk : dK[r][oc] / nk;
      }
    }
  }

  // ---- reductions (deterministic): dbeta and the GDN per-token db over the 16 lanes of a row
  float* sDB = sm + S::DB;
  float* sDBETA = sm + S::DBETA;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float tb = sum16(dbeta_p[r]);
    const float td = sum16(dbp[r]);
    if (tj == 0) {
      sDBETA[4 * ti + r] = tb;
      sDB[4 * ti + r] = td;
    }
  }
  __syncthreads();
  if (GATE == DELTA_SCALAR) {
    // dlast: sum over every thread, in a fixed order (warp shuffles, then warps in order)
    float* red = sX;  // Gq is no longer read
    const float wsum = sum32(dlast);
    if ((tid & 31) == 0) red[tid >> 5] = wsum;
    __syncthreads();
    // db_i += (row i of M) - (column i of M), M_ij = dP_ij P_ij (P_ij = e^{b_i - b_j}, j <= i):
    // threads 0..63 sum rows, 64..127 columns, each in a fixed order
    float* rowc = red + 8;  // [2][C]
    if (tid < C) {
      float acc = 0.f;
      for (int j = 0; j <= tid; ++j) acc += sM[tid * LDA + j];
      rowc[tid] = acc;
    } else if (tid < 2 * C) {
      const int j = tid - C;
      float acc = 0.f;
      for (int i = j; i < C; ++i) acc += sM[i * LDA + j];
      rowc[C + j] = acc;
    } else if (tid < 3 * C) {
      // d b_last from the carry e^{b_last}, expanded over the 128 features: two features per thread
      const int d = 2 * (tid - 2 * C);
      rowc[2 * C + (tid - 2 * C)] = (dcar[d] + dcar[d + 1]) * __expf(sb[C - 1]);
    }
    __syncthreads();
    if (tid == 0) {
      float last = 0.f;
      for (int w = 0; w < NT / 32; ++w) last += red[w];
      for (int e = 0; e < C; ++e) last += rowc[2 * C + e];
      float acc = 0.f;  // dg_t = sum_{s >= t} db_s
      for (int i = C - 1; i >= 0; --i) {
        acc += sDB[i] + rowc[i] - rowc[C + i] + (i == C - 1 ? last : 0.f);
        sDB[i] = acc;
      }
    }
    __syncthreads();
  } else if (GATE == DELTA_FEATURE) {
    // per-feature db tile into shared memory (Q / K tiles are no longer read), then the reverse
    // cumulative sum over the chunk per feature; d b_last gets sum_i dkc kc + dcarry e^{b_last}
    __syncthreads();
    float* sDBT = sm + S::Q;
    float* sLast = sm + S::K;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int oc = 0; oc < 8; ++oc) {
        sDBT[(4 * ti + r) * LDF + tj + 16 * oc] = dBt[r][oc];
        sLast[(4 * ti + r) * LDF + tj + 16 * oc] = dKI[r][oc];
      }
    __syncthreads();
    if (a.g_raw) {
      // the gate's pre-activation tile comes in with 16-byte loads (KI is free: the normalisation
      // above has read its rows before the reductions' barrier)
      float* sraw = sm + S::KI;
      constexpr int LPR = D / 8, RPP = NT / LPR, PASSES = C / RPP;
      const int d0 = (tid % LPR) * 8, i0 = tid / LPR;
      float rv[PASSES][8];
#pragma unroll
      for (int ps = 0; ps < PASSES; ++ps) {
        const int t = n * C + i0 + ps * RPP;
        if (t < a.T) {
          load_vec<__nv_bfloat16>(a.g_raw + ((static_cast<int64_t>(b) * a.T + t) * a.H + h) * D + d0, rv[ps]);
        } else {
#pragma unroll
          for (int u = 0; u < 8; ++u) rv[ps][u] = 0.f;
        }
      }
#pragma unroll
      for (int ps = 0; ps < PASSES; ++ps)
#pragma unroll
        for (int u = 0; u < 8; ++u) sraw[(i0 + ps * RPP) * LDF + d0 + u] = rv[ps][u];
    }
    __syncthreads();
    if (tid < D) {
      // reverse cumulative sum per feature: dg_t = sum_{s >= t} db_s (+ d b_last at the last token)
      const int d = tid;
      float last = 0.f;
      for (int i = 0; i < C; ++i) last += sLast[i * LDF + d];
      last = fmaf(dcar[d], __expf(sb[(C - 1) * LDF + d]), last);
      float acc = 0.f;
      for (int i = C - 1; i >= 0; --i) {
        acc += sDBT[i * LDF + d] + (i == C - 1 ? last : 0.f);
        if (a.g_raw) sDBT[i * LDF + d] = acc;
        else if (n * C + i < a.T) a.dg[(tok_base + static_cast<int64_t>(i) * a.H) * D + d] = acc;
      }
    }
    if (a.g_raw) {
      // g = -e^{A} softplus(z), z = g_raw + bias:  dz = -dg e^{A} sigmoid(z),  d A = dg g.  Every
      // thread takes one feature (tid mod 128) and every other token; the two partial sums of a
      // feature are added in a fixed order.
      __syncthreads();
      const int d = tid & (D - 1), half = tid >> 7;
      const float ea = expf(a.g_log[h * D + d]), bias = a.g_bias[h * D + d];
      const float* sraw = sm + S::KI;
      float pa = 0.f, pb = 0.f;
      for (int i = half; i < C; i += 2) {
        if (n * C + i >= a.T) break;
        const float z = sraw[i * LDF + d] + bias, dg = sDBT[i * LDF + d];
        const float ez = expf(z);
        const float sp = z > 20.f ? z : log1pf(ez);
        const float sg = z > 20.f ? 1.f : ez / (1.f + ez);
        const float dz = -dg * ea * sg;
        a.dg_raw[(tok_base + static_cast<int64_t>(i) * a.H) * D + d] = __float2bfloat16_rn(dz);
        pb += dz;
        pa = fmaf(dg, -ea * sp, pa);
      }
      float* red = sm + S::K;  // sLast is read
      __syncthreads();
      red[tid] = pa;
      red[NT + tid] = pb;
      __syncthreads();
      if (tid < D) {
        const int64_t part = ((static_cast<int64_t>(b) * N + n) * a.H + h) * D + tid;
        a.dg_log_part[part] = red[tid] + red[tid + D];
        a.dg_bias_part[part] = red[NT + tid] + red[NT + tid + D];
      }
    }
  }

  // ---- GDN: back through the L2 normalisation; write dq, dk, dg, dbeta
  if (GATE == DELTA_SCALAR) {
    const float s = a.qk_scale;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = 4 * ti + r;
      float pq = 0.f, pk = 0.f;
#pragma unroll
      for (int oc = 0; oc < 8; ++oc) {
        const int d = tj + 16 * oc;
        pq = fmaf(sm[S::Q + i * LDF + d], dQ[r][oc], pq);
        pk = fmaf(sm[S::K + i * LDF + d], dK[r][oc], pk);
      }
      pq = sum16(pq);
      pk = sum16(pk);
      const float nq = sm[S::NQ + i], nk = sm[S::NK + i];
      const bool liveq = nq > 1e-12f, livek = nk > 1e-12f;
#pragma unroll
      for (int oc = 0; oc < 8; ++oc) {
        const int d = tj + 16 * oc;
        // q^ = s q / |q|:  dq = (s / |q|) (dq^ - q^ (q^ . dq^) / s^2)
        const float qh = sm[S::Q + i * LDF + d], kh = sm[S::K + i * LDF + d];
        dQ[r][oc] = liveq ? (s / nq) * (dQ[r][oc] - qh * pq / (s * s)) : (s / nq) * dQ[r][oc];
        dK[r][oc] = livek ? (dK[r][oc] - kh * pk) / nk : dK[r][oc] / nk;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = 4 * ti + r;
    if (n * C + i >= a.T) continue;
    const int64_t o = (tok_base + static_cast<int64_t>(i) * a.H) * D;
#pragma unroll
    for (int oc = 0; oc < 8; ++oc) {
      const int d = tj + 16 * oc;
      a.dq[o + d] = dQ[r][oc];
      a.dk[o + d] = dK[r][oc];
    }
  }
  if (tid < C && n * C + tid < a.T) {
    const int64_t t = tok_base + static_cast<int64_t>(tid) * a.H;
    a.dbeta[t] = sDBETA[tid];
    if (GATE == DELTA_SCALAR) a.dg[t] = sDB[tid];
  }
}

template <int GATE, typename TIn>
int launch(const DeltaPrepArgs& a, cudaStream_t s, bool bwd) {
  using S = Smem<GATE>;
  const int N = (a.T + C - 1) / C;
  dim3 grid(N, a.H, a.B);
  if (bwd) {
    static std::atomic<uint64_t> set{0};
    smem_limit(set, prep_bwd_kernel<GATE, TIn>, S::BYTES);
    prep_bwd_kernel<GATE, TIn><<<grid, NT, S::BYTES, s>>>(a);
  } else {
    static std::atomic<uint64_t> set{0};
    smem_limit(set, prep_fwd_kernel<GATE, TIn>, S::BYTES);
    prep_fwd_kernel<GATE, TIn><<<grid, NT, S::BYTES, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

template <typename TIn>
int dispatch(const DeltaPrepArgs& a, cudaStream_t s, bool bwd) {
  switch (a.gate) {
    case DELTA_NONE: return launch<DELTA_NONE, TIn>(a, s, bwd);
    case DELTA_SCALAR: return launch<DELTA_SCALAR, TIn>(a, s, bwd);
    case DELTA_FEATURE: return launch<DELTA_FEATURE, TIn>(a, s, bwd);
    default: return -1;
  }
}

static_assert(Smem<DELTA_FEATURE>::BYTES <= 232448, "KDA chunk terms exceed the shared-memory limit");
static_assert(Smem<DELTA_SCALAR>::BYTES <= 232448, "GDN chunk terms exceed the shared-memory limit");

}  // namespace dprep
}  // namespace nt

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The chunk loads are 16-byte vectors: q / k / v, the per-feature gate and the forward's w / u0
// must start on 16-byte boundaries (rows are 128 features, so every row then does too).
static bool prep_args_ok(const DeltaPrepArgs& a) {
  const bool raw = a.gate == DELTA_FEATURE && a.g_raw;
  if (a.g_raw && (a.gate != DELTA_FEATURE || !a.g_log || !a.g_bias || !aligned16(a.g_raw))) return false;
  if (a.qk_norm && a.gate != DELTA_FEATURE) return false;
  return a.B > 0 && a.T > 0 && a.H > 0 && a.q && a.k && a.v && a.beta && (a.gate == DELTA_NONE || a.g || raw) &&
         aligned16(a.q) && aligned16(a.k) && aligned16(a.v) && (a.gate != DELTA_FEATURE || raw || aligned16(a.g)) &&
         (!a.w || aligned16(a.w)) && (!a.u0 || aligned16(a.u0));
}

int nt_delta_prep_fwd(const DeltaPrepArgs& a, cudaStream_t s) {
  nt::current_context();
  if (!prep_args_ok(a) || !a.w || !a.u0 || !a.qt || !a.kc || !a.aqk || !a.carry) return -1;
  return a.in_bf16 ? nt::dprep::dispatch<__nv_bfloat16>(a, s, false) : nt::dprep::dispatch<float>(a, s, false);
}

int nt_delta_prep_bwd(const DeltaPrepArgs& a, cudaStream_t s) {
  nt::current_context();
  if (!prep_args_ok(a) || !a.w || !a.u0 || !a.dw || !a.du0 || !a.dqt || !a.dkc || !a.daqk || !a.dcarry || !a.dq ||
      !a.dk || !a.dv ||
      !a.dbeta)
    return -1;
  if (a.g_raw ? (!a.dg_raw || !a.dg_log_part || !a.dg_bias_part) : (a.gate != DELTA_NONE && !a.dg)) return -1;
  return a.in_bf16 ? nt::dprep::dispatch<__nv_bfloat16>(a, s, true) : nt::dprep::dispatch<float>(a, s, true);
}
