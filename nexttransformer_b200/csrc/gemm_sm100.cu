// K0: persistent warp-specialized bf16 GEMM engine for sm_100a.
//
//   D[b, m, n] = epilogue( sum_k A[b, m, k] * B[b, n, k] )
//
// A is stored K-major ([M, K], K contiguous) or M-major ([K, M], M contiguous); B is stored
// K-major ([N, K]) or N-major ([K, N]).  Those four storage orders cover a Linear layer's
// forward (A K-major, B K-major), input gradient (B N-major) and weight gradient (both
// MN-major), and the Newton-Schulz chain of the Muon optimizer.
//
// Structure (one CTA per SM, 192 threads):
//   warp 0      TMA producer: 128x64 A tiles and BNx64 B tiles, 128-byte swizzle, into a
//               STAGES-deep shared-memory ring guarded by full/empty mbarriers.
//   warp 1      allocates TMEM (2 x BN fp32 columns = double-buffered accumulator) and issues
//               tcgen05.mma (M=128, N=BN, K=16) from one thread; tcgen05.commit frees ring
//               slots and publishes finished accumulators.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (one accumulator row per thread),
//               apply the fused epilogue, store to global memory.  While they drain one
//               accumulator, warp 1 fills the other.
// Tiles are visited in a grouped raster (GROUP_M row-blocks at a time) so that A and B tiles
// are re-read from L2.  No TMA load here uses cluster multicast.
#include "common.cuh"
#include "gemm_sm100.h"

#include <cudaTypedefs.h>
#include <mutex>
#include <cstdlib>
#include <stdexcept>
#include <string>

namespace nt {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int GROUP_M = 16;
constexpr int NUM_THREADS = 192;

// Bulk-store epilogue: each epilogue warp stages [32 rows x 32 columns] bf16 boxes (2 KB, 64-byte
// swizzle) in two alternating buffers; a second output (the ReLU^2 pre-activation) doubles them.
constexpr int STG_BOX = 2048;
constexpr int STG_WARP = 2 * 2 * STG_BOX;      // 2 buffers x (C box + P box)
constexpr int STG_BYTES = 4 * STG_WARP;        // 4 epilogue warps = 32 KB

template <int BN, int STAGES>
struct Smem {
  static constexpr int A_BYTES = BM * BK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STG_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFFSET = STG_OFFSET + STG_BYTES;
  // full[S], empty[S], tmem_full[2], tmem_empty[2], tmem holder, abort flag
  static constexpr int BAR_BYTES = (2 * STAGES + 4) * 8 + 16;
  static constexpr int TOTAL = BAR_OFFSET + BAR_BYTES + 1024;  // + alignment slack
  static_assert(TOTAL <= 232448, "GEMM shared memory exceeds the sm_100 limit");
};

struct Params {
  int M, N, K, batch;
  int tiles_m, tiles_n;
  int epi;
  void* C;
  int64_t ldc, strideC;  // elements
  const void* R;         // residual / pre-activation input (bf16)
  int64_t ldr, strideR;
  void* P;               // second output (bf16 pre-activation)
  int64_t ldp, strideP;
  float s_acc, s_res;
  const float* s_ptr;
  int split;           // K slices (1 = no split-K)
  int kb_per_split;    // k-blocks per slice
  int64_t strideSplit; // elements between the partial-output slices of the workspace
  CeArgs ce;           // cross-entropy epilogues only
  int tma_out;         // 1: bf16 outputs leave through shared memory and bulk tensor stores
  // Grouped (expert) modes.  grp_m: per 128-row tile of A/C, the batch index of B (-1: no work);
  // A and C unbatched.  grp_k: per batch of C, the row range [grp_k[b], grp_k[b+1]) of the
  // reduction dimension (multiples of 64); A and B unbatched.
  const int* grp_m;
  const int* grp_k;
};

// Epilogue threads release an accumulator buffer on the MMA issuer's barrier (the leader's for a pair).
template <bool PAIR>
NT_DEVICE void arrive_tempty(uint64_t* bar, uint32_t crank) {
  if (PAIR && crank != 0) mbar_arrive_cluster(bar, 0);
  else mbar_arrive(bar);
}

struct TileWork {
  int zA, zB, zC, kb_lo, kb_hi;
};
// Batch coordinates of the three operands and the k-block range of one tile; false = no work.
NT_DEVICE bool tile_work(const Params& p, int b, int mb, int ks, int num_kb, TileWork& w) {
  w.zA = w.zB = w.zC = b;
  w.kb_lo = ks * p.kb_per_split;
  w.kb_hi = min(num_kb, w.kb_lo + p.kb_per_split);
  if (p.grp_m) {
    w.zA = w.zC = 0;
    w.zB = p.grp_m[mb];
    return w.zB >= 0;
  }
  if (p.grp_k) {
    w.zA = w.zB = 0;
    w.kb_lo = p.grp_k[b] / BK;
    w.kb_hi = p.grp_k[b + 1] / BK;
    return w.kb_hi > w.kb_lo;
  }
  return true;
}

NT_DEVICE void tile_coords(int t, const Params& p, int& b, int& mb, int& nb, int& ks) {
  const int per_slice = p.tiles_m * p.tiles_n;
  const int per_batch = per_slice * p.split;
  b = t / per_batch;
  int r = t - b * per_batch;
  ks = r / per_slice;
  r -= ks * per_slice;
  const int group_span = GROUP_M * p.tiles_n;
  const int g = r / group_span;
  const int first_m = g * GROUP_M;
  const int rows_in_group = min(GROUP_M, p.tiles_m - first_m);
  const int in_g = r - g * group_span;
  mb = first_m + in_g % rows_in_group;
  nb = in_g / rows_in_group;
}

// Soft-capped cross-entropy, forward: G = e (1 - t^2) over 32 columns of one row; returns the
// sum of e over those columns and records z at the target column.
// Soft-capped cross-entropy terms of one logit x (cap c): with E = e^{2x/c} and r = 1 / (1 + E),
//   t = tanh(x / c) = 1 - 2r,  z = c t,  e = exp(z - c) = exp(-2 c r),  1 - t^2 = 4 r (1 - r).
// Two base-2 exponentials and one reciprocal on the SFU and a few FMA-pipe operations, against a
// full-precision tanh per logit before: the LM-head GEMM's epilogue was three times its MMA time.
// Every step stays finite as |x| grows: E -> inf gives r = 0, e = 1, 1 - t^2 = 0; E -> 0 gives
// r = 1, z = -c, 1 - t^2 = 0.  The absolute error of z is about c * 2^-21.
struct CeConst {
  float k_in, k_out, cap;  // 2 log2(e) / c, -2 c log2(e), c
};
NT_DEVICE CeConst ce_const(float cap) {
  constexpr float kLog2e = 1.4426950408889634f;
  return CeConst{2.f * kLog2e / cap, -2.f * cap * kLog2e, cap};
}
NT_DEVICE void ce_terms(float x, const CeConst& k, float& e, float& g, float& z) {
  float big, r, ex;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(big) : "f"(x * k.k_in));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + big));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(ex) : "f"(r * k.k_out));
  e = ex;
  g = ex * 4.f * fmaf(-r, r, r);
  z = k.cap * fmaf(-2.f, r, 1.f);
}

NT_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
NT_DEVICE float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A row chunk of 32 live logits without branches, in packed fp32 pairs: out = bf16 e (1 - t^2),
// returns the chunk's sum of e.
NT_DEVICE float ce_chunk32(const uint32_t (&acc)[32], const CeConst& k, uint32_t (&out)[16]) {
  const float2 kin = make_float2(k.k_in, k.k_in), kout = make_float2(k.k_out, k.k_out);
  const float2 one = make_float2(1.f, 1.f), four = make_float2(4.f, 4.f);
  float2 se = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 y = mul2(make_float2(__uint_as_float(acc[2 * i]), __uint_as_float(acc[2 * i + 1])), kin);
    const float2 big = add2(make_float2(ex2_approx(y.x), ex2_approx(y.y)), one);
    const float2 r = make_float2(rcp_approx(big.x), rcp_approx(big.y));
    const float2 w = mul2(r, kout);
    const float2 ex = make_float2(ex2_approx(w.x), ex2_approx(w.y));
    se = add2(se, ex);
    const float2 q = fma2(make_float2(-r.x, -r.y), r, r);  // r (1 - r)
    const float2 g = mul2(mul2(ex, four), q);
    out[i] = pack_bf16x2(g.x, g.y);
  }
  return se.x + se.y;
}

// z of the target column when it falls in this chunk (one thread in 2048 chunks per row)
NT_DEVICE void ce_target(const CeArgs& ce, const CeConst& k, int64_t tgt, int row, int col0, int lim,
                         const uint32_t (&acc)[32]) {
  if (tgt < col0 || tgt >= col0 + lim) return;
  const int j = static_cast<int>(tgt - col0);
  float x = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) x = i == j ? __uint_as_float(acc[i]) : x;
  float e, g, z;
  ce_terms(x, k, e, g, z);
  ce.ztgt[row] = z;
}

NT_DEVICE float ce_fwd32(const Params& p, int row, int col0, const uint32_t (&acc)[32]) {
  const CeArgs& ce = p.ce;
  const CeConst k = ce_const(ce.cap);
  const int64_t tgt = ce.tgt[row];
  const int ncols = min(32, p.N - col0);
  float se = 0.f;
  uint32_t out[16];
  const int lim = min(ncols, ce.vocab - col0);
  if (lim >= 32) {
    se = ce_chunk32(acc, k, out);
    ce_target(ce, k, tgt, row, col0, lim, acc);
  } else {
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float g[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int col = col0 + i + e;
      g[e] = 0.f;
      if (col < ce.vocab) {
        float ex, gv, z;
        ce_terms(__uint_as_float(acc[i + e]), k, ex, gv, z);
        se += ex;
        g[e] = gv;
        if (col == tgt) ce.ztgt[row] = z;
      }
    }
    out[i / 2] = pack_bf16x2(g[0], g[1]);
  }
  }
  __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(row) * p.ldc + col0;
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(c) & 15) == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<uint4*>(c + 8 * i) = make_uint4(out[4 * i], out[4 * i + 1], out[4 * i + 2], out[4 * i + 3]);
  } else {
    for (int i = 0; i < ncols; ++i) {
      const uint32_t w = out[i / 2];
      c[i] = __ushort_as_bfloat16(static_cast<unsigned short>((i & 1) ? (w >> 16) : (w & 0xFFFFu)));
    }
  }
  return se;
}

// Soft-capped cross-entropy, input gradient: s (rscale acc - rcorr W[target, col]) over 32 columns.
NT_DEVICE void ce_dgrad32(const Params& p, float sacc, int row, int col0, const uint32_t (&acc)[32]) {
  const CeArgs& ce = p.ce;
  const int ncols = min(32, p.N - col0);
  const int64_t tgt = ce.tgt[row];
  const float rs = ce.rscale[row] * sacc;
  const float rc = tgt >= 0 ? ce.rcorr[row] * sacc : 0.f;
  const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(ce.w) + (tgt >= 0 ? tgt : 0) * ce.ldw + col0;
  float wv[32];
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 q = *reinterpret_cast<const uint4*>(w + 8 * i);
      float2 f0 = unpack_bf16x2(q.x), f1 = unpack_bf16x2(q.y), f2 = unpack_bf16x2(q.z), f3 = unpack_bf16x2(q.w);
      wv[8 * i + 0] = f0.x; wv[8 * i + 1] = f0.y; wv[8 * i + 2] = f1.x; wv[8 * i + 3] = f1.y;
      wv[8 * i + 4] = f2.x; wv[8 * i + 5] = f2.y; wv[8 * i + 6] = f3.x; wv[8 * i + 7] = f3.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) wv[i] = (i < ncols) ? bf2f(w[i]) : 0.f;
  }
  uint32_t out[16];
#pragma unroll
  for (int i = 0; i < 32; i += 2)
    out[i / 2] = pack_bf16x2(rs * __uint_as_float(acc[i]) - rc * wv[i], rs * __uint_as_float(acc[i + 1]) - rc * wv[i + 1]);
  __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + static_cast<int64_t>(row) * p.ldc + col0;
  if (ncols == 32 && (reinterpret_cast<uintptr_t>(c) & 15) == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
      *reinterpret_cast<uint4*>(c + 8 * i) = make_uint4(out[4 * i], out[4 * i + 1], out[4 * i + 2], out[4 * i + 3]);
  } else {
    for (int i = 0; i < ncols; ++i) {
      const uint32_t v = out[i / 2];
      c[i] = __ushort_as_bfloat16(static_cast<unsigned short>((i & 1) ? (v >> 16) : (v & 0xFFFFu)));
    }
  }
}

// bf16 epilogues: the 32 packed output values (and the ReLU^2 pre-activation) of one row chunk.
// Rows past M and columns past N read no operand; the bulk store clips them.
template <int EPI>
NT_DEVICE void epi_pack(const Params& p, float sacc, int b, int row, int col0, const uint32_t (&acc)[32],
                        uint32_t (&out)[16], uint32_t (&pre)[16], float& se) {
  const bool live = row < p.M;
  const int ncols = live ? max(0, min(32, p.N - col0)) : 0;
  if constexpr (EPI == EPI_CE_FWD) {
    const CeArgs& ce = p.ce;
    const CeConst k = ce_const(ce.cap);
    const int64_t tgt = live ? ce.tgt[row] : -1;
    const int lim = min(ncols, ce.vocab - col0);
    if (lim >= 32) {
      se += ce_chunk32(acc, k, out);
      ce_target(ce, k, tgt, row, col0, lim, acc);
      return;
    }
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float g[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = col0 + i + e;
        g[e] = 0.f;
        if (i + e < ncols && col < ce.vocab) {
          float ex, gv, z;
          ce_terms(__uint_as_float(acc[i + e]), k, ex, gv, z);
          se += ex;
          g[e] = gv;
          if (col == tgt) ce.ztgt[row] = z;
        }
      }
      out[i / 2] = pack_bf16x2(g[0], g[1]);
    }
    return;
  } else if constexpr (EPI == EPI_CE_DGRAD) {
    const CeArgs& ce = p.ce;
    const int64_t tgt = live ? ce.tgt[row] : -1;
    const float rs = live ? ce.rscale[row] * sacc : 0.f;
    const float rc = tgt >= 0 ? ce.rcorr[row] * sacc : 0.f;
    const __nv_bfloat16* w = reinterpret_cast<const __nv_bfloat16*>(ce.w) + (tgt >= 0 ? tgt : 0) * ce.ldw + col0;
    const bool vec = ncols == 32 && (reinterpret_cast<uintptr_t>(w) & 15) == 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float wv[8];
      if (vec) {
        const uint4 u = *reinterpret_cast<const uint4*>(w + 8 * q);
        const float2 f0 = unpack_bf16x2(u.x), f1 = unpack_bf16x2(u.y), f2 = unpack_bf16x2(u.z), f3 = unpack_bf16x2(u.w);
        wv[0] = f0.x; wv[1] = f0.y; wv[2] = f1.x; wv[3] = f1.y; wv[4] = f2.x; wv[5] = f2.y; wv[6] = f3.x; wv[7] = f3.y;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) wv[e] = (8 * q + e < ncols) ? bf2f(w[8 * q + e]) : 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; e += 2)
        out[4 * q + e / 2] = pack_bf16x2(rs * __uint_as_float(acc[8 * q + e]) - rc * wv[e],
                                         rs * __uint_as_float(acc[8 * q + e + 1]) - rc * wv[e + 1]);
    }
    return;
  } else {
    float rv[32];
    if constexpr (EPI == EPI_BF16_AXPBY || EPI == EPI_RELU2_BWD) {
      const __nv_bfloat16* r =
          reinterpret_cast<const __nv_bfloat16*>(p.R) + b * p.strideR + static_cast<int64_t>(live ? row : 0) * p.ldr + col0;
      if (ncols == 32 && ((reinterpret_cast<uintptr_t>(r) & 15) == 0)) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 q = *reinterpret_cast<const uint4*>(r + 8 * i);
          float2 f0 = unpack_bf16x2(q.x), f1 = unpack_bf16x2(q.y), f2 = unpack_bf16x2(q.z), f3 = unpack_bf16x2(q.w);
          rv[8 * i + 0] = f0.x; rv[8 * i + 1] = f0.y; rv[8 * i + 2] = f1.x; rv[8 * i + 3] = f1.y;
          rv[8 * i + 4] = f2.x; rv[8 * i + 5] = f2.y; rv[8 * i + 6] = f3.x; rv[8 * i + 7] = f3.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) rv[i] = (i < ncols) ? bf2f(r[i]) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const float v0 = __uint_as_float(acc[i]), v1 = __uint_as_float(acc[i + 1]);
      float o0, o1;
      if constexpr (EPI == EPI_BF16) {
        o0 = v0 * sacc;
        o1 = v1 * sacc;
      } else if constexpr (EPI == EPI_BF16_AXPBY) {
        o0 = bf2f(f2bf(v0 * sacc)) + p.s_res * rv[i];
        o1 = bf2f(f2bf(v1 * sacc)) + p.s_res * rv[i + 1];
      } else if constexpr (EPI == EPI_RELU2) {
        const float h0 = bf2f(f2bf(v0)), h1 = bf2f(f2bf(v1));
        pre[i / 2] = pack_bf16x2(h0, h1);
        const float r0 = fmaxf(h0, 0.f), r1 = fmaxf(h1, 0.f);
        o0 = r0 * r0;
        o1 = r1 * r1;
      } else {  // EPI_RELU2_BWD
        const float g0 = bf2f(f2bf(v0)), g1 = bf2f(f2bf(v1));
        o0 = g0 * 2.f * fmaxf(rv[i], 0.f);
        o1 = g1 * 2.f * fmaxf(rv[i + 1], 0.f);
      }
      out[i / 2] = pack_bf16x2(o0, o1);
    }
  }
}

template <int EPI>
__host__ __device__ constexpr bool bf16_out() {
  return EPI == EPI_BF16 || EPI == EPI_BF16_AXPBY || EPI == EPI_RELU2 || EPI == EPI_RELU2_BWD || EPI == EPI_CE_FWD ||
         EPI == EPI_CE_DGRAD;
}

// Epilogue for 32 consecutive columns of one row.
template <int EPI>
NT_DEVICE void epilogue32(const Params& p, float sacc, int b, int ks, int row, int col0, const uint32_t (&acc)[32]) {
  if (row >= p.M) return;
  const int ncols = min(32, p.N - col0);
  if (ncols <= 0) return;
  if constexpr (EPI == EPI_CE_DGRAD) {
    ce_dgrad32(p, sacc, row, col0, acc);
    return;
  }
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(acc[i]);
  const bool full = (ncols == 32);

  if constexpr (EPI == EPI_F32 || EPI == EPI_F32_ACC) {
    float* c = reinterpret_cast<float*>(p.C) + b * p.strideC + ks * p.strideSplit +
               static_cast<int64_t>(row) * p.ldc + col0;
    const bool acc_into = (EPI == EPI_F32_ACC) && p.split == 1;
    if (full && ((reinterpret_cast<uintptr_t>(c) & 15) == 0)) {
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        float4 o = make_float4(v[i] * sacc, v[i + 1] * sacc, v[i + 2] * sacc, v[i + 3] * sacc);
        if (acc_into) {
          float4 old = *reinterpret_cast<float4*>(c + i);
          o.x += old.x; o.y += old.y; o.z += old.z; o.w += old.w;
        }
        *reinterpret_cast<float4*>(c + i) = o;
      }
    } else {
      for (int i = 0; i < ncols; ++i) {
        float o = v[i] * sacc;
        if (acc_into) o += c[i];
        c[i] = o;
      }
    }
    return;
  } else {
    __nv_bfloat16* c =
        reinterpret_cast<__nv_bfloat16*>(p.C) + b * p.strideC + static_cast<int64_t>(row) * p.ldc + col0;
    const __nv_bfloat16* r = nullptr;
    if constexpr (EPI == EPI_BF16_AXPBY || EPI == EPI_RELU2_BWD) {
      r = reinterpret_cast<const __nv_bfloat16*>(p.R) + b * p.strideR + static_cast<int64_t>(row) * p.ldr + col0;
    }
    __nv_bfloat16* pp = nullptr;
    if constexpr (EPI == EPI_RELU2) {
      pp = reinterpret_cast<__nv_bfloat16*>(p.P) + b * p.strideP + static_cast<int64_t>(row) * p.ldp + col0;
    }
    uint32_t out[16];
    uint32_t pre[16];
    float rv[32];
    if constexpr (EPI == EPI_BF16_AXPBY || EPI == EPI_RELU2_BWD) {
      if (full && ((reinterpret_cast<uintptr_t>(r) & 15) == 0)) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          uint4 q = *reinterpret_cast<const uint4*>(r + 8 * i);
          float2 f0 = unpack_bf16x2(q.x), f1 = unpack_bf16x2(q.y), f2 = unpack_bf16x2(q.z), f3 = unpack_bf16x2(q.w);
          rv[8 * i + 0] = f0.x; rv[8 * i + 1] = f0.y; rv[8 * i + 2] = f1.x; rv[8 * i + 3] = f1.y;
          rv[8 * i + 4] = f2.x; rv[8 * i + 5] = f2.y; rv[8 * i + 6] = f3.x; rv[8 * i + 7] = f3.y;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) rv[i] = (i < ncols) ? bf2f(r[i]) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float o0, o1;
      if constexpr (EPI == EPI_BF16) {
        o0 = v[i] * sacc;
        o1 = v[i + 1] * sacc;
      } else if constexpr (EPI == EPI_BF16_AXPBY) {
        // Round the product first, as a bf16 matmul followed by a bf16 add would.
        o0 = bf2f(f2bf(v[i] * sacc)) + p.s_res * rv[i];
        o1 = bf2f(f2bf(v[i + 1] * sacc)) + p.s_res * rv[i + 1];
      } else if constexpr (EPI == EPI_RELU2) {
        const float h0 = bf2f(f2bf(v[i])), h1 = bf2f(f2bf(v[i + 1]));
        pre[i / 2] = pack_bf16x2(h0, h1);
        const float r0 = fmaxf(h0, 0.f), r1 = fmaxf(h1, 0.f);
        o0 = r0 * r0;
        o1 = r1 * r1;
      } else {  // EPI_RELU2_BWD: d(relu(h)^2)/dh = 2 relu(h)
        const float g0 = bf2f(f2bf(v[i])), g1 = bf2f(f2bf(v[i + 1]));
        o0 = g0 * 2.f * fmaxf(rv[i], 0.f);
        o1 = g1 * 2.f * fmaxf(rv[i + 1], 0.f);
      }
      out[i / 2] = pack_bf16x2(o0, o1);
    }
    if (full && ((reinterpret_cast<uintptr_t>(c) & 15) == 0)) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(c + 8 * i) = make_uint4(out[4 * i], out[4 * i + 1], out[4 * i + 2], out[4 * i + 3]);
      if constexpr (EPI == EPI_RELU2) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          *reinterpret_cast<uint4*>(pp + 8 * i) = make_uint4(pre[4 * i], pre[4 * i + 1], pre[4 * i + 2], pre[4 * i + 3]);
      }
    } else {
      for (int i = 0; i < ncols; ++i) {
        const uint32_t w = out[i / 2];
        c[i] = __ushort_as_bfloat16(static_cast<unsigned short>((i & 1) ? (w >> 16) : (w & 0xFFFFu)));
        if constexpr (EPI == EPI_RELU2) {
          const uint32_t q = pre[i / 2];
          pp[i] = __ushort_as_bfloat16(static_cast<unsigned short>((i & 1) ? (q >> 16) : (q & 0xFFFFu)));
        }
      }
    }
  }
}

// PAIR: a cluster of two CTAs computes 256 x BN tiles with cta_group::2 MMAs issued by the leader
// (rank 0): each CTA stages its 128 rows of A and its BN / 2 rows of B, so each SM reads half of
// the B operand per MMA; each CTA's tensor memory receives its own 128 rows of the accumulator.
template <int BN, int A_MN, int B_MN, int EPI, int STAGES, bool PAIR = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmP, Params p) {
  using S = Smem<PAIR ? BN / 2 : BN, STAGES>;
  constexpr int BNC = PAIR ? BN / 2 : BN;  // B rows staged by this CTA
  constexpr int TM = PAIR ? 2 * BM : BM;    // rows per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFFSET);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_kb = (p.K + BK - 1) / BK;
  const int total_tiles = p.batch * p.split * p.tiles_m * p.tiles_n;
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const int tile0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int tstride = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  const bool leader = crank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 256 : 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_holder, 2 * BN);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, 2 * BN);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = tile0; t < total_tiles && ok; t += tstride) {
        int b, mb, nb, ks;
        tile_coords(t, p, b, mb, nb, ks);
        TileWork tw;
        if (!tile_work(p, b, mb, ks, num_kb, tw)) continue;
        const int m0 = mb * TM + static_cast<int>(crank) * BM, n0 = nb * BN + static_cast<int>(crank) * BNC;
        const int kb_lo = tw.kb_lo, kb_hi = tw.kb_hi;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, 0x100u + stage, abort_flag)) { ok = false; break; }
          uint8_t* sA = smem + stage * S::STAGE_BYTES;
          uint8_t* sB = sA + S::A_BYTES;
          const int k0 = kb * BK;
          if constexpr (PAIR) {
            // both CTAs' copies count on the leader's barrier; only the leader arms it
            if (leader) mbar_expect_tx(&full[stage], 2 * S::STAGE_BYTES);
            const uint32_t fb = leader_bar(&full[stage]);
            if constexpr (A_MN == 0) {
              tma_load_3d_pair(sA, &tmA, fb, k0, m0, tw.zA);
            } else {
              tma_load_3d_pair(sA, &tmA, fb, m0, k0, tw.zA);
              tma_load_3d_pair(sA + 8192, &tmA, fb, m0 + 64, k0, tw.zA);
            }
            if constexpr (B_MN == 0) {
              tma_load_3d_pair(sB, &tmB, fb, k0, n0, tw.zB);
            } else {
#pragma unroll
              for (int j = 0; j < BNC / 64; ++j) tma_load_3d_pair(sB + j * 8192, &tmB, fb, n0 + 64 * j, k0, tw.zB);
            }
          } else {
            mbar_expect_tx(&full[stage], S::STAGE_BYTES);
            if constexpr (A_MN == 0) {
              tma_load_3d(sA, &tmA, &full[stage], k0, m0, tw.zA);
            } else {
              tma_load_3d(sA, &tmA, &full[stage], m0, k0, tw.zA);
              tma_load_3d(sA + 8192, &tmA, &full[stage], m0 + 64, k0, tw.zA);
            }
            if constexpr (B_MN == 0) {
              tma_load_3d(sB, &tmB, &full[stage], k0, n0, tw.zB);
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_3d(sB + j * 8192, &tmB, &full[stage], n0 + 64 * j, k0, tw.zB);
            }
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      // Drain: wait (bounded) until the copies of the last issued stages have landed (a pair's
      // copies all count on the leader's barriers).
      const int outstanding = (!PAIR || leader) ? (issued < STAGES ? issued : STAGES) : 0;
      int s = stage;
      uint32_t ph = phase;
      for (int i = 0; i < outstanding; ++i) {
        if (--s < 0) { s = STAGES - 1; ph ^= 1u; }
        mbar_wait(&full[s], ph, 0x180u + s, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_bf16_f32(TM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = tile0; t < total_tiles && ok; t += tstride, ++local) {
        int tb, tmb, tnb, tks;
        tile_coords(t, p, tb, tmb, tnb, tks);
        TileWork tw;
        if (!tile_work(p, tb, tmb, tks, num_kb, tw)) { --local; continue; }
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, 0x200u + acc, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int kb_lo = tw.kb_lo, kb_hi = tw.kb_hi;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&full[stage], phase, 0x300u + stage, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * S::STAGE_BYTES);
          const uint32_t b_addr = a_addr + S::A_BYTES;
#pragma unroll
          for (int j = 0; j < BK / 16; ++j) {
            // K-major: step 32 bytes along the swizzled 128-byte row.
            // MN-major: step 16 rows of 128 bytes (two 8-row swizzle atoms).
            const uint64_t ad = A_MN ? smem_desc(a_addr + j * 2048, 8192, 1024) : smem_desc(a_addr + j * 32, 16, 1024);
            const uint64_t bd = B_MN ? smem_desc(b_addr + j * 2048, 8192, 1024) : smem_desc(b_addr + j * 32, 16, 1024);
            if constexpr (PAIR) umma_bf16_pair(d_tmem, ad, bd, idesc, (kb > kb_lo || j != 0) ? 1u : 0u);
            else umma_bf16(d_tmem, ad, bd, idesc, (kb > kb_lo || j != 0) ? 1u : 0u);
          }
          if constexpr (PAIR) umma_commit_pair(&empty[stage], 0x3);
          else umma_commit(&empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (ok) {
          if constexpr (PAIR) umma_commit_pair(&tfull[acc], 0x3);
          else umma_commit(&tfull[acc]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    const float sacc = p.s_ptr ? p.s_acc * *p.s_ptr : p.s_acc;
    if constexpr (EPI == EPI_F32 || EPI == EPI_F32_ACC) {
      if (p.tma_out) {
        // fp32 outputs: [32 rows x 32 fp32] boxes (128-byte rows, 128-byte swizzle) leave by bulk
        // tensor store, or by bulk tensor add-reduction for the accumulating weight gradient (each
        // output element receives exactly one addition, so the result stays deterministic)
        uint8_t* stg = smem + S::STG_OFFSET + (warp - 2) * STG_WARP;
        const bool reduce = EPI == EPI_F32_ACC && p.split == 1;
        int g = 0;
        int local = 0;
        for (int t = tile0; t < total_tiles; t += tstride, ++local) {
          int b, mb, nb, ks;
          tile_coords(t, p, b, mb, nb, ks);
          TileWork tw;
          if (!tile_work(p, b, mb, ks, num_kb, tw)) { --local; continue; }
          b = tw.zC;
          const int acc = local & 1;
          const uint32_t acc_phase = (local >> 1) & 1;
          if (!mbar_wait(&tfull[acc], acc_phase, 0x400u + acc, abort_flag)) break;
          __syncwarp();
          tc_fence_after();
          const int row0 = (mb * TM + static_cast<int>(crank) * BM) + quad * 32;
          const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c, ++g) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld32(t_row + c * 32, r);
            tmem_wait_ld();
            if (c == BN / 32 - 1) {
              tc_fence_before();
              arrive_tempty<PAIR>(&tempty[acc], crank);
            }
            const int col0 = nb * BN + c * 32;
            uint8_t* sc = stg + (g & 1) * (2 * STG_BOX);  // 4 KB box
            if (lane == 0) tma_store_wait_read1();
            __syncwarp();
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int pos = lane * 128 + ((k ^ (lane & 7)) << 4);
              *reinterpret_cast<float4*>(sc + pos) =
                  make_float4(__uint_as_float(r[4 * k]) * sacc, __uint_as_float(r[4 * k + 1]) * sacc,
                              __uint_as_float(r[4 * k + 2]) * sacc, __uint_as_float(r[4 * k + 3]) * sacc);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && row0 < p.M && col0 < p.N) {
              // the split-K workspace is addressed as [split, M, N]: slice = z
              const int z = p.split > 1 ? ks : b;
              if (reduce) tma_reduce_add_3d(&tmC, sc, col0, row0, z);
              else tma_store_3d(&tmC, sc, col0, row0, z);
            }
            if (lane == 0) tma_store_commit();
          }
        }
        if (lane == 0) tma_store_wait0();
      }
    }
    if constexpr (bf16_out<EPI>()) {
      if (p.tma_out) {
        // staged path: values -> swizzled shared-memory box -> bulk tensor store (no per-thread
        // global stores, so the L1/LSU path stays free for the operand loads)
        uint8_t* stg = smem + S::STG_OFFSET + (warp - 2) * STG_WARP;
        const int nparts = (p.N + 127) / 128;
        int g = 0;
        int local = 0;
        for (int t = tile0; t < total_tiles; t += tstride, ++local) {
          int b, mb, nb, ks;
          tile_coords(t, p, b, mb, nb, ks);
          TileWork tw;
          if (!tile_work(p, b, mb, ks, num_kb, tw)) { --local; continue; }
          b = tw.zC;
          const int acc = local & 1;
          const uint32_t acc_phase = (local >> 1) & 1;
          if (!mbar_wait(&tfull[acc], acc_phase, 0x400u + acc, abort_flag)) break;
          __syncwarp();
          tc_fence_after();
          const int row = (mb * TM + static_cast<int>(crank) * BM) + row_in_tile;
          const int row0 = (mb * TM + static_cast<int>(crank) * BM) + quad * 32;
          const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
          float se = 0.f;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c, ++g) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld32(t_row + c * 32, r);
            tmem_wait_ld();
            if (c == BN / 32 - 1) {
              tc_fence_before();
              arrive_tempty<PAIR>(&tempty[acc], crank);  // the accumulator is in registers: MMA may reuse it
            }
            const int col0 = nb * BN + c * 32;
            uint32_t out[16], pre[16];
            epi_pack<EPI>(p, sacc, b, row, col0, r, out, pre, se);
            if constexpr (EPI == EPI_CE_FWD) {
              const int group0 = nb * BN + (c & ~3) * 32;
              if ((c & 3) == 3 && row < p.M && group0 < p.N) {
                p.ce.part[static_cast<int64_t>(row) * nparts + group0 / 128] = se;
                se = 0.f;
              }
            }
            uint8_t* sc = stg + (g & 1) * (2 * STG_BOX);
            if (lane == 0) tma_store_wait_read1();  // the store that used this buffer two chunks ago has read it
            __syncwarp();
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const int pos = lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4);
              *reinterpret_cast<uint4*>(sc + pos) = make_uint4(out[4 * k], out[4 * k + 1], out[4 * k + 2], out[4 * k + 3]);
              if constexpr (EPI == EPI_RELU2)
                *reinterpret_cast<uint4*>(sc + STG_BOX + pos) =
                    make_uint4(pre[4 * k], pre[4 * k + 1], pre[4 * k + 2], pre[4 * k + 3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && row0 < p.M && col0 < p.N) {
              tma_store_3d(&tmC, sc, col0, row0, b);
              if constexpr (EPI == EPI_RELU2) tma_store_3d(&tmP, sc + STG_BOX, col0, row0, b);
            }
            if (lane == 0) tma_store_commit();
          }
          if constexpr (EPI == EPI_CE_FWD) {
            if ((BN / 32) % 4 != 0 && row < p.M) p.ce.part[static_cast<int64_t>(row) * nparts + (nb * BN) / 128] = se;
          }
        }
        if (lane == 0) tma_store_wait0();
      }
    }
    if (!(bf16_out<EPI>() || EPI == EPI_F32 || EPI == EPI_F32_ACC) || !p.tma_out) {
      int local = 0;
      for (int t = tile0; t < total_tiles; t += tstride, ++local) {
        int b, mb, nb, ks;
        tile_coords(t, p, b, mb, nb, ks);
        TileWork tw;
        if (!tile_work(p, b, mb, ks, num_kb, tw)) { --local; continue; }
        b = tw.zC;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tfull[acc], acc_phase, 0x400u + acc, abort_flag)) break;
        __syncwarp();
        tc_fence_after();
        const int row = (mb * TM + static_cast<int>(crank) * BM) + row_in_tile;
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN;
        if constexpr (EPI == EPI_CE_FWD) {
          const int nparts = (p.N + 127) / 128;
          float se = 0.f;
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            __syncwarp();  // the previous chunk's epilogue may have diverged (partial tiles)
            tmem_ld32(t_row + c * 32, r);
            tmem_wait_ld();
            const int col0 = nb * BN + c * 32;
            if (row < p.M && col0 < p.N) se += ce_fwd32(p, row, col0, r);
            const int group0 = nb * BN + (c & ~3) * 32;  // first column of this 128-column part
            if ((c & 3) == 3 && row < p.M && group0 < p.N) {
              p.ce.part[static_cast<int64_t>(row) * nparts + group0 / 128] = se;
              se = 0.f;
            }
          }
          if ((BN / 32) % 4 != 0 && row < p.M) p.ce.part[static_cast<int64_t>(row) * nparts + (nb * BN) / 128] = se;
        } else {
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            __syncwarp();  // the previous chunk's epilogue may have diverged (partial tiles)
            tmem_ld32(t_row + c * 32, r);
            tmem_wait_ld();
            epilogue32<EPI>(p, sacc, b, ks, row, nb * BN + c * 32, r);
          }
        }
        tc_fence_before();
        arrive_tempty<PAIR>(&tempty[acc], crank);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's epilogue has read its tensor memory
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, 2 * BN);
    else tmem_dealloc(tmem_base, 2 * BN);
  }
}

// C (+)= sum_s W[s]  in a fixed order (deterministic split-K reduction); n elements per slice.
__global__ void splitk_reduce_kernel(const float* __restrict__ w, int split, int64_t n, float* __restrict__ c,
                                     int64_t ldc, int cols, int accumulate) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i >= n) return;
  float4 a = *reinterpret_cast<const float4*>(w + i);
  for (int s = 1; s < split; ++s) {
    const float4 b = *reinterpret_cast<const float4*>(w + s * n + i);
    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
  }
  const int64_t r = i / cols;
  const int col = static_cast<int>(i - r * cols);
  float4* dst = reinterpret_cast<float4*>(c + r * ldc + col);
  if (accumulate) {
    const float4 o = *dst;
    a.x += o.x; a.y += o.y; a.z += o.z; a.w += o.w;
  }
  *dst = a;
}

// Cross-entropy row statistics (one warp per row, fixed summation order).
__global__ void ce_finish_kernel(const float* __restrict__ part, int nparts, const int64_t* __restrict__ tgt,
                                 const float* __restrict__ ztgt, float* __restrict__ loss, float* __restrict__ rscale,
                                 float* __restrict__ rcorr, int rows, float cap) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float s = 0.f;
  for (int i = lane; i < nparts; i += 32) s += part[static_cast<int64_t>(row) * nparts + i];
  s = warp_sum(s);
  if (lane == 0) {
    const bool live = tgt[row] >= 0;
    const float z = live ? ztgt[row] : 0.f;
    loss[row] = live ? cap + logf(s) - z : 0.f;
    rscale[row] = live ? 1.f / s : 0.f;
    const float t = z / cap;
    rcorr[row] = live ? 1.f - t * t : 0.f;
  }
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// 3-D bf16 tensor map: dims {inner, outer, batch}, box {64, box_outer, 1}, 128-byte swizzle.
static CUtensorMap make_map(const void* base, int64_t inner, int64_t outer, int64_t ld, int64_t batch,
                            int64_t batch_stride, int box_outer) {
  if (reinterpret_cast<uintptr_t>(base) % 16) throw std::runtime_error("gemm operand is not 16-byte aligned");
  if ((ld * 2) % 16 || (batch > 1 && (batch_stride * 2) % 16))
    throw std::runtime_error("gemm operand strides must be multiples of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2),
                           static_cast<cuuint64_t>((batch > 1 ? batch_stride : ld * outer) * 2)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_outer), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = get_encode()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return map;
}

// bf16 output map for the bulk-store epilogue: dims {N, M, batch}, box {32, 32, 1}, 64-byte swizzle.
// Returns false (direct stores are used) when the layout does not allow bulk tensor stores.
static bool out_map(CUtensorMap& map, const void* base, int64_t N, int64_t M, int64_t ld, int64_t batch,
                    int64_t batch_stride) {
  if (!base || reinterpret_cast<uintptr_t>(base) % 16 || (ld * 2) % 16 || (batch > 1 && (batch_stride * 2) % 16))
    return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2),
                           static_cast<cuuint64_t>((batch > 1 ? batch_stride : ld * M) * 2)};
  cuuint32_t box[3] = {32u, 32u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return get_encode()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp32 output map: dims {N, M, depth}, box {32, 32, 1}, 128-byte swizzle (depth = batch or split slices).
static bool out_map_f32(CUtensorMap& map, const void* base, int64_t N, int64_t M, int64_t ld, int64_t depth,
                        int64_t depth_stride) {
  if (!base || reinterpret_cast<uintptr_t>(base) % 16 || (ld * 4) % 16 || (depth > 1 && (depth_stride * 4) % 16))
    return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(depth)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 4),
                           static_cast<cuuint64_t>((depth > 1 ? depth_stride : ld * M) * 4)};
  cuuint32_t box[3] = {32u, 32u, 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return get_encode()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int A_MN, int B_MN, int EPI, bool PAIR = false>
static void launch_t(const GemmArgs& g, cudaStream_t stream) {
  constexpr int BNC = PAIR ? BN / 2 : BN;   // B rows per CTA
  constexpr int TM = PAIR ? 2 * BM : BM;    // rows per tile
  constexpr int STAGES = BNC == 256 ? 4 : 6;
  using S = Smem<BNC, STAGES>;
  // A: logical [M, K].  K-major storage [M rows, K cols] (inner = K); M-major [K rows, M cols].
  const bool grouped = g.grp_m || g.grp_k;
  const int bA = grouped ? 1 : g.batch;
  const int bB = g.grp_m ? g.groups : (g.grp_k ? 1 : g.batch);
  const int bC = g.grp_m ? 1 : (g.grp_k ? g.groups : g.batch);
  CUtensorMap ta = A_MN == 0 ? make_map(g.A, g.K, g.M, g.lda, bA, g.strideA, BM)
                             : make_map(g.A, g.M, g.K, g.lda, bA, g.strideA, BK);
  CUtensorMap tb = B_MN == 0 ? make_map(g.B, g.K, g.N, g.ldb, bB, g.strideB, BNC)
                             : make_map(g.B, g.N, g.K, g.ldb, bB, g.strideB, BK);
  Params p;
  p.M = g.M; p.N = g.N; p.K = g.K; p.batch = bC;
  p.grp_m = g.grp_m;
  p.grp_k = g.grp_k;
  p.tiles_m = (g.M + TM - 1) / TM;
  p.tiles_n = (g.N + BN - 1) / BN;
  p.epi = EPI;
  p.C = g.C; p.ldc = g.ldc; p.strideC = g.strideC;
  p.R = g.R; p.ldr = g.ldr; p.strideR = g.strideR;
  p.P = g.P; p.ldp = g.ldp; p.strideP = g.strideP;
  p.s_acc = g.s_acc; p.s_res = g.s_res; p.s_ptr = g.s_ptr;
  p.ce = g.ce;
  p.split = g.split_k > 1 ? g.split_k : 1;
  const int num_kb = (g.K + BK - 1) / BK;
  p.kb_per_split = (num_kb + p.split - 1) / p.split;
  p.strideSplit = p.split > 1 ? static_cast<int64_t>(g.M) * g.N : 0;
  if (p.split > 1) {
    p.C = g.workspace;  // partial products: [split, M, N] fp32, contiguous
    p.ldc = g.N;
    p.strideC = 0;
  }
  CUtensorMap tc = ta, tp = ta;  // placeholders when the direct epilogue runs
  p.tma_out = 0;
  if (bf16_out<EPI>() && p.split == 1 && g.tma_out_ok) {
    bool ok = out_map(tc, g.C, g.N, g.M, g.ldc, bC, g.strideC);
    if (EPI == EPI_RELU2) ok = ok && out_map(tp, g.P, g.N, g.M, g.ldp, bC, g.strideP);
    p.tma_out = ok ? 1 : 0;
  }
  if ((EPI == EPI_F32 || EPI == EPI_F32_ACC) && g.tma_out_ok) {
    const bool ok = p.split > 1 ? out_map_f32(tc, p.C, g.N, g.M, p.ldc, p.split, p.strideSplit)
                                : out_map_f32(tc, g.C, g.N, g.M, g.ldc, bC, g.strideC);
    p.tma_out = ok ? 1 : 0;
  }
  auto kern = gemm_kernel<BN, A_MN, B_MN, EPI, STAGES, PAIR>;
  static std::atomic<uint64_t> smem_set{0};
  nt::smem_limit(smem_set, kern, S::TOTAL);
  const int tiles = p.batch * p.split * p.tiles_m * p.tiles_n;
  if constexpr (PAIR) {
    const int pairs = tiles < g.num_sms / 2 ? tiles : g.num_sms / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.blockDim = dim3(NUM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = S::TOTAL;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, tp, p);
  } else {
    const int grid = tiles < g.num_sms ? tiles : g.num_sms;
    kern<<<grid, NUM_THREADS, S::TOTAL, stream>>>(ta, tb, tc, tp, p);
  }
  if (p.split > 1) {
    const int64_t n = static_cast<int64_t>(g.M) * g.N;
    splitk_reduce_kernel<<<static_cast<unsigned>((n / 4 + 255) / 256), 256, 0, stream>>>(
        reinterpret_cast<const float*>(g.workspace), p.split, n, reinterpret_cast<float*>(g.C), g.ldc, g.N,
        g.epi == EPI_F32_ACC ? 1 : 0);
  }
}

template <int BN, int A_MN, int B_MN, bool PAIR>
static void dispatch_epi(const GemmArgs& g, cudaStream_t s) {
  switch (g.epi) {
    case EPI_BF16: return launch_t<BN, A_MN, B_MN, EPI_BF16, PAIR>(g, s);
    case EPI_F32: return launch_t<BN, A_MN, B_MN, EPI_F32, PAIR>(g, s);
    case EPI_F32_ACC: return launch_t<BN, A_MN, B_MN, EPI_F32_ACC, PAIR>(g, s);
    case EPI_BF16_AXPBY: return launch_t<BN, A_MN, B_MN, EPI_BF16_AXPBY, PAIR>(g, s);
    case EPI_RELU2: return launch_t<BN, A_MN, B_MN, EPI_RELU2, PAIR>(g, s);
    case EPI_RELU2_BWD: return launch_t<BN, A_MN, B_MN, EPI_RELU2_BWD, PAIR>(g, s);
    case EPI_CE_FWD:
      if constexpr (A_MN == 0 && B_MN == 0) return launch_t<BN, 0, 0, EPI_CE_FWD, PAIR>(g, s);
      throw std::runtime_error("cross-entropy forward epilogue needs K-major operands");
    case EPI_CE_DGRAD:
      if constexpr (A_MN == 0 && B_MN == 1) return launch_t<BN, 0, 1, EPI_CE_DGRAD, PAIR>(g, s);
      throw std::runtime_error("cross-entropy input-gradient epilogue needs A K-major, B N-major");
    default: throw std::runtime_error("unknown gemm epilogue");
  }
}

template <int BN, bool PAIR = false>
static void dispatch_major(const GemmArgs& g, cudaStream_t s) {
  if (!g.a_mn && !g.b_mn) return dispatch_epi<BN, 0, 0, PAIR>(g, s);
  if (!g.a_mn && g.b_mn) return dispatch_epi<BN, 0, 1, PAIR>(g, s);
  if (g.a_mn && !g.b_mn) return dispatch_epi<BN, 1, 0, PAIR>(g, s);
  return dispatch_epi<BN, 1, 1, PAIR>(g, s);
}

}  // namespace gemm
}  // namespace nt

namespace {
// Split-K pays when an fp32-output problem has a long reduction but too few 128x256 tiles to fill
// the machine (weight gradients reduce over all tokens).  Returns the slice count (1 = none).
// The persistent grid gives each CTA ceil(tiles * split / SMs) tiles, so the slice count is picked
// by a cost model: rounds of tiles x the time of one tile's share of K, plus writing and reading the
// fp32 partial products (s x M x N x 8 bytes).  Per-SM tensor rate and memory bandwidth are nominal
// (about 11 TFLOP/s per SM, 6 TB/s); only their ratio matters.
int choose_split(const GemmArgs& g) {
  if (g.epi != EPI_F32 && g.epi != EPI_F32_ACC) return 1;
  if (g.batch != 1 || g.N < 256 || g.M % 4 || g.N % 4 || g.ldc % 4) return 1;
  const long tiles = static_cast<long>((g.M + 127) / 128) * ((g.N + 255) / 256);
  const int sms = g.num_sms > 0 ? g.num_sms : 148;
  // NT_GEMM_SPLIT_MODEL=0 selects the plain rule (enough slices for two tiles per SM; measurement only)
  static const bool plain = [] {
    const char* e = std::getenv("NT_GEMM_SPLIT_MODEL");
    return e && e[0] == '0';
  }();
  if (plain) {
    if (tiles >= 2L * sms) return 1;
    const int kb = (g.K + 63) / 64;
    int split = static_cast<int>((2L * sms + tiles - 1) / tiles);
    split = split > 16 ? 16 : split;
    while (split > 1 && kb / split < 16) --split;
    return split;
  }
  if (tiles >= 4L * sms) return 1;
  const int num_kb = (g.K + 63) / 64;
  const double tile_s = 2.0 * 128 * 256 * static_cast<double>(g.K) / 11e12;
  const double slice_s = 8.0 * static_cast<double>(g.M) * g.N / 6e12;
  int best = 1;
  double best_t = static_cast<double>((tiles + sms - 1) / sms) * tile_s;
  for (int s = 2; s <= 16 && num_kb / s >= 16; ++s) {  // >= 16 k-blocks per slice
    const double t = static_cast<double>((tiles * s + sms - 1) / sms) * tile_s / s + s * slice_s;
    if (t < 0.98 * best_t) {
      best = s;
      best_t = t;
    }
  }
  return best;
}
}  // namespace

// CTA-pair tiles are the default; NT_GEMM_PAIRS=0 in the environment keeps single-CTA tiles.
bool gemm_pairs_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("NT_GEMM_PAIRS");
    return !(v && v[0] == '0');
  }();
  return on;
}

size_t nt_gemm_splitk_bytes(const GemmArgs& g) {
  const int split = choose_split(g);
  return split > 1 ? static_cast<size_t>(split) * g.M * g.N * sizeof(float) : 0;
}

void nt_gemm_launch(const GemmArgs& g_in, cudaStream_t stream) {
  nt::current_context();
  using namespace nt::gemm;
  GemmArgs g = g_in;
  if (g.M <= 0 || g.N <= 0 || g.K <= 0 || g.batch <= 0) return;
  if (g.grp_m || g.grp_k) {
    if (g.groups <= 0 || (g.grp_m && g.grp_k) || (g.grp_k && g.epi != EPI_F32_ACC))
      throw std::runtime_error("grouped GEMM: one table, groups > 0, and EPI_F32_ACC for grp_k");
    g.batch = g.grp_k ? g.groups : 1;
  }
  g.split_k = 1;
  const int split = (g.grp_m || g.grp_k) ? 1 : choose_split(g);
  if (split > 1 && g.workspace && g.workspace_bytes >= static_cast<size_t>(split) * g.M * g.N * sizeof(float))
    g.split_k = split;
  // BN = 256 halves B-operand shared-memory traffic per MMA (128-wide tiles are bound by
  // shared-memory bandwidth); 128-wide tiles are kept only when 256-wide ones cannot fill the GPU.
  const long tiles256 = static_cast<long>(g.batch) * g.split_k * ((g.M + 127) / 128) * ((g.N + 255) / 256);
  const bool wide = g.N >= 256 && tiles256 >= g.num_sms;
  // CTA pairs (256 x 256 tiles over two SMs) when the problem still fills every SM pair
  const long pair_tiles = static_cast<long>(g.batch) * ((g.M + 255) / 256) * ((g.N + 255) / 256);
  const bool pair = wide && g.split_k == 1 && !g.grp_m && !g.grp_k && pair_tiles >= g.num_sms / 2 &&
                    gemm_pairs_enabled();
  if (pair) dispatch_major<256, true>(g, stream);
  else if (wide) dispatch_major<256>(g, stream);
  else dispatch_major<128>(g, stream);
}

int nt_gemm_read_error(unsigned* where) {
  nt::ErrorWord w{0, 0};
  cudaMemcpyFromSymbol(&w, nt::g_nt_error, sizeof(w));
  if (where) *where = w.where;
  return static_cast<int>(w.code);
}

int nt_ce_finish(const float* part, int nparts, const int64_t* tgt, const float* ztgt, float* loss, float* rscale,
                 float* rcorr, int rows, float cap, cudaStream_t stream) {
  if (rows <= 0) return 0;
  nt::gemm::ce_finish_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(part, nparts, tgt, ztgt, loss, rscale, rcorr, rows,
                                                                  cap);
  return 0;
}
