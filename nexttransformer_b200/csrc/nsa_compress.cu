// NSA compressed branch: attention over the compressed keys of complete blocks, the selection-block
// importance and the top-k block choice, and the backward of the attention.
//
// Compressed key c summarises tokens [cstride c, cstride c + csize); query t sees it once the block is
// complete (cstride c + csize - 1 <= t).  Per query row: p_c = softmax_c(scale q . k_c) over the
// visible keys, o = sum_c p_c v_c, importance of selection block s = sum of p_c over the compressed
// blocks that overlap it, and the chosen blocks = the top-k complete blocks other than the row's own
// (ties to the lower block) plus the row's own block.
//
// Forward: one CTA per (64-query tile, head, batch), 4 warps of 16 query rows.  Pass 1 streams the
// key tiles for the row log-sum-exp; pass 2 recomputes the scores, forms the normalised p once,
// adds it into the importance (shared memory) and into O = P V with the probabilities reused as the
// A operand of the second MMA from registers; then each warp picks its rows' top-k by repeated warp
// arg-max.  Nothing of size [B, H, T, Nc] is stored.
// Backward: one CTA per (64-key tile, head, batch), 4 warps of 16 keys; for every query tile that
// sees the key tile: S^T, P^T, dP^T and dS^T in registers, dV += P^T dO and dK += dS^T Q from
// registers, dS through shared memory into dQ = dS K; dQ, dK and dV are added to fp32 buffers
// (the 16 query heads of a KV head share dK / dV).
// Tensor-core MMAs are mma.sync m16n8k16 (bf16 in, fp32 accumulate).  The torch expression of the
// reference path is models/sparse.py's compressed branch (nexttransformer/models/sparse.py:182-276).
#include "nsa_compress.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>

namespace nt {
namespace nsa {

constexpr int TQ = 64, TK = 64, HD = 128;
constexpr int LDS = HD + 8;   // bf16 stride of row-major [64 x 128] tiles
constexpr int LDT = TK + 8;   // bf16 stride of transposed [128 x 64] tiles
constexpr int THREADS = 128;
constexpr int MAX_SEL = 256;

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t ld32(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }

// rows [r0, r0 + 64) of a [.., 128] bf16 matrix (row stride ld) into a row-major tile, and / or
// transposed into a [128 x 64] tile; rows at or past `valid` are zero
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, __nv_bfloat16* dstT, const __nv_bfloat16* src,
                                          int64_t ld, int r0, int valid) {
  for (int e = threadIdx.x; e < 64 * (HD / 8); e += THREADS) {
    const int r = e / (HD / 8), c = (e % (HD / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r0 + r < valid) v = *reinterpret_cast<const uint4*>(src + static_cast<int64_t>(r0 + r) * ld + c);
    if (dst) *reinterpret_cast<uint4*>(dst + r * LDS + c) = v;
    if (dstT) {
      const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int u = 0; u < 8; ++u) dstT[(c + u) * LDT + r] = x[u];
    }
  }
}

// acc (16 rows of A from `a_rows` x 64 columns) = A . B^T with B rows from `b_rows` (row-major, both
// [.. x 128]): acc[n][0..1] row g, columns 8n + 2t, +1; acc[n][2..3] row g + 8
__device__ __forceinline__ void rows_dot_rows(const __nv_bfloat16* a_rows, const __nv_bfloat16* b_rows,
                                              float (&acc)[8][4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
  const __nv_bfloat16* pa = a_rows + g * LDS + 2 * t;
#pragma unroll
  for (int k0 = 0; k0 < HD; k0 += 16) {
    uint32_t a[4] = {ld32(pa + k0), ld32(pa + 8 * LDS + k0), ld32(pa + k0 + 8), ld32(pa + 8 * LDS + k0 + 8)};
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const __nv_bfloat16* pb = b_rows + (8 * n + g) * LDS + k0 + 2 * t;
      uint32_t b[2] = {ld32(pb), ld32(pb + 8)};
      mma_bf16(acc[n], a, b);
    }
  }
}

// out (16 rows x 128 columns) += P (16 x 64, fp32 fragments of rows_dot_rows layout) . M with M^T
// given as a transposed [128 x 64] tile (mT[col][k])
__device__ __forceinline__ void frag_times_tile(const float (&p)[8][4], const __nv_bfloat16* mT, float (&out)[16][4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    uint32_t a[4] = {pack2(p[2 * kk][0], p[2 * kk][1]), pack2(p[2 * kk][2], p[2 * kk][3]),
                     pack2(p[2 * kk + 1][0], p[2 * kk + 1][1]), pack2(p[2 * kk + 1][2], p[2 * kk + 1][3])};
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const __nv_bfloat16* pb = mT + (8 * n + g) * LDT + 16 * kk + 2 * t;
      uint32_t b[2] = {ld32(pb), ld32(pb + 8)};
      mma_bf16(out[n], a, b);
    }
  }
}

__device__ __forceinline__ bool visible(const NsaArgs& a, int c, int t) {
  return c < a.Nc && t < a.T && a.cstride * c + a.csize - 1 <= t;
}

struct FwdSmem {
  static constexpr int Q = 0;
  static constexpr int K = Q + TQ * LDS * 2;
  static constexpr int VT = K + TK * LDS * 2;
  static constexpr int IMP = VT + HD * LDT * 2;
  // the importance rows take TQ x nsel floats: sized per launch, so short sequences fit two CTAs / SM
  static int bytes(int nsel) { return IMP + TQ * nsel * 4; }
  static constexpr int MAX_BYTES = IMP + TQ * MAX_SEL * 4;
};

__global__ void __launch_bounds__(THREADS) fwd_kernel(const NsaArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem + FwdSmem::Q);
  __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(smem + FwdSmem::K);
  __nv_bfloat16* svT = reinterpret_cast<__nv_bfloat16*>(smem + FwdSmem::VT);
  float* imp = reinterpret_cast<float*>(smem + FwdSmem::IMP);
  const int q0 = blockIdx.x * TQ, h = blockIdx.y, b = blockIdx.z, hk = h / (a.H / a.Hk);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  const int nsel = (a.T + a.ssize - 1) / a.ssize;
  const int64_t ldq = static_cast<int64_t>(a.H) * HD, ldk = static_cast<int64_t>(a.Hk) * HD;
  const __nv_bfloat16* qb = a.q + static_cast<int64_t>(b) * a.T * ldq + h * HD;
  const __nv_bfloat16* kb = a.k + static_cast<int64_t>(b) * a.Nc * ldk + hk * HD;
  const __nv_bfloat16* vb = a.v + static_cast<int64_t>(b) * a.Nc * ldk + hk * HD;
  const int qmax = min(q0 + TQ, a.T) - 1;
  const int n_keys = qmax >= a.csize - 1 ? min(a.Nc, (qmax - (a.csize - 1)) / a.cstride + 1) : 0;
  load_tile(sq, nullptr, qb, ldq, q0, a.T);
  for (int e = threadIdx.x; e < TQ * nsel; e += THREADS) imp[e] = 0.f;
  const int row[2] = {q0 + 16 * warp + g, q0 + 16 * warp + g + 8};
  // pass 1: row log-sum-exp of the scaled scores over the visible keys
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  for (int c0 = 0; c0 < n_keys; c0 += TK) {
    __syncthreads();
    load_tile(sk, nullptr, kb, ldk, c0, a.Nc);
    __syncthreads();
    float s[8][4];
    rows_dot_rows(sq + 16 * warp * LDS, sk, s);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float& x = s[n][2 * hf + e];
          x = visible(a, c0 + 8 * n + 2 * t + e, row[hf]) ? x * a.scale : -INFINITY;
          mx = fmaxf(mx, x);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m[hf], mx), ref = mn == -INFINITY ? 0.f : mn;
      float sum = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) sum += expf(s[n][2 * hf + e] - ref);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      l[hf] = l[hf] * expf(m[hf] - ref) + sum;
      m[hf] = mn;
    }
  }
  const float lse[2] = {l[0] > 0.f ? m[0] + logf(l[0]) : -INFINITY, l[1] > 0.f ? m[1] + logf(l[1]) : -INFINITY};
  // pass 2: normalised probabilities -> importance and O = P V
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[n][e] = 0.f;
  for (int c0 = 0; c0 < n_keys; c0 += TK) {
    __syncthreads();
    load_tile(sk, nullptr, kb, ldk, c0, a.Nc);
    load_tile(nullptr, svT, vb, ldk, c0, a.Nc);
    __syncthreads();
    float s[8][4];
    rows_dot_rows(sq + 16 * warp * LDS, sk, s);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hf = e >> 1, c = c0 + 8 * n + 2 * t + (e & 1);
        const float p = visible(a, c, row[hf]) ? expf(s[n][e] * a.scale - lse[hf]) : 0.f;
        s[n][e] = p;
        if (p > 0.f) {
          const int lo = a.cstride * c / a.ssize, hi = (a.cstride * c + a.csize - 1) / a.ssize;
          float* ir = imp + (row[hf] - q0) * nsel;
          for (int sb = lo; sb <= hi && sb < nsel; ++sb) atomicAdd(ir + sb, p);
        }
      }
    frag_times_tile(s, svT, o);
  }
  // O and lse
  __nv_bfloat16* ob = a.o + static_cast<int64_t>(b) * a.T * ldq + h * HD;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    if (row[hf] >= a.T) continue;
#pragma unroll
    for (int n = 0; n < 16; ++n)
      *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(row[hf]) * ldq + 8 * n + 2 * t) =
          pack2(o[n][2 * hf], o[n][2 * hf + 1]);
    if (t == 0) a.lse[(static_cast<int64_t>(b) * a.H + h) * a.T + row[hf]] = lse[hf];
  }
  __syncthreads();
  // top-k complete blocks other than the row's own, plus the own block
  const int per_lane = (nsel + 31) / 32;
  for (int r = 16 * warp; r < 16 * warp + 16; ++r) {
    const int tr = q0 + r;
    if (tr >= a.T) break;
    const int cur = tr / a.ssize;
    float v[MAX_SEL / 32];
    unsigned chosen = 0;
#pragma unroll
    for (int j = 0; j < MAX_SEL / 32; ++j) {
      const int sb = lane + 32 * j;
      const bool ok = j < per_lane && sb < nsel && (sb + 1) * a.ssize - 1 <= tr && sb != cur;
      v[j] = ok ? imp[r * nsel + sb] : -INFINITY;
    }
    for (int round = 0; round < a.topk; ++round) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < MAX_SEL / 32; ++j)
        if (v[j] > bv) {
          bv = v[j];
          bi = lane + 32 * j;
        }
#pragma unroll
      for (int off = 16; off; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (bv == -INFINITY) break;
      if ((bi & 31) == lane) {
#pragma unroll
        for (int j = 0; j < MAX_SEL / 32; ++j)
          if (j == (bi >> 5)) {
            v[j] = -INFINITY;
            chosen |= 1u << j;
          }
      }
    }
    uint8_t* out = a.sel + ((static_cast<int64_t>(b) * a.H + h) * a.T + tr) * nsel;
    for (int j = 0; j < per_lane; ++j) {
      const int sb = lane + 32 * j;
      if (sb < nsel) out[sb] = ((chosen >> j) & 1u) || sb == cur ? 1 : 0;
    }
  }
}

struct BwdSmem {
  static constexpr int K = 0;
  static constexpr int KT = K + TK * LDS * 2;
  static constexpr int V = KT + HD * LDT * 2;
  static constexpr int Q = V + TK * LDS * 2;
  static constexpr int QT = Q + TQ * LDS * 2;
  static constexpr int DO = QT + HD * LDT * 2;
  static constexpr int DOT = DO + TQ * LDS * 2;
  static constexpr int DS = DOT + HD * LDT * 2;
  static constexpr int STAT = DS + TQ * LDT * 2;
  static constexpr int BYTES = STAT + 2 * TQ * 4;
};

__global__ void __launch_bounds__(THREADS) bwd_kernel(const NsaArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sk = reinterpret_cast<__nv_bfloat16*>(smem + BwdSmem::K);
  __nv_bfloat16* skT = reinterpret_cast<__nv_bfloat16*>(smem + BwdSmem::KT);
  __nv_bfloat16* sv = reinterpret_cast<__nv_bfloat16*>(smem + BwdSmem::V);
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem + BwdSmem::Q);
  __nv_bfloat16* sqT = reinterpret_cast<__nv_bfloat16*>(smem + BwdSmem::QT);
  __nv_bfloat16* sdo = reinterpret_cast<__nv_bfloat16*>(smem + BwdSmem::DO);
  __nv_bfloat16* sdoT = reinterpret_cast<__nv_bfloat16*>(smem + BwdSmem::DOT);
  __nv_bfloat16* sds = reinterpret_cast<__nv_bfloat16*>(smem + BwdSmem::DS);   // dS [query][key]
  float* slse = reinterpret_cast<float*>(smem + BwdSmem::STAT);
  float* sdel = slse + TQ;
  // the query tiles of a key tile are split round-robin over `splits` CTAs (dK / dV are added atomically)
  const int splits = a.bwd_splits > 0 ? a.bwd_splits : 1;
  const int c0 = (blockIdx.x / splits) * TK, part = blockIdx.x % splits;
  const int h = blockIdx.y, b = blockIdx.z, hk = h / (a.H / a.Hk);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
  const int first = a.cstride * c0 + a.csize - 1;  // first query that sees key c0
  if (first >= a.T) return;
  const int64_t ldq = static_cast<int64_t>(a.H) * HD, ldk = static_cast<int64_t>(a.Hk) * HD;
  const __nv_bfloat16* qb = a.q + static_cast<int64_t>(b) * a.T * ldq + h * HD;
  const __nv_bfloat16* dob = a.dout + static_cast<int64_t>(b) * a.T * ldq + h * HD;
  load_tile(sk, skT, a.k + static_cast<int64_t>(b) * a.Nc * ldk + hk * HD, ldk, c0, a.Nc);
  load_tile(sv, nullptr, a.v + static_cast<int64_t>(b) * a.Nc * ldk + hk * HD, ldk, c0, a.Nc);
  float dk[16][4], dv[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[n][e] = dv[n][e] = 0.f;
  const int key[2] = {c0 + 16 * warp + g, c0 + 16 * warp + g + 8};
  for (int q0 = (first / TQ + part) * TQ; q0 < a.T; q0 += splits * TQ) {
    __syncthreads();
    load_tile(sq, sqT, qb, ldq, q0, a.T);
    load_tile(sdo, sdoT, dob, ldq, q0, a.T);
    for (int r = threadIdx.x; r < TQ; r += THREADS) {
      const int tr = q0 + r;
      const int64_t o = (static_cast<int64_t>(b) * a.H + h) * a.T + tr;
      slse[r] = tr < a.T ? a.lse[o] : INFINITY;
      sdel[r] = tr < a.T ? a.delta[o] : 0.f;
    }
    __syncthreads();
    float st[8][4], dpt[8][4];
    rows_dot_rows(sk + 16 * warp * LDS, sq, st);    // S^T: this warp's 16 keys x 64 queries
    rows_dot_rows(sv + 16 * warp * LDS, sdo, dpt);  // dP^T = V dO^T
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = 8 * n + 2 * t + (e & 1);
        const bool vis = visible(a, key[e >> 1], q0 + ql);
        const float p = vis ? expf(st[n][e] * a.scale - slse[ql]) : 0.f;
        st[n][e] = p;                                   // P^T
        dpt[n][e] = vis ? p * (dpt[n][e] - sdel[ql]) : 0.f;   // dS^T
      }
    frag_times_tile(st, sdoT, dv);   // dV += P^T dO
    frag_times_tile(dpt, sqT, dk);   // dK += dS^T Q
    // dS [query][key] for dQ = dS K
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = 8 * n + 2 * t + (e & 1), kl = 16 * warp + g + 8 * (e >> 1);
        sds[ql * LDT + kl] = __float2bfloat16_rn(dpt[n][e]);
      }
    __syncthreads();
    float dq[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) dq[n][e] = 0.f;
    {
      // this warp's 16 queries: A = dS rows (k = keys, 4 steps of 16), B = K (k = key, n = dim) from K^T
      const __nv_bfloat16* pa = sds + (16 * warp + g) * LDT + 2 * t;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t af[4] = {ld32(pa + 16 * kk), ld32(pa + 8 * LDT + 16 * kk), ld32(pa + 16 * kk + 8),
                          ld32(pa + 8 * LDT + 16 * kk + 8)};
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          const __nv_bfloat16* pb = skT + (8 * n + g) * LDT + 16 * kk + 2 * t;
          uint32_t bf[2] = {ld32(pb), ld32(pb + 8)};
          mma_bf16(dq[n], af, bf);
        }
      }
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int tr = q0 + 16 * warp + g + 8 * hf;
      if (tr >= a.T) continue;
      float* dst = a.dq_acc + (static_cast<int64_t>(b) * a.T + tr) * ldq + h * HD;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        atomicAdd(dst + 8 * n + 2 * t, dq[n][2 * hf] * a.scale);
        atomicAdd(dst + 8 * n + 2 * t + 1, dq[n][2 * hf + 1] * a.scale);
      }
    }
  }
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    if (key[hf] >= a.Nc) continue;
    const int64_t o = (static_cast<int64_t>(b) * a.Nc + key[hf]) * ldk + hk * HD;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      atomicAdd(a.dk_acc + o + 8 * n + 2 * t, dk[n][2 * hf] * a.scale);
      atomicAdd(a.dk_acc + o + 8 * n + 2 * t + 1, dk[n][2 * hf + 1] * a.scale);
      atomicAdd(a.dv_acc + o + 8 * n + 2 * t, dv[n][2 * hf]);
      atomicAdd(a.dv_acc + o + 8 * n + 2 * t + 1, dv[n][2 * hf + 1]);
    }
  }
}

template <class Kernel>
static cudaError_t smem_once(std::atomic<uint64_t>& done, Kernel kern, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit && (done.load() & bit)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit);
  return e;
}

}  // namespace nsa
}  // namespace nt

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static bool nsa_ok(const NsaArgs& a) {
  const auto al = al16;
  const int nsel = a.ssize > 0 ? (a.T + a.ssize - 1) / a.ssize : 0;
  return a.D == nt::nsa::HD && a.B > 0 && a.T > 0 && a.H > 0 && a.Hk > 0 && a.H % a.Hk == 0 && a.Nc > 0 &&
         a.cstride > 0 && a.csize > 0 && a.ssize > 0 && nsel <= nt::nsa::MAX_SEL && a.topk >= 0 && a.q && a.k &&
         a.v && al(a.q) && al(a.k) && al(a.v);
}

int nt_nsa_compressed_fwd(const NsaArgs& a, cudaStream_t s) {
  using namespace nt::nsa;
  if (!nsa_ok(a) || !a.o || !a.lse || !a.sel) return -1;
  static std::atomic<uint64_t> set{0};
  if (smem_once(set, fwd_kernel, FwdSmem::MAX_BYTES) != cudaSuccess) return -1;
  const int nsel = (a.T + a.ssize - 1) / a.ssize;
  fwd_kernel<<<dim3((a.T + TQ - 1) / TQ, a.H, a.B), THREADS, FwdSmem::bytes(nsel), s>>>(a);
  return 0;
}

int nt_nsa_compressed_bwd(const NsaArgs& a, cudaStream_t s) {
  using namespace nt::nsa;
  if (!nsa_ok(a) || !a.dout || !a.lse || !a.delta || !a.dq_acc || !a.dk_acc || !a.dv_acc || !al16(a.dout)) return -1;
  static std::atomic<uint64_t> set{0};
  if (smem_once(set, bwd_kernel, BwdSmem::BYTES) != cudaSuccess) return -1;
  NsaArgs b = a;
  // enough CTAs to cover the SMs twice: split each key tile's query tiles over CTAs
  const int base = ((a.Nc + TK - 1) / TK) * a.H * a.B;
  b.bwd_splits = std::max(1, std::min((2 * 148 + base - 1) / base, (a.T + TQ - 1) / TQ));
  bwd_kernel<<<dim3(((a.Nc + TK - 1) / TK) * b.bwd_splits, a.H, a.B), THREADS, BwdSmem::BYTES, s>>>(b);
  return 0;
}
