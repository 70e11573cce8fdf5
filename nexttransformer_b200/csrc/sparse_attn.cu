// Block-sparse attention for the sparse mixers on sm_100a (NSA selected blocks, MoBA blocks).
//
// Each query tile (128 rows of one head) walks a list of 64-key blocks: the union of the blocks
// its rows selected, each with a 128-bit row mask (bit r: row r selected the block).  Row r
// sees key j of a listed block iff its bit is set and j <= its position (causal), the selection
// semantics of the reference's indexed attention (nexttransformer/models/sparse.py:35-68) when
// the selection unit is a multiple of 64 keys.  Lists are shared by the heads of a list group
// (NSA: the KV group; MoBA: one list per head).
//
// Forward (one CTA per (query tile, head, batch); 192 threads):
//   warp 0      TMA: the Q tile once, then the K / V blocks (64 keys) of the list into a 2-stage ring.
//   warp 1      MMA: S_l = Q K_l^T (M 128, N 64) into one of two TMEM S buffers, one block ahead;
//               O += P_l V_l (P from shared memory) into the TMEM O accumulator.
//   warps 2..5  online softmax, one query row per thread, lazy rescaling of O (only when the row
//               maximum grows by more than 2^8); at the end O / l and the log-sum-exp.
// Backward (same grid, Q-stationary; 320 threads): per block S = Q K^T and dP = dO V^T in TMEM,
//   the softmax warps form P and dS = P (dP - delta) scale in shared memory, then dQ += dS K
//   accumulates in TMEM over the list while dV^T = dO^T P and dK^T = Q^T dS (M = 128 over the
//   head dimension) go to the drain warps, which transpose them through shared memory and add
//   them into fp32 dK / dV buffers with bulk tensor add-reductions (heads of a KV group and
//   query tiles that share a block add into the same rows).  dQ is complete per tile.
// Optional additive relative bias (Inkling REL, nexttransformer/methods/inkling_rel of the
// reference): logit(i, j) += rel[b, h, i, i - j]; the backward writes d rel at (i, i - j) once per
// selected pair (no atomics: a distance has one key per row).
// Every wait is bounded (common.cuh).  No TMA load uses cluster multicast.
#include <cudaTypedefs.h>
#include <math.h>
#include <mutex>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "sparse_attn.h"

namespace nt {
namespace bsa {

constexpr int QT = 128;
constexpr int KB = 64;
constexpr int HD = 128;
constexpr int QBOX = QT * 128;   // [128 rows x 64 bf16] = 16 KB
constexpr int KBOX = KB * 128;   // [64 rows x 64 bf16] = 8 KB
constexpr float LOG2E = 1.4426950408889634f;

struct Params {
  int B, T, H, Hk, G, Lmax, n_qt;
  float scale_log2, scale;
  const int* lists;
  const uint32_t* masks;
  __nv_bfloat16* o;
  int64_t ldo;
  float* lse;
  const float* delta;
  __nv_bfloat16* dq;
  int64_t lddq;
  const float* rel;
  float* drel;
  int rel_extent;
};

NT_DEVICE uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}
NT_DEVICE uint32_t swz(int r, int c) { return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4)); }
NT_DEVICE float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
NT_DEVICE bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t where, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, where, abort);
  return __all_sync(0xffffffffu, ok);
}
// Q tile (two 64-column boxes of 128 rows), k-step j of 16 columns, K-major.
NT_DEVICE uint64_t q_kmajor(uint32_t base, int j) { return smem_desc(base + (j >> 2) * QBOX + (j & 3) * 32, 16, 1024); }
// Key block (two 64-column boxes of 64 rows) as the K-major B operand (N = 64 keys).
NT_DEVICE uint64_t kb_kmajor(uint32_t base, int j) { return smem_desc(base + (j >> 2) * KBOX + (j & 3) * 32, 16, 1024); }
// Key block as the MN-major B operand (rows = keys = reduction, N = 128 features in two boxes).
NT_DEVICE uint64_t kb_mnmajor(uint32_t base, int j) { return smem_desc(base + j * 2048, KBOX, 1024); }

NT_DEVICE int list_base(const Params& p, int b, int h, int qt) {
  const int g = h / (p.H / p.G);
  return ((b * p.G + g) * p.n_qt + qt) * p.Lmax;
}
NT_DEVICE int list_len(const Params& p, int base) {
  int n = 0;
  while (n < p.Lmax && p.lists[base + n] >= 0) ++n;
  return n;
}

// ------------------------------------------------------------------------------ forward
struct FwdSmem {
  static constexpr int Q = 0;
  static constexpr int K0 = Q + 2 * QBOX;        // 2 stages x 16 KB
  static constexpr int V0 = K0 + 4 * KBOX;       // 2 stages x 16 KB
  static constexpr int P0 = V0 + 4 * KBOX;       // 2 buffers x [128 rows x 64 keys] bf16
  static constexpr int BAR = P0 + 2 * QBOX;
  static constexpr int NBAR = 10;                // q_full kv_full[2] kv_empty[2] s_full[2] p_full[2] o_done
  static constexpr int TOTAL = BAR + NBAR * 8 + 16 + 1024;
};
static_assert(FwdSmem::TOTAL <= 232448, "block-sparse forward shared memory");

__global__ void __launch_bounds__(192, 1)
    bsa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + FwdSmem::BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 7;
  uint64_t* o_done = bars + 9;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + FwdSmem::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.H / p.Hk);
  const int q0 = qt * QT;
  const int lbase = list_base(p, b, h, qt);
  const int L = list_len(p, lbase);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
    }
    mbar_init(o_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const uint32_t t_o = tbase, t_s0 = tbase + 128;

  if (warp == 0) {
    if (lane == 0 && L > 0) {
      mbar_expect_tx(q_full, 2 * QBOX);
      tma_load_3d(sm + FwdSmem::Q, &tmQ, q_full, h * HD, q0, b);
      tma_load_3d(sm + FwdSmem::Q + QBOX, &tmQ, q_full, h * HD + 64, q0, b);
      int issued = 0;
      for (int l = 0; l < L; ++l) {
        const int st = l & 1;
        if (!mbar_wait(&kv_empty[st], ((l >> 1) & 1) ^ 1u, 0xC00u + st, abort_flag)) break;
        const int k0 = p.lists[lbase + l] * KB;
        mbar_expect_tx(&kv_full[st], 4 * KBOX);
        uint8_t* kd = sm + FwdSmem::K0 + st * 2 * KBOX;
        uint8_t* vd = sm + FwdSmem::V0 + st * 2 * KBOX;
        tma_load_3d(kd, &tmK, &kv_full[st], hk * HD, k0, b);
        tma_load_3d(kd + KBOX, &tmK, &kv_full[st], hk * HD + 64, k0, b);
        tma_load_3d(vd, &tmV, &kv_full[st], hk * HD, k0, b);
        tma_load_3d(vd + KBOX, &tmV, &kv_full[st], hk * HD + 64, k0, b);
        ++issued;
      }
      mbar_wait(q_full, 0, 0xC10u, nullptr);
      for (int l = (issued > 2 ? issued - 2 : 0); l < issued; ++l)
        mbar_wait(&kv_full[l & 1], (l >> 1) & 1, 0xC11u, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0 && L > 0) {
      const uint32_t qa = smem_u32(sm + FwdSmem::Q);
      constexpr uint32_t id_s = idesc_bf16_f32(128, KB, 0, 0);
      constexpr uint32_t id_o = idesc_bf16_f32(128, HD, 0, 1);
      bool ok = mbar_wait(q_full, 0, 0xC20u, abort_flag);
      auto issue_s = [&](int l) -> bool {
        const int st = l & 1;
        if (!mbar_wait(&kv_full[st], (l >> 1) & 1, 0xC21u, abort_flag)) return false;
        tc_fence_after();
        const uint32_t kb = smem_u32(sm + FwdSmem::K0 + st * 2 * KBOX);
#pragma unroll
        for (int j = 0; j < 8; ++j) umma_bf16(t_s0 + st * 64, q_kmajor(qa, j), kb_kmajor(kb, j), id_s, j > 0);
        umma_commit(&s_full[st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int l = 0; l < L && ok; ++l) {
        const int st = l & 1;
        if (l + 1 < L && !issue_s(l + 1)) break;
        if (!mbar_wait(&p_full[st], (l >> 1) & 1, 0xC22u, abort_flag)) break;
        tc_fence_after();
        const uint32_t pb = smem_u32(sm + FwdSmem::P0 + st * QBOX);
        const uint32_t vb = smem_u32(sm + FwdSmem::V0 + st * 2 * KBOX);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          umma_bf16(t_o, smem_desc(pb + j * 32, 16, 1024), kb_mnmajor(vb, j), id_o, (l > 0 || j > 0) ? 1u : 0u);
        umma_commit(o_done);
        umma_commit(&kv_empty[st]);
      }
    }
  } else {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qpos = q0 + r;
    const uint32_t lrow = static_cast<uint32_t>(quad * 32) << 16;
    float m_used = -INFINITY, lsum = 0.f;
    int consumed = 0;  // completions of o_done observed (consumed == l or l - 1 at step l)
    bool ok = true;
    for (int l = 0; l < L && ok; ++l) {
      const int st = l & 1;
      if (!warp_wait(&s_full[st], (l >> 1) & 1, 0xC30u, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int k0 = p.lists[lbase + l] * KB;
      const uint32_t bit = (p.masks[(lbase + l) * 4 + (r >> 5)] >> (r & 31)) & 1u;
      float x[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t a[32];
        tmem_ld32(t_s0 + st * 64 + lrow + c * 32, a);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(a[i]) * p.scale_log2;
      }
      // keys past this row's position (or past T) and unselected blocks are masked
      const int lim = bit ? min(qpos, p.T - 1) - k0 : -1;
      if (p.rel && qpos < p.T) {
        // relative bias of row qpos at distances qpos - (k0 + i), i <= lim (contiguous, descending)
        const float* rrow = p.rel + ((static_cast<int64_t>(b) * p.H + h) * p.T + qpos) * p.rel_extent + (qpos - k0);
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i <= lim) x[i] += rrow[-i] * LOG2E;
      }
      float mx = -INFINITY;
      if (lim < KB - 1) {
#pragma unroll
        for (int i = 0; i < 64; ++i) x[i] = i <= lim ? x[i] : -INFINITY;
      }
#pragma unroll
      for (int i = 0; i < 64; ++i) mx = fmaxf(mx, x[i]);
      const float m_new = fmaxf(m_used, mx);
      const bool grow = m_new > m_used + 8.f;
      // o_done completes once per block.  Completion l - 1 is waited for here, at step l and before
      // this step's p_full arrival: completion l needs that arrival, so the barrier is in phase
      // l - 1 or l and the parity wait is unambiguous (a lazier wait could fall two phases behind).
      if (consumed < l) {
        if (!warp_wait(o_done, (l - 1) & 1, 0xC31u, abort_flag)) { ok = false; break; }
        consumed = l;
      }
      if (__any_sync(0xffffffffu, grow && m_used != -INFINITY)) {
        // rescale O: every product issued so far has landed (waited above)
        tc_fence_after();
        const float f = (grow && m_used != -INFINITY) ? fast_exp2(m_used - m_new) : 1.f;
#pragma unroll 1
        for (int c = 0; c < 8; ++c) {
          uint32_t a[16];
          tmem_ld16(t_o + lrow + c * 16, a);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) a[i] = __float_as_uint(__uint_as_float(a[i]) * f);
          tmem_st16(t_o + lrow + c * 16, a);
        }
        tmem_wait_st();
      }
      if (grow) {
        if (m_used != -INFINITY) lsum *= fast_exp2(m_used - m_new);
        m_used = m_new;
      }
      // the P buffer of this parity was last read by the product of block l - 2 (waited above)
      uint8_t* pb = sm + FwdSmem::P0 + st * QBOX;
      const float mu = m_used == -INFINITY ? 0.f : m_used;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float e[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          e[i] = fast_exp2(x[c * 8 + i] - mu);
          lsum += e[i];
        }
        *reinterpret_cast<uint4*>(pb + swz(r, c)) =
            make_uint4(pack_bf16x2(e[0], e[1]), pack_bf16x2(e[2], e[3]), pack_bf16x2(e[4], e[5]),
                       pack_bf16x2(e[6], e[7]));
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[st]);
    }
    if (ok && L > 0 && consumed < L) {
      // completion L - 1 (the last product); consumed == L - 1 here
      if (!warp_wait(o_done, (L - 1) & 1, 0xC33u, abort_flag)) ok = false;
      else consumed = L;
    }
    tc_fence_after();
    const bool live = qpos < p.T;
    const bool empty = !(lsum > 0.f);
    const float inv = empty ? 0.f : 1.f / lsum;
    __nv_bfloat16* orow = p.o + (static_cast<int64_t>(b) * p.T + (live ? qpos : 0)) * p.ldo + h * HD;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t a[32];
      if (L > 0 && ok) {
        tmem_ld32(t_o + lrow + c * 32, a);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) a[i] = 0u;
      }
      if (live) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(a[j * 8 + i]) * inv;
          *reinterpret_cast<uint4*>(orow + c * 32 + j * 8) =
              make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                         pack_bf16x2(f[6], f[7]));
        }
      }
    }
    if (live) {
      p.lse[(static_cast<int64_t>(b) * p.H + h) * p.T + qpos] =
          empty ? INFINITY : (m_used + __log2f(lsum)) / LOG2E;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
  }
}

// ------------------------------------------------------------------------------ backward
struct BwdSmem {
  static constexpr int Q = 0;
  static constexpr int DO = Q + 2 * QBOX;
  static constexpr int K0 = DO + 2 * QBOX;       // 2 stages x 16 KB
  static constexpr int V0 = K0 + 4 * KBOX;       // 2 stages x 16 KB
  static constexpr int P = V0 + 4 * KBOX;        // [128 rows x 64 keys] bf16
  static constexpr int DS = P + QBOX;
  static constexpr int STG = DS + QBOX;          // fp32 [64 keys x 128 features]: four [64 x 32] boxes
  static constexpr int BAR = STG + 4 * 8192;
  // qd_full kv_full[2] kv_empty[2] s_full ds_ready mma2_done dkv_free stg_full stg_free
  static constexpr int NBAR = 11;
  static constexpr int TOTAL = BAR + NBAR * 8 + 16 + 1024;
};
static_assert(BwdSmem::TOTAL <= 232448, "block-sparse backward shared memory");

__global__ void __launch_bounds__(320, 1)
    bsa_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                   const __grid_constant__ CUtensorMap tmDK, const __grid_constant__ CUtensorMap tmDV, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BwdSmem::BAR);
  uint64_t* qd_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* ds_ready = bars + 6;
  uint64_t* mma2_done = bars + 7;
  uint64_t* dkv_free = bars + 8;
  uint64_t* stg_full = bars + 9;
  uint64_t* stg_free = bars + 10;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + BwdSmem::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.H / p.Hk);
  const int q0 = qt * QT;
  const int lbase = list_base(p, b, h, qt);
  const int L = list_len(p, lbase);

  if (threadIdx.x == 0) {
    mbar_init(qd_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(ds_ready, 128);
    mbar_init(mma2_done, 1);
    mbar_init(dkv_free, 128);
    mbar_init(stg_full, 128);
    mbar_init(stg_free, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const uint32_t t_s = tbase, t_dp = tbase + 64, t_dq = tbase + 128, t_dv = tbase + 256, t_dk = tbase + 320;

  if (warp == 0) {
    if (lane == 0 && L > 0) {
      mbar_expect_tx(qd_full, 4 * QBOX);
      tma_load_3d(sm + BwdSmem::Q, &tmQ, qd_full, h * HD, q0, b);
      tma_load_3d(sm + BwdSmem::Q + QBOX, &tmQ, qd_full, h * HD + 64, q0, b);
      tma_load_3d(sm + BwdSmem::DO, &tmDO, qd_full, h * HD, q0, b);
      tma_load_3d(sm + BwdSmem::DO + QBOX, &tmDO, qd_full, h * HD + 64, q0, b);
      int issued = 0;
      for (int l = 0; l < L; ++l) {
        const int st = l & 1;
        if (!mbar_wait(&kv_empty[st], ((l >> 1) & 1) ^ 1u, 0xD00u + st, abort_flag)) break;
        const int k0 = p.lists[lbase + l] * KB;
        mbar_expect_tx(&kv_full[st], 4 * KBOX);
        uint8_t* kd = sm + BwdSmem::K0 + st * 2 * KBOX;
        uint8_t* vd = sm + BwdSmem::V0 + st * 2 * KBOX;
        tma_load_3d(kd, &tmK, &kv_full[st], hk * HD, k0, b);
        tma_load_3d(kd + KBOX, &tmK, &kv_full[st], hk * HD + 64, k0, b);
        tma_load_3d(vd, &tmV, &kv_full[st], hk * HD, k0, b);
        tma_load_3d(vd + KBOX, &tmV, &kv_full[st], hk * HD + 64, k0, b);
        ++issued;
      }
      mbar_wait(qd_full, 0, 0xD10u, nullptr);
      for (int l = (issued > 2 ? issued - 2 : 0); l < issued; ++l)
        mbar_wait(&kv_full[l & 1], (l >> 1) & 1, 0xD11u, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0 && L > 0) {
      const uint32_t qa = smem_u32(sm + BwdSmem::Q), da = smem_u32(sm + BwdSmem::DO);
      const uint32_t pa = smem_u32(sm + BwdSmem::P), sa = smem_u32(sm + BwdSmem::DS);
      constexpr uint32_t id_s = idesc_bf16_f32(128, KB, 0, 0);
      constexpr uint32_t id_dq = idesc_bf16_f32(128, HD, 0, 1);
      constexpr uint32_t id_t = idesc_bf16_f32(128, KB, 1, 1);
      bool ok = mbar_wait(qd_full, 0, 0xD20u, abort_flag);
      for (int l = 0; l < L && ok; ++l) {
        const int st = l & 1;
        if (!mbar_wait(&kv_full[st], (l >> 1) & 1, 0xD21u, abort_flag)) break;
        if (l > 0 && !mbar_wait(ds_ready, (l - 1) & 1, 0xD22u, abort_flag)) break;
        tc_fence_after();
        const uint32_t kb = smem_u32(sm + BwdSmem::K0 + st * 2 * KBOX);
        const uint32_t vb = smem_u32(sm + BwdSmem::V0 + st * 2 * KBOX);
#pragma unroll
        for (int j = 0; j < 8; ++j) umma_bf16(t_s, q_kmajor(qa, j), kb_kmajor(kb, j), id_s, j > 0);
#pragma unroll
        for (int j = 0; j < 8; ++j) umma_bf16(t_dp, q_kmajor(da, j), kb_kmajor(vb, j), id_s, j > 0);
        umma_commit(s_full);
        if (!mbar_wait(ds_ready, l & 1, 0xD23u, abort_flag)) break;
        if (l > 0 && !mbar_wait(dkv_free, (l - 1) & 1, 0xD24u, abort_flag)) break;
        tc_fence_after();
        // dQ += dS K
#pragma unroll
        for (int j = 0; j < 4; ++j)
          umma_bf16(t_dq, smem_desc(sa + j * 32, 16, 1024), kb_mnmajor(kb, j), id_dq, (l > 0 || j > 0) ? 1u : 0u);
        // dV^T = dO^T P ; dK^T = Q^T dS   (M = 128 features, N = 64 keys, reduction over the 128 rows)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          umma_bf16(t_dv, smem_desc(da + j * 2048, QBOX, 1024), smem_desc(pa + j * 2048, 8192, 1024), id_t, j > 0);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          umma_bf16(t_dk, smem_desc(qa + j * 2048, QBOX, 1024), smem_desc(sa + j * 2048, 8192, 1024), id_t, j > 0);
        umma_commit(mma2_done);
        umma_commit(&kv_empty[st]);
      }
    }
  } else if (warp < 6) {
    // softmax: one query row per thread
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qpos = q0 + r;
    const bool live = qpos < p.T;
    const uint32_t lrow = static_cast<uint32_t>(quad * 32) << 16;
    const int64_t srow = (static_cast<int64_t>(b) * p.H + h) * p.T + (live ? qpos : 0);
    const float lse2 = live ? p.lse[srow] * LOG2E : INFINITY;
    const float dlt = live ? p.delta[srow] : 0.f;
    bool ok = true;
    for (int l = 0; l < L; ++l) {
      if (!warp_wait(s_full, l & 1, 0xD30u, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int k0 = p.lists[lbase + l] * KB;
      const uint32_t bit = (p.masks[(lbase + l) * 4 + (r >> 5)] >> (r & 31)) & 1u;
      const int lim = (bit && live && lse2 != INFINITY) ? min(qpos, p.T - 1) - k0 : -1;
      // the P / dS buffers were last read by the products of block l - 1
      if (l > 0 && !warp_wait(mma2_done, (l - 1) & 1, 0xD31u, abort_flag)) { ok = false; break; }
      uint8_t* pbuf = sm + BwdSmem::P;
      uint8_t* sbuf = sm + BwdSmem::DS;
      const float* rrow = nullptr;
      float* drow = nullptr;
      if (p.rel && live) {
        const int64_t off = ((static_cast<int64_t>(b) * p.H + h) * p.T + qpos) * p.rel_extent + (qpos - k0);
        rrow = p.rel + off;
        drow = p.drel + off;
      }
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t a[32];
        float pr[32];
        tmem_ld32(t_s + lrow + c * 32, a);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) pr[i] = __uint_as_float(a[i]) * p.scale_log2 - lse2;
        if (rrow) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i <= lim) pr[i] += rrow[-(c * 32 + i)] * LOG2E;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) pr[i] = c * 32 + i <= lim ? fast_exp2(pr[i]) : 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(pbuf + swz(r, c * 4 + j)) =
              make_uint4(pack_bf16x2(pr[j * 8], pr[j * 8 + 1]), pack_bf16x2(pr[j * 8 + 2], pr[j * 8 + 3]),
                         pack_bf16x2(pr[j * 8 + 4], pr[j * 8 + 5]), pack_bf16x2(pr[j * 8 + 6], pr[j * 8 + 7]));
        tmem_ld32(t_dp + lrow + c * 32, a);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) pr[i] *= __uint_as_float(a[i]) - dlt;   // dL / d(logit)
        if (drow) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c * 32 + i <= lim) drow[-(c * 32 + i)] = pr[i];
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) pr[i] *= p.scale;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(sbuf + swz(r, c * 4 + j)) =
              make_uint4(pack_bf16x2(pr[j * 8], pr[j * 8 + 1]), pack_bf16x2(pr[j * 8 + 2], pr[j * 8 + 3]),
                         pack_bf16x2(pr[j * 8 + 4], pr[j * 8 + 5]), pack_bf16x2(pr[j * 8 + 6], pr[j * 8 + 7]));
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    if (ok && L > 0 && !warp_wait(mma2_done, (L - 1) & 1, 0xD32u, abort_flag)) ok = false;
    tc_fence_after();
    // the aligned TMEM loads run on every lane (warp-uniform condition); only live rows store
    __nv_bfloat16* drow = p.dq + (static_cast<int64_t>(b) * p.T + (live ? qpos : 0)) * p.lddq + h * HD;
    const bool have = L > 0 && ok;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t a[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = 0u;
      if (have) {
        tmem_ld32(t_dq + lrow + c * 32, a);
        tmem_wait_ld();
      }
      if (live) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          *reinterpret_cast<uint4*>(drow + c * 32 + j * 8) =
              make_uint4(pack_bf16x2(__uint_as_float(a[j * 8]), __uint_as_float(a[j * 8 + 1])),
                         pack_bf16x2(__uint_as_float(a[j * 8 + 2]), __uint_as_float(a[j * 8 + 3])),
                         pack_bf16x2(__uint_as_float(a[j * 8 + 4]), __uint_as_float(a[j * 8 + 5])),
                         pack_bf16x2(__uint_as_float(a[j * 8 + 6]), __uint_as_float(a[j * 8 + 7])));
      }
    }
  } else {
    // drain: feature row d of dV^T / dK^T per thread, transposed into the fp32 staging boxes
    const int quad = warp & 3;
    const int d = quad * 32 + lane;
    const uint32_t lrow = static_cast<uint32_t>(quad * 32) << 16;
    const bool leader = threadIdx.x == 192;
    uint8_t* stg = sm + BwdSmem::STG;
    int rounds = 0;
    for (int l = 0; l < L; ++l) {
      if (!warp_wait(mma2_done, l & 1, 0xD40u, abort_flag)) break;
      tc_fence_after();
      const int k0 = p.lists[lbase + l] * KB;
      bool ok = true;
#pragma unroll 1
      for (int which = 0; which < 2 && ok; ++which, ++rounds) {
        const uint32_t tsrc = which == 0 ? t_dv : t_dk;
        if (!warp_wait(stg_free, (rounds & 1) ^ 1u, 0xD41u, abort_flag)) { ok = false; break; }
        uint8_t* box = stg + (d >> 5) * 8192 + (d & 3) * 4;
        const int ch = (d & 31) >> 2;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t a[32];
          tmem_ld32(tsrc + lrow + c * 32, a);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int key = c * 32 + i;
            *reinterpret_cast<float*>(box + key * 128 + ((ch ^ (key & 7)) << 4)) = __uint_as_float(a[i]);
          }
        }
        if (which == 1) {  // both accumulators have been read: the MMA may reuse them
          tc_fence_before();
          mbar_arrive(dkv_free);
        }
        fence_proxy_async_smem();
        mbar_arrive(stg_full);
        int lok = 1;
        if (leader) {
          lok = mbar_wait(stg_full, rounds & 1, 0xD42u, abort_flag) ? 1 : 0;
          if (lok) {
            const CUtensorMap* map = which == 0 ? &tmDV : &tmDK;
#pragma unroll
            for (int bx = 0; bx < 4; ++bx) tma_reduce_add_3d(map, stg + bx * 8192, hk * HD + bx * 32, k0, b);
            tma_store_commit();
            tma_store_wait_read0();
            mbar_arrive(stg_free);
          }
        }
        // the leader's outcome is its whole warp's (the others learn of a failure from their own waits)
        if (warp == 6) ok = __shfl_sync(0xffffffffu, lok, 0) != 0;
      }
      if (!ok) break;
    }
    if (leader) tma_store_wait0();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------------------ host
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// bf16 [B, T, cols] with row stride ld: dims {cols, T, B}, box {64, rows, 1}, 128B swizzle.
CUtensorMap row_map(const void* base, int64_t cols, int64_t ld, int T, int B, int rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || (ld * 2) % 16) throw std::runtime_error("sparse attention alignment");
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(ld * 2 * T)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(rows), 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (sparse attention) failed: " + std::to_string(int(r)));
  return m;
}

// fp32 [B, T, cols] accumulator: dims {cols, T, B}, box {32, 64, 1}, 128B swizzle.
CUtensorMap acc_map(float* base, int64_t cols, int T, int B) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || cols % 4) throw std::runtime_error("sparse attention dK/dV alignment");
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols * 4), static_cast<cuuint64_t>(cols * 4 * T)};
  cuuint32_t box[3] = {32u, 64u, 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (sparse dK/dV) failed: " + std::to_string(int(r)));
  return m;
}

Params make_params(const SparseAttnArgs& a) {
  Params p{};
  p.B = a.B; p.T = a.T; p.H = a.H; p.Hk = a.Hk; p.G = a.G; p.Lmax = a.Lmax;
  p.n_qt = (a.T + QT - 1) / QT;
  p.scale = a.scale;
  p.scale_log2 = a.scale * LOG2E;
  p.lists = a.lists;
  p.masks = a.masks;
  p.o = a.o; p.ldo = a.ldo;
  p.lse = a.lse;
  p.delta = a.delta;
  p.dq = a.dq; p.lddq = a.lddq;
  p.rel = a.rel;
  p.drel = a.drel;
  p.rel_extent = a.rel_extent;
  return p;
}

}  // namespace bsa
}  // namespace nt

using namespace nt::bsa;

int nt_sparse_attn_fwd(const SparseAttnArgs& a, cudaStream_t s) {
  nt::current_context();
  if (a.D != HD || a.H % a.Hk || a.H % a.G || a.Lmax <= 0 || a.T <= 0) return -1;
  if (a.rel && a.rel_extent < a.T) return -1;
  const Params p = make_params(a);
  const CUtensorMap tq = row_map(a.q, static_cast<int64_t>(a.H) * HD, a.ldq, a.T, a.B, QT);
  const CUtensorMap tk = row_map(a.k, static_cast<int64_t>(a.Hk) * HD, a.ldk, a.T, a.B, KB);
  const CUtensorMap tv = row_map(a.v, static_cast<int64_t>(a.Hk) * HD, a.ldv, a.T, a.B, KB);
  static std::atomic<uint64_t> smem_set{0};
  nt::smem_limit(smem_set, bsa_fwd_kernel, FwdSmem::TOTAL);
  bsa_fwd_kernel<<<dim3(p.n_qt, a.H, a.B), 192, FwdSmem::TOTAL, s>>>(tq, tk, tv, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int nt_sparse_attn_bwd(const SparseAttnArgs& a, cudaStream_t s) {
  nt::current_context();
  if (a.D != HD || a.H % a.Hk || a.H % a.G || a.Lmax <= 0 || a.T <= 0) return -1;
  if (a.rel && (a.rel_extent < a.T || !a.drel)) return -1;
  const Params p = make_params(a);
  const CUtensorMap tq = row_map(a.q, static_cast<int64_t>(a.H) * HD, a.ldq, a.T, a.B, QT);
  const CUtensorMap tk = row_map(a.k, static_cast<int64_t>(a.Hk) * HD, a.ldk, a.T, a.B, KB);
  const CUtensorMap tv = row_map(a.v, static_cast<int64_t>(a.Hk) * HD, a.ldv, a.T, a.B, KB);
  const CUtensorMap td = row_map(a.dout, static_cast<int64_t>(a.H) * HD, a.lddo, a.T, a.B, QT);
  const CUtensorMap tdk = acc_map(a.dk_acc, static_cast<int64_t>(a.Hk) * HD, a.T, a.B);
  const CUtensorMap tdv = acc_map(a.dv_acc, static_cast<int64_t>(a.Hk) * HD, a.T, a.B);
  static std::atomic<uint64_t> smem_set{0};
  nt::smem_limit(smem_set, bsa_bwd_kernel, BwdSmem::TOTAL);
  bsa_bwd_kernel<<<dim3(p.n_qt, a.H, a.B), 320, BwdSmem::TOTAL, s>>>(tq, tk, tv, td, tdk, tdv, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int nt_sparse_attn_read_error(unsigned* where) {
  nt::ErrorWord e{};
  cudaMemcpyFromSymbol(&e, nt::g_nt_error, sizeof(e));
  if (where) *where = e.where;
  if (e.code) {
    const nt::ErrorWord z{};
    cudaMemcpyToSymbol(nt::g_nt_error, &z, sizeof(z));
  }
  return static_cast<int>(e.code);
}
