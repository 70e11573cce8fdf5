// K1: flash attention for sm_100a (causal, optional left window, GQA, head dim 128).
//
// Forward (one CTA per (query tile of 128, head, batch); 192 threads):
//   warp 0      TMA: the Q tile once, then K/V tiles (128 keys) into a 2-stage ring.
//   warp 1      TMEM owner and MMA issuer: S_t = Q K_t^T into one of two TMEM S buffers
//               (issued one tile ahead), then O += P_{t-1} V_{t-1} into the TMEM O accumulator.
//   warps 2..5  softmax, one query row per thread: tcgen05.ld of the S row, online softmax in
//               the log2 domain, lazy rescaling of O in TMEM (only when the running max grows by
//               more than 2^8), P written to shared memory in the 128-byte-swizzled K-major
//               layout the next MMA reads; at the end O / l and the log-sum-exp are stored.
// Backward (one CTA per (key tile of 128, KV head, batch)), loops over the query heads of the
// KV group and the query tiles that see the key tile:
//   S^T = K Q^T and dP^T = V dO^T in TMEM; one thread per key row forms P^T and
//   dS^T = P^T (dP^T - delta) in shared memory; dV += P^T dO and dK += dS^T Q accumulate in
//   TMEM over the whole loop; dQ = dS K lands in TMEM and is added to an fp32 buffer with
//   vector atomics.  Small kernels compute delta = rowsum(dO * O) and convert dQ to bf16.
// Every mbarrier wait is bounded (see common.cuh).  No TMA load uses cluster multicast.
#include "attention_sm100.h"
#include "common.cuh"

#include <type_traits>

#include <cudaTypedefs.h>
#include <math.h>
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <string>

namespace nt {
namespace attn {

constexpr int TILE = 128;
constexpr int HD = 128;
constexpr int BOX_BYTES = TILE * 64 * 2;      // [128 rows x 64 bf16] = 16 KB
constexpr int TILE_BYTES = 2 * BOX_BYTES;     // [128 rows x 128 bf16] = 32 KB
constexpr float LOG2E = 1.4426950408889634f;

struct Params {
  int B, T, H, Hk;
  int window;
  float scale_log2;  // softmax scale * log2(e)
  float scale;
  __nv_bfloat16* o;
  int64_t ldo;
  float* lse;
  // backward
  const __nv_bfloat16* dout;
  int64_t lddo;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t lddk, lddv;
  float* dq_acc;
  const float* delta;
  long long* trace;
  int dq_slices;  // 0: dQ added into one fp32 buffer (bulk reductions); else one slice per key tile
  int dq_direct;  // drain: 0 staged bulk reductions, 1 register reductions only, 2 half and half
  float* dq_base; // dq_acc (row stride H * 128) for the direct drain
  int order_window;  // CTA order: 0 = (batch, head)-major; W > 0 = longest first within W (batch, head) groups
};

// Clock stamp of (role, pair, event) for the first CTA when a trace buffer is given.
NT_DEVICE void stamp(const Params& p, int role, int it, int ev) {
  if (p.trace && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && it < 64)
    p.trace[(role * 64 + it) * 8 + ev] = clock64();
}

// K-major operand made of two [128 rows x 64] swizzled boxes; k-step j covers 16 columns.
NT_DEVICE uint64_t kmajor_desc(uint32_t base, int j) {
  return smem_desc(base + (j >> 2) * BOX_BYTES + (j & 3) * 32, 16, 1024);
}
// MN-major operand: rows are the reduction index (128 rows), two 64-wide MN boxes.
NT_DEVICE uint64_t mnmajor_desc(uint32_t base, int j) {
  return smem_desc(base + j * 2048, BOX_BYTES, 1024);
}

// Byte offsets of k-step j from step 0 in the two operand forms above.  An MMA loop builds the step-0
// descriptor once and adds offset >> 4 to its start-address field (address >> 4 in 14 bits; every tile
// lies below 256 KB, so the sum never carries out of the field): fully unrolled, the issuing thread
// spends no instructions on descriptors between MMAs.
__host__ __device__ constexpr uint32_t kmajor_step(int j) { return ((j >> 2) * BOX_BYTES + (j & 3) * 32) >> 4; }
__host__ __device__ constexpr uint32_t mnmajor_step(int j) { return (j * 2048) >> 4; }

// The MMAs of one k-step loop: step-0 descriptors plus immediate steps, added inside the asm statement
// so that the compiler neither keeps every step's descriptor live across the loop nor spends
// registers of the issuing warp (which runs with few after its register split) on them.
template <uint32_t SA, uint32_t SB>
NT_DEVICE void umma_step(uint32_t tmem_d, uint64_t a0, uint64_t b0, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "add.s64 da, %1, %5;\n\t"
      "add.s64 db, %2, %6;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a0), "l"(b0), "r"(idesc), "r"(accumulate), "n"(static_cast<uint64_t>(SA)), "n"(static_cast<uint64_t>(SB))
      : "memory");
}
// The same with A read from tensor memory at column offset TA.
template <uint32_t TA, uint32_t SB>
NT_DEVICE void umma_step_tmem_a(uint32_t tmem_d, uint32_t tmem_a0, uint64_t b0, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 ta;\n\t.reg .b64 db;\n\t"
      "add.u32 ta, %1, %5;\n\t"
      "add.s64 db, %2, %6;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], db, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a0), "l"(b0), "r"(idesc), "r"(accumulate), "n"(TA), "n"(static_cast<uint64_t>(SB))
      : "memory");
}
// Eight k-steps (K = 128) of one operand-form pair, unrolled at compile time.
template <int J = 0, class F>
NT_DEVICE void for_steps(F&& f) {
  if constexpr (J < 8) {
    f(std::integral_constant<int, J>{});
    for_steps<J + 1>(f);
  }
}

// Byte offset of 16-byte chunk `c` (0..15) of row `r` in a two-box 128B-swizzled tile.
// Work unit of flat block index x for `units` work units per (batch, head) group, `groups` groups,
// unit 0 the longest.  Window 0: group-major (a group's units run together, so their shared tiles stay
// in L2).  Window W: longest first within each run of W groups, which keeps long CTAs out of the
// grid's tail while W groups' tiles share L2.
NT_DEVICE void work_unit(int x, int units, int groups, int window, int& unit, int& group) {
  if (window <= 0) {
    unit = x % units;
    group = x / units;
    return;
  }
  const int span = window * units;
  const int w = x / span, local = x - w * span;
  const int wl = min(window, groups - w * window);
  unit = local / wl;
  group = w * window + local % wl;
}

NT_DEVICE uint32_t swz_off(int r, int c) {
  return (c >> 3) * BOX_BYTES + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

// 2^x with the SFU's approximate base-2 exponential (ex2.approx.ftz: inputs far below -126 give 0).
NT_DEVICE float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for a pair on the FMA pipe instead of the MUFU unit, which caps the softmax at 16
// exponentials per clock per SM.  Range reduction to the nearest integer j (adding 1.5 x 2^23
// rounds x into the low mantissa bits), then 2^f for f in [-1/2, 1/2] by a cubic fitted here for
// minimum relative error (Lawson-weighted least squares; max relative error 7.5e-5, below bf16's
// 2^-9 rounding of P), and j added to the exponent field.  The split of a softmax between this and
// ex2.approx follows the FlashAttention-4 write-up (software exponentials on the FMA units).
// Inputs are clamped at -125 (2^-125 stands in for 0: far below any row maximum's share).
NT_DEVICE float2 exp2_fma2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 x 2^23
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 t = add2(x, make_float2(kRound, kRound));
  const float2 r = add2(t, make_float2(-kRound, -kRound));
  const float2 f = add2(x, make_float2(-r.x, -r.y));
  float2 q = fma2(make_float2(0.05517166853f, 0.05517166853f), f, make_float2(0.24261112511f, 0.24261112511f));
  q = fma2(q, f, make_float2(0.69326096773f, 0.69326096773f));
  q = fma2(q, f, make_float2(0.99992805719f, 0.99992805719f));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}
// Of every 8 exponential pairs of a softmax row, FWD_EMU go to exp2_fma2 (the rest to MUFU);
// NT_ATTN_FWD_EMU selects another compiled split (0, 2, 3 or 4) for measurement.
constexpr int FWD_EMU_DEFAULT = 0;

// ------------------------------------------------------------------------------ forward
// One CTA per pair of consecutive query tiles (A = 2c, B = 2c + 1) of one (head, batch); 320 threads.
// The two tiles share every K/V tile load, and their softmax warpgroups alternate with the MMAs:
//   warp 0      TMA: Q_A, Q_B once, then K/V tiles into a 2-stage ring.
//   warp 1      TMEM owner and MMA issuer: S_A = Q_A K^T, S_B = Q_B K^T, O_A += P_A V (P from tensor
//               memory), S_A of the next key tile, O_B += P_B V, S_B of the next key tile, ...
//   warps 2..5  softmax of tile A, warps 6..9 softmax of tile B, one query row per thread: row max
//               over the S row (first pass), then P = exp2(S - m) written back over the first 64
//               columns of S as bf16 (second pass), lazy rescaling of O only when the running max
//               grows by more than 2^8; at the end O / l goes out through shared memory (the tile's Q
//               buffer, whose last reader has finished) with a bulk tensor store, and the lse.
// Tensor memory: O_A [0,128) | O_B [128,256) | S_A [256,384) | S_B [384,512).
// Under the causal mask tile A has one key tile less than B (the diagonal tile of B).
struct FwdSmem {
  static constexpr int QA = 0;
  static constexpr int QB = QA + TILE_BYTES;
  static constexpr int K0 = QB + TILE_BYTES;      // 2 stages
  static constexpr int V0 = K0 + 2 * TILE_BYTES;  // 2 stages
  static constexpr int BAR = V0 + 2 * TILE_BYTES;
  // q_full, kv_full[2], kv_empty[2], s_full[2], p_full[2], o_done[2]
  static constexpr int NBAR = 11;
  static constexpr int TOTAL = BAR + NBAR * 8 + 32 + 1024;  // + tmem holder, abort and veto flags
};
static_assert(FwdSmem::TOTAL <= 232448, "forward shared memory exceeds the sm_100 limit");
// 12 warps in three warpgroups: warpgroup 0 = TMA producer (warp 0), MMA issuer (warp 1) and two
// idle warps; warpgroups 1 and 2 = the softmax of query tiles A and B.  Launched at 168 registers a
// thread (the most 384 threads may hold); warpgroup 0 gives registers back so each softmax thread
// can keep a whole 128-key S row in registers: 128 x FWD_REGS_LOW + 256 x FWD_REGS_HIGH = 384 x 168.
constexpr int FWD_THREADS = 384;
constexpr uint32_t FWD_REGS_LAUNCH = 168;
constexpr uint32_t FWD_REGS_LOW = 56;
constexpr uint32_t FWD_REGS_HIGH = 224;
static_assert(128 * FWD_REGS_LOW + 256 * FWD_REGS_HIGH <= FWD_THREADS * FWD_REGS_LAUNCH,
              "forward register split exceeds the launch budget");

// Key-tile range [lo, hi] of query tile qt (causal, optional left window); empty when qt is past T.
NT_DEVICE void fwd_kv_range(const Params& p, int qt, int& lo, int& hi) {
  const int q0 = qt * TILE;
  lo = 0;
  if (p.window >= 0) lo = max(0, (q0 - p.window) / TILE);
  hi = qt;
}

template <int FWD_EMU>
__global__ void __launch_bounds__(FWD_THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + FwdSmem::BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [A, B]
  uint64_t* p_full = bars + 7;    // [A, B]
  uint64_t* o_done = bars + 9;    // [A, B]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + FwdSmem::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [abort, veto A, veto B]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.T + TILE - 1) / TILE;
  const int n_pairs = (n_qt + 1) / 2;
  int unit, bh;  // unit 0 = the last (longest) query-tile pair
  work_unit(static_cast<int>(blockIdx.x), n_pairs, p.H * p.B, p.order_window, unit, bh);
  const int pair = n_pairs - 1 - unit;
  const int h = bh % p.H, b = bh / p.H;
  const int hk = h / (p.H / p.Hk);
  const int qtA = 2 * pair, qtB = 2 * pair + 1;
  const bool hasB = qtB < n_qt;
  int loA, hiA, loB = 0, hiB = -1;
  fwd_kv_range(p, qtA, loA, hiA);
  if (hasB) fwd_kv_range(p, qtB, loB, hiB);
  const int j_lo = loA, j_hi = hasB ? hiB : hiA;  // loA <= loB, hiA < hiB
  const int n_kv = j_hi - j_lo + 1;
  const int nA = hiA - loA + 1, nB = hasB ? hiB - loB + 1 : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    abort_flag[0] = 0;
    abort_flag[1] = 0;
    abort_flag[2] = 0;
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
  if (warp < 4) {
   setmaxnreg_dec<FWD_REGS_LOW>();
   if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_expect_tx(q_full, (hasB ? 2 : 1) * TILE_BYTES);
      tma_load_3d(sm + FwdSmem::QA, &tmQ, q_full, h * HD, qtA * TILE, b);
      tma_load_3d(sm + FwdSmem::QA + BOX_BYTES, &tmQ, q_full, h * HD + 64, qtA * TILE, b);
      if (hasB) {
        tma_load_3d(sm + FwdSmem::QB, &tmQ, q_full, h * HD, qtB * TILE, b);
        tma_load_3d(sm + FwdSmem::QB + BOX_BYTES, &tmQ, q_full, h * HD + 64, qtB * TILE, b);
      }
      int issued = 0;
      for (int t = 0; t < n_kv; ++t) {
        const int st = t & 1;
        if (!mbar_wait(&kv_empty[st], ((t >> 1) & 1) ^ 1u, 0x10u + st, abort_flag)) break;
        const int k0 = (j_lo + t) * TILE;
        uint8_t* ks = sm + FwdSmem::K0 + st * TILE_BYTES;
        uint8_t* vs = sm + FwdSmem::V0 + st * TILE_BYTES;
        mbar_expect_tx(&kv_full[st], 2 * TILE_BYTES);
        tma_load_3d(ks, &tmK, &kv_full[st], hk * HD, k0, b);
        tma_load_3d(ks + BOX_BYTES, &tmK, &kv_full[st], hk * HD + 64, k0, b);
        tma_load_3d(vs, &tmV, &kv_full[st], hk * HD, k0, b);
        tma_load_3d(vs + BOX_BYTES, &tmV, &kv_full[st], hk * HD + 64, k0, b);
        ++issued;
      }
      mbar_wait(q_full, 0, 0x1Fu, nullptr);
      for (int t = max(0, issued - 2); t < issued; ++t) mbar_wait(&kv_full[t & 1], (t >> 1) & 1, 0x1Du, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(TILE, TILE, 0, 0);   // S = Q K^T
      constexpr uint32_t idesc_pv = idesc_bf16_f32(TILE, HD, 0, 1);    // O += P V  (P from tensor memory)
      const uint32_t qa_addr = smem_u32(sm + FwdSmem::QA), qb_addr = smem_u32(sm + FwdSmem::QB);
      const uint32_t t_oA = tbase, t_oB = tbase + 128, t_sA = tbase + 256, t_sB = tbase + 384;
      int iA = 0, iB = 0;  // S tiles issued per query tile
      int uA = 0, uB = 0;  // PV products issued per query tile
      bool ok = mbar_wait(q_full, 0, 0x20u, abort_flag);
      // S_X of key tile t for query tile X (0: A, 1: B) when X sees that tile
      auto sees = [&](int X, int t) -> bool {
        const int j = j_lo + t;
        return X == 0 ? (j >= loA && j <= hiA) : (hasB && j >= loB && j <= hiB);
      };
      auto issue_s = [&](int X, int t) -> bool {
        const int st = t & 1;
        if (!mbar_wait(&kv_full[st], (t >> 1) & 1, 0x21u, abort_flag)) return false;
        stamp(p, 1, t, 4 + X);
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm + FwdSmem::K0 + st * TILE_BYTES);
        const uint32_t qx = X ? qb_addr : qa_addr, tsx = X ? t_sB : t_sA;
        const uint64_t da = kmajor_desc(qx, 0), db = kmajor_desc(k_addr, 0);
        for_steps([&](auto q) {
          constexpr int Q = decltype(q)::value;
          umma_step<kmajor_step(Q), kmajor_step(Q)>(tsx, da, db, idesc_s, Q > 0);
        });
        umma_commit(&s_full[X]);
        stamp(p, 1, t, X);
        if (X) ++iB; else ++iA;
        return true;
      };
      auto issue_pv = [&](int X, int t) -> bool {
        int& u = X ? uB : uA;
        if (!mbar_wait(&p_full[X], u & 1, 0x23u + X, abort_flag)) return false;
        stamp(p, 1, t, 6 + X);
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm + FwdSmem::V0 + (t & 1) * TILE_BYTES);
        const uint32_t tox = X ? t_oB : t_oA, tsx = X ? t_sB : t_sA;
        const uint64_t dv = mnmajor_desc(v_addr, 0);
        const uint32_t acc0 = u > 0 ? 1u : 0u;
        for_steps([&](auto q) {
          constexpr int Q = decltype(q)::value;
          umma_step_tmem_a<Q * 8, mnmajor_step(Q)>(tox, tsx, dv, idesc_pv, Q > 0 ? 1u : acc0);
        });
        umma_commit(&o_done[X]);
        stamp(p, 1, t, 2 + X);
        ++u;
        return true;
      };
      // Order: S_A(0) S_B(0) | PV_A(t) S_A(t+1) PV_B(t) S_B(t+1) | ...  Each tile's next S follows its own
      // PV at once, so one warpgroup's softmax overlaps the other tile's PV and S.  S_X(t+1) overwrites
      // the columns P_X(t) occupies; it is issued after PV_X(t), and MMAs from one thread run in order.
      if (ok && n_kv > 0) {
        if (sees(0, 0)) ok = issue_s(0, 0);
        if (ok && sees(1, 0)) ok = issue_s(1, 0);
      }
      for (int t = 0; ok && t < n_kv; ++t) {
        for (int X = 0; ok && X < 2; ++X) {
          if (sees(X, t)) ok = issue_pv(X, t);
          if (ok && t + 1 < n_kv && sees(X, t + 1)) ok = issue_s(X, t + 1);
        }
        if (ok) umma_commit(&kv_empty[t & 1]);
      }
      (void)iA;
      (void)iB;
    }
   }
  } else {
    setmaxnreg_inc<FWD_REGS_HIGH>();
    // ------------------------------------------------------------ softmax warpgroups
    const int grp = warp < 8 ? 0 : 1;  // 0: tile A, 1: tile B
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int qt = grp ? qtB : qtA;
    const int lo = grp ? loB : loA;
    const int n = grp ? nB : nA;
    const int q0 = qt * TILE;
    const int qi = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t t_o = tbase + grp * 128, t_s = tbase + 256 + grp * 128;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n; ++i) {
      const int k0 = (lo + i) * TILE;
      if (!mbar_wait(&s_full[grp], i & 1, 0x30u, abort_flag)) { ok = false; break; }
      if (r == 0) stamp(p, 2 + grp, i, 0);
      __syncwarp();
      tc_fence_after();
      const bool boundary = (k0 + TILE - 1 > q0) || (k0 + TILE > p.T) ||
                            (p.window >= 0 && q0 + TILE - 1 - k0 > p.window);
      // the whole S row (128 keys) comes into registers with four loads and one wait; it is read
      // from tensor memory once, scaled (log2 domain) and masked in place
      uint32_t v[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(t_s + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&v[c * 32]));
      tmem_wait_ld();
      if (r == 0) stamp(p, 2 + grp, i, 1);
      if (boundary) {
#pragma unroll
        for (int e = 0; e < 128; ++e) {
          const int kj = k0 + e;
          const bool keep = kj <= qi && kj < p.T && (p.window < 0 || qi - kj <= p.window);
          if (!keep) v[e] = __float_as_uint(-INFINITY);
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int e = 0; e < 128; e += 4) {
        mx0 = fmaxf(mx0, __uint_as_float(v[e]));
        mx1 = fmaxf(mx1, __uint_as_float(v[e + 1]));
        mx2 = fmaxf(mx2, __uint_as_float(v[e + 2]));
        mx3 = fmaxf(mx3, __uint_as_float(v[e + 3]));
      }
      // raw scores are scaled after the max (the scale is positive)
      const float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * p.scale_log2;
      // lazy rescale: keep the old reference max unless the row grew by more than 2^8
      float m_new = m;
      if (i == 0 || mx > m + 8.f) m_new = fmaxf(m, mx);
      const float alpha = (i == 0 || m_new == m) ? 1.f : fast_exp2(m - m_new);
      const float mref = (m_new == -INFINITY) ? 0.f : m_new;
      if (r == 0) stamp(p, 2 + grp, i, 2);
      if (i > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        // O holds every earlier product: wait for the last one, then scale O in place
        if (!mbar_wait(&o_done[grp], (i - 1) & 1, 0x31u, abort_flag)) { ok = false; break; }
        __syncwarp();
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t w[32];
          tmem_ld32(t_o + lane_off + c * 32, w);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) w[e] = __float_as_uint(__uint_as_float(w[e]) * alpha);
          tmem_st16(t_o + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[16]>(&w[0]));
          tmem_st16(t_o + lane_off + c * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&w[16]));
        }
        tmem_wait_st();
      }
      m = m_new;
      if (r == 0) stamp(p, 2 + grp, i, 3);
      // P = exp2(S scale - m) as bf16 over columns [0, 64) of this tile's S (S is in registers);
      // FWD_EMU of every 8 pairs on the FMA pipe, the others on MUFU
      const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-mref, -mref);
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 x = fma2(make_float2(__uint_as_float(v[c * 32 + e]), __uint_as_float(v[c * 32 + e + 1])),
                                sc2, nm2);
          const float2 ev = ((e >> 1) & 7) < FWD_EMU ? exp2_fma2(x)
                                                            : make_float2(fast_exp2(x.x), fast_exp2(x.y));
          acc = add2(acc, ev);
          pk[e / 2] = pack_bf16x2(ev.x, ev.y);
        }
        tmem_st16(t_s + lane_off + c * 16, pk);
      }
      const float sum = acc.x + acc.y;
      l = l * alpha + sum;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[grp]);
      if (r == 0) stamp(p, 2 + grp, i, 4);
    }
    // epilogue: O / l -> this tile's Q buffer (its last reader, S of the last key tile, is done once
    // the last PV product is) -> bulk tensor store; lse per row.  Every thread of the group reaches
    // the group barrier, whether or not its waits succeeded; a shared flag vetoes the store.
    volatile int* veto = abort_flag + 1 + grp;
    const bool fin = ok && n > 0 && mbar_wait(&o_done[grp], (n - 1) & 1, 0x32u, abort_flag);
    uint8_t* ob = sm + (grp ? FwdSmem::QB : FwdSmem::QA);
    if (!fin) *veto = 1;
    if (fin) {
      __syncwarp();
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(t_o + lane_off + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int i = 8 * g;
          uint4 w = make_uint4(pack_bf16x2(__uint_as_float(v[i]) * inv, __uint_as_float(v[i + 1]) * inv),
                               pack_bf16x2(__uint_as_float(v[i + 2]) * inv, __uint_as_float(v[i + 3]) * inv),
                               pack_bf16x2(__uint_as_float(v[i + 4]) * inv, __uint_as_float(v[i + 5]) * inv),
                               pack_bf16x2(__uint_as_float(v[i + 6]) * inv, __uint_as_float(v[i + 7]) * inv));
          *reinterpret_cast<uint4*>(ob + swz_off(r, c * 4 + g)) = w;
        }
      }
      if (qi < p.T) p.lse[(static_cast<int64_t>(b) * p.H + h) * p.T + qi] = (m * 0.6931471805599453f) + logf(l);
    }
    fence_proxy_async_smem();
    named_bar_sync(2 + grp, 128);
    if (r == 0 && n > 0 && !*veto) {
      tma_store_3d(&tmO, ob, h * HD, q0, b);
      tma_store_3d(&tmO, ob + BOX_BYTES, h * HD + 64, q0, b);
      tma_store_commit();
      tma_store_wait0();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------------------ backward
// One CTA per (key tile of 128, KV head, batch); 512 threads in four warpgroups (the first one
// gives registers back to the dQ drain).  Key tiles are the fastest-varying
// block index: CTAs running at the same time then share one (batch, KV head), so the fp32 dQ rows
// they all add into stay resident in L2.
//   warp 0      TMA: K and V once, then Q tiles of every (query head, query tile) pair into a
//               2-stage ring and the dO tiles into one buffer (refilled once dV of the pair is done).
//   warp 1      TMEM owner and MMA issuer, per pair i:
//                 dP^T = V dO^T -> tDP (after dQ of pair i-1 left tDP);
//                 dV += P^T dO with P^T read from tensor memory (tS, bf16);
//                 S^T of pair i+1 = K Q^T -> tS at once (MMAs from one thread run in order, and the
//                 softmax keeps P^T in registers, so nothing reads tS after the dV product);
//                 dK += dS^T Q;  dQ = dS K -> tDP.
//   warps 4..11 two warpgroups, one key row per thread, warpgroup g on queries [64 g, 64 g + 64):
//               P^T = exp2(S^T scale - lse) written back as bf16 into the group's own S^T columns
//               (queries 64 g .. go to columns [64 g, 64 g + 32)) and kept in registers, then
//               dS^T = P^T (dP^T - delta) into shared memory (128B-swizzled) once dK and dQ of the
//               previous pair have read it.  Each pair's lse / delta are loaded a pair ahead.
//   warps 12..15 drain dQ: tcgen05.ld of the 128 x 128 fp32 tile, release tDP, stage it in
//               quarters of 32 columns through a two-slot ring and add each quarter to the fp32 dQ
//               buffer with a bulk tensor reduction (performed in L2); two reductions in flight.
// Tensor-memory columns: tS [0,128) | tDP [128,256) | dV [256,384) | dK [384,512); P^T of queries
// [64 g, 64 g + 64) in bf16 pairs at columns [64 g, 64 g + 32) of tS.
struct BwdSmem {
  static constexpr int K = 0;
  static constexpr int V = K + TILE_BYTES;
  static constexpr int Q = V + TILE_BYTES;        // 2 stages
  static constexpr int DO = Q + 2 * TILE_BYTES;   // 1 stage
  static constexpr int DST = DO + TILE_BYTES;     // dS^T [keys x queries]
  static constexpr int STG = DST + TILE_BYTES;    // dQ staging: 2 slots of [128 rows x 32 fp32]
  static constexpr int STAT = STG + TILE_BYTES;   // lse * log2(e) [128], delta [128] of the current pair
  static constexpr int BAR = STAT + 1024;
  // kv_full, q_full[2], q_empty[2], do_full, do_empty, s_full, p_full, dp_full, ds_full, dq_full,
  // dq_free, stg_full, stg_free[2], stat_ready, stat_free
  static constexpr int NBAR = 18;
  static constexpr int TOTAL = BAR + NBAR * 8 + 16 + 1024;
};
static_assert(BwdSmem::TOTAL <= 232448, "backward shared memory exceeds the sm_100 limit");

constexpr int BWD_THREADS = 512;
constexpr uint32_t BWD_REGS_LAUNCH = 128;  // the two softmax warpgroups keep the launch count
constexpr uint32_t BWD_REGS_LOW = 72;      // TMA / MMA warpgroup
constexpr uint32_t BWD_REGS_DRAIN = 184;   // dQ drain (a whole fp32 dQ row in registers)
static_assert(128 * BWD_REGS_LOW + 256 * BWD_REGS_LAUNCH + 128 * BWD_REGS_DRAIN <= BWD_THREADS * BWD_REGS_LAUNCH,
              "backward register split exceeds the launch budget");
constexpr int STG_SLOT = 16384;

NT_DEVICE void bwd_q_range(const Params& p, int k0, int& i_lo, int& i_hi) {
  const int n_qt = (p.T + TILE - 1) / TILE;
  i_lo = k0 / TILE;  // causal: queries >= keys
  i_hi = n_qt - 1;
  if (p.window >= 0) i_hi = min(i_hi, (k0 + TILE - 1 + p.window) / TILE);
}

__global__ void __launch_bounds__(BWD_THREADS, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BwdSmem::BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* q_full = bars + 1;    // [2]
  uint64_t* q_empty = bars + 3;   // [2]
  uint64_t* do_full = bars + 5;
  uint64_t* do_empty = bars + 6;
  uint64_t* s_full = bars + 7;
  uint64_t* p_full = bars + 8;
  uint64_t* dp_full = bars + 9;
  uint64_t* ds_full = bars + 10;
  uint64_t* dq_full = bars + 11;
  uint64_t* dq_free = bars + 12;
  uint64_t* stg_full = bars + 13;
  uint64_t* stg_free = bars + 14;  // [2]
  uint64_t* stat_ready = bars + 16;
  uint64_t* stat_free = bars + 17;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + BwdSmem::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int kt, bk;  // causal: key tile 0 has the most query tiles
  work_unit(static_cast<int>(blockIdx.x), (p.T + TILE - 1) / TILE, p.Hk * p.B, p.order_window, kt, bk);
  const int hk = bk % p.Hk, b = bk / p.Hk;
  const int group = p.H / p.Hk;
  const int k0 = kt * TILE;
  int i_lo, i_hi;
  bwd_q_range(p, k0, i_lo, i_hi);
  const int n_q = i_hi - i_lo + 1;
  const int n_it = group * n_q;  // (query head in the group, query tile) pairs

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&stg_free[i], 1);
    }
    mbar_init(do_full, 1);
    mbar_init(do_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(p_full, 256);
    mbar_init(dp_full, 1);
    mbar_init(ds_full, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 128);
    mbar_init(stg_full, 128);
    mbar_init(stat_ready, 256);
    mbar_init(stat_free, 256);
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
  const uint32_t t_s = tbase;          // S^T, then P^T (bf16, 64 columns)
  const uint32_t t_dp = tbase + 128;   // dP^T, then dQ
  const uint32_t t_dv = tbase + 256;
  const uint32_t t_dk = tbase + 384;

  if (warp < 4) {
   setmaxnreg_dec<BWD_REGS_LOW>();
   if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDO);
      mbar_expect_tx(kv_full, 2 * TILE_BYTES);
      tma_load_3d(sm + BwdSmem::K, &tmK, kv_full, hk * HD, k0, b);
      tma_load_3d(sm + BwdSmem::K + BOX_BYTES, &tmK, kv_full, hk * HD + 64, k0, b);
      tma_load_3d(sm + BwdSmem::V, &tmV, kv_full, hk * HD, k0, b);
      tma_load_3d(sm + BwdSmem::V + BOX_BYTES, &tmV, kv_full, hk * HD + 64, k0, b);
      int q_issued = 0, do_issued = 0;
      for (int it = 0; it < n_it; ++it) {
        const int st = it & 1;
        const int h = hk * group + it / n_q;
        const int q0 = (i_lo + it % n_q) * TILE;
        if (!mbar_wait(&q_empty[st], ((it >> 1) & 1) ^ 1u, 0x50u + st, abort_flag)) break;
        stamp(p, 0, it, 0);
        uint8_t* qs = sm + BwdSmem::Q + st * TILE_BYTES;
        mbar_expect_tx(&q_full[st], TILE_BYTES);
        tma_load_3d(qs, &tmQ, &q_full[st], h * HD, q0, b);
        tma_load_3d(qs + BOX_BYTES, &tmQ, &q_full[st], h * HD + 64, q0, b);
        ++q_issued;
        // dO of this pair once the dV product of the previous pair has read the buffer
        if (!mbar_wait(do_empty, (it & 1) ^ 1u, 0x52u, abort_flag)) break;
        stamp(p, 0, it, 1);
        uint8_t* ds = sm + BwdSmem::DO;
        mbar_expect_tx(do_full, TILE_BYTES);
        tma_load_3d(ds, &tmDO, do_full, h * HD, q0, b);
        tma_load_3d(ds + BOX_BYTES, &tmDO, do_full, h * HD + 64, q0, b);
        ++do_issued;
      }
      // no copy may still be in flight when the CTA exits
      mbar_wait(kv_full, 0, 0x5Eu, nullptr);
      for (int it = max(0, q_issued - 2); it < q_issued; ++it) mbar_wait(&q_full[it & 1], (it >> 1) & 1, 0x5Fu, nullptr);
      if (do_issued > 0) mbar_wait(do_full, (do_issued - 1) & 1, 0x5Du, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16_f32(TILE, TILE, 0, 0);   // S^T = K Q^T ; dP^T = V dO^T
      constexpr uint32_t id_kv = idesc_bf16_f32(TILE, HD, 0, 1);    // dV += P^T dO ; dK += dS^T Q
      constexpr uint32_t id_q = idesc_bf16_f32(TILE, HD, 1, 1);     // dQ = dS K  (A = dS^T read M-major)
      const uint32_t k_addr = smem_u32(sm + BwdSmem::K), v_addr = smem_u32(sm + BwdSmem::V);
      const uint32_t ds_addr = smem_u32(sm + BwdSmem::DST), do_addr = smem_u32(sm + BwdSmem::DO);
      // S^T of pair `it` into tS (Q of the pair must have landed)
      auto issue_s = [&](int it) -> bool {
        if (!mbar_wait(&q_full[it & 1], (it >> 1) & 1, 0x61u, abort_flag)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sm + BwdSmem::Q + (it & 1) * TILE_BYTES);
        // unrolled over k-steps from two step-0 descriptors (the steps are immediates)
        const uint64_t dk = kmajor_desc(k_addr, 0), dq = kmajor_desc(q_addr, 0);
        for_steps([&](auto j) {
          constexpr int J = decltype(j)::value;
          umma_step<kmajor_step(J), kmajor_step(J)>(t_s, dk, dq, id_s, J > 0);
        });
        umma_commit(s_full);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, 0x60u, abort_flag) && (n_it == 0 || issue_s(0));
      for (int it = 0; ok && it < n_it; ++it) {
        const int st = it & 1;
        const uint32_t q_addr = smem_u32(sm + BwdSmem::Q + st * TILE_BYTES);
        if (!mbar_wait(do_full, it & 1, 0x66u, abort_flag)) break;
        if (it > 0 && !mbar_wait(dq_free, (it - 1) & 1, 0x62u, abort_flag)) break;  // dQ of it-1 left tDP
        stamp(p, 1, it, 1);
        tc_fence_after();
        const uint64_t dvk = kmajor_desc(v_addr, 0), ddo = kmajor_desc(do_addr, 0);
        for_steps([&](auto j) {
          constexpr int J = decltype(j)::value;
          umma_step<kmajor_step(J), kmajor_step(J)>(t_dp, dvk, ddo, id_s, J > 0);
        });
        umma_commit(dp_full);
        if (!mbar_wait(p_full, it & 1, 0x63u, abort_flag)) break;
        stamp(p, 1, it, 2);
        tc_fence_after();
        const uint64_t ddo_mn = mnmajor_desc(do_addr, 0);
        const uint32_t acc_kv = it > 0 ? 1u : 0u;
        for_steps([&](auto j) {
          constexpr int J = decltype(j)::value;
          umma_step_tmem_a<(J >> 2) * 64 + (J & 3) * 8, mnmajor_step(J)>(t_dv, t_s, ddo_mn, id_kv, J > 0 ? 1u : acc_kv);
        });
        umma_commit(do_empty);
        if (it + 1 < n_it && !issue_s(it + 1)) break;
        if (!mbar_wait(ds_full, it & 1, 0x64u, abort_flag)) break;
        stamp(p, 1, it, 3);
        tc_fence_after();
        const uint64_t dds = kmajor_desc(ds_addr, 0), dq_mn = mnmajor_desc(q_addr, 0);
        const uint64_t dds_mn = mnmajor_desc(ds_addr, 0), dk_mn = mnmajor_desc(k_addr, 0);
        for_steps([&](auto j) {
          constexpr int J = decltype(j)::value;
          umma_step<kmajor_step(J), mnmajor_step(J)>(t_dk, dds, dq_mn, id_kv, J > 0 ? 1u : acc_kv);
        });
        for_steps([&](auto j) {
          constexpr int J = decltype(j)::value;
          umma_step<mnmajor_step(J), mnmajor_step(J)>(t_dp, dds_mn, dk_mn, id_q, J > 0);
        });
        umma_commit(dq_full);
        umma_commit(&q_empty[st]);
        stamp(p, 1, it, 4);
      }
    }
   }
  } else if (warp < 12) {
    // ------------------------------------------------------------ P^T and dS^T (one key row each)
    const int grp = (warp - 4) >> 2;   // queries [64 grp, 64 grp + 64)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const int kj = k0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t t_sg = t_s + grp * 64;
    uint8_t* dsb = sm + BwdSmem::DST;
    float* s_lse = reinterpret_cast<float*>(sm + BwdSmem::STAT);
    float* s_del = s_lse + 128;
    // lse (group 0) or delta (group 1) of query row r of a pair, read a pair ahead
    auto stat_of = [&](int it) -> float {
      const int h = hk * group + it / n_q;
      const int qi = (i_lo + it % n_q) * TILE + r;
      const int64_t o = (static_cast<int64_t>(b) * p.H + h) * p.T + min(qi, p.T - 1);
      return grp ? p.delta[o] : p.lse[o] * LOG2E;
    };
    float stat_next = n_it > 0 ? stat_of(0) : 0.f;
    for (int it = 0; it < n_it; ++it) {
      const int q0 = (i_lo + it % n_q) * TILE;
      const float stat_cur = stat_next;
      if (it + 1 < n_it) stat_next = stat_of(it + 1);
      // statistics of this pair into shared memory once every row is done with the previous pair's.
      // stat_free and stat_ready are mbarriers, so a row that leaves the loop after a timed-out wait
      // cannot strand the others.
      if (it > 0 && !mbar_wait(stat_free, (it - 1) & 1, 0x74u, abort_flag)) break;
      (grp ? s_del : s_lse)[r] = stat_cur;
      mbar_arrive(stat_ready);
      if (!mbar_wait(stat_ready, it & 1, 0x75u, abort_flag)) break;
      if (r == 0 && grp == 0) stamp(p, 2, it, 0);
      const bool boundary = (k0 + TILE - 1 > q0) || (q0 + TILE > p.T) || (k0 + TILE > p.T) ||
                            (p.window >= 0 && q0 + TILE - 1 - k0 > p.window);
      if (!mbar_wait(s_full, it & 1, 0x70u, abort_flag)) break;
      if (r == 0 && grp == 0) stamp(p, 2, it, 1);
      __syncwarp();
      tc_fence_after();
      // P^T of this key row over the group's 64 queries, bf16 pairs: written to tS for the dV
      // product and kept here for dS^T (tS takes the next pair's S^T right after the dV product)
      uint32_t pk[32];
      {
        uint32_t sv[64];  // the group's 64 S^T columns, two loads in flight
        tmem_ld32(t_sg + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
        tmem_ld32(t_sg + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          const float2 l2 = *reinterpret_cast<const float2*>(s_lse + grp * 64 + i);
          sv[i] = __float_as_uint(fmaf(__uint_as_float(sv[i]), p.scale_log2, -l2.x));
          sv[i + 1] = __float_as_uint(fmaf(__uint_as_float(sv[i + 1]), p.scale_log2, -l2.y));
        }
        // the mask is applied in a separate loop so the unrolled exp loop carries no branches
        if (boundary) {
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int qi = q0 + grp * 64 + i;
            const bool valid = kj <= qi && qi < p.T && kj < p.T && (p.window < 0 || qi - kj <= p.window);
            if (!valid) sv[i] = __float_as_uint(-INFINITY);
          }
        }
#pragma unroll
        for (int i = 0; i < 64; i += 2)
          pk[i / 2] = pack_bf16x2(fast_exp2(__uint_as_float(sv[i])), fast_exp2(__uint_as_float(sv[i + 1])));
      }
      // columns [64 grp, 64 grp + 32): this group's own S^T, already read above
      tmem_st16(t_sg + lane_off, *reinterpret_cast<uint32_t(*)[16]>(&pk[0]));
      tmem_st16(t_sg + lane_off + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk[16]));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full);
      if (r == 0 && grp == 0) stamp(p, 2, it, 2);
      if (!mbar_wait(dp_full, it & 1, 0x71u, abort_flag)) break;
      if (r == 0 && grp == 0) stamp(p, 2, it, 3);
      // dS^T buffer: the dK and dQ products of the previous pair read it last
      if (it > 0 && !mbar_wait(dq_full, (it - 1) & 1, 0x73u, abort_flag)) break;
      if (r == 0 && grp == 0) stamp(p, 2, it, 4);
      __syncwarp();
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t dv[32];
        tmem_ld32(t_dp + lane_off + grp * 64 + c * 32, dv);
        tmem_wait_ld();
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int i = 8 * g + 2 * e;
            const float2 pp = unpack_bf16x2(pk[c * 16 + i / 2]);
            const float2 dl = *reinterpret_cast<const float2*>(s_del + grp * 64 + c * 32 + i);
            w[e] = pack_bf16x2(pp.x * (__uint_as_float(dv[i]) - dl.x), pp.y * (__uint_as_float(dv[i + 1]) - dl.y));
          }
          *reinterpret_cast<uint4*>(dsb + swz_off(r, grp * 8 + c * 4 + g)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(ds_full);
      mbar_arrive(stat_free);
      if (r == 0 && grp == 0) stamp(p, 2, it, 5);
    }
    // dK of this key tile (columns [64 grp, 64 grp + 64)) once every MMA has completed
    if (!*abort_flag && n_it > 0 && mbar_wait(dq_full, (n_it - 1) & 1, 0x72u, abort_flag)) {
      __syncwarp();
      tc_fence_after();
      // every lane takes part in the aligned TMEM loads; only rows inside the sequence store
      const bool live = kj < p.T;
      __nv_bfloat16* dkr = p.dk + (static_cast<int64_t>(b) * p.T + (live ? kj : 0)) * p.lddk + hk * HD;
#pragma unroll 1
      for (int c = 2 * grp; c < 2 * grp + 2; ++c) {
        uint32_t k[32];
        tmem_ld32(t_dk + lane_off + c * 32, k);
        tmem_wait_ld();
        const float sc = p.scale;
        if (live) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 z = make_uint4(pack_bf16x2(__uint_as_float(k[i]) * sc, __uint_as_float(k[i + 1]) * sc),
                                 pack_bf16x2(__uint_as_float(k[i + 2]) * sc, __uint_as_float(k[i + 3]) * sc),
                                 pack_bf16x2(__uint_as_float(k[i + 4]) * sc, __uint_as_float(k[i + 5]) * sc),
                                 pack_bf16x2(__uint_as_float(k[i + 6]) * sc, __uint_as_float(k[i + 7]) * sc));
            *reinterpret_cast<uint4*>(dkr + c * 32 + i) = z;
          }
        }
        __syncwarp();
      }
    }
  } else {
    setmaxnreg_inc<BWD_REGS_DRAIN>();
    // ------------------------------------------------------------ dQ drain (one query row each)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const bool leader = threadIdx.x == 384;  // warp 12, lane 0: issues the bulk reductions
    int n_q4 = 0;                            // quarters staged so far
    for (int it = 0; it < n_it; ++it) {
      const int h = hk * group + it / n_q;
      const int q0 = (i_lo + it % n_q) * TILE;
      if (!mbar_wait(dq_full, it & 1, 0x78u, abort_flag)) break;
      if (leader) stamp(p, 3, it, 0);
      __syncwarp();
      tc_fence_after();
      // the whole dQ row comes into registers first, so tDP is released for the next dP^T at once
      uint32_t vq[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(t_dp + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&vq[c * 32]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(dq_free);  // tDP may take the next dP^T
      // columns [4 j0, 4 j1) of this thread's query row added from registers: vector reductions of 4
      // fp32 (plain vector stores into the key tile's slice in deterministic mode)
      auto add_direct = [&](int j0, int j1) {
        const int qi = q0 + r;
        if (qi >= p.T) return;
        float* dst = p.dq_base +
                     ((p.dq_slices ? static_cast<int64_t>(kt) * p.B * p.T : 0) + static_cast<int64_t>(b) * p.T + qi) *
                         (static_cast<int64_t>(p.H) * HD) + h * HD;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (j < j0 || j >= j1) continue;
          const float a0 = __uint_as_float(vq[4 * j]) * p.scale, a1 = __uint_as_float(vq[4 * j + 1]) * p.scale;
          const float a2 = __uint_as_float(vq[4 * j + 2]) * p.scale, a3 = __uint_as_float(vq[4 * j + 3]) * p.scale;
          if (p.dq_slices)
            *reinterpret_cast<float4*>(dst + 4 * j) = make_float4(a0, a1, a2, a3);
          else
            asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst + 4 * j), "f"(a0), "f"(a1),
                         "f"(a2), "f"(a3)
                         : "memory");
        }
      };
      if (p.dq_direct == 1) {
        add_direct(0, 32);
        if (leader) stamp(p, 3, it, 2);
        continue;
      }
      // staged quarters: all four, or (dq_direct 2) the first two while the last two go out directly,
      // so bulk reductions and register reductions are in flight together
      const int nst = p.dq_direct == 2 ? 2 : 4;
      bool fine = true;
#pragma unroll
      for (int qq = 0; qq < 4; ++qq) {
        if (qq >= nst) break;
        const int n = n_q4 + qq;
        const int slot = n & 1;
        uint8_t* stg = sm + BwdSmem::STG + slot * STG_SLOT;
        // the slot's previous reduction (quarter n - 2) must have read it
        if (n >= 2 && !mbar_wait(&stg_free[slot], ((n - 2) >> 1) & 1, 0x7Au, abort_flag)) { fine = false; break; }
        if (leader && qq == 0) stamp(p, 3, it, 1);
        __syncwarp();
        // one box of [128 rows x 32 fp32], 128-byte rows, 128-byte swizzle
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int i = qq * 32 + c * 4;
          float4 w = make_float4(__uint_as_float(vq[i]) * p.scale, __uint_as_float(vq[i + 1]) * p.scale,
                                 __uint_as_float(vq[i + 2]) * p.scale, __uint_as_float(vq[i + 3]) * p.scale);
          *reinterpret_cast<float4*>(stg + r * 128 + ((c ^ (r & 7)) << 4)) = w;
        }
        fence_proxy_async_smem();
        mbar_arrive(stg_full);
        if (leader) {
          if (mbar_wait(stg_full, n & 1, 0x7Bu, abort_flag)) {
            if (p.dq_slices) {
              // deterministic mode: this key tile's contribution goes to its own slice (plain stores);
              // the convert kernel sums the slices in key-tile order
              tma_store_3d(&tmDQ, stg, h * HD + qq * 32, q0, kt * p.B + b);
            } else {
              tma_reduce_add_3d(&tmDQ, stg, h * HD + qq * 32, q0, b);
            }
            tma_store_commit();
            // the reduction before this one has read its slot: release that slot
            tma_store_wait_read1();
            if (n >= 1) mbar_arrive(&stg_free[(n - 1) & 1]);
            if (qq == nst - 1) stamp(p, 3, it, 2);
          } else {
            fine = false;
          }
        }
        __syncwarp();
      }
      n_q4 += nst;
      if (!fine) break;
      if (nst < 4) add_direct(8 * nst, 32);
    }
    if (leader) tma_store_wait0();  // every reduction has landed before the CTA retires
    // dV of this key tile (every MMA has completed once the last dq_full fired)
    const int kj = k0 + r;
    if (!*abort_flag && n_it > 0 && mbar_wait(dq_full, (n_it - 1) & 1, 0x79u, abort_flag)) {
      __syncwarp();
      tc_fence_after();
      const bool live = kj < p.T;
      __nv_bfloat16* dvr = p.dv + (static_cast<int64_t>(b) * p.T + (live ? kj : 0)) * p.lddv + hk * HD;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t w[32];
        tmem_ld32(t_dv + lane_off + c * 32, w);
        tmem_wait_ld();
        if (live) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 a = make_uint4(pack_bf16x2(__uint_as_float(w[i]), __uint_as_float(w[i + 1])),
                                 pack_bf16x2(__uint_as_float(w[i + 2]), __uint_as_float(w[i + 3])),
                                 pack_bf16x2(__uint_as_float(w[i + 4]), __uint_as_float(w[i + 5])),
                                 pack_bf16x2(__uint_as_float(w[i + 6]), __uint_as_float(w[i + 7])));
            *reinterpret_cast<uint4*>(dvr + c * 32 + i) = a;
          }
        }
        __syncwarp();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// delta[b, h, t] = sum_d dO[b t, h d] * O[b t, h d]   (one warp per (row, head))
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo, const __nv_bfloat16* __restrict__ dout,
                                  int64_t lddo, float* __restrict__ delta, int B, int T, int H) {
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(B) * T * H) return;
  const int h = static_cast<int>(gw % H);
  const int64_t row = gw / H;
  const __nv_bfloat16* a = o + row * ldo + h * HD + lane * 4;
  const __nv_bfloat16* g = dout + row * lddo + h * HD + lane * 4;
  const uint2 av = *reinterpret_cast<const uint2*>(a);
  const uint2 gv = *reinterpret_cast<const uint2*>(g);
  const float2 a0 = unpack_bf16x2(av.x), a1 = unpack_bf16x2(av.y), g0 = unpack_bf16x2(gv.x), g1 = unpack_bf16x2(gv.y);
  float s = a0.x * g0.x + a0.y * g0.y + a1.x * g1.x + a1.y * g1.y;
  s = warp_sum(s);
  if (lane == 0) {
    const int b = static_cast<int>(row / T), t = static_cast<int>(row % T);
    delta[(static_cast<int64_t>(b) * H + h) * T + t] = s;
  }
}

// dq (bf16, strided rows) = sum over `slices` slices of dq_acc (fp32 [slices][B*T, H*128]), in slice
// order (one slice: a plain conversion)
__global__ void attn_dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int64_t lddq,
                                       int64_t rows, int cols, int slices) {
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  const int64_t n = rows * cols;
  if (i >= n) return;
  const int64_t r = i / cols;
  const int c = static_cast<int>(i - r * cols);
  float4 v = *reinterpret_cast<const float4*>(acc + i);
  for (int s = 1; s < slices; ++s) {
    const float4 u = *reinterpret_cast<const float4*>(acc + s * n + i);
    v.x += u.x; v.y += u.y; v.z += u.z; v.w += u.w;
  }
  uint2 w = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  *reinterpret_cast<uint2*>(dq + r * lddq + c) = w;
}

// ------------------------------------------------------------------------------ host
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// dims {cols, T, B} over rows of stride ld (elements); box {64, 128, 1}; 128B swizzle.
static CUtensorMap tile_map(const void* base, int64_t cols, int64_t ld, int T, int B) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || (ld * 2) % 16) throw std::runtime_error("attention operand alignment");
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld * 2), static_cast<cuuint64_t>(ld * 2 * T)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(TILE), 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return m;
}

// fp32 dQ accumulator [B, T, H*128]: dims {cols, T, B}, box {32, 128, 1} (128-byte rows), 128B swizzle.
static CUtensorMap dq_map(float* base, int64_t cols, int T, int B) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || cols % 4) throw std::runtime_error("dQ buffer alignment");
  CUtensorMap m;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(cols * 4), static_cast<cuuint64_t>(cols * 4 * T)};
  cuuint32_t box[3] = {32u, static_cast<cuuint32_t>(TILE), 1u};
  cuuint32_t es[3] = {1u, 1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (dQ) failed: " + std::to_string(int(r)));
  return m;
}

static Params make_params(const AttnArgs& a) {
  Params p{};
  p.B = a.B; p.T = a.T; p.H = a.H; p.Hk = a.Hk;
  p.window = a.window;
  p.scale = a.scale;
  p.scale_log2 = a.scale * LOG2E;
  p.o = reinterpret_cast<__nv_bfloat16*>(a.o);
  p.ldo = a.ldo;
  p.lse = a.lse;
  return p;
}

}  // namespace attn
}  // namespace nt

using namespace nt::attn;

// CTA order: longest first within runs of W (batch, head) groups.  At the benchmark shape (B 32,
// T 2048, 10 / 5 heads) W = 16 measured 1.66 ms backward / 0.488 ms forward against 1.90 / 0.510 for
// the plain group-major order (W = 0) and 1.72 / 0.505 for W = 8; a global longest-first order (every
// group in one run) was slower than both, since concurrent CTAs then share no K / V tiles in L2.
// NT_ATTN_ORDER overrides W (0: group-major).
static int order_window() {
  static const int w = [] {
    const char* e = std::getenv("NT_ATTN_ORDER");
    return e ? std::max(0, std::atoi(e)) : 16;
  }();
  return w;
}

static bool supported(const AttnArgs& a) {
  return a.D == HD && a.B > 0 && a.T > 0 && a.H > 0 && a.Hk > 0 && a.H % a.Hk == 0;
}

int nt_attention_fwd(const AttnArgs& a, cudaStream_t s) {
  nt::current_context();
  if (!supported(a)) return -1;
  CUtensorMap tq = tile_map(a.q, static_cast<int64_t>(a.H) * HD, a.ldq, a.T, a.B);
  CUtensorMap tk = tile_map(a.k, static_cast<int64_t>(a.Hk) * HD, a.ldk, a.T, a.B);
  CUtensorMap tv = tile_map(a.v, static_cast<int64_t>(a.Hk) * HD, a.ldv, a.T, a.B);
  CUtensorMap to = tile_map(a.o, static_cast<int64_t>(a.H) * HD, a.ldo, a.T, a.B);
  Params p = make_params(a);
  p.trace = a.trace;
  static const int emu = [] {
    const char* e = std::getenv("NT_ATTN_FWD_EMU");
    return e ? std::atoi(e) : FWD_EMU_DEFAULT;
  }();
  const int n_qt = (a.T + TILE - 1) / TILE;
  dim3 grid(static_cast<unsigned>((n_qt + 1) / 2) * a.H * a.B);
  p.order_window = order_window();
  auto launch = [&](auto kern, std::atomic<uint64_t>& set) {
    nt::smem_limit(set, kern, FwdSmem::TOTAL);
    kern<<<grid, FWD_THREADS, FwdSmem::TOTAL, s>>>(tq, tk, tv, to, p);
  };
  static std::atomic<uint64_t> set0{0}, set2{0}, set3{0}, set4{0};
  switch (emu) {
    case 0: launch(attn_fwd_kernel<0>, set0); break;
    case 2: launch(attn_fwd_kernel<2>, set2); break;
    case 4: launch(attn_fwd_kernel<4>, set4); break;
    default: launch(attn_fwd_kernel<3>, set3); break;
  }
  return 0;
}

int nt_attention_bwd(const AttnArgs& a, cudaStream_t s) {
  nt::current_context();
  if (!supported(a)) return -1;
  if (reinterpret_cast<uintptr_t>(a.dq) % 8 || a.lddq % 4) return -1;
  const int64_t rows = static_cast<int64_t>(a.B) * a.T;
  const int64_t warps = rows * a.H;
  attn_delta_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, s>>>(
      reinterpret_cast<const __nv_bfloat16*>(a.o), a.ldo, reinterpret_cast<const __nv_bfloat16*>(a.dout), a.lddo,
      a.delta, a.B, a.T, a.H);
  CUtensorMap tq = tile_map(a.q, static_cast<int64_t>(a.H) * HD, a.ldq, a.T, a.B);
  CUtensorMap tk = tile_map(a.k, static_cast<int64_t>(a.Hk) * HD, a.ldk, a.T, a.B);
  CUtensorMap tv = tile_map(a.v, static_cast<int64_t>(a.Hk) * HD, a.ldv, a.T, a.B);
  CUtensorMap tdo = tile_map(a.dout, static_cast<int64_t>(a.H) * HD, a.lddo, a.T, a.B);
  const int n_kt = (a.T + TILE - 1) / TILE;
  if (a.dq_slices && a.dq_slices != n_kt) return -1;
  CUtensorMap tdq = dq_map(a.dq_acc, static_cast<int64_t>(a.H) * HD, a.T, a.dq_slices ? a.B * n_kt : a.B);
  Params p = make_params(a);
  p.dq_slices = a.dq_slices;
  p.dout = reinterpret_cast<const __nv_bfloat16*>(a.dout);
  p.lddo = a.lddo;
  p.dk = reinterpret_cast<__nv_bfloat16*>(a.dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(a.dv);
  p.lddk = a.lddk;
  p.lddv = a.lddv;
  p.dq_acc = a.dq_acc;
  p.delta = a.delta;
  p.trace = a.trace;
  // NT_ATTN_DQ_DIRECT=1: the drain adds dQ with vector reductions from registers instead of staging it
  // through shared memory for bulk reductions; 2: half of each row each way (selectable for measurement)
  static const int direct = [] {
    const char* e = std::getenv("NT_ATTN_DQ_DIRECT");
    return e ? std::atoi(e) : 0;
  }();
  p.dq_direct = direct;
  p.dq_base = a.dq_acc;
  static std::atomic<uint64_t> smem_set{0};
  nt::smem_limit(smem_set, attn_bwd_kernel, BwdSmem::TOTAL);
  p.order_window = order_window();
  dim3 grid(static_cast<unsigned>((a.T + TILE - 1) / TILE) * a.Hk * a.B);
  attn_bwd_kernel<<<grid, BWD_THREADS, BwdSmem::TOTAL, s>>>(tq, tk, tv, tdo, tdq, p);
  const int cols = a.H * HD;
  const int64_t n = rows * cols;
  attn_dq_convert_kernel<<<static_cast<unsigned>((n / 4 + 255) / 256), 256, 0, s>>>(
      a.dq_acc, reinterpret_cast<__nv_bfloat16*>(a.dq), a.lddq, rows, cols, a.dq_slices ? a.dq_slices : 1);
  return 0;
}

int nt_attention_read_error(unsigned* where) {
  nt::ErrorWord w{0, 0};
  cudaMemcpyFromSymbol(&w, nt::g_nt_error, sizeof(w));
  if (where) *where = w.where;
  return static_cast<int>(w.code);
}
