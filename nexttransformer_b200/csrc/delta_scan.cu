// Inter-chunk scan of the chunked (gated) delta rule on sm_100a (tcgen05 + TMEM + TMA).
//
// The chunk form of DeltaNet / Gated DeltaNet / KDA (nexttransformer/models/linear.py:198-276 of
// the reference; the torch restatement is models/linear.py `_delta_chunks` here) splits into a
// part that is independent per chunk (the WY representation w, u0 from the unit-lower-triangular
// solve, the masked intra-chunk scores aqk, the decayed q~ and k_c) and a sequential scan over
// chunks that carries the fp32 state S [Dk = 128 keys x V = 128 values]:
//
//     u_n = u0_n - w_n S_n
//     o_n = q~_n S_n + aqk_n u_n
//     S_{n+1} = c_n (.) S_n + k_c,n^T u_n        (c_n: per-key decay of chunk n, 1 for DeltaNet)
//
// These kernels run that scan.  Forward: one CTA per (batch*head, 64-value block); the state
// block [128 x 64] lives in TMEM as the fp32 accumulator of the update MMA; per chunk one MMA
// computes [w; q~] S (M = 128: rows 0-63 w S, rows 64-127 q~ S), the compute warps form u and
// its bf16 copy in shared memory, then one MMA adds aqk u into the q~ S rows (A zero-padded to
// 128 rows) and one MMA adds k_c^T u into the state after the threads scaled it by c_n in TMEM.
// Chunk operands are double-buffered by TMA.  The states S_n (bf16) and u_n (bf16) are saved
// for the backward.
//
// Backward (reverse scan, one CTA per batch*head, all 128 values): with dS = dL/dS_{n+1},
//     du_n   = aqk_n^T do_n + k_c,n dS           (computed transposed, du^T [128 v x 64], M = 128)
//     dS_n   = c_n (.) dS + q~_n^T do_n - w_n^T du_n
// and dS_{n+1} (bf16), du_n^T (bf16) and dc_n = rowsum(S_n (.) dS_{n+1}) are written out; the
// remaining products (dq~ = do S^T, dw = -du S^T, daqk = do u^T, dk_c = u dS^T) have no chain
// dependency and run afterwards as batched GEMMs.
//
// Every wait is bounded (common.cuh): a broken pipeline records an error and the kernel ends.
#include <cudaTypedefs.h>
#include <mutex>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "delta_scan.h"

namespace nt {
namespace {

constexpr int CH = 64;    // chunk length
constexpr int DK = 128;   // key features
constexpr int VB = 64;    // value columns per forward CTA
constexpr int DV = 128;   // value features

NT_DEVICE uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Byte offset of 16-byte chunk j of row r in a 128-byte-swizzled tile of 128-byte rows.
NT_DEVICE uint32_t swz(int r, int j) { return static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4)); }

NT_DEVICE bool warp_wait(uint64_t* bar, uint32_t parity, uint32_t where, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, where, abort);
  return __all_sync(0xffffffffu, ok);
}

NT_DEVICE uint4 pack8(const float* f) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}
NT_DEVICE void unpack8(uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

struct FwdParams {
  int N;             // chunks per sequence
  const float* carry;        // [BH, N, 128]
  __nv_bfloat16* o;          // [BH, N, 64, 128]
  __nv_bfloat16* states;     // [BH, N, 128, 128]  (S_n, state entering chunk n)
  __nv_bfloat16* u;          // [BH, N, 64, 128]
};

struct FwdSmem {
  static constexpr uint32_t A1 = 0;          // [2 key blocks][128 rows: w 0-63, q~ 64-127][128 B]
  static constexpr uint32_t KC = 32768;      // [2 key blocks][64 rows][128 B]
  static constexpr uint32_t A3 = 49152;      // [128 rows: zeros 0-63, aqk 64-127][128 B]
  static constexpr uint32_t U0 = 65536;      // [64 rows][128 B]   (64 values)
  static constexpr uint32_t STAGE = 73728;
  static constexpr uint32_t SB = 2 * STAGE;  // S_n bf16 [128 key rows][128 B]
  static constexpr uint32_t UB = SB + 16384; // u bf16 [64 rows][128 B]
  static constexpr uint32_t BAR = UB + 8192;
  static constexpr int NBAR = 8;
  static constexpr uint32_t MISC = BAR + NBAR * 8;
  static constexpr uint32_t TOTAL = MISC + 16 + 1024;
};
static_assert(FwdSmem::TOTAL <= 232448, "forward scan shared memory");

__global__ void __launch_bounds__(192, 1)
delta_scan_fwd_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmKC, const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmU0, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + FwdSmem::BAR);
  uint64_t* full = bar;
  uint64_t* empty = bar + 2;
  uint64_t* sb_ready = bar + 4;
  uint64_t* d1_full = bar + 5;
  uint64_t* u_ready = bar + 6;
  uint64_t* mma2_done = bar + 7;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + FwdSmem::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + FwdSmem::MISC + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int v0 = blockIdx.x * VB, bh = blockIdx.y, N = p.N;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(sb_ready, 128);
    mbar_init(d1_full, 1);
    mbar_init(u_ready, 64);
    mbar_init(mma2_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  // rows 0-63 of both A3 tiles stay zero (TMA fills rows 64-127 only)
  for (int i = threadIdx.x; i < 1024; i += blockDim.x)
    *reinterpret_cast<uint4*>(smem + (i >> 9) * FwdSmem::STAGE + FwdSmem::A3 + (i & 511) * 16) = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(tmem_holder, 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_holder;
  const uint32_t tD1 = tbase, tS = tbase + 64;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int n = 0; n < N; ++n) {
        const int s = n & 1;
        const uint32_t ph = (n >> 1) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1u, 0x500u + s, abort_flag)) break;
        uint8_t* st = smem + s * FwdSmem::STAGE;
        const int row0 = (bh * N + n) * CH;
        mbar_expect_tx(&full[s], 65536);
        tma_load_2d(st + FwdSmem::A1, &tmW, &full[s], 0, row0);
        tma_load_2d(st + FwdSmem::A1 + 16384, &tmW, &full[s], 64, row0);
        tma_load_2d(st + FwdSmem::A1 + 8192, &tmQ, &full[s], 0, row0);
        tma_load_2d(st + FwdSmem::A1 + 16384 + 8192, &tmQ, &full[s], 64, row0);
        tma_load_2d(st + FwdSmem::KC, &tmKC, &full[s], 0, row0);
        tma_load_2d(st + FwdSmem::KC + 8192, &tmKC, &full[s], 64, row0);
        tma_load_2d(st + FwdSmem::A3 + 8192, &tmA, &full[s], 0, row0);
        tma_load_2d(st + FwdSmem::U0, &tmU0, &full[s], v0, row0);
        ++issued;
      }
      // wait (bounded) for the copies still in flight before the CTA can exit
      for (int n = (issued > 2 ? issued - 2 : 0); n < issued; ++n)
        mbar_wait(&full[n & 1], (n >> 1) & 1, 0x510u, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t sb = smem_u32(smem + FwdSmem::SB), ub = smem_u32(smem + FwdSmem::UB);
      constexpr uint32_t id_km = idesc_bf16_f32(128, VB, 0, 1);   // A K-major, B MN-major
      constexpr uint32_t id_mm = idesc_bf16_f32(128, VB, 1, 1);   // both MN-major
      for (int n = 0; n < N; ++n) {
        const int s = n & 1;
        const uint32_t st = smem_u32(smem + s * FwdSmem::STAGE);
        if (!mbar_wait(&full[s], (n >> 1) & 1, 0x520u, abort_flag)) break;
        if (!mbar_wait(sb_ready, n & 1, 0x521u, abort_flag)) break;
        tc_fence_after();
        // D1 = [w; q~] S_n
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_bf16(tD1, smem_desc(st + FwdSmem::A1 + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024),
                    smem_desc(sb + ks * 2048, 16384, 1024), id_km, ks > 0);
        umma_commit(d1_full);
        if (!mbar_wait(u_ready, n & 1, 0x522u, abort_flag)) break;
        tc_fence_after();
        // D1[64:128] += aqk u ;  S += k_c^T u
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tD1, smem_desc(st + FwdSmem::A3 + ks * 32, 16, 1024), smem_desc(ub + ks * 2048, 8192, 1024),
                    id_km, 1);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tS, smem_desc(st + FwdSmem::KC + ks * 2048, 8192, 1024), smem_desc(ub + ks * 2048, 8192, 1024),
                    id_mm, 1);
        umma_commit(mma2_done);
        umma_commit(&empty[s]);
      }
    }
  } else {
    const int q = warp & 3;           // TMEM lane quarter of this warp
    const int r = q * 32 + lane;      // key row (state) / chunk row (D1)
    const uint32_t lrow = static_cast<uint32_t>(q * 32) << 16;
    {
      uint32_t z[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) z[i] = 0u;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_st16(tS + lrow + c * 16, z);
      tmem_wait_st();
    }
    bool ok = true;
    for (int n = 0; n <= N && ok; ++n) {
      if (n > 0) {
        if (!warp_wait(mma2_done, (n - 1) & 1, 0x530u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        if (q >= 2) {  // o rows of chunk n-1
          uint32_t a[32];
          __nv_bfloat16* orow = p.o + (static_cast<int64_t>(bh * N + n - 1) * CH + (r - 64)) * DV + v0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            tmem_ld32(tD1 + lrow + h * 32, a);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float f[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(a[j * 8 + e]);
              *reinterpret_cast<uint4*>(orow + h * 32 + j * 8) = pack8(f);
            }
          }
        }
      }
      if (n == N) break;
      // state entering chunk n: bf16 copy (MMA operand + saved), then scale by the chunk decay
      const float c = p.carry[static_cast<int64_t>(bh * N + n) * DK + r];
      __nv_bfloat16* srow = p.states + (static_cast<int64_t>(bh * N + n) * DK + r) * DV + v0;
      uint8_t* sb = smem + FwdSmem::SB;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t a[32];
        tmem_ld32(tS + lrow + h * 32, a);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(a[j * 8 + e]);
          const uint4 pk = pack8(f);
          *reinterpret_cast<uint4*>(sb + swz(r, h * 4 + j)) = pk;
          *reinterpret_cast<uint4*>(srow + h * 32 + j * 8) = pk;
        }
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          lo[e] = __float_as_uint(__uint_as_float(a[e]) * c);
          hi[e] = __float_as_uint(__uint_as_float(a[16 + e]) * c);
        }
        tmem_st16(tS + lrow + h * 32, lo);
        tmem_st16(tS + lrow + h * 32 + 16, hi);
      }
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(sb_ready);
      if (q < 2) {  // u = u0 - w S for chunk row r
        const int s = n & 1;
        if (!warp_wait(d1_full, n & 1, 0x531u, abort_flag)) { ok = false; break; }
        if (!warp_wait(&full[s], (n >> 1) & 1, 0x532u, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint8_t* u0 = smem + s * FwdSmem::STAGE + FwdSmem::U0;
        uint8_t* ub = smem + FwdSmem::UB;
        __nv_bfloat16* urow = p.u + (static_cast<int64_t>(bh * N + n) * CH + r) * DV + v0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t a[32];
          tmem_ld32(tD1 + lrow + h * 32, a);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float f[8];
            unpack8(*reinterpret_cast<const uint4*>(u0 + swz(r, h * 4 + j)), f);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] -= __uint_as_float(a[j * 8 + e]);
            const uint4 pk = pack8(f);
            *reinterpret_cast<uint4*>(ub + swz(r, h * 4 + j)) = pk;
            *reinterpret_cast<uint4*>(urow + h * 32 + j * 8) = pk;
          }
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(u_ready);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 128);
  }
}

// ------------------------------------------------------------------------------ backward
struct BwdParams {
  int N;
  const float* carry;            // [BH, N, 128]
  const __nv_bfloat16* states;   // [BH, N, 128, 128]
  __nv_bfloat16* ds;             // [BH, N, 128, 128]  dL/dS_{n+1}
  __nv_bfloat16* dut;            // [BH, N, 128 v, 64] du_n^T
  float* dcarry;                 // [BH, N, 128]
};

struct BwdSmem {
  static constexpr uint32_t DO = 0;          // [2 value blocks][64 rows][128 B]
  static constexpr uint32_t AQ = 16384;      // [64 rows][128 B]
  static constexpr uint32_t KC = 24576;      // [2 key blocks][64 rows][128 B]
  static constexpr uint32_t QT = 40960;
  static constexpr uint32_t W = 57344;
  static constexpr uint32_t STAGE = 73728;
  static constexpr uint32_t DSB = 2 * STAGE;     // dS bf16 [2 value blocks][128 key rows][128 B]
  static constexpr uint32_t DUB = DSB + 32768;   // -du^T bf16 [128 value rows][128 B]
  static constexpr uint32_t BAR = DUB + 16384;
  static constexpr int NBAR = 8;
  static constexpr uint32_t MISC = BAR + NBAR * 8;
  static constexpr uint32_t TOTAL = MISC + 16 + 1024;
};
static_assert(BwdSmem::TOTAL <= 232448, "backward scan shared memory");

__global__ void __launch_bounds__(192, 1)
delta_scan_bwd_kernel(const __grid_constant__ CUtensorMap tmDO, const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmKC, const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmW, const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + BwdSmem::BAR);
  uint64_t* full = bar;
  uint64_t* empty = bar + 2;
  uint64_t* dsb_ready = bar + 4;
  uint64_t* du_full = bar + 5;
  uint64_t* dub_ready = bar + 6;
  uint64_t* ds_full = bar + 7;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + BwdSmem::MISC);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + BwdSmem::MISC + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x, N = p.N;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(dsb_ready, 128);
    mbar_init(du_full, 1);
    mbar_init(dub_ready, 128);
    mbar_init(ds_full, 1);
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
  const uint32_t tDS = tbase, tDU = tbase + 128;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int m = 0; m < N; ++m) {
        const int n = N - 1 - m, s = m & 1;
        if (!mbar_wait(&empty[s], ((m >> 1) & 1) ^ 1u, 0x600u + s, abort_flag)) break;
        uint8_t* st = smem + s * BwdSmem::STAGE;
        const int row0 = (bh * N + n) * CH;
        mbar_expect_tx(&full[s], BwdSmem::STAGE);
        tma_load_2d(st + BwdSmem::DO, &tmDO, &full[s], 0, row0);
        tma_load_2d(st + BwdSmem::DO + 8192, &tmDO, &full[s], 64, row0);
        tma_load_2d(st + BwdSmem::AQ, &tmA, &full[s], 0, row0);
        tma_load_2d(st + BwdSmem::KC, &tmKC, &full[s], 0, row0);
        tma_load_2d(st + BwdSmem::KC + 8192, &tmKC, &full[s], 64, row0);
        tma_load_2d(st + BwdSmem::QT, &tmQ, &full[s], 0, row0);
        tma_load_2d(st + BwdSmem::QT + 8192, &tmQ, &full[s], 64, row0);
        tma_load_2d(st + BwdSmem::W, &tmW, &full[s], 0, row0);
        tma_load_2d(st + BwdSmem::W + 8192, &tmW, &full[s], 64, row0);
        ++issued;
      }
      for (int m = (issued > 2 ? issued - 2 : 0); m < issued; ++m)
        mbar_wait(&full[m & 1], (m >> 1) & 1, 0x610u, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t dsb = smem_u32(smem + BwdSmem::DSB), dub = smem_u32(smem + BwdSmem::DUB);
      constexpr uint32_t id_du_mm = idesc_bf16_f32(128, 64, 1, 1);
      constexpr uint32_t id_du_mk = idesc_bf16_f32(128, 64, 1, 0);
      constexpr uint32_t id_ds_mm = idesc_bf16_f32(128, 128, 1, 1);
      constexpr uint32_t id_ds_mk = idesc_bf16_f32(128, 128, 1, 0);
      for (int m = 0; m < N; ++m) {
        const int s = m & 1;
        const uint32_t st = smem_u32(smem + s * BwdSmem::STAGE);
        if (!mbar_wait(&full[s], (m >> 1) & 1, 0x620u, abort_flag)) break;
        if (!mbar_wait(dsb_ready, m & 1, 0x621u, abort_flag)) break;
        tc_fence_after();
        // du^T = do^T aqk + dS^T k_c^T
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tDU, smem_desc(st + BwdSmem::DO + ks * 2048, 8192, 1024),
                    smem_desc(st + BwdSmem::AQ + ks * 2048, 8192, 1024), id_du_mm, ks > 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          umma_bf16(tDU, smem_desc(dsb + ks * 2048, 16384, 1024),
                    smem_desc(st + BwdSmem::KC + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024), id_du_mk, 1);
        umma_commit(du_full);
        if (!mbar_wait(dub_ready, m & 1, 0x622u, abort_flag)) break;
        tc_fence_after();
        // dS += q~^T do - w^T du
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tDS, smem_desc(st + BwdSmem::QT + ks * 2048, 8192, 1024),
                    smem_desc(st + BwdSmem::DO + ks * 2048, 8192, 1024), id_ds_mm, 1);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_bf16(tDS, smem_desc(st + BwdSmem::W + ks * 2048, 8192, 1024), smem_desc(dub + ks * 32, 16, 1024),
                    id_ds_mk, 1);
        umma_commit(ds_full);
        umma_commit(&empty[s]);
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;     // key row of dS; value row of du^T
    const uint32_t lrow = static_cast<uint32_t>(q * 32) << 16;
    {
      uint32_t z[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) z[i] = 0u;
#pragma unroll
      for (int c = 0; c < 8; ++c) tmem_st16(tDS + lrow + c * 16, z);
      tmem_wait_st();
    }
    for (int m = 0; m < N; ++m) {
      const int n = N - 1 - m;
      if (m > 0) {
        if (!warp_wait(ds_full, (m - 1) & 1, 0x630u, abort_flag)) break;
        tc_fence_after();
      }
      // dS_{n+1}: bf16 copy (MMA operand + saved), dc_n, then scale by c_n
      const int64_t srow = (static_cast<int64_t>(bh * N + n) * DK + r) * DV;
      const float c = p.carry[static_cast<int64_t>(bh * N + n) * DK + r];
      float dc = 0.f;
      uint8_t* dsb = smem + BwdSmem::DSB;
#pragma unroll 1
      for (int h = 0; h < 4; ++h) {
        uint32_t a[32];
        tmem_ld32(tDS + lrow + h * 32, a);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f[8], sv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(a[j * 8 + e]);
          const uint4 pk = pack8(f);
          *reinterpret_cast<uint4*>(dsb + (h >> 1) * 16384 + swz(r, (h & 1) * 4 + j)) = pk;
          *reinterpret_cast<uint4*>(p.ds + srow + h * 32 + j * 8) = pk;
          unpack8(*reinterpret_cast<const uint4*>(p.states + srow + h * 32 + j * 8), sv);
#pragma unroll
          for (int e = 0; e < 8; ++e) dc += sv[e] * f[e];
        }
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          lo[e] = __float_as_uint(__uint_as_float(a[e]) * c);
          hi[e] = __float_as_uint(__uint_as_float(a[16 + e]) * c);
        }
        tmem_st16(tDS + lrow + h * 32, lo);
        tmem_st16(tDS + lrow + h * 32 + 16, hi);
      }
      p.dcarry[static_cast<int64_t>(bh * N + n) * DK + r] = dc;
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(dsb_ready);
      // du^T row r (value r): saved, and -du as the K-major operand of the dS update
      if (!warp_wait(du_full, m & 1, 0x631u, abort_flag)) break;
      tc_fence_after();
      uint8_t* dub = smem + BwdSmem::DUB;
      __nv_bfloat16* drow = p.dut + (static_cast<int64_t>(bh * N + n) * DV + r) * CH;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t a[32];
        tmem_ld32(tDU + lrow + h * 32, a);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f[8], nf[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            f[e] = __uint_as_float(a[j * 8 + e]);
            nf[e] = -f[e];
          }
          *reinterpret_cast<uint4*>(drow + h * 32 + j * 8) = pack8(f);
          *reinterpret_cast<uint4*>(dub + swz(r, h * 4 + j)) = pack8(nf);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(dub_ready);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 256);
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

// bf16 [rows, cols] row-major, box {64 columns, 64 rows}, 128-byte swizzle.
CUtensorMap map2d(const void* base, int64_t cols, int64_t rows) {
  if (reinterpret_cast<uintptr_t>(base) % 16 || (cols * 2) % 16) throw std::runtime_error("delta scan operand alignment");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  cuuint32_t box[2] = {64u, 64u};
  cuuint32_t es[2] = {1u, 1u};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (delta scan) failed: " + std::to_string(int(r)));
  return m;
}

}  // namespace
}  // namespace nt

using namespace nt;

int nt_delta_scan_fwd(const DeltaScanFwdArgs& a, cudaStream_t stream) {
  nt::current_context();
  if (a.BH <= 0 || a.N <= 0) return -1;
  const int64_t rows = static_cast<int64_t>(a.BH) * a.N * CH;
  const CUtensorMap tw = map2d(a.w, DK, rows), tq = map2d(a.qt, DK, rows), tk = map2d(a.kc, DK, rows),
                    ta = map2d(a.aqk, CH, rows), tu = map2d(a.u0, DV, rows);
  FwdParams p{a.N, a.carry, a.o, a.states, a.u};
  static std::atomic<uint64_t> smem_set{0};
  nt::smem_limit(smem_set, delta_scan_fwd_kernel, FwdSmem::TOTAL);
  delta_scan_fwd_kernel<<<dim3(DV / VB, a.BH), 192, FwdSmem::TOTAL, stream>>>(tw, tq, tk, ta, tu, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int nt_delta_scan_bwd(const DeltaScanBwdArgs& a, cudaStream_t stream) {
  nt::current_context();
  if (a.BH <= 0 || a.N <= 0) return -1;
  const int64_t rows = static_cast<int64_t>(a.BH) * a.N * CH;
  const CUtensorMap td = map2d(a.dout, DV, rows), ta = map2d(a.aqk, CH, rows), tk = map2d(a.kc, DK, rows),
                    tq = map2d(a.qt, DK, rows), tw = map2d(a.w, DK, rows);
  BwdParams p{a.N, a.carry, a.states, a.ds, a.dut, a.dcarry};
  static std::atomic<uint64_t> smem_set{0};
  nt::smem_limit(smem_set, delta_scan_bwd_kernel, BwdSmem::TOTAL);
  delta_scan_bwd_kernel<<<a.BH, 192, BwdSmem::TOTAL, stream>>>(td, ta, tk, tq, tw, p);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int nt_delta_scan_read_error(unsigned* where) {
  ErrorWord e{};
  cudaMemcpyFromSymbol(&e, g_nt_error, sizeof(e));
  if (where) *where = e.where;
  if (e.code) {
    const ErrorWord z{};
    cudaMemcpyToSymbol(g_nt_error, &z, sizeof(z));
  }
  return static_cast<int>(e.code);
}
