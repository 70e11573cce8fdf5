// NSA compressed branch on sm_100a (nsa_compress.cu): attention of every query over the compressed
// keys whose blocks are complete, the selection-block importance and the top-k block choice.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime_api.h>
#include <stdint.h>

struct NsaArgs {
  int B = 0, T = 0, H = 0, Hk = 0, Nc = 0, D = 128;
  int cstride = 16, csize = 32;   // compressed block c covers tokens [cstride c, cstride c + csize)
  int ssize = 64, topk = 16;      // selection blocks of ssize tokens; top-k complete blocks per row
  float scale = 1.f;
  // q [B, T, H, D], k / v (compressed) [B, Nc, Hk, D], o [B, T, H, D]: bf16, rows of H*D / Hk*D
  const __nv_bfloat16* q = nullptr;
  const __nv_bfloat16* k = nullptr;
  const __nv_bfloat16* v = nullptr;
  __nv_bfloat16* o = nullptr;
  float* lse = nullptr;            // [B, H, T] natural log; -inf for a row without complete blocks
  uint8_t* sel = nullptr;          // [B, H, T, nsel] 1 = selected (top-k complete blocks + the current one)
  // backward
  const __nv_bfloat16* dout = nullptr;  // [B, T, H, D]
  const float* delta = nullptr;         // [B, H, T] rowsum(dO * O)
  float* dq_acc = nullptr;              // fp32 [B, T, H, D], zeroed
  float* dk_acc = nullptr;              // fp32 [B, Nc, Hk, D], zeroed
  float* dv_acc = nullptr;              // fp32 [B, Nc, Hk, D], zeroed
  int bwd_splits = 0;                   // set by the launcher: CTAs sharing one key tile's query tiles
};

// Return 0, -1 for unsupported shapes (D 128, nsel <= 256, 16-byte aligned rows).
int nt_nsa_compressed_fwd(const NsaArgs& a, cudaStream_t s);
int nt_nsa_compressed_bwd(const NsaArgs& a, cudaStream_t s);
