// Host interface of the block-sparse attention kernels (sparse_attn.cu).  Head dimension 128;
// q / o / dout / dq are [B, T, H*128] bf16 with row strides, k / v [B, T, Hk*128]; lists
// [B, G, ceil(T/128), Lmax] int32 block ids of 64 keys (-1 ends a list); masks
// [B, G, ceil(T/128), Lmax, 4] uint32 row bits; head h uses list group h / (H / G).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime_api.h>
#include <stdint.h>

struct SparseAttnArgs {
  int B = 0, T = 0, H = 0, Hk = 0, D = 128, G = 1, Lmax = 0;
  float scale = 0.f;
  const void* q = nullptr;
  int64_t ldq = 0;
  const void* k = nullptr;
  int64_t ldk = 0;
  const void* v = nullptr;
  int64_t ldv = 0;
  const int* lists = nullptr;
  const uint32_t* masks = nullptr;
  __nv_bfloat16* o = nullptr;   // forward output
  int64_t ldo = 0;
  float* lse = nullptr;         // [B, H, T] natural-log sum-exp (+inf for rows that see no key)
  // backward
  const void* dout = nullptr;
  int64_t lddo = 0;
  const float* delta = nullptr; // [B, H, T] rowsum(dout * o)
  __nv_bfloat16* dq = nullptr;
  int64_t lddq = 0;
  float* dk_acc = nullptr;      // fp32 [B, T, Hk*128], added into
  float* dv_acc = nullptr;
  // optional additive relative bias (Inkling REL): logit(i, j) += rel[b, h, i, i - j] for j <= i
  const float* rel = nullptr;   // fp32 [B, H, T, rel_extent], rel_extent >= T
  float* drel = nullptr;        // backward: fp32 [B, H, T, rel_extent], entry (i, i - j) written once
  int rel_extent = 0;
};

int nt_sparse_attn_fwd(const SparseAttnArgs& a, cudaStream_t s);
int nt_sparse_attn_bwd(const SparseAttnArgs& a, cudaStream_t s);
int nt_sparse_attn_read_error(unsigned* where);
