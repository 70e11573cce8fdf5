// Head-mean distillation teacher of the learned sparse indexers (sparse_teacher.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime_api.h>
#include <stdint.h>

struct TeacherArgs {
  int B = 0, H = 0, Hk = 0, Q = 0, T = 0, D = 128;
  int q_start = 0;          // absolute position of query row 0
  float scale = 1.f;
  const __nv_bfloat16* q = nullptr;   // element (b, h, i, d) at b sqb + h sqh + i sqt + d
  int64_t sqb = 0, sqh = 0, sqt = 0;
  const __nv_bfloat16* k = nullptr;   // element (b, hk, j, d) at b skb + hk skh + j skt + d
  int64_t skb = 0, skh = 0, skt = 0;
  const uint8_t* mask = nullptr;      // [B, Q, T] (1 = in the domain) or null: causal only
  float* lse = nullptr;               // [B, H, Q] workspace
  float* out = nullptr;               // [B, Q, T] fp32, zero-filled by the caller
};

// Return 0, -1 for unsupported arguments (head dim 128, 16-byte aligned rows).
int nt_sparse_teacher(const TeacherArgs& a, cudaStream_t s);
