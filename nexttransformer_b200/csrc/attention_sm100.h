// Host interface of the sm_100a flash-attention kernels (attention_sm100.cu).
//
// Layout: q/k/v/o rows are tokens ([B*T, ...]); head h of a row starts at h * D within the
// row.  Rows may be strided (q, k and v are usually column slices of the packed qkv
// projection).  lse is [B, H, T] fp32 (natural log).  window < 0 means full causal attention;
// otherwise a query at position t sees keys t - window .. t.
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

struct AttnArgs {
  const void* q = nullptr;
  const void* k = nullptr;
  const void* v = nullptr;
  void* o = nullptr;
  float* lse = nullptr;
  int64_t ldq = 0, ldk = 0, ldv = 0, ldo = 0;  // row strides in elements
  int B = 0, T = 0, H = 0, Hk = 0, D = 128;
  int window = -1;
  float scale = 0.f;
  int num_sms = 148;
  // backward only
  const void* dout = nullptr;
  int64_t lddo = 0;
  void* dq = nullptr;
  void* dk = nullptr;
  void* dv = nullptr;
  int64_t lddq = 0, lddk = 0, lddv = 0;
  float* dq_acc = nullptr;  // fp32 [B*T, H*D] workspace (zeroed), or [dq_slices][B*T, H*D] (zeroed)
  // 0: dQ contributions of the key tiles are added into dq_acc with bulk reductions (order not
  // fixed); ceil(T / 128): deterministic mode, one slice per key tile written with plain stores
  // and summed in key-tile order by the conversion
  int dq_slices = 0;
  float* delta = nullptr;   // fp32 [B, H, T] workspace
  // Optional pipeline trace of the first CTA (int64 [4 roles][64 pairs][8 events] of SM clock
  // stamps; zero-filled by the caller).  Diagnostics only.
  long long* trace = nullptr;
};

// Return 0 on success, -1 when the shape is not supported by the kernels.
int nt_attention_fwd(const AttnArgs& a, cudaStream_t s);
int nt_attention_bwd(const AttnArgs& a, cudaStream_t s);
int nt_attention_read_error(unsigned* where);
