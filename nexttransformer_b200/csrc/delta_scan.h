// Host interface of the inter-chunk delta-rule scan (delta_scan.cu).  Chunk length 64, 128 key
// and 128 value features; every bf16 operand is a contiguous [BH, N, rows, cols] tensor.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime_api.h>
#include <stdint.h>

struct DeltaScanFwdArgs {
  int BH = 0, N = 0;
  const void* w = nullptr;       // [BH, N, 64, 128]  WY keys  (T beta k~)
  const void* qt = nullptr;      // [BH, N, 64, 128]  decayed queries q~
  const void* kc = nullptr;      // [BH, N, 64, 128]  keys decayed to the chunk end
  const void* aqk = nullptr;     // [BH, N, 64, 64]   masked intra-chunk scores
  const void* u0 = nullptr;      // [BH, N, 64, 128]  WY values (T beta v)
  const float* carry = nullptr;  // [BH, N, 128]      per-key decay over the chunk
  __nv_bfloat16* o = nullptr;       // out [BH, N, 64, 128]
  __nv_bfloat16* states = nullptr;  // out [BH, N, 128, 128] state entering each chunk
  __nv_bfloat16* u = nullptr;       // out [BH, N, 64, 128]  u = u0 - w S
};

struct DeltaScanBwdArgs {
  int BH = 0, N = 0;
  const void* dout = nullptr;    // [BH, N, 64, 128]
  const void* w = nullptr;
  const void* qt = nullptr;
  const void* kc = nullptr;
  const void* aqk = nullptr;
  const float* carry = nullptr;
  const __nv_bfloat16* states = nullptr;
  __nv_bfloat16* ds = nullptr;      // out [BH, N, 128, 128] gradient of the state leaving each chunk
  __nv_bfloat16* dut = nullptr;     // out [BH, N, 128, 64]  du^T
  float* dcarry = nullptr;          // out [BH, N, 128]
};

int nt_delta_scan_fwd(const DeltaScanFwdArgs& a, cudaStream_t stream);
int nt_delta_scan_bwd(const DeltaScanBwdArgs& a, cudaStream_t stream);
int nt_delta_scan_read_error(unsigned* where);
