// Per-chunk terms of the chunked (gated) delta rule, forward and backward (delta_prep.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime_api.h>
#include <stdint.h>

// Gate modes: no decay (DeltaNet), one log decay per token and head (Gated DeltaNet, with the
// q / k L2 normalisation done here), one log decay per token, head and key feature (KDA).
enum DeltaGate : int { DELTA_NONE = 0, DELTA_SCALAR = 1, DELTA_FEATURE = 2 };

struct DeltaPrepArgs {
  int B = 0, T = 0, H = 0;   // inputs [B, T, H, 128] (q, k, v), g [B, T, H] or [B, T, H, 128], beta [B, T, H]
  int gate = DELTA_NONE;
  int in_bf16 = 1;           // q / k / v element type: bf16 (1) or fp32 (0)
  float qk_scale = 1.f;      // DELTA_SCALAR: q <- qk_scale q / |q|, k <- k / |k|
  const void* q = nullptr;
  const void* k = nullptr;
  const void* v = nullptr;
  const float* g = nullptr;
  const float* beta = nullptr;
  // forward outputs, chunk-major [B*H, N, 64, ...]: w, u0, qt, kc bf16 [.., 128]; aqk bf16 [.., 64];
  // carry fp32 [B*H, N, 128]
  void* w = nullptr;
  void* u0 = nullptr;
  void* qt = nullptr;
  void* kc = nullptr;
  void* aqk = nullptr;
  float* carry = nullptr;
  // backward inputs: the forward's w and u0 above, and (fp32, chunk-major as above) the gradients;
  // outputs fp32 in the input layouts
  const float* dw = nullptr;
  const float* du0 = nullptr;
  const float* dqt = nullptr;
  const float* dkc = nullptr;
  const float* daqk = nullptr;
  const float* dcarry = nullptr;
  float* dq = nullptr;
  float* dk = nullptr;
  float* dv = nullptr;
  float* dg = nullptr;
  float* dbeta = nullptr;
  // DELTA_FEATURE options.  qk_norm: q <- qk_scale q / |q| and k <- k / |k| here, as DELTA_SCALAR
  // always does.  g_raw: the gate from its pre-activation instead of g,
  //   g = -exp(g_log[h, d]) softplus(g_raw + g_bias[h, d])   (g_raw bf16 [B, T, H, 128]; g_log, g_bias fp32 [H, 128]);
  // its backward writes dg_raw (bf16, the layout of g_raw) and per-chunk partial sums of the g_log / g_bias
  // gradients, fp32 [B, N, H, 128], that the caller sums over (B, N); dg is then not written.
  int qk_norm = 0;
  const __nv_bfloat16* g_raw = nullptr;
  const float* g_log = nullptr;
  const float* g_bias = nullptr;
  __nv_bfloat16* dg_raw = nullptr;
  float* dg_log_part = nullptr;
  float* dg_bias_part = nullptr;
};

// Return 0 on success, -1 for an unsupported shape.
int nt_delta_prep_fwd(const DeltaPrepArgs& a, cudaStream_t stream);
int nt_delta_prep_bwd(const DeltaPrepArgs& a, cudaStream_t stream);
