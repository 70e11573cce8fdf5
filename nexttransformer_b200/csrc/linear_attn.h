// Host interface of the linear-attention elementwise kernels (linear_attn.cu).  bf16 activations,
// fp32 weights / gains / reductions.  Return 0, or -1 for an unsupported shape.
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

// x, y, pre: [B, T, C] (C % 8 == 0); w: [C, K] fp32, 2 <= K <= 4.  pre (optional) keeps the conv output.
int nt_causal_conv_silu_fwd(const void* x, const float* w, void* y, void* pre, int B, int T, int C, int K,
                            cudaStream_t s);
// dw (fp32 [C, K]) is accumulated into (zero it first).
int nt_causal_conv_silu_bwd(const void* x, const void* pre, const void* dy, const float* w, void* dx, float* dw,
                            int B, int T, int C, int K, cudaStream_t s);
// Canon layer: y = x + causal depthwise conv(x) (no activation); dw accumulated as above.
int nt_canon_conv_fwd(const void* x, const float* w, void* y, int B, int T, int C, int K, cudaStream_t s);
int nt_canon_conv_bwd(const void* x, const void* dy, const float* w, void* dx, float* dw, int B, int T, int C, int K,
                      cudaStream_t s);
// rows of D (64 or 128) channels; gain fp32 [D]; rstd fp32 [rows] saved for the backward.
int nt_gated_rmsnorm_fwd(const void* x, const void* g, const float* gain, void* y, float* rstd, int64_t rows, int D,
                         cudaStream_t s);
// dgain (fp32 [D]) is accumulated into (zero it first); work: fp32 [NT_GATED_NORM_PARTS, D] scratch for
// the per-block partial sums (deterministic: no atomics).
constexpr int NT_GATED_NORM_PARTS = 592;
int nt_gated_rmsnorm_bwd(const void* x, const void* g, const float* gain, const float* rstd, const void* dy, void* dx,
                         void* dg, float* dgain, float* work, int64_t rows, int D, cudaStream_t s);
