// Elementwise heads of the attention plugins (plugin_ops.cu).  bf16 tensors, contiguous rows of
// H heads x 128 channels (v: Hk heads).  Return 0, or -1 for an unsupported shape.
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

// z = y sigmoid(g); g has G = 128 channels per head (elementwise) or G = 1 (headwise).
int nt_gate_mul_fwd(const void* y, const void* g, void* z, int64_t rows, int H, int G, cudaStream_t s);
int nt_gate_mul_bwd(const void* y, const void* g, const void* dz, void* dy, void* dg, int64_t rows, int H, int G,
                    cudaStream_t s);
// z = y - <y, u> u, u = v / max(|v|, 1e-12) of the query head's KV head.
int nt_xsa_fwd(const void* y, const void* v, void* z, int64_t rows, int H, int Hk, cudaStream_t s);
int nt_xsa_bwd(const void* y, const void* v, const void* dz, void* dy, void* dv, int64_t rows, int H, int Hk,
               cudaStream_t s);
