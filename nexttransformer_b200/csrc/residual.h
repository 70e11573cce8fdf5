// Host interface of the residual-stream kernels (residual.cu).  fp32 [rows, n, n] matrices, n = 4.
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

int nt_sinkhorn_fwd(const float* logits, float* out, int64_t rows, int n, int iterations, cudaStream_t s);
int nt_sinkhorn_bwd(const float* logits, const float* dout, float* dlogits, int64_t rows, int n, int iterations,
                    cudaStream_t s);
