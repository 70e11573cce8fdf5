// Host interface of the optimizer kernels (optim.cu).
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

struct AdamWHyper {
  float lr, beta1, beta2, eps, wd, bias1, bias2;
};

int nt_adamw(void* p, int p_is_bf16, const float* g, float* m, float* v, void* shadow, int64_t n, AdamWHyper h,
             cudaStream_t s);
// Pointer tables (grads, moms, smbs, params, shadows) live in device memory.
int nt_muon_prep(float* const* grads, float* const* moms, void* X, float* rowss, int K, int m, int n, float mu,
                 cudaStream_t s);
int nt_muon_normalize(void* X, const float* rowss, float* tot, int K, int m, int n, cudaStream_t s);
int nt_muon_finish(const void* X, float* red, float* tot, float* const* smbs, float* fscale, float* const* params,
                   void* const* shadows, int K, int m, int n, float beta2, float lr, float wd, cudaStream_t s);
