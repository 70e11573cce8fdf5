// Host interface of the elementwise / row-reduction kernels (elementwise.cu).
// Every bf16 row pointer must be 16-byte aligned and every row length a multiple of 8;
// the Python wrappers check this before calling.  Return value: 0 ok, -1 unsupported shape.
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

int nt_mix_norm_fwd(const void* x, const void* x0, const float* ab, void* xm, void* h, float* rstd, int M, int d,
                    float out_scale, cudaStream_t s);
int nt_norm_bwd(const void* x, const void* dy, const void* dres, void* dx, int M, int d, cudaStream_t s);
int nt_mix_norm_bwd(const void* x, const void* x0, const void* xm, const void* dh, const void* dres,
                    const float* ab, void* dx, float* dx0_acc, float* part, int M, int d, cudaStream_t s);
int nt_rope_norm_fwd(void* qkv, const void* cosb, const void* sinb, float* rstd, int M, int T, int H, int Hk, int D,
                     float scale, const void* ve_table, const int64_t* idx, const void* hrow, int ldh,
                     const void* wg, int G, float* gate_out, cudaStream_t s);
int nt_rope_norm_bwd(void* dqkv, const void* qkv, const void* cosb, const void* sinb, const float* rstd, int M,
                     int T, int H, int Hk, int D, float scale, const void* ve_table, const int64_t* idx,
                     const float* gate, float* dz, float* ve_grad, cudaStream_t s);
// variant is reserved for alternative kernels (0 = default)
int nt_softcap_ce(void* logits, int64_t ld, const int64_t* tgt, float* loss, float* lse, int rows, int V, int Vp,
                  float cap, int variant, cudaStream_t s);
int nt_embed_smear(const void* wte, const int64_t* idx, const void* wsm, const float* lam, void* n_out, void* x_out,
                   float* gate_out, int M, int T, int d, int G, cudaStream_t s);
int nt_embed_scatter(const void* dy, int dy_is_f32, const int64_t* idx, float* grad, int M, int d, cudaStream_t s);
int nt_cast_bf16(const float* src, void* dst, int64_t n, cudaStream_t s);
