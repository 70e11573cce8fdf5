// Host interface of the mixture-of-experts row movement kernels (moe.cu).  bf16 rows of d
// features (d % 8 == 0); index tables are int32.  Return 0, -1 for bad arguments.
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

int nt_moe_gather_rows(const void* src, const int* src_of, void* out, int64_t rows, int d, cudaStream_t s);
int nt_moe_combine(const void* rows, const int* row_of, const float* w, const void* add, void* out, int T, int k, int d,
                   cudaStream_t s);
int nt_moe_combine_bwd(const void* dy, const void* rows, const int* row_of, const float* w, void* d_rows, float* dw,
                       int T, int k, int d, cudaStream_t s);
int nt_moe_pull_rows(const uint64_t* peers, const int* src_rank, const int* src_row, void* out, int64_t rows, int d,
                     cudaStream_t s);
int nt_moe_push_rows(const void* rows, const uint64_t* peers, const int* dst_rank, const int* dst_row, int64_t n, int d,
                     cudaStream_t s);
