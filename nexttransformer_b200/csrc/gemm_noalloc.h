/* C interface of the allocation-free weight-gradient GEMM (gemm_noalloc.cu).
 *
 * No counterpart in the reference: this entry point exists only in this library.
 *
 * For callers that cannot allocate device memory while they run: a host runtime that plans
 * every allocation up front, a caller holding a lock the caching allocator may also take, or
 * C / C++ / Rust code that links the library without PyTorch and so has no allocator at all.
 * The split-K scratch comes from a fixed 64 MiB device array that the library reserves per GPU
 * when it is loaded; see gemm_noalloc.cu for the sharing rules.
 *
 * Plain C: no C++ types and no exceptions cross this interface.
 */
#ifndef NT_GEMM_NOALLOC_H
#define NT_GEMM_NOALLOC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes of nt_wgrad_splitk_noalloc. */
enum {
  NT_NOALLOC_OK = 0,
  NT_NOALLOC_TOO_LARGE = 1,     /* split-K partial products exceed the scratch array; nothing launched */
  NT_NOALLOC_SETUP_FAILED = 2,  /* the scratch array's device address or the SM count could not be read */
  NT_NOALLOC_BAD_ARGUMENT = 3,  /* null pointer, non-positive size, misaligned operand or short stride */
  NT_NOALLOC_BAD_DEVICE = 4,    /* current device id outside 0..63 */
  NT_NOALLOC_LAUNCH_FAILED = 5, /* the kernel launch itself reported an error */
  NT_NOALLOC_INTERNAL = 6       /* the launcher rejected the problem (for example tensor-map encoding) */
};

/* C[M, N] (fp32, row stride ldc) = alpha * A^T B  (+ C when accumulate != 0), with
 * A stored [K, M] (bf16, row stride lda) and B stored [K, N] (bf16, row stride ldb):
 * the weight gradient dW = dY^T X of a Linear layer over K tokens.  Operands 16-byte aligned,
 * lda and ldb multiples of 8 elements, ldc a multiple of 4.  `stream` is a cudaStream_t (NULL:
 * the legacy default stream).  The call is asynchronous: a launch that succeeded can still
 * time out on the GPU, which nt_wgrad_noalloc_read_error reports after the stream has
 * finished. */
int nt_wgrad_splitk_noalloc(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc, int M,
                            int N, int K, float alpha, int accumulate, void* stream);

/* Capacity of the scratch array in bytes: the largest split-K partial-product buffer a call may need. */
size_t nt_wgrad_splitk_noalloc_scratch_bytes(void);

/* First error recorded by a bounded wait inside a GEMM kernel of this library (0 = none); `where`
 * (may be NULL) receives the location code.  Synchronous: call it after the stream has finished.
 * A nonzero value means the results of the GEMMs since the error are not valid. */
int nt_wgrad_noalloc_read_error(unsigned* where);

#ifdef __cplusplus
}
#endif

#endif /* NT_GEMM_NOALLOC_H */
