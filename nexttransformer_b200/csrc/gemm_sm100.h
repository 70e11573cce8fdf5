// Host interface of the sm_100a GEMM engine (gemm_sm100.cu).
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

// Fused epilogues.  acc is the fp32 accumulator of sum_k A[m,k] B[n,k].
enum NtGemmEpilogue : int {
  EPI_BF16 = 0,        // C(bf16) = s_acc * acc
  EPI_F32 = 1,         // C(f32)  = s_acc * acc
  EPI_F32_ACC = 2,     // C(f32) += s_acc * acc              (weight-gradient accumulation)
  EPI_BF16_AXPBY = 3,  // C(bf16) = bf16(s_acc * acc) + s_res * R   (residual add, Newton-Schulz)
  EPI_RELU2 = 4,       // P(bf16) = acc ; C(bf16) = relu(P)^2        (MLP up-projection)
  EPI_RELU2_BWD = 5,   // C(bf16) = bf16(acc) * 2 relu(R)            (R = saved pre-activation)
  // Soft-capped cross-entropy fused into the LM head (acc = logit x, t = tanh(x / cap),
  // z = cap t, e = exp(z - cap); columns >= vocab are padding):
  EPI_CE_FWD = 6,      // C(bf16) = e (1 - t^2); ce.part[row, col / 128] = sum of e over the 128
                       // columns; ce.ztgt[row] = z at column ce.tgt[row]
  EPI_CE_DGRAD = 7,    // C(bf16) = s_acc (ce.rscale[row] acc - ce.rcorr[row] ce.w[ce.tgt[row], col])
};

// Extra operands of the cross-entropy epilogues.
struct CeArgs {
  const int64_t* tgt = nullptr;   // [M] target ids (-1: ignored row)
  float* part = nullptr;          // EPI_CE_FWD: [M, ceil(N / 128)] partial sums of e
  float* ztgt = nullptr;          // EPI_CE_FWD: [M] soft-capped target logit (left as is for ignored rows)
  int vocab = 0;
  float cap = 15.f;
  const float* rscale = nullptr;  // EPI_CE_DGRAD: [M] 1 / sum_e (0 for ignored rows)
  const float* rcorr = nullptr;   // EPI_CE_DGRAD: [M] 1 - (z_target / cap)^2 (0 for ignored rows)
  const void* w = nullptr;        // EPI_CE_DGRAD: head weight [vocab rows, N] (bf16)
  int64_t ldw = 0;
};

struct GemmArgs {
  int M = 0, N = 0, K = 0, batch = 1;
  // A is logical [M, K]: a_mn = 0 -> stored [M, K] with row stride lda (elements);
  //                      a_mn = 1 -> stored [K, M] with row stride lda.
  const void* A = nullptr;
  int64_t lda = 0, strideA = 0;
  int a_mn = 0;
  // B is logical [N, K]: b_mn = 0 -> stored [N, K]; b_mn = 1 -> stored [K, N].
  const void* B = nullptr;
  int64_t ldb = 0, strideB = 0;
  int b_mn = 0;
  void* C = nullptr;
  int64_t ldc = 0, strideC = 0;
  const void* R = nullptr;
  int64_t ldr = 0, strideR = 0;
  void* P = nullptr;
  int64_t ldp = 0, strideP = 0;
  float s_acc = 1.f, s_res = 1.f;
  const float* s_ptr = nullptr;  // optional device scalar multiplying s_acc
  int epi = EPI_BF16;
  int num_sms = 148;
  // Optional fp32 workspace for split-K (EPI_F32 / EPI_F32_ACC only): the reduction dimension
  // is cut into slices whose partial products land in the workspace and are summed in a fixed
  // order by a second kernel, so results are deterministic.
  void* workspace = nullptr;
  size_t workspace_bytes = 0;
  int split_k = 1;  // set by the launcher
  CeArgs ce;
  // bf16 outputs leave through shared memory and bulk tensor stores when the layout allows it
  // (16-byte aligned base and row stride); 0 forces per-thread global stores.
  int tma_out_ok = 1;
  // Grouped (expert) modes, at most one set; device tables, so the host never reads the counts.
  //  grp_m [ceil(M/128)]: batch index of B for each 128-row tile of A and C (-1: tile has no
  //        rows); A and C are single matrices, B is a stack of `groups` matrices (strideB).
  //  grp_k [groups + 1]: row offsets (multiples of 64) of each group along the reduction
  //        dimension; A and B are single matrices, C a stack of `groups` (strideC).  Groups with
  //        no rows leave C untouched, so only EPI_F32_ACC is allowed.
  const int* grp_m = nullptr;
  const int* grp_k = nullptr;
  int groups = 0;
};

// Bytes of workspace nt_gemm_launch would use for split-K on this problem (0 = no split).
size_t nt_gemm_splitk_bytes(const GemmArgs& args);

void nt_gemm_launch(const GemmArgs& args, cudaStream_t stream);
// Cross-entropy row statistics from the EPI_CE_FWD partial sums: per row S = sum(part),
// loss = cap + log S - ztgt, rscale = 1 / S, rcorr = 1 - (ztgt / cap)^2 (all 0 for ignored rows).
int nt_ce_finish(const float* part, int nparts, const int64_t* tgt, const float* ztgt, float* loss, float* rscale,
                 float* rcorr, int rows, float cap, cudaStream_t stream);
// Returns the first error code recorded by a bounded wait in a GEMM kernel (0 = none).
int nt_gemm_read_error(unsigned* where);
