// Fused mixture-of-experts routing (moe_route.cu): softmax router, biased top-k choice, normalised
// weights, the grouped-GEMM row plan and the balance / z losses, in three launches; and the
// router-logit gradient in one.
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

constexpr int NT_ROUTE_TOKENS = 128;  // tokens per routing block
constexpr int NT_ROUTE_PAD = 128;     // rows of one grouped-GEMM tile: expert segments are padded to it

struct MoeRouteArgs {
  int N = 0, E = 0, k = 0;      // tokens, experts (E % 32 == 0, E <= 256), choices per token (k <= 16)
  int P = 0;                    // capacity of the padded row layout: round_up(N k, 128) + 128 E
  const float* logits = nullptr;  // [N, E] fp32
  const float* bias = nullptr;    // [E] selection bias (aux-free balancing) or null
  float aux_coeff = 0.f, z_coeff = 0.f;
  // per-token outputs
  int* choice = nullptr;   // [N, k] expert ids, by decreasing biased score
  float* w = nullptr;      // [N, k] softmax probabilities of the choices, normalised over the k
  float* lse = nullptr;    // [N] log-sum-exp of the logits
  // workspace, [ceil(N / 128), E] each, and [ceil(N / 128)]
  int* blk_counts = nullptr;
  float* blk_probs = nullptr;
  float* blk_z = nullptr;
  // plan
  int* counts = nullptr;     // [E]
  int* seg_start = nullptr;  // [E] first row of each expert's padded segment
  int* blk_offset = nullptr; // [ceil(N / 128), E] rows of earlier blocks within each segment
  int* grp_m = nullptr;      // [P / 128] expert of each row tile, -1 past the last segment
  int* grp_k = nullptr;      // [E + 1] segment boundaries
  int* row_of = nullptr;     // [N k] row of each (token, choice)
  int* src_of = nullptr;     // [P] token of each row, -1 for padding
  float* load = nullptr;     // [E] += counts (optional)
  float* aux_grad = nullptr; // [E] d(balance loss) / d(prob of expert e at one token)
  float* aux = nullptr;      // [2] balance loss, z loss
};

// Return 0, -1 for unsupported arguments.
int nt_moe_route(const MoeRouteArgs& a, cudaStream_t s);
// dlogits [N, E] = d(w, aux) / d logits given dw [N, k] (null: zero) and the gradient of the summed
// losses daux (a device scalar, read on the device; null: zero).
int nt_moe_route_bwd(const float* logits, const float* lse, const int* choice, const float* w, const float* dw,
                     const float* aux_grad, const float* daux, float z_coeff, float* dlogits, int N, int E, int k,
                     cudaStream_t s);
