// Residual-stream kernels on sm_100a: the log-domain Sinkhorn-Knopp projection of mHC.
//
// sinkhorn_knopp (nexttransformer/models/residual.py of the reference; models/residual.py here)
// alternates a column and a row log-normalisation of an n x n logit matrix `iterations` times
// and returns exp of the result.  The PyTorch form launches ~5 kernels per normalisation (200
// forward, ~300 backward for 20 iterations) on tiny [tokens, 4, 4] tensors.  Here one thread owns
// one token's matrix in registers:
//   forward   z <- lognorm_cols(z); z <- lognorm_rows(z)  (x iterations), out = exp(z)
//   backward  the log-softmax rule per normalisation, dz = dy - softmax . sum(dy), walked back
//             through the iterations from the normalised states (every state is kept in local
//             memory by the backward's own re-run of the forward).
// The max subtracted inside each normalisation is detached in the reference, which makes each
// step exactly a log-softmax, so the rule above is its full gradient.
#include <math.h>

#include "common.cuh"
#include "residual.h"

namespace nt {
namespace res {

constexpr int N = 4;
constexpr int MAX_IT = 32;

// log-softmax of the 4 x 4 matrix along columns (dim -2, over i) or rows (dim -1, over j)
NT_DEVICE void lognorm(float (&z)[N][N], bool cols) {
#pragma unroll
  for (int a = 0; a < N; ++a) {
    float m = -INFINITY;
#pragma unroll
    for (int b = 0; b < N; ++b) m = fmaxf(m, cols ? z[b][a] : z[a][b]);
    float s = 0.f;
#pragma unroll
    for (int b = 0; b < N; ++b) s += __expf((cols ? z[b][a] : z[a][b]) - m);
    const float lse = m + __logf(s);
#pragma unroll
    for (int b = 0; b < N; ++b) {
      if (cols) z[b][a] -= lse;
      else z[a][b] -= lse;
    }
  }
}

// dz = dy - exp(y) * sum(dy) along the normalised dimension (y = the normalisation's output)
NT_DEVICE void lognorm_bwd(const float (&y)[N][N], float (&g)[N][N], bool cols) {
#pragma unroll
  for (int a = 0; a < N; ++a) {
    float s = 0.f;
#pragma unroll
    for (int b = 0; b < N; ++b) s += cols ? g[b][a] : g[a][b];
#pragma unroll
    for (int b = 0; b < N; ++b) {
      if (cols) g[b][a] -= __expf(y[b][a]) * s;
      else g[a][b] -= __expf(y[a][b]) * s;
    }
  }
}

__global__ void sinkhorn_fwd_kernel(const float* __restrict__ logits, float* __restrict__ out, int64_t rows,
                                    int iterations) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows) return;
  float z[N][N];
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) z[i][j] = logits[t * N * N + i * N + j];
  for (int it = 0; it < iterations; ++it) {
    lognorm(z, true);
    lognorm(z, false);
  }
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) out[t * N * N + i * N + j] = __expf(z[i][j]);
}

__global__ void sinkhorn_bwd_kernel(const float* __restrict__ logits, const float* __restrict__ dout,
                                    float* __restrict__ dlogits, int64_t rows, int iterations) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= rows) return;
  // states after every normalisation (2 per iteration), kept in thread-local memory
  float st[2 * MAX_IT][N][N];
  float z[N][N];
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) z[i][j] = logits[t * N * N + i * N + j];
  for (int it = 0; it < iterations; ++it) {
    lognorm(z, true);
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) st[2 * it][i][j] = z[i][j];
    lognorm(z, false);
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) st[2 * it + 1][i][j] = z[i][j];
  }
  // out = exp(z): dz = dout * out
  float g[N][N];
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) g[i][j] = dout[t * N * N + i * N + j] * __expf(z[i][j]);
  for (int k = 2 * iterations - 1; k >= 0; --k) {
    float y[N][N];
#pragma unroll
    for (int i = 0; i < N; ++i)
#pragma unroll
      for (int j = 0; j < N; ++j) y[i][j] = st[k][i][j];
    lognorm_bwd(y, g, (k & 1) == 0);
  }
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < N; ++j) dlogits[t * N * N + i * N + j] = g[i][j];
}

}  // namespace res
}  // namespace nt

int nt_sinkhorn_fwd(const float* logits, float* out, int64_t rows, int n, int iterations, cudaStream_t s) {
  if (n != nt::res::N || iterations < 0 || iterations > nt::res::MAX_IT) return -1;
  if (!rows) return 0;
  nt::res::sinkhorn_fwd_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0, s>>>(logits, out, rows, iterations);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int nt_sinkhorn_bwd(const float* logits, const float* dout, float* dlogits, int64_t rows, int n, int iterations,
                    cudaStream_t s) {
  if (n != nt::res::N || iterations < 0 || iterations > nt::res::MAX_IT) return -1;
  if (!rows) return 0;
  nt::res::sinkhorn_bwd_kernel<<<static_cast<unsigned>((rows + 127) / 128), 128, 0, s>>>(logits, dout, dlogits, rows,
                                                                                         iterations);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}
