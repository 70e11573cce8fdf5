// Allocation-free weight-gradient GEMM entry point.
//
// No counterpart in the reference: this entry point exists only in this library.
//
// Who needs it: code that drives the GPU but is not allowed to allocate device memory at the
// moment it runs - for example a host runtime that pre-plans every allocation up front and
// forbids further cudaMalloc/cudaFree calls, a caller that holds a lock the caching allocator
// may also need, or foreign code (C, Rust, another framework) that links this library without
// PyTorch and therefore has no allocator to borrow.  The PyTorch binding of the GEMM asks the
// caching allocator for its split-K workspace on every call; this entry point instead uses a
// fixed scratch array that the library reserves once, when it is loaded.
//
// What it computes: the weight-gradient product of a Linear layer,
//     C[M, N] (fp32) = alpha * sum_k A[k, m] * B[k, n]   (+ C when accumulate != 0)
// with A stored [K, M] (bf16, row stride lda) and B stored [K, N] (bf16, row stride ldb), i.e.
// dW = dY^T X with the reduction over K tokens.  When the problem has too few output tiles to
// fill the GPU, the reduction is split into slices whose fp32 partial products are written to
// the scratch array and summed in a fixed order (deterministic), exactly as the allocating path
// does with its workspace.
//
// Limits and sharing:
//  * The scratch array holds NT_NOALLOC_SCRATCH_BYTES (64 MiB) per GPU.  Every GPU that loads the
//    library reserves it until the process exits.  A problem whose split-K partial products would
//    not fit is rejected with NT_NOALLOC_TOO_LARGE; nothing is launched.
//  * All calls on a GPU share the one array and it keeps whatever the previous call left in it.
//    Nothing needs to start at zero: every partial-product element a call reads was written by
//    that same call first.  Two calls whose kernels overlap on the GPU (different streams without
//    ordering) race on the array; order them on one stream, or with events.
//  * Errors: the C declarations and return codes are in gemm_noalloc.h.  A bounded wait that
//    times out inside the kernel is reported by nt_wgrad_noalloc_read_error once the stream
//    has finished (the launch itself has already returned NT_NOALLOC_OK by then).
//  * Set-up: the first call on each device looks up the array's device address with
//    cudaGetSymbolAddress while that device is current (host code cannot use the array's name as
//    a device pointer).  That first call should therefore come before any stream capture.
#include <cuda_runtime.h>
#include <stdint.h>

#include <exception>
#include <mutex>

#include "gemm_noalloc.h"
#include "gemm_sm100.h"

namespace {

constexpr size_t NT_NOALLOC_SCRATCH_BYTES = size_t(64) << 20;
constexpr int NT_NOALLOC_MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[NT_NOALLOC_SCRATCH_BYTES];

struct DeviceSlot {
  void* ptr = nullptr;
  int sms = 0;
  bool ready = false;
};
DeviceSlot g_slots[NT_NOALLOC_MAX_DEVICES];
std::mutex g_setup_lock;

// Once per device, with that device current: the scratch array's device address and SM count.
int setup_device(int dev, DeviceSlot** out) {
  if (dev < 0 || dev >= NT_NOALLOC_MAX_DEVICES) return NT_NOALLOC_BAD_DEVICE;
  std::lock_guard<std::mutex> guard(g_setup_lock);
  DeviceSlot& slot = g_slots[dev];
  if (!slot.ready) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return NT_NOALLOC_SETUP_FAILED;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
      return NT_NOALLOC_SETUP_FAILED;
    slot.ptr = ptr;
    slot.sms = sms;
    slot.ready = true;
  }
  *out = &slot;
  return 0;
}

}  // namespace

extern "C" int nt_wgrad_splitk_noalloc(const void* A, int64_t lda, const void* B, int64_t ldb, float* C, int64_t ldc,
                                       int M, int N, int K, float alpha, int accumulate, void* stream) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0) return NT_NOALLOC_BAD_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(A) % 16 || reinterpret_cast<uintptr_t>(B) % 16 ||
      reinterpret_cast<uintptr_t>(C) % 16 || (lda * 2) % 16 || (ldb * 2) % 16 || ldc % 4 || lda < M || ldb < N ||
      ldc < N)
    return NT_NOALLOC_BAD_ARGUMENT;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return NT_NOALLOC_SETUP_FAILED;
  DeviceSlot* slot = nullptr;
  const int rc = setup_device(dev, &slot);
  if (rc) return rc;

  GemmArgs g;
  g.M = M;
  g.N = N;
  g.K = K;
  g.batch = 1;
  g.A = A;
  g.lda = lda;
  g.a_mn = 1;  // A logical [M, K] stored [K, M]
  g.B = B;
  g.ldb = ldb;
  g.b_mn = 1;  // B logical [N, K] stored [K, N]
  g.C = C;
  g.ldc = ldc;
  g.s_acc = alpha;
  g.epi = accumulate ? EPI_F32_ACC : EPI_F32;
  g.num_sms = slot->sms;
  const size_t need = nt_gemm_splitk_bytes(g);
  if (need > NT_NOALLOC_SCRATCH_BYTES) return NT_NOALLOC_TOO_LARGE;
  if (need) {
    g.workspace = slot->ptr;
    g.workspace_bytes = NT_NOALLOC_SCRATCH_BYTES;
  }
  // An error left pending by unrelated earlier work is cleared first, so that the error read
  // after the launch is this launch's own.  No C++ exception may cross the C interface.
  (void)cudaGetLastError();
  try {
    nt_gemm_launch(g, static_cast<cudaStream_t>(stream));
  } catch (const std::exception&) {
    return NT_NOALLOC_INTERNAL;
  } catch (...) {
    return NT_NOALLOC_INTERNAL;
  }
  return cudaGetLastError() == cudaSuccess ? NT_NOALLOC_OK : NT_NOALLOC_LAUNCH_FAILED;
}

extern "C" size_t nt_wgrad_splitk_noalloc_scratch_bytes(void) { return NT_NOALLOC_SCRATCH_BYTES; }

extern "C" int nt_wgrad_noalloc_read_error(unsigned* where) {
  try {
    return nt_gemm_read_error(where);
  } catch (...) {
    return -1;
  }
}
