// MSAR element kernels (msar.cu): temporal augmentation and the depth-read gate.
#pragma once
#include <cuda_runtime_api.h>
#include <stdint.h>

struct MsarTemporalArgs {
  int B = 0, T = 0, C = 0;
  int bf16 = 1;                 // element type of x / y / dy / dx: bf16 (1) or fp32 (0)
  const void* x = nullptr;      // [B, T, C]
  const float* taps = nullptr;  // [C, 24]: widths 4, 8, 12 back to back
  void* y = nullptr;            // [B, T, 4, C]
  const void* dy = nullptr;     // [B, T, 4, C]
  void* dx = nullptr;           // [B, T, C]
  float* part = nullptr;        // nt_msar_temporal_part_floats(B, T, C) floats
  float* dtaps = nullptr;       // [C, 24]
};

struct MsarGateArgs {
  int N = 0, C = 0;
  int bf16 = 1;                 // element type of s / out / dout / ds
  const void* s = nullptr;      // [N, 4, C]
  const float* P = nullptr;     // [4 C, 4]
  const float* alpha = nullptr; // [1] (read on the device)
  const float* bias = nullptr;  // [4]
  void* out = nullptr;          // [N, C]
  float* zr = nullptr;          // [N, 5]: z and r per token (r = 0 marks an all-zero row)
  const void* dout = nullptr;   // [N, C]
  void* ds = nullptr;           // [N, 4, C]
  float* y = nullptr;           // [N, 4] workspace
  float* ab_part = nullptr;     // [N, 5]: per-token d alpha and d bias
  float* p_part = nullptr;      // [nt_msar_gate_proj_slices(N), 4 C, 4]
};

int nt_msar_temporal_fwd(const MsarTemporalArgs& a, cudaStream_t s);
int nt_msar_temporal_bwd(const MsarTemporalArgs& a, cudaStream_t s);
int nt_msar_temporal_part_floats(int B, int T, int C);
int nt_msar_gate_fwd(const MsarGateArgs& a, cudaStream_t s);
int nt_msar_gate_bwd(const MsarGateArgs& a, cudaStream_t s);
int nt_msar_gate_proj_slices(int N);
