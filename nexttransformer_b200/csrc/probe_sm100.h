// tcgen05.mma issue-rate probe (probe_sm100.cu).
#pragma once
#include <cuda_runtime_api.h>

// out: int64 [ctas, 3] = (issue clocks, clocks to the last completion, wait succeeded).  Returns 0,
// -1 for bad arguments, -2 for a launch error.
int nt_mma_rate(int variant, int groups, int ctas, long long* out, cudaStream_t s);
