// K1: flash attention for sm_100a (forward and backward) -- see attention_sm100.h.
#include "attention_sm100.h"
#include "common.cuh"

int nt_attention_fwd(const AttnArgs&, cudaStream_t) { return -1; }
int nt_attention_bwd(const AttnArgs&, cudaStream_t) { return -1; }
int nt_attention_read_error(unsigned* where) {
  nt::ErrorWord w{0, 0};
  cudaMemcpyFromSymbol(&w, nt::g_nt_error, sizeof(w));
  if (where) *where = w.where;
  return static_cast<int>(w.code);
}
