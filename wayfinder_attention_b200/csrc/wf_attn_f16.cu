// Sparse attention kernels for __half inputs (all output types and head dims).
#include "wf_attn.cuh"

namespace wf {
int launch_sparse_attention_f16(const AttnParams& p, int out_dtype, cudaStream_t s) {
  return launch_ti<__half>(p, out_dtype, s);
}
}  // namespace wf
