// Sparse attention kernels for float inputs (all output types and head dims).
#include "wf_attn.cuh"

namespace wf {
int launch_sparse_attention_f32(const AttnParams& p, int out_dtype, cudaStream_t s) {
  return launch_ti<float>(p, out_dtype, s);
}
}  // namespace wf
