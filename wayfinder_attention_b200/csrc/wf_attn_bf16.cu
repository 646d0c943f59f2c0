// Sparse attention kernels for __nv_bfloat16 inputs (all output types and head dims).
#include "wf_attn.cuh"

namespace wf {
int launch_sparse_attention_bf16(const AttnParams& p, int out_dtype, cudaStream_t s) {
  return launch_ti<__nv_bfloat16>(p, out_dtype, s);
}
}  // namespace wf
