// Sparse attention entry: dtype dispatch to the per-input-dtype translation units.
#include "wf_common.cuh"
#include "wf_kernels.h"

namespace wf {

int launch_sparse_attention_bf16(const AttnParams& p, int out_dtype, cudaStream_t s);
int launch_sparse_attention_f16(const AttnParams& p, int out_dtype, cudaStream_t s);
int launch_sparse_attention_f32(const AttnParams& p, int out_dtype, cudaStream_t s);

int attn_max_k() { return 512; }

int launch_sparse_attention(const AttnParams& p, int dtype, int out_dtype, cudaStream_t stream) {
  if (p.K < 1 || p.K > attn_max_k()) return -1;
  switch (dtype) {
    case kBF16: return launch_sparse_attention_bf16(p, out_dtype, stream);
    case kF16: return launch_sparse_attention_f16(p, out_dtype, stream);
    case kF32: return launch_sparse_attention_f32(p, out_dtype, stream);
    default: return -1;
  }
}

}  // namespace wf
