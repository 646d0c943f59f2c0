// Host-side launch interface between the C ABI (wf_abi.cu) and the kernels.
// Not part of the public ABI: include/wayfinder.h is.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace wf {

// Causal top-K over address vectors.
//   query rows:  q[b, l, :]  for local row l in [0, Tq); its sequence position
//                g(l) = ((l / rt) * rs + r0) * rt + l % rt   (identity when rs=1, r0=0, rt>=Tq)
//   keys:        k[b, j, :]  for j in [0, Tk); row g may retrieve j <= g only.
//   output:      idx[(b * Tq + l) * K + s], s = slot (descending score, ties -> lower index)
struct TopkParams {
  const void* q;
  const void* k;
  int64_t qsb, qst, qsr;
  int64_t ksb, kst, ksr;
  int B, Tq, Tk, R, K;
  int pad_mode;          // 0: reference pads (g + K + s + 1) % Tk; 1: -1 (masked)
  int rt, rs, r0;        // query row map
  int32_t* idx;
  int cap;               // candidate buffer capacity per row (multiple of 32)
  int32_t* status;       // nullable; bit 1 set if a bounded wait timed out
  void* ws;              // workspace of the tensor-core kernel (see topk_tc_workspace_bytes)
  size_t ws_bytes;
  // Optional [B][Tq] per-row key limits (replaces the row map): row l of batch b may
  // retrieve keys j < lim[b][l]; non-decreasing along the rows.  Null: causal row map.
  const int32_t* lim;
};

// Sparse attention over retrieved rows, indices shared across heads.
struct AttnParams {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* idx;
  void* out;
  int64_t qsb, qsh, qst;
  int64_t ksb, ksh, kst;
  int64_t vsb, vsh, vst;
  int64_t osb, osh, ost;
  int64_t isb, ist, iss;
  int B, H, Tq, Tk, D, K;
  float scale;
  int mask_negative;     // 1: negative index = masked slot; 0: wraps like torch indexing
  int out_vec_ok;        // output rows are 16-byte aligned (vector stores allowed)
  // Keys of a sequence sharded in cyclic row blocks and all-gathered rank-major:
  // key j lives in rank (j / kv_tile) % kv_world at local row
  // (j / kv_tile / kv_world) * kv_tile + j % kv_tile.  kv_world = 1: identity.
  int kv_tile, kv_world;
  int64_t k_rank_stride, v_rank_stride;
  // > 0: the gathered rows arrive in chunks of kv_chunk_rows local rows, stored
  // chunk-major: local row lr of rank r is row lr % kv_chunk_rows of block
  // (lr / kv_chunk_rows) * kv_world + r, blocks k/v_rank_stride apart.
  int kv_chunk_rows;
  int32_t* status;       // nullable; bit 0 set on an out-of-range index
  // Attention-probability dropout (training): rate in [0, 1), 0 = off.  Element
  // (b, h, t, k) is kept when dropout_uniform(seed, ((b*H + h)*Tq + t)*K + k) >= rate.
  float drop_rate;
  uint64_t drop_seed;
};

// Returns a cudaError_t; a negative value means "unsupported configuration"
// (the caller formats the message).
int launch_causal_topk(const TopkParams& p, int dtype, cudaStream_t stream);
int launch_sparse_attention(const AttnParams& p, int dtype, int out_dtype, cudaStream_t stream);

// Tensor-core (tcgen05) top-K: bf16/fp16 addresses, R in {16, 32, 64}, K <= 128,
// Tk <= 65536, unit address stride, 16-byte aligned rows.
bool topk_tc_supported(const TopkParams& p, int dtype);
int launch_causal_topk_tc(const TopkParams& p, int dtype, cudaStream_t stream);
// Test hook: the next tensor-core top-K launch withholds CTA 1's arrive of bisection
// exchange `round` (0..7; negative: off) and bounds those waits by wait_ns.
void topk_tc_test_withhold(int round, uint64_t wait_ns);
// Allocation-free retrieval: capacity of the library's built-in scratch array and
// its device address on the current device (first call per device looks it up).
size_t noalloc_scratch_capacity();
int noalloc_scratch(void** out);

// Workspace bytes the tensor-core path needs for B*Tq query rows (0 if K > 128).
size_t topk_tc_workspace_bytes(int64_t B, int64_t Tq, int64_t Tk, int R, int K, int dtype);

// Shared-memory bytes the top-K kernel needs for (R, K); 0 if unsupported.
size_t topk_smem_bytes(int R, int K);
int topk_max_k();
int attn_max_k();

// Fused address projection (wf_addr_proj.cu): out[m, :] = normalize_group(x[m] W^T + b).
int launch_address_projection(const void* x, int dtype, int64_t M, int K, int64_t x_stride, const void* w,
                              const void* bias, int N, int group, int normalize, void* out, int64_t out_stride,
                              int32_t* status, cudaStream_t stream);

// Top-K over the keys a (B, T) padding mask keeps (wf_keymask.cu).  `prep` holds
// topk_key_mask_prep_bytes; p.ws the top-K workspace for (B, T, T).
size_t topk_key_mask_prep_bytes(int64_t B, int64_t T, int R, int esz);
int launch_topk_key_mask(TopkParams p, int dtype, const uint8_t* mask, int64_t msb, int64_t mst, void* prep,
                         cudaStream_t stream);

// Backward of the sparse attention (wf_attn_bwd.cu).
struct AttnBwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* dout;
  const int32_t* idx;
  void* dq;
  void* dk;
  void* dv;
  int64_t qsb, qsh, qst, ksb, ksh, kst, vsb, vsh, vst, osb, osh, ost;
  int64_t dqsb, dqsh, dqst, dksb, dksh, dkst, dvsb, dvsh, dvst;
  int64_t isb, ist, iss;
  int B, H, Tq, Tk, D, K;
  float scale;
  int mask_negative;
  int dq_vec_ok, dk_vec_ok, dv_vec_ok;
  float drop_rate;       // the forward's dropout (see AttnParams); 0 = off
  uint64_t drop_seed;
  float* P;      // [B][Tq][K][H] softmax probabilities (workspace)
  float* DS;     // [B][Tq][K][H] scale * ds (workspace)
  int32_t* cnt;  // [B][Tk] per-key counts, then fill cursors (workspace)
  int32_t* off;  // [B][Tk + 1] list offsets (workspace)
  int32_t* list; // [B][Tq * K] (t * K + slot) entries grouped by key (workspace)
  int32_t* status;
};
size_t attn_bwd_workspace_bytes(int64_t B, int64_t H, int64_t Tq, int64_t Tk, int K);
int launch_sparse_attention_backward(AttnBwdParams p, void* ws, size_t ws_bytes, int dtype, int grad_dtype,
                                     cudaStream_t stream);

// Gather-rate ceiling (wf_bench.cu): K and V rows of row_bytes (<= 1024) at the
// indices idx[n_query][K], 16-byte loads, nothing computed; -1 for bad sizes.
int launch_gather_rows_bench(const void* k, const void* v, int64_t row_bytes, int64_t stride_bytes,
                             const int32_t* idx, int64_t n_query, int K, int64_t n_rows, uint32_t* sink,
                             cudaStream_t stream);
// The same 1 KB rows moved by cp.async.bulk into shared memory (read back or not).
int launch_gather_rows_bulk_bench(const void* k, const void* v, int64_t stride_bytes, const int32_t* idx,
                                  int64_t n_query, int K, int64_t n_rows, int read_back, uint32_t* sink,
                                  cudaStream_t stream);

}  // namespace wf
