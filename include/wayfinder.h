/*
 * wayfinder.h — C ABI of libwayfinder_sm100.so, the B200 (sm_100a) kernels for
 * Wayfinder's causal learned-address retrieval + sparse attention forward.
 *
 * Every entry point takes plain device pointers, sizes and element strides,
 * enqueues work on the given CUDA stream and returns without synchronising.
 * Return value: WF_OK (0) or an error code; wf_last_error() then holds a
 * message for the calling thread.  Inputs are never written.
 *
 * Reference interfaces replaced (paths inside Wayland-The-Smith/wayfinder-attention):
 *   wf_causal_topk            <- routing_attention/kernels/causal_topk.py:470-521   causal_topk()
 *   wf_sparse_attention       <- routing_attention/kernels/fused_sparse.py:275-324  sparse_meat_attention()
 *   wf_fused_sparse_attention <- routing_attention/kernels/fused_sparse.py:327-356  fused_sparse_attention()
 *   wf_fused_sparse_attention_host: the same operator on host-resident tensors (copies overlapped)
 *   wf_address_projection     <- routing_attention/models/learned_address.py:39-46  forward_query_key()
 */
#ifndef WAYFINDER_H_
#define WAYFINDER_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WF_API __attribute__((visibility("default")))
#else
#define WF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types. */
#define WF_DTYPE_BF16 0
#define WF_DTYPE_F16 1
#define WF_DTYPE_F32 2

/* Return codes. */
#define WF_OK 0
#define WF_ERR_INVALID_ARGUMENT 1 /* bad shape, stride, pointer or value (Python: ValueError)   */
#define WF_ERR_UNSUPPORTED 2      /* valid request this build does not cover (Python: ValueError) */
#define WF_ERR_CUDA 3             /* CUDA launch/runtime failure (Python: RuntimeError)          */

/* Pad policy for query rows that have fewer than K causal keys (rows i < K-1). */
#define WF_PAD_REFERENCE 0 /* slot s >= i+1 gets index (i + K + s + 1) % T, attended unmasked,
                              as routing_attention/kernels/causal_topk.py:37-57 does        */
#define WF_PAD_MASKED 1    /* slot s >= i+1 gets -1 and is excluded from the softmax        */

/* Attention flags. */
#define WF_ATTN_MASK_NEGATIVE 1 /* a negative index is a masked slot (otherwise it wraps by T,
                                   like torch advanced indexing)                              */

/* Library version (major * 100 + minor). */
WF_API int wf_version(void);

/* Message describing the last error returned on this thread ("" if none). */
WF_API const char* wf_last_error(void);

/* Largest top_k that wf_causal_topk / wf_fused_sparse_attention accept. */
WF_API int wf_max_top_k(void);

/*
 * Exact causal top-K inner-product retrieval.  Replaces causal_topk()
 * (routing_attention/kernels/causal_topk.py:470-521; default path
 * _causal_topk_row_blocked :133-171 + _finalize_causal_topk :37-57).
 *
 *   q_addr  : (B, Tq, R) query addresses, strides q_strides[3] in elements
 *   k_addr  : (B, Tk, R) key addresses,   strides k_strides[3] in elements
 *   dtype   : WF_DTYPE_* of both address tensors (scores are computed in fp32)
 *   top_k   : requested K; K_eff = min(top_k, Tk) slots are written per row
 *   pad_mode: WF_PAD_REFERENCE or WF_PAD_MASKED
 *   row map : local query row l sits at sequence position
 *             g(l) = ((l / row_tile) * row_stride + row_start) * row_tile + l % row_tile
 *             and may retrieve keys j <= g(l).  row_tile = 0 selects the identity map
 *             (g(l) = l).  Otherwise row_tile must be a multiple of 64, row_stride >= 1,
 *             0 <= row_start < row_stride, and every g(l) < Tk.  This is how a rank of a
 *             query-row-sharded long sequence addresses its cyclic row blocks.
 *   idx_out : (B, Tq, K_eff) int32, contiguous.  Slots hold the retrieved key indices in
 *             an unspecified (deterministic) order; equal scores break to the lower
 *             index at the K-th place; pad slots come last.
 *   workspace, workspace_bytes: device scratch of at least wf_causal_topk_workspace_bytes();
 *             may be NULL/0 when that returns 0.
 *   status  : optional device int32; bit 1 is OR-ed in if a bounded internal wait of the
 *             tensor-core kernel timed out (the output is then invalid).  May be NULL.
 */
WF_API int wf_causal_topk(const void* q_addr, const void* k_addr, int32_t dtype, int64_t B, int64_t Tq,
                   int64_t Tk, int32_t R, const int64_t* q_strides, const int64_t* k_strides,
                   int32_t top_k, int32_t pad_mode, int32_t row_tile, int32_t row_stride,
                   int32_t row_start, int32_t* idx_out, void* workspace, size_t workspace_bytes,
                   int32_t* status, void* stream);

/*
 * Device workspace (bytes, 16-byte aligned) that wf_causal_topk and
 * wf_fused_sparse_attention need for these sizes: the tensor-core retrieval
 * kernel parks each row's exact candidates there (about 4 KB per query row for
 * K <= 128) for its finalisation pass.  0 means none is needed.
 */
WF_API size_t wf_causal_topk_workspace_bytes(int64_t B, int64_t Tq, int64_t Tk, int32_t R, int32_t top_k,
                                             int32_t dtype);

/*
 * Allocation-free variant of wf_causal_topk.  It has no counterpart in the
 * reference.  It is for callers that cannot allocate device memory at all (an
 * allocator-less runtime, or code running where cudaMalloc is not permitted): the
 * retrieval scratch comes from a fixed 16 MiB device array built into this library,
 * which every GPU that loads the library keeps reserved until the process exits.
 * Same arguments and results as wf_causal_topk without the workspace.  A request
 * fits when wf_causal_topk_workspace_bytes() for its sizes is at most 16 MiB:
 * 2044 query rows (B*Tq) for K <= 128 with bf16/fp16 addresses; fp32 addresses also
 * keep bf16 copies of the address rows there ((Tq + Tk) * R * 2 bytes per batch
 * element), so fewer rows fit (2012 at B = 1, Tq = Tk, R = 32).  Larger requests
 * return WF_ERR_UNSUPPORTED with the byte counts.  The first call on a device
 * looks up the array's device address, so make that first call before any stream
 * capture.  All calls share the one array: calls that overlap on the GPU (other
 * streams, other host threads) race on it and must be serialised by the caller.
 */
WF_API int wf_causal_topk_noalloc(const void* q_addr, const void* k_addr, int32_t dtype, int64_t B, int64_t Tq,
                                  int64_t Tk, int32_t R, const int64_t* q_strides, const int64_t* k_strides,
                                  int32_t top_k, int32_t pad_mode, int32_t row_tile, int32_t row_stride,
                                  int32_t row_start, int32_t* idx_out, int32_t* status, void* stream);

/*
 * Softmax attention over the K rows named by idx, shared by all heads.  Replaces
 * sparse_meat_attention() (routing_attention/kernels/fused_sparse.py:275-324; the
 * arithmetic of sparse_meat_attention_reference :80-94), computed in fp32.
 *
 *   q        : (B, H, Tq, D)      strides q_strides[4]   (last stride must be 1)
 *   k, v     : (B, H, Tk, D)      strides k_strides[4], v_strides[4] (last stride 1)
 *   dtype    : WF_DTYPE_* of q, k and v
 *   idx      : (B, Tq, K) int32   strides idx_strides[3]
 *   D        : 16, 32, 64, 128 or 256; rows must start on 16-byte boundaries
 *   flags    : WF_ATTN_MASK_NEGATIVE or 0
 *   out      : (B, H, Tq, D) of out_dtype, strides out_strides[4] (last stride 1)
 *   status   : optional device int32; bit 0 is OR-ed in when an index lies outside
 *              [-Tk, Tk) (that row's output is NaN).  May be NULL.
 */
WF_API int wf_sparse_attention(const void* q, const void* k, const void* v, int32_t dtype,
                        const int32_t* idx, int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t D,
                        int32_t K, const int64_t* q_strides, const int64_t* k_strides,
                        const int64_t* v_strides, const int64_t* idx_strides, float scale,
                        int32_t flags, void* out, int32_t out_dtype, const int64_t* out_strides,
                        int32_t* status, void* stream);

/*
 * wf_sparse_attention for one long sequence split over ranks in cyclic row blocks
 * (the query-row sharding of the multi-GPU path) whose K/V were all-gathered
 * rank-major, so no reordering copy is needed.  It has no counterpart in the
 * reference, which is single-GPU.  Keys are addressed by their global position j:
 * j lives on rank (j / kv_row_tile) % kv_world at local row
 * (j / kv_row_tile / kv_world) * kv_row_tile + j % kv_row_tile.  k and v point at
 * rank 0's block, k_strides / v_strides describe one rank's (B, H, Tk / kv_world, D)
 * block and k_rank_stride / v_rank_stride (elements) step from one rank to the next.
 */
WF_API int wf_sparse_attention_cyclic_kv(const void* q, const void* k, const void* v, int32_t dtype,
                                         const int32_t* idx, int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                                         int32_t D, int32_t K, const int64_t* q_strides,
                                         const int64_t* k_strides, const int64_t* v_strides,
                                         const int64_t* idx_strides, float scale, int32_t flags, void* out,
                                         int32_t out_dtype, const int64_t* out_strides, int32_t kv_row_tile,
                                         int32_t kv_world, int64_t k_rank_stride, int64_t v_rank_stride,
                                         int32_t* status, void* stream);

/*
 * wf_sparse_attention with attention-probability dropout, for training.  The
 * reference's training path applies nn.Dropout to the softmax probabilities before
 * the weighted sum (routing_attention/models/attention.py:50-54); here probability
 * (b, h, t, k) is kept with probability 1 - drop_rate and scaled by 1 / (1 - drop_rate),
 * the keep decision being u >= drop_rate for u = a counter-based uniform of drop_seed
 * and the element's flat index ((b*H + h)*Tq + t)*K + k (SplitMix64 output function,
 * 24 bits; the backward recomputes the same mask).  drop_rate in [0, 1).
 */
WF_API int wf_sparse_attention_dropout(const void* q, const void* k, const void* v, int32_t dtype,
                                       const int32_t* idx, int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t D,
                                       int32_t K, const int64_t* q_strides, const int64_t* k_strides,
                                       const int64_t* v_strides, const int64_t* idx_strides, float scale,
                                       int32_t flags, float drop_rate, uint64_t drop_seed, void* out,
                                       int32_t out_dtype, const int64_t* out_strides, int32_t* status, void* stream);

/*
 * wf_sparse_attention_cyclic_kv with the gathered K/V stored chunk by chunk, so a
 * rank can attend with the chunks that have already arrived (no counterpart in the
 * reference).  Each rank's local rows are split into chunks of kv_chunk_rows (a
 * multiple of kv_row_tile dividing Tk / kv_world); block (chunk c, rank r) holds
 * local rows [c * kv_chunk_rows, (c + 1) * kv_chunk_rows) of rank r and starts
 * (c * kv_world + r) * k_block_stride (v_block_stride) elements after k (v), whose
 * strides describe one block as (B, H, kv_chunk_rows, D).  At most 64 blocks.
 */
WF_API int wf_sparse_attention_cyclic_kv_chunked(const void* q, const void* k, const void* v, int32_t dtype,
                                                 const int32_t* idx, int64_t B, int64_t H, int64_t Tq, int64_t Tk,
                                                 int32_t D, int32_t K, const int64_t* q_strides,
                                                 const int64_t* k_strides, const int64_t* v_strides,
                                                 const int64_t* idx_strides, float scale, int32_t flags, void* out,
                                                 int32_t out_dtype, const int64_t* out_strides, int32_t kv_row_tile,
                                                 int32_t kv_world, int32_t kv_chunk_rows, int64_t k_block_stride,
                                                 int64_t v_block_stride, int32_t* status, void* stream);

/*
 * Retrieval + attention in one call.  Replaces fused_sparse_attention()
 * (routing_attention/kernels/fused_sparse.py:327-356): wf_causal_topk into idx_out,
 * then wf_sparse_attention over it (masking pads when pad_mode == WF_PAD_MASKED).
 * Arguments have the meanings given above; addr_dtype may differ from dtype.
 */
WF_API int wf_fused_sparse_attention(const void* q_addr, const void* k_addr, int32_t addr_dtype, int32_t R,
                              const int64_t* q_addr_strides, const int64_t* k_addr_strides,
                              const void* q, const void* k, const void* v, int32_t dtype, int64_t B,
                              int64_t H, int64_t Tq, int64_t Tk, int32_t D,
                              const int64_t* q_strides, const int64_t* k_strides,
                              const int64_t* v_strides, int32_t top_k, float scale,
                              int32_t pad_mode, int32_t row_tile, int32_t row_stride,
                              int32_t row_start, int32_t* idx_out, void* out, int32_t out_dtype,
                              const int64_t* out_strides, void* workspace, size_t workspace_bytes,
                              int32_t* status, void* stream);

/*
 * wf_fused_sparse_attention for HOST-resident inputs and outputs, with the copies
 * overlapped with the kernels.  No counterpart in the reference (whose operator
 * takes device tensors); it serves callers whose activations live in pinned host
 * memory.  Schedule (three caller streams):
 *   h2d_stream : q_addr, k_addr | q,k,v rows of chunk 0 | ... | chunk chunks-1
 *   stream     : retrieval of all rows | attention of chunk 0 | ... (each chunk
 *                waits for its rows; attention of rows [a, e) reads K/V rows < e only)
 *   d2h_stream : idx | out rows of chunk 0 | ...
 * On return everything is enqueued and `stream` waits for the last download, so
 * the host outputs are valid once `stream` has completed.  Results are identical
 * to wf_fused_sparse_attention on the same data.
 *
 *   q_addr_h, k_addr_h : (B, T, R) host addresses, contiguous
 *   q_h, k_h, v_h      : (B, H, T, D) host tensors with element strides q/k/v_strides,
 *                        stride(D) = 1 and either (B,T,H,D)-major rows (stride(T) = H*D,
 *                        stride(H) = D) or head-major rows (stride(T) = D)
 *   idx_h              : (B, T, K_eff) int32 host output, contiguous; NULL leaves the
 *                        indices in d_idx only (no download)
 *   out_h              : (B, H, T, D) host output with out_strides (same layout rule)
 *   d_*                : device staging buffers of the same shapes and strides as the host
 *                        tensors (addresses and idx contiguous), reused across calls
 *   workspace          : device scratch of wf_causal_topk_workspace_bytes(B, T, T, R, top_k, addr_dtype)
 *   chunks             : number of query-row chunks (1 .. min(64, T)); 4-8 suits T >= 4096
 * top_k must be >= 1 (K_eff = min(top_k, T)).  Host buffers that are not page-locked
 * still work, with copies that no longer overlap.
 */
WF_API int wf_fused_sparse_attention_host(const void* q_addr_h, const void* k_addr_h, int32_t addr_dtype, int32_t R,
                                          const void* q_h, const void* k_h, const void* v_h, int32_t dtype,
                                          int64_t B, int64_t H, int64_t T, int32_t D, const int64_t* q_strides,
                                          const int64_t* k_strides, const int64_t* v_strides, int32_t top_k,
                                          float scale, int32_t pad_mode, int32_t chunks, int32_t* idx_h,
                                          void* out_h, int32_t out_dtype, const int64_t* out_strides,
                                          void* d_q_addr, void* d_k_addr, void* d_q, void* d_k, void* d_v,
                                          int32_t* d_idx, void* d_out, void* workspace, size_t workspace_bytes,
                                          int32_t* status, void* stream, void* h2d_stream, void* d2h_stream);

/*
 * Fused learned-address projection.  Replaces LearnedAddressModule.forward_query_key
 * (routing_attention/models/learned_address.py:39-46: nn.Linear(d_model, d_A) for the
 * query and the key address, then F.normalize(dim=-1) on each) with one pass over x:
 *   out[m, n] = (x[m, :] . w[n, :] + bias[n]), then every consecutive `group` outputs
 *   are divided by max(||.||_2, 1e-12) when `normalize` is nonzero.
 * Stack the query and key weights ([W_q; W_k], n_out = 2 * d_A, group = d_A) to get
 * both addresses at once.
 *   x    : (M, d_model) rows of x_row_stride elements, dtype WF_DTYPE_*
 *   w    : (n_out, d_model) contiguous, same dtype; bias: (n_out) same dtype or NULL
 *   out  : (M, n_out) rows of out_row_stride elements, same dtype
 * bf16/fp16 with n_out in {32, 64, 128} run on tcgen05 (fp32 accumulate, fp32
 * normalisation, one rounding); fp32 and other widths on CUDA cores in fp32.
 * group: power of two <= 32 dividing n_out; n_out: a divisor of 32 or a multiple
 * of 32 up to 256.
 */
WF_API int wf_address_projection(const void* x, int32_t dtype, int64_t M, int32_t d_model, int64_t x_row_stride,
                                 const void* w, const void* bias, int32_t n_out, int32_t group, int32_t normalize,
                                 void* out, int64_t out_row_stride, int32_t* status, void* stream);

/*
 * Causal top-K that retrieves only keys a padding mask keeps.  The reference's
 * sparse path accepts attn_mask (a (B, T) key-padding mask, `input_ids != pad`,
 * routing_attention/models/transformer.py:269-284) and ignores it
 * (models/attention.py:456-490); here query t retrieves the K best keys j <= t with
 * key_mask[b, j] != 0.  Slots a row cannot fill are -1 (masked pads; give
 * WF_ATTN_MASK_NEGATIVE to the attention).  Queries and keys are the same T
 * positions.  key_mask: (B, T) uint8, element strides mask_strides[2].  workspace:
 * wf_causal_topk_key_mask_workspace_bytes(...) bytes, 256-byte aligned (the
 * compacted key addresses, prefix counts and the position map, then the top-K
 * workspace).  Other arguments as wf_causal_topk.
 */
WF_API size_t wf_causal_topk_key_mask_workspace_bytes(int64_t B, int64_t T, int32_t R, int32_t top_k, int32_t dtype);
WF_API int wf_causal_topk_key_mask(const void* q_addr, const void* k_addr, int32_t dtype, int64_t B, int64_t T,
                                   int32_t R, const int64_t* q_strides, const int64_t* k_strides,
                                   const uint8_t* key_mask, const int64_t* mask_strides, int32_t top_k,
                                   int32_t* idx_out, void* workspace, size_t workspace_bytes, int32_t* status,
                                   void* stream);

/*
 * Backward of wf_sparse_attention (the reference's fused path is forward-only; its
 * non-fused training path gets these gradients from autograd through the gather,
 * routing_attention/models/attention.py:35-56).  Given dout = dL/dout (B, H, Tq, D):
 *   dq (B, H, Tq, D), dk and dv (B, H, Tk, D) = gradients of q, k, v; the indices
 * carry no gradient.  Masked slots (flags & WF_ATTN_MASK_NEGATIVE) contribute
 * nothing; duplicate indices add up.  Every dk/dv row is written (zeros for keys
 * no query retrieved).  grad_dtype: WF_DTYPE_F32 or the input dtype; accumulation
 * is fp32 and each gradient element is rounded once.  D in {32, 64, 128}.
 * drop_rate / drop_seed: those of the forward (wf_sparse_attention_dropout); 0 = none.
 * workspace: wf_sparse_attention_backward_workspace_bytes(B, H, Tq, Tk, K) bytes,
 * 256-byte aligned (softmax probabilities and scaled ds per slot and head, and the
 * key -> (query, slot) inverse index).
 */
WF_API size_t wf_sparse_attention_backward_workspace_bytes(int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t K);
WF_API int wf_sparse_attention_backward(const void* q, const void* k, const void* v, int32_t dtype,
                                        const int32_t* idx, int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t D,
                                        int32_t K, const int64_t* q_strides, const int64_t* k_strides,
                                        const int64_t* v_strides, const int64_t* idx_strides, const void* dout,
                                        const int64_t* dout_strides, float scale, int32_t flags, float drop_rate,
                                        uint64_t drop_seed, void* dq, void* dk, void* dv, int32_t grad_dtype, const int64_t* dq_strides,
                                        const int64_t* dk_strides, const int64_t* dv_strides, void* workspace,
                                        size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Peer-memory K/V exchange of the sequence-sharded path, one process per GPU of a
 * node.  No counterpart in the reference (single-GPU); it replaces the NCCL
 * all-gather of the K/V row shards with copy-engine pulls over NVLink, which leave
 * the SMs to retrieval and attention.
 *   wf_peer_buffer_alloc : cudaMalloc `bytes` and export a 64-byte CUDA IPC handle
 *   wf_peer_buffer_open  : map another process's buffer from its handle (close with
 *                          wf_peer_buffer_close before that process frees it)
 *   wf_pack_row_blocks   : copy this rank's (B, Tl) rows of row_bytes each (batch
 *                          stride src_batch_stride_bytes) into blocks (c, rank) of a
 *                          chunk-major buffer: block (c, r) of Tl/chunks rows per batch
 *                          element at base + c*chunk_stride + r*rank_stride
 *   wf_peer_pull_blocks  : for every chunk c in increasing order, copy blocks (c, p) of
 *                          every tensor t from each peer p's buffer (bases[p], mapped) into
 *                          the same place of bases[rank]; chunk c's copies go to
 *                          streams[c % n_streams] (with one stream, chunk_events[c] also
 *                          marks every earlier chunk),
 *                          which first wait start_event (NULL: none), and chunk_events[c]
 *                          is recorded after them.  The caller orders the pulls after every
 *                          rank packed its blocks, and its next pack after every rank's
 *                          pulls (e.g. with a small collective on each side).
 */
WF_API int wf_peer_buffer_alloc(size_t bytes, void** ptr, void* handle_out);
WF_API int wf_peer_buffer_free(void* ptr);
WF_API int wf_peer_buffer_open(const void* handle, void** ptr);
WF_API int wf_peer_buffer_close(void* ptr);
WF_API int wf_pack_row_blocks(void* base, const void* src, int64_t B, int64_t Tl, int64_t row_bytes,
                              int64_t src_batch_stride_bytes, int32_t chunks, int64_t chunk_stride,
                              int64_t rank_stride, int32_t rank, void* stream);
WF_API int wf_peer_pull_blocks(void* const* bases, int32_t world, int32_t rank, int32_t chunks, int32_t tensors,
                               int64_t block_bytes, int64_t rank_stride, int64_t chunk_stride, int64_t tensor_stride,
                               void* start_event, void* const* streams, int32_t n_streams, void* const* chunk_events);

/*
 * Measurement aid, no counterpart in the reference: the gather-rate ceiling of the
 * attention kernel's access pattern.  For each of n_query queries, reads the K and
 * V rows (row_bytes each, 16..1024 in 16-byte steps, row_stride_bytes apart) at its
 * K indices idx[q][0..K) with the attention kernel's 16-byte loads and computes
 * nothing; one word per query goes to sink (n_query uint32).  Indices outside
 * [0, n_rows) read row 0.  Bytes moved: 2 * n_query * K * row_bytes.
 */
WF_API int wf_gather_rows_bench(const void* k, const void* v, int64_t row_bytes, int64_t row_stride_bytes,
                                const int32_t* idx, int64_t n_query, int32_t K, int64_t n_rows, uint32_t* sink,
                                void* stream);
/* The same gather with 1 KB rows moved by the bulk-copy engine (cp.async.bulk, global
 * to shared, two-stage ring per warp), each row read back from shared memory with
 * 16-byte loads when read_back != 0: the alternative to loading rows into registers.
 * K a multiple of 4.  A query whose wait gave up gets 0xffffffff in sink. */
WF_API int wf_gather_rows_bulk_bench(const void* k, const void* v, int64_t row_stride_bytes, const int32_t* idx,
                                     int64_t n_query, int32_t K, int64_t n_rows, int32_t read_back, uint32_t* sink,
                                     void* stream);

/*
 * Test hook, no counterpart in the reference: makes the next tensor-core retrieval
 * launch on this process exercise its timeout path without any fault.  CTA 1 of
 * every CTA pair skips its send to the peer CTA in bisection exchange
 * `round` (0..7; negative turns the hook off), and the exchange waits give up after
 * wait_limit_ns.  The waiting CTA then sets status bits 1 and 8 (wait site 256),
 * drains its own copies and MMAs, frees its tensor memory and returns; the output
 * of that launch is invalid.  Returns WF_OK.
 */
WF_API int wf_testing_withhold_pair_arrive(int32_t round, uint64_t wait_limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* WAYFINDER_H_ */
