// C ABI of libwayfinder_sm100.so: argument validation, error reporting and
// dispatch to the kernels.  See include/wayfinder.h for the contract.
#include "../../include/wayfinder.h"
#include "wf_kernels.h"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int ok() {
  g_err.clear();
  return WF_OK;
}

int cuda_fail(int rc, const char* what) {
  if (rc == -3) return fail(WF_ERR_INVALID_ARGUMENT, "%s: workspace missing, misaligned or too small "
                            "(query wf_causal_topk_workspace_bytes)", what);
  if (rc < 0) return fail(WF_ERR_UNSUPPORTED, "%s: unsupported configuration", what);
  return fail(WF_ERR_CUDA, "%s: CUDA error %d (%s)", what, rc, cudaGetErrorString((cudaError_t)rc));
}

bool valid_dtype(int32_t d) { return d == WF_DTYPE_BF16 || d == WF_DTYPE_F16 || d == WF_DTYPE_F32; }
int dtype_size(int32_t d) { return d == WF_DTYPE_F32 ? 4 : 2; }

constexpr int64_t kI32Max = 2147483647;

int check_topk(const void* q_addr, const void* k_addr, int32_t dtype, int64_t B, int64_t Tq,
               int64_t Tk, int32_t R, const int64_t* qs, const int64_t* ks, int32_t top_k,
               int32_t pad_mode, int32_t& rt, int32_t& rs, int32_t& r0, const int32_t* idx_out,
               int32_t* k_eff_out) {
  if (B < 0 || Tq < 0 || Tk < 0) return fail(WF_ERR_INVALID_ARGUMENT, "negative size (B=%lld, Tq=%lld, Tk=%lld)",
                                             (long long)B, (long long)Tq, (long long)Tk);
  if (R < 1) return fail(WF_ERR_INVALID_ARGUMENT, "address dim R must be >= 1, got %d", R);
  if (top_k < 0) return fail(WF_ERR_INVALID_ARGUMENT, "top_k must be >= 0, got %d", top_k);
  if (!valid_dtype(dtype)) return fail(WF_ERR_INVALID_ARGUMENT, "unknown address dtype %d", dtype);
  if (pad_mode != WF_PAD_REFERENCE && pad_mode != WF_PAD_MASKED)
    return fail(WF_ERR_INVALID_ARGUMENT, "unknown pad_mode %d", pad_mode);
  if (Tk > kI32Max || Tq > kI32Max || B > 65535)
    return fail(WF_ERR_UNSUPPORTED, "sizes too large (B <= 65535 and T < 2^31 required)");
  const int64_t k_eff = top_k < Tk ? top_k : Tk;
  *k_eff_out = (int32_t)k_eff;
  if (k_eff == 0 || B == 0 || Tq == 0) return ok();
  if (!q_addr || !k_addr || !idx_out || !qs || !ks) return fail(WF_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (k_eff > wf::topk_max_k())
    return fail(WF_ERR_UNSUPPORTED, "top_k=%lld exceeds this build's maximum of %d", (long long)k_eff,
                wf::topk_max_k());
  if (wf::topk_smem_bytes(R, (int)k_eff) == 0)
    return fail(WF_ERR_UNSUPPORTED, "address dim R=%d with top_k=%lld exceeds shared memory", R, (long long)k_eff);
  if (rt == 0) {
    rt = (int32_t)(((Tq + 63) / 64) * 64);
    rs = 1;
    r0 = 0;
  } else {
    if (rt < 0 || rt % 64 != 0) return fail(WF_ERR_INVALID_ARGUMENT, "row_tile must be a positive multiple of 64, got %d", rt);
    if (rs < 1 || r0 < 0 || r0 >= rs)
      return fail(WF_ERR_INVALID_ARGUMENT, "need row_stride >= 1 and 0 <= row_start < row_stride (got %d, %d)", rs, r0);
  }
  const int64_t l = Tq - 1;
  const int64_t gmax = ((l / rt) * rs + r0) * (int64_t)rt + l % rt;
  if (gmax >= Tk)
    return fail(WF_ERR_INVALID_ARGUMENT, "query row map reaches position %lld but only Tk=%lld keys exist",
                (long long)gmax, (long long)Tk);
  if (rs == 1 && r0 == 0 && Tq > Tk)
    return fail(WF_ERR_INVALID_ARGUMENT, "Tq=%lld exceeds Tk=%lld", (long long)Tq, (long long)Tk);
  return WF_OK;
}

int check_attn_tensor(const char* name, const void* p, const int64_t* s, int esz) {
  if (!p || !s) return fail(WF_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (s[3] != 1) return fail(WF_ERR_INVALID_ARGUMENT, "%s: last dimension must be contiguous (stride %lld)", name,
                             (long long)s[3]);
  if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
    return fail(WF_ERR_UNSUPPORTED, "%s: base address must be 16-byte aligned", name);
  for (int i = 0; i < 3; ++i)
    if ((s[i] * esz) % 16 != 0)
      return fail(WF_ERR_UNSUPPORTED, "%s: stride %d (%lld elements) is not a multiple of 16 bytes", name, i,
                  (long long)s[i]);
  return WF_OK;
}

int check_attn(const void* q, const void* k, const void* v, int32_t dtype, const int32_t* idx, int64_t B,
               int64_t H, int64_t Tq, int64_t Tk, int32_t D, int32_t K, const int64_t* qs,
               const int64_t* ks, const int64_t* vs, const int64_t* is, float scale, int32_t flags,
               const void* out, int32_t out_dtype, const int64_t* os) {
  if (B < 0 || H < 0 || Tq < 0 || Tk < 0 || K < 0)
    return fail(WF_ERR_INVALID_ARGUMENT, "negative size argument");
  if (!valid_dtype(dtype)) return fail(WF_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (!valid_dtype(out_dtype)) return fail(WF_ERR_INVALID_ARGUMENT, "unknown out_dtype %d", out_dtype);
  if (flags & ~WF_ATTN_MASK_NEGATIVE) return fail(WF_ERR_INVALID_ARGUMENT, "unknown flags 0x%x", flags);
  if (!std::isfinite(scale)) return fail(WF_ERR_INVALID_ARGUMENT, "scale must be finite");
  if (D != 16 && D != 32 && D != 64 && D != 128 && D != 256)
    return fail(WF_ERR_UNSUPPORTED, "head_dim D=%d not supported (16, 32, 64, 128, 256)", D);
  if (Tk > kI32Max || Tq > kI32Max || B > kI32Max || H > kI32Max)
    return fail(WF_ERR_UNSUPPORTED, "sizes too large");
  if (B == 0 || H == 0 || Tq == 0) return WF_OK;
  if (K == 0) return fail(WF_ERR_INVALID_ARGUMENT, "softmax over K=0 retrieved rows is undefined");
  if (K > wf::attn_max_k())
    return fail(WF_ERR_UNSUPPORTED, "K=%d exceeds this build's maximum of %d", K, wf::attn_max_k());
  if (Tk == 0) return fail(WF_ERR_INVALID_ARGUMENT, "no keys to attend to (Tk=0)");
  if (!idx || !is) return fail(WF_ERR_INVALID_ARGUMENT, "indices: null pointer");
  const int esz = dtype_size(dtype);
  int rc;
  if ((rc = check_attn_tensor("q", q, qs, esz))) return rc;
  if ((rc = check_attn_tensor("k", k, ks, esz))) return rc;
  if ((rc = check_attn_tensor("v", v, vs, esz))) return rc;
  if (!out || !os) return fail(WF_ERR_INVALID_ARGUMENT, "out: null pointer");
  if (os[3] != 1) return fail(WF_ERR_INVALID_ARGUMENT, "out: last dimension must be contiguous");
  const int64_t work = B * H * Tq;
  if ((work + 7) / 8 > kI32Max) return fail(WF_ERR_UNSUPPORTED, "B*H*Tq too large for one launch");
  return WF_OK;
}

}  // namespace

extern "C" {

int wf_version(void) { return 100; }

const char* wf_last_error(void) { return g_err.c_str(); }

int wf_max_top_k(void) { return wf::topk_max_k(); }

int wf_gather_rows_bench(const void* k, const void* v, int64_t row_bytes, int64_t row_stride_bytes,
                         const int32_t* idx, int64_t n_query, int32_t K, int64_t n_rows, uint32_t* sink,
                         void* stream) {
  if (!k || !v || !idx || !sink) return fail(WF_ERR_INVALID_ARGUMENT, "wf_gather_rows_bench: null pointer");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) % 16)
    return fail(WF_ERR_INVALID_ARGUMENT, "wf_gather_rows_bench: rows must be 16-byte aligned");
  const int rc = wf::launch_gather_rows_bench(k, v, row_bytes, row_stride_bytes, idx, n_query, K, n_rows, sink,
                                              static_cast<cudaStream_t>(stream));
  if (rc < 0) return fail(WF_ERR_UNSUPPORTED, "wf_gather_rows_bench: rows of 16..1024 bytes in 16-byte steps");
  if (rc) return cuda_fail(rc, "wf_gather_rows_bench");
  return ok();
}

// ---------------------------------------------------------------- peer-memory K/V exchange
// Buffers shared between the processes of one node through CUDA IPC, and the
// copy-engine pulls of the sequence-sharded path (see include/wayfinder.h).

int wf_peer_buffer_alloc(size_t bytes, void** ptr, void* handle_out) {
  if (!ptr || !handle_out || bytes == 0) return fail(WF_ERR_INVALID_ARGUMENT, "wf_peer_buffer_alloc: bad argument");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail((int)e, "wf_peer_buffer_alloc: cudaMalloc");
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail((int)e, "wf_peer_buffer_alloc: cudaIpcGetMemHandle");
  }
  memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return ok();
}

int wf_peer_buffer_free(void* ptr) {
  if (!ptr) return ok();
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail((int)e, "wf_peer_buffer_free");
  return ok();
}

int wf_peer_buffer_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return fail(WF_ERR_INVALID_ARGUMENT, "wf_peer_buffer_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail((int)e, "wf_peer_buffer_open: cudaIpcOpenMemHandle");
  return ok();
}

int wf_peer_buffer_close(void* ptr) {
  if (!ptr) return ok();
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_fail((int)e, "wf_peer_buffer_close");
  return ok();
}

int wf_pack_row_blocks(void* base, const void* src, int64_t B, int64_t Tl, int64_t row_bytes,
                       int64_t src_batch_stride_bytes, int32_t chunks, int64_t chunk_stride, int64_t rank_stride,
                       int32_t rank, void* stream) {
  if (!base || !src || B < 1 || Tl < 1 || row_bytes < 1 || chunks < 1 || Tl % chunks)
    return fail(WF_ERR_INVALID_ARGUMENT, "wf_pack_row_blocks: bad sizes (Tl must be a multiple of chunks)");
  const int64_t tc = Tl / chunks;
  const size_t width = (size_t)(tc * row_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int c = 0; c < chunks; ++c) {
    char* dst = static_cast<char*>(base) + c * chunk_stride + (int64_t)rank * rank_stride;
    const char* from = static_cast<const char*>(src) + c * tc * row_bytes;
    const cudaError_t e = B == 1 ? cudaMemcpyAsync(dst, from, width, cudaMemcpyDeviceToDevice, st)
                                 : cudaMemcpy2DAsync(dst, width, from, (size_t)src_batch_stride_bytes, width,
                                                     (size_t)B, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_fail((int)e, "wf_pack_row_blocks");
  }
  return ok();
}

int wf_peer_pull_blocks(void* const* bases, int32_t world, int32_t rank, int32_t chunks, int32_t tensors,
                        int64_t block_bytes, int64_t rank_stride, int64_t chunk_stride, int64_t tensor_stride,
                        void* start_event, void* const* streams, int32_t n_streams, void* const* chunk_events) {
  if (!bases || world < 1 || rank < 0 || rank >= world || chunks < 1 || tensors < 1 || block_bytes < 1 ||
      !streams || n_streams < 1 || !chunk_events)
    return fail(WF_ERR_INVALID_ARGUMENT, "wf_peer_pull_blocks: bad argument");
  for (int p = 0; p < world; ++p)
    if (!bases[p]) return fail(WF_ERR_INVALID_ARGUMENT, "wf_peer_pull_blocks: base of rank %d is NULL", p);
  for (int s = 0; s < n_streams && s < chunks; ++s)
    if (start_event) {
      const cudaError_t e = cudaStreamWaitEvent(static_cast<cudaStream_t>(streams[s]),
                                                static_cast<cudaEvent_t>(start_event), 0);
      if (e != cudaSuccess) return cuda_fail((int)e, "wf_peer_pull_blocks: wait");
    }
  char* mine = static_cast<char*>(bases[rank]);
  // chunks in order: the attention of query chunk c reads key chunks <= c
  for (int c = 0; c < chunks; ++c) {
    cudaStream_t st = static_cast<cudaStream_t>(streams[c % n_streams]);
    // peers in rank order starting after this rank, so the ranks spread their pulls
    for (int i = 1; i < world; ++i) {
      const int p = (rank + i) % world;
      for (int t = 0; t < tensors; ++t) {
        const int64_t off = t * tensor_stride + c * chunk_stride + p * rank_stride;
        const cudaError_t e = cudaMemcpyAsync(mine + off, static_cast<const char*>(bases[p]) + off,
                                              (size_t)block_bytes, cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return cuda_fail((int)e, "wf_peer_pull_blocks: copy");
      }
    }
    const cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(chunk_events[c]), st);
    if (e != cudaSuccess) return cuda_fail((int)e, "wf_peer_pull_blocks: event");
  }
  return ok();
}

int wf_gather_rows_bulk_bench(const void* k, const void* v, int64_t row_stride_bytes, const int32_t* idx,
                              int64_t n_query, int32_t K, int64_t n_rows, int32_t read_back, uint32_t* sink,
                              void* stream) {
  if (!k || !v || !idx || !sink) return fail(WF_ERR_INVALID_ARGUMENT, "wf_gather_rows_bulk_bench: null pointer");
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) % 16)
    return fail(WF_ERR_INVALID_ARGUMENT, "wf_gather_rows_bulk_bench: rows must be 16-byte aligned");
  const int rc = wf::launch_gather_rows_bulk_bench(k, v, row_stride_bytes, idx, n_query, K, n_rows, read_back, sink,
                                                   static_cast<cudaStream_t>(stream));
  if (rc < 0) return fail(WF_ERR_UNSUPPORTED, "wf_gather_rows_bulk_bench: K must be a multiple of 4");
  if (rc) return cuda_fail(rc, "wf_gather_rows_bulk_bench");
  return ok();
}

int wf_testing_withhold_pair_arrive(int32_t round, uint64_t wait_limit_ns) {
  wf::topk_tc_test_withhold(round, wait_limit_ns);
  return ok();
}

size_t wf_causal_topk_workspace_bytes(int64_t B, int64_t Tq, int64_t Tk, int32_t R, int32_t top_k, int32_t dtype) {
  if (B <= 0 || Tq <= 0 || Tk <= 0 || top_k <= 0) return 0;
  const int64_t k_eff = top_k < Tk ? top_k : Tk;
  if (!valid_dtype(dtype)) return 0;
  if (R != 16 && R != 32 && R != 64) return 0;
  if (Tk > 65536) return 0;
  return wf::topk_tc_workspace_bytes(B, Tq, Tk, R, (int)k_eff, dtype);
}

int wf_causal_topk(const void* q_addr, const void* k_addr, int32_t dtype, int64_t B, int64_t Tq,
                   int64_t Tk, int32_t R, const int64_t* q_strides, const int64_t* k_strides,
                   int32_t top_k, int32_t pad_mode, int32_t row_tile, int32_t row_stride,
                   int32_t row_start, int32_t* idx_out, void* workspace, size_t workspace_bytes,
                   int32_t* status, void* stream) {
  int32_t k_eff = 0;
  int rc = check_topk(q_addr, k_addr, dtype, B, Tq, Tk, R, q_strides, k_strides, top_k, pad_mode, row_tile,
                      row_stride, row_start, idx_out, &k_eff);
  if (rc) return rc;
  if (k_eff == 0 || B == 0 || Tq == 0) return ok();
  wf::TopkParams p{};
  p.q = q_addr;
  p.k = k_addr;
  p.qsb = q_strides[0]; p.qst = q_strides[1]; p.qsr = q_strides[2];
  p.ksb = k_strides[0]; p.kst = k_strides[1]; p.ksr = k_strides[2];
  p.B = (int)B; p.Tq = (int)Tq; p.Tk = (int)Tk; p.R = R; p.K = k_eff;
  p.pad_mode = pad_mode;
  p.rt = row_tile; p.rs = row_stride; p.r0 = row_start;
  p.idx = idx_out;
  p.status = status;
  p.ws = workspace;
  p.ws_bytes = workspace_bytes;
  rc = wf::launch_causal_topk(p, dtype, static_cast<cudaStream_t>(stream));
  if (rc) return cuda_fail(rc, "wf_causal_topk");
  return ok();
}

namespace {
int attention_impl(const void* q, const void* k, const void* v, int32_t dtype, const int32_t* idx, int64_t B,
                   int64_t H, int64_t Tq, int64_t Tk, int32_t D, int32_t K, const int64_t* q_strides,
                   const int64_t* k_strides, const int64_t* v_strides, const int64_t* idx_strides, float scale,
                   int32_t flags, void* out, int32_t out_dtype, const int64_t* out_strides, int32_t* status,
                   void* stream, int32_t kv_tile, int32_t kv_world, int64_t k_rank_stride, int64_t v_rank_stride,
                   float drop_rate = 0.f, uint64_t drop_seed = 0, int32_t kv_chunk_rows = 0) {
  int rc = check_attn(q, k, v, dtype, idx, B, H, Tq, Tk, D, K, q_strides, k_strides, v_strides, idx_strides,
                      scale, flags, out, out_dtype, out_strides);
  if (rc) return rc;
  if (B == 0 || H == 0 || Tq == 0) return ok();
  wf::AttnParams p{};
  p.q = q; p.k = k; p.v = v; p.idx = idx; p.out = out;
  p.qsb = q_strides[0]; p.qsh = q_strides[1]; p.qst = q_strides[2];
  p.ksb = k_strides[0]; p.ksh = k_strides[1]; p.kst = k_strides[2];
  p.vsb = v_strides[0]; p.vsh = v_strides[1]; p.vst = v_strides[2];
  p.osb = out_strides[0]; p.osh = out_strides[1]; p.ost = out_strides[2];
  p.isb = idx_strides[0]; p.ist = idx_strides[1]; p.iss = idx_strides[2];
  p.B = (int)B; p.H = (int)H; p.Tq = (int)Tq; p.Tk = (int)Tk; p.D = D; p.K = K;
  p.scale = scale;
  p.mask_negative = (flags & WF_ATTN_MASK_NEGATIVE) ? 1 : 0;
  p.status = status;
  p.kv_tile = kv_tile;
  p.kv_world = kv_world;
  p.k_rank_stride = k_rank_stride;
  p.v_rank_stride = v_rank_stride;
  p.drop_rate = drop_rate;
  p.drop_seed = drop_seed;
  p.kv_chunk_rows = kv_chunk_rows;
  {
    const int osz = dtype_size(out_dtype);
    p.out_vec_ok = (reinterpret_cast<uintptr_t>(out) % 16 == 0) && (out_strides[0] * osz) % 16 == 0 &&
                   (out_strides[1] * osz) % 16 == 0 && (out_strides[2] * osz) % 16 == 0;
  }
  rc = wf::launch_sparse_attention(p, dtype, out_dtype, static_cast<cudaStream_t>(stream));
  if (rc) return cuda_fail(rc, "wf_sparse_attention");
  return ok();
}
}  // namespace

int wf_sparse_attention(const void* q, const void* k, const void* v, int32_t dtype, const int32_t* idx,
                        int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t D, int32_t K,
                        const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                        const int64_t* idx_strides, float scale, int32_t flags, void* out, int32_t out_dtype,
                        const int64_t* out_strides, int32_t* status, void* stream) {
  return attention_impl(q, k, v, dtype, idx, B, H, Tq, Tk, D, K, q_strides, k_strides, v_strides, idx_strides,
                        scale, flags, out, out_dtype, out_strides, status, stream, 0, 1, 0, 0);
}

int wf_sparse_attention_dropout(const void* q, const void* k, const void* v, int32_t dtype, const int32_t* idx,
                                int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t D, int32_t K,
                                const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                const int64_t* idx_strides, float scale, int32_t flags, float drop_rate,
                                uint64_t drop_seed, void* out, int32_t out_dtype, const int64_t* out_strides,
                                int32_t* status, void* stream) {
  if (!(drop_rate >= 0.f && drop_rate < 1.f))
    return fail(WF_ERR_INVALID_ARGUMENT, "drop_rate must be in [0, 1), got %g", (double)drop_rate);
  return attention_impl(q, k, v, dtype, idx, B, H, Tq, Tk, D, K, q_strides, k_strides, v_strides, idx_strides,
                        scale, flags, out, out_dtype, out_strides, status, stream, 0, 1, 0, 0, drop_rate, drop_seed);
}

int wf_sparse_attention_cyclic_kv(const void* q, const void* k, const void* v, int32_t dtype, const int32_t* idx,
                                  int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t D, int32_t K,
                                  const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                  const int64_t* idx_strides, float scale, int32_t flags, void* out,
                                  int32_t out_dtype, const int64_t* out_strides, int32_t kv_row_tile,
                                  int32_t kv_world, int64_t k_rank_stride, int64_t v_rank_stride,
                                  int32_t* status, void* stream) {
  if (kv_world < 1 || kv_world > 64) return fail(WF_ERR_INVALID_ARGUMENT, "kv_world must be in [1, 64], got %d", kv_world);
  if (kv_row_tile < 1) return fail(WF_ERR_INVALID_ARGUMENT, "kv_row_tile must be >= 1, got %d", kv_row_tile);
  if (Tk >= (int64_t(1) << 25)) return fail(WF_ERR_UNSUPPORTED, "Tk=%lld too large for the rank-major key layout", (long long)Tk);
  if (Tk % ((int64_t)kv_row_tile * kv_world))
    return fail(WF_ERR_INVALID_ARGUMENT, "Tk=%lld is not a whole number of %d-row blocks on %d ranks", (long long)Tk,
                kv_row_tile, kv_world);
  const int esz = dtype_size(dtype);
  if ((k_rank_stride * esz) % 16 || (v_rank_stride * esz) % 16)
    return fail(WF_ERR_UNSUPPORTED, "rank strides must be multiples of 16 bytes");
  return attention_impl(q, k, v, dtype, idx, B, H, Tq, Tk, D, K, q_strides, k_strides, v_strides, idx_strides,
                        scale, flags, out, out_dtype, out_strides, status, stream, kv_row_tile, kv_world,
                        k_rank_stride, v_rank_stride);
}

int wf_sparse_attention_cyclic_kv_chunked(const void* q, const void* k, const void* v, int32_t dtype,
                                          const int32_t* idx, int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t D,
                                          int32_t K, const int64_t* q_strides, const int64_t* k_strides,
                                          const int64_t* v_strides, const int64_t* idx_strides, float scale,
                                          int32_t flags, void* out, int32_t out_dtype, const int64_t* out_strides,
                                          int32_t kv_row_tile, int32_t kv_world, int32_t kv_chunk_rows,
                                          int64_t k_block_stride, int64_t v_block_stride, int32_t* status,
                                          void* stream) {
  if (kv_world < 1 || kv_row_tile < 1 || kv_chunk_rows < 1)
    return fail(WF_ERR_INVALID_ARGUMENT, "kv_world, kv_row_tile and kv_chunk_rows must be >= 1");
  if (Tk >= (int64_t(1) << 25)) return fail(WF_ERR_UNSUPPORTED, "Tk=%lld too large for the gathered key layout", (long long)Tk);
  if (Tk % ((int64_t)kv_row_tile * kv_world))
    return fail(WF_ERR_INVALID_ARGUMENT, "Tk=%lld is not a whole number of %d-row blocks on %d ranks", (long long)Tk,
                kv_row_tile, kv_world);
  const int64_t local = Tk / kv_world;
  if (kv_chunk_rows % kv_row_tile || local % kv_chunk_rows)
    return fail(WF_ERR_INVALID_ARGUMENT, "kv_chunk_rows=%d must be a multiple of kv_row_tile and divide the %lld local rows",
                kv_chunk_rows, (long long)local);
  if ((local / kv_chunk_rows) * kv_world > 64)
    return fail(WF_ERR_UNSUPPORTED, "at most 64 (chunk, rank) blocks");
  const int esz = dtype_size(dtype);
  if ((k_block_stride * esz) % 16 || (v_block_stride * esz) % 16)
    return fail(WF_ERR_UNSUPPORTED, "block strides must be multiples of 16 bytes");
  return attention_impl(q, k, v, dtype, idx, B, H, Tq, Tk, D, K, q_strides, k_strides, v_strides, idx_strides,
                        scale, flags, out, out_dtype, out_strides, status, stream, kv_row_tile, kv_world,
                        k_block_stride, v_block_stride, 0.f, 0, kv_chunk_rows);
}

int wf_fused_sparse_attention(const void* q_addr, const void* k_addr, int32_t addr_dtype, int32_t R,
                              const int64_t* q_addr_strides, const int64_t* k_addr_strides, const void* q,
                              const void* k, const void* v, int32_t dtype, int64_t B, int64_t H, int64_t Tq,
                              int64_t Tk, int32_t D, const int64_t* q_strides, const int64_t* k_strides,
                              const int64_t* v_strides, int32_t top_k, float scale, int32_t pad_mode,
                              int32_t row_tile, int32_t row_stride, int32_t row_start, int32_t* idx_out,
                              void* out, int32_t out_dtype, const int64_t* out_strides, void* workspace,
                              size_t workspace_bytes, int32_t* status, void* stream) {
  int32_t k_eff = 0;
  int32_t rt = row_tile, rs = row_stride, r0 = row_start;
  int rc = check_topk(q_addr, k_addr, addr_dtype, B, Tq, Tk, R, q_addr_strides, k_addr_strides, top_k, pad_mode,
                      rt, rs, r0, idx_out, &k_eff);
  if (rc) return rc;
  if (B == 0 || H == 0 || Tq == 0) return ok();
  const int64_t idx_strides[3] = {Tq * (int64_t)k_eff, (int64_t)k_eff, 1};
  rc = check_attn(q, k, v, dtype, idx_out, B, H, Tq, Tk, D, k_eff, q_strides, k_strides, v_strides, idx_strides,
                  scale, pad_mode == WF_PAD_MASKED ? WF_ATTN_MASK_NEGATIVE : 0, out, out_dtype, out_strides);
  if (rc) return rc;
  rc = wf_causal_topk(q_addr, k_addr, addr_dtype, B, Tq, Tk, R, q_addr_strides, k_addr_strides, top_k, pad_mode,
                      row_tile, row_stride, row_start, idx_out, workspace, workspace_bytes, status, stream);
  if (rc) return rc;
  return wf_sparse_attention(q, k, v, dtype, idx_out, B, H, Tq, Tk, D, k_eff, q_strides, k_strides, v_strides,
                             idx_strides, scale, pad_mode == WF_PAD_MASKED ? WF_ATTN_MASK_NEGATIVE : 0, out,
                             out_dtype, out_strides, status, stream);
}

int wf_causal_topk_noalloc(const void* q_addr, const void* k_addr, int32_t dtype, int64_t B, int64_t Tq,
                           int64_t Tk, int32_t R, const int64_t* q_strides, const int64_t* k_strides,
                           int32_t top_k, int32_t pad_mode, int32_t row_tile, int32_t row_stride,
                           int32_t row_start, int32_t* idx_out, int32_t* status, void* stream) {
  // Same retrieval as wf_causal_topk, with the scratch taken from the library's
  // built-in device array instead of a caller workspace; no allocation anywhere.
  const size_t need = wf_causal_topk_workspace_bytes(B, Tq, Tk, R, top_k, dtype);
  void* scratch = nullptr;
  if (need > 0) {
    const size_t cap = wf::noalloc_scratch_capacity();
    if (need > cap)
      return fail(WF_ERR_UNSUPPORTED,
                  "wf_causal_topk_noalloc: B*Tq=%lld query rows need %zu bytes of scratch but the built-in "
                  "buffer holds %zu; use wf_causal_topk with a workspace",
                  (long long)(B * Tq), need, cap);
    const int rc = wf::noalloc_scratch(&scratch);
    if (rc) return cuda_fail(rc, "wf_causal_topk_noalloc: scratch address lookup");
  }
  return wf_causal_topk(q_addr, k_addr, dtype, B, Tq, Tk, R, q_strides, k_strides, top_k, pad_mode, row_tile,
                        row_stride, row_start, idx_out, scratch, need, status, stream);
}


namespace {
// Row-chunk copy plan of a (B, H, T, D) tensor: rows [a, e) of every (b[, h]) as
// 2D copies.  kind 1: (B,T,H,D)-major rows, kind 2: head-major rows.
int row_layout(const int64_t* s, int64_t H, int32_t D) {
  if (s[3] != 1) return 0;
  if (s[1] == D && s[2] == H * D) return 1;
  if (s[2] == D) return 2;
  return 0;
}

cudaError_t copy_rows(char* dst, const char* src, int esz, int kind, int64_t B, int64_t H, int32_t D,
                      const int64_t* s, int64_t a, int64_t e, cudaMemcpyKind dir, cudaStream_t st) {
  if (kind == 1) {
    const size_t width = (size_t)(e - a) * H * D * esz, off = (size_t)(a * s[2]) * esz;
    if (B == 1) return cudaMemcpyAsync(dst + off, src + off, width, dir, st);
    const size_t pitch = (size_t)s[0] * esz;
    return cudaMemcpy2DAsync(dst + off, pitch, src + off, pitch, width, (size_t)B, dir, st);
  }
  const size_t width = (size_t)(e - a) * D * esz, off = (size_t)(a * D) * esz, pitch = (size_t)s[1] * esz;
  if (s[0] == H * s[1]) return cudaMemcpy2DAsync(dst + off, pitch, src + off, pitch, width, (size_t)(B * H), dir, st);
  for (int64_t b = 0; b < B; ++b) {
    const size_t ob = off + (size_t)(b * s[0]) * esz;
    cudaError_t rc = cudaMemcpy2DAsync(dst + ob, pitch, src + ob, pitch, width, (size_t)H, dir, st);
    if (rc != cudaSuccess) return rc;
  }
  return cudaSuccess;
}

// Events of one host-pipelined call; destroyed once recorded (the runtime frees
// them after they complete).
struct EventSet {
  cudaEvent_t ev[256];
  int n = 0;
  cudaEvent_t make() {
    cudaEvent_t e = nullptr;
    if (n < 256 && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess) ev[n++] = e;
    return e;
  }
  ~EventSet() {
    for (int i = 0; i < n; ++i) cudaEventDestroy(ev[i]);
  }
};
}  // namespace

int wf_fused_sparse_attention_host(const void* q_addr_h, const void* k_addr_h, int32_t addr_dtype, int32_t R,
                                   const void* q_h, const void* k_h, const void* v_h, int32_t dtype, int64_t B,
                                   int64_t H, int64_t T, int32_t D, const int64_t* q_strides,
                                   const int64_t* k_strides, const int64_t* v_strides, int32_t top_k, float scale,
                                   int32_t pad_mode, int32_t chunks, int32_t* idx_h, void* out_h,
                                   int32_t out_dtype, const int64_t* out_strides, void* d_q_addr, void* d_k_addr,
                                   void* d_q, void* d_k, void* d_v, int32_t* d_idx, void* d_out, void* workspace,
                                   size_t workspace_bytes, int32_t* status, void* stream, void* h2d_stream,
                                   void* d2h_stream) {
  if (top_k < 1) return fail(WF_ERR_INVALID_ARGUMENT, "wf_fused_sparse_attention_host: top_k must be >= 1, got %d", top_k);
  if (!q_addr_h || !k_addr_h || !q_h || !k_h || !v_h || !out_h || !d_q_addr || !d_k_addr || !d_q ||
      !d_k || !d_v || !d_idx || !d_out || !q_strides || !k_strides || !v_strides || !out_strides)
    return fail(WF_ERR_INVALID_ARGUMENT, "wf_fused_sparse_attention_host: null pointer argument");
  if (B < 1 || H < 1 || T < 1) return fail(WF_ERR_INVALID_ARGUMENT, "wf_fused_sparse_attention_host: empty problem");
  if (chunks < 1 || chunks > 64 || chunks > T)
    return fail(WF_ERR_INVALID_ARGUMENT, "chunks must be in [1, min(64, T)], got %d", chunks);
  if (!valid_dtype(dtype) || !valid_dtype(out_dtype) || !valid_dtype(addr_dtype))
    return fail(WF_ERR_INVALID_ARGUMENT, "unknown dtype");
  const int kq = row_layout(q_strides, H, D), kk = row_layout(k_strides, H, D), kv = row_layout(v_strides, H, D),
            ko = row_layout(out_strides, H, D);
  if (!kq || !kk || !kv || !ko)
    return fail(WF_ERR_UNSUPPORTED, "host q/k/v/out need unit stride(D) and (B,T,H,D)-major or head-major rows");
  const int32_t k_eff = (int32_t)(top_k < T ? top_k : T);
  const int64_t as[3] = {T * R, (int64_t)R, 1};
  const int64_t is[3] = {T * (int64_t)k_eff, (int64_t)k_eff, 1};
  // full validation of both launches before anything is enqueued
  {
    int32_t rt = 0, rs = 1, r0 = 0, ke = 0;
    int rc = check_topk(d_q_addr, d_k_addr, addr_dtype, B, T, T, R, as, as, top_k, pad_mode, rt, rs, r0, d_idx, &ke);
    if (rc) return rc;
    rc = check_attn(d_q, d_k, d_v, dtype, d_idx, B, H, T, T, D, k_eff, q_strides, k_strides, v_strides, is, scale,
                    pad_mode == WF_PAD_MASKED ? WF_ATTN_MASK_NEGATIVE : 0, d_out, out_dtype, out_strides);
    if (rc) return rc;
  }
  cudaStream_t sm = static_cast<cudaStream_t>(stream), si = static_cast<cudaStream_t>(h2d_stream),
               so = static_cast<cudaStream_t>(d2h_stream);
  const int esz = dtype_size(dtype), osz = dtype_size(out_dtype), asz = dtype_size(addr_dtype);
  EventSet evs;
  cudaError_t ce = cudaSuccess;
#define WF_CK(x)                                                            \
  do {                                                                      \
    ce = (x);                                                               \
    if (ce != cudaSuccess) return cuda_fail((int)ce, "wf_fused_sparse_attention_host"); \
  } while (0)
#define WF_EV(name)                                                                             \
  cudaEvent_t name = evs.make();                                                                \
  if (!name) return fail(WF_ERR_CUDA, "wf_fused_sparse_attention_host: event creation failed")
  // the copy streams start after the work already queued on `stream` (the previous
  // call's kernels may still read the staging buffers)
  WF_EV(e_start);
  WF_CK(cudaEventRecord(e_start, sm));
  WF_CK(cudaStreamWaitEvent(si, e_start, 0));
  WF_CK(cudaStreamWaitEvent(so, e_start, 0));
  const size_t abytes = (size_t)(B * T * R) * asz;
  WF_CK(cudaMemcpyAsync(d_q_addr, q_addr_h, abytes, cudaMemcpyHostToDevice, si));
  WF_CK(cudaMemcpyAsync(d_k_addr, k_addr_h, abytes, cudaMemcpyHostToDevice, si));
  WF_EV(e_addr);
  WF_CK(cudaEventRecord(e_addr, si));
  cudaEvent_t e_rows[64];
  for (int c = 0; c < chunks; ++c) {
    const int64_t a = T * c / chunks, e = T * (c + 1) / chunks;
    WF_CK(copy_rows((char*)d_q, (const char*)q_h, esz, kq, B, H, D, q_strides, a, e, cudaMemcpyHostToDevice, si));
    WF_CK(copy_rows((char*)d_k, (const char*)k_h, esz, kk, B, H, D, k_strides, a, e, cudaMemcpyHostToDevice, si));
    WF_CK(copy_rows((char*)d_v, (const char*)v_h, esz, kv, B, H, D, v_strides, a, e, cudaMemcpyHostToDevice, si));
    WF_EV(er);
    WF_CK(cudaEventRecord(er, si));
    e_rows[c] = er;
  }
  WF_CK(cudaStreamWaitEvent(sm, e_addr, 0));
  int rc = wf_causal_topk(d_q_addr, d_k_addr, addr_dtype, B, T, T, R, as, as, top_k, pad_mode, 0, 1, 0, d_idx,
                          workspace, workspace_bytes, status, stream);
  if (rc) return rc;
  WF_EV(e_idx);
  WF_CK(cudaEventRecord(e_idx, sm));
  WF_CK(cudaStreamWaitEvent(so, e_idx, 0));
  if (idx_h)  // NULL: the indices stay in d_idx only
    WF_CK(cudaMemcpyAsync(idx_h, d_idx, (size_t)(B * T) * k_eff * sizeof(int32_t), cudaMemcpyDeviceToHost, so));
  // Chunk c's causal indices read K/V rows < e only, so it needs uploads 0..c.  With
  // pad_mode=reference, rows i < K-1 also attend their pad rows (i + K + s + 1) % T,
  // s < K, which reach row 3K-2 (and wrap to any row when 3K-2 >= T): a chunk holding
  // such rows waits for the chunk of the highest pad row.  Chunks run in order of the
  // upload they wait for, so the pad chunks go last and never hold up the others.
  int need[64], order[64];
  {
    const int64_t pad_rows = pad_mode == WF_PAD_MASKED ? 0 : (int64_t)k_eff - 1;
    const int64_t hi = 3 * (int64_t)top_k - 2 < T ? 3 * (int64_t)top_k - 2 : T - 1;
    int c_hi = 0;
    while (c_hi + 1 < chunks && T * (c_hi + 1) / chunks <= hi) ++c_hi;
    int n = 0;
    for (int c = 0; c < chunks; ++c) {
      const int64_t a = T * c / chunks;
      need[c] = (a < pad_rows && c_hi > c) ? c_hi : c;
    }
    for (int w = 0; w < chunks; ++w)
      for (int c = 0; c < chunks; ++c)
        if (need[c] == w) order[n++] = c;
  }
  for (int oi = 0; oi < chunks; ++oi) {
    const int c = order[oi];
    const int64_t a = T * c / chunks, e = T * (c + 1) / chunks;
    WF_CK(cudaStreamWaitEvent(sm, e_rows[need[c]], 0));
    rc = wf_sparse_attention(static_cast<const char*>(d_q) + (size_t)(a * q_strides[2]) * esz, d_k, d_v, dtype,
                             d_idx + a * k_eff, B, H, e - a, T, D, k_eff, q_strides, k_strides, v_strides, is, scale,
                             pad_mode == WF_PAD_MASKED ? WF_ATTN_MASK_NEGATIVE : 0,
                             static_cast<char*>(d_out) + (size_t)(a * out_strides[2]) * osz, out_dtype, out_strides,
                             status, stream);
    if (rc) return rc;
    WF_EV(ed);
    WF_CK(cudaEventRecord(ed, sm));
    WF_CK(cudaStreamWaitEvent(so, ed, 0));
    WF_CK(copy_rows((char*)out_h, (const char*)d_out, osz, ko, B, H, D, out_strides, a, e, cudaMemcpyDeviceToHost, so));
  }
  WF_EV(e_fin);
  WF_CK(cudaEventRecord(e_fin, so));
  WF_CK(cudaStreamWaitEvent(sm, e_fin, 0));
#undef WF_CK
#undef WF_EV
  return ok();
}


int wf_address_projection(const void* x, int32_t dtype, int64_t M, int32_t d_model, int64_t x_row_stride,
                          const void* w, const void* bias, int32_t n_out, int32_t group, int32_t normalize,
                          void* out, int64_t out_row_stride, int32_t* status, void* stream) {
  if (!valid_dtype(dtype)) return fail(WF_ERR_INVALID_ARGUMENT, "unknown dtype %d", dtype);
  if (M < 0 || d_model < 1 || n_out < 1) return fail(WF_ERR_INVALID_ARGUMENT, "bad sizes (M=%lld, d_model=%d, n_out=%d)",
                                                     (long long)M, d_model, n_out);
  if (M > kI32Max) return fail(WF_ERR_UNSUPPORTED, "M=%lld rows exceed 2^31", (long long)M);
  if (group < 1 || group > 32 || (group & (group - 1)) || n_out % group)
    return fail(WF_ERR_INVALID_ARGUMENT, "group must be a power of two <= 32 dividing n_out, got %d", group);
  if (n_out > 256 || (n_out <= 32 ? 32 % n_out != 0 : n_out % 32 != 0))
    return fail(WF_ERR_UNSUPPORTED, "n_out=%d: supported are divisors of 32 and multiples of 32 up to 256", n_out);
  if (x_row_stride < d_model || out_row_stride < n_out)
    return fail(WF_ERR_INVALID_ARGUMENT, "row strides must cover the rows");
  if (M == 0) return ok();
  if (!x || !w || !out) return fail(WF_ERR_INVALID_ARGUMENT, "null pointer argument");
  const int rc = wf::launch_address_projection(x, dtype, M, d_model, x_row_stride, w, bias, n_out, group, normalize,
                                               out, out_row_stride, status, static_cast<cudaStream_t>(stream));
  if (rc) return cuda_fail(rc, "wf_address_projection");
  return ok();
}


size_t wf_sparse_attention_backward_workspace_bytes(int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t K) {
  if (B <= 0 || H <= 0 || Tq <= 0 || Tk <= 0 || K <= 0) return 0;
  return wf::attn_bwd_workspace_bytes(B, H, Tq, Tk, K);
}

int wf_sparse_attention_backward(const void* q, const void* k, const void* v, int32_t dtype, const int32_t* idx,
                                 int64_t B, int64_t H, int64_t Tq, int64_t Tk, int32_t D, int32_t K,
                                 const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                 const int64_t* idx_strides, const void* dout, const int64_t* dout_strides, float scale,
                                 int32_t flags, float drop_rate, uint64_t drop_seed, void* dq, void* dk, void* dv,
                                 int32_t grad_dtype,
                                 const int64_t* dq_strides, const int64_t* dk_strides, const int64_t* dv_strides,
                                 void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  int rc = check_attn(q, k, v, dtype, idx, B, H, Tq, Tk, D, K, q_strides, k_strides, v_strides, idx_strides, scale,
                      flags, dq, grad_dtype, dq_strides);
  if (rc) return rc;
  if (B == 0 || H == 0 || (Tq == 0 && Tk == 0)) return ok();
  if (D != 32 && D != 64 && D != 128) return fail(WF_ERR_UNSUPPORTED, "backward: head_dim D=%d not supported (32, 64, 128)", D);
  if (grad_dtype != WF_DTYPE_F32 && grad_dtype != dtype)
    return fail(WF_ERR_UNSUPPORTED, "backward: gradients are produced in fp32 or in the input dtype");
  if (Tq * (int64_t)K > kI32Max || Tq >= (int64_t(1) << 22))
    return fail(WF_ERR_UNSUPPORTED, "backward: Tq*K must be below 2^31 and Tq below 2^22");
  const int esz = dtype_size(dtype), gsz = dtype_size(grad_dtype);
  if ((rc = check_attn_tensor("dout", dout, dout_strides, esz))) return rc;
  if (!dk || !dv || !dk_strides || !dv_strides) return fail(WF_ERR_INVALID_ARGUMENT, "dk/dv: null pointer");
  if (dk_strides[3] != 1 || dv_strides[3] != 1) return fail(WF_ERR_INVALID_ARGUMENT, "dk/dv: last dimension must be contiguous");
  auto vec_ok = [&](const void* ptr, const int64_t* s) {
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (s[0] * gsz) % 16 == 0 && (s[1] * gsz) % 16 == 0 &&
           (s[2] * gsz) % 16 == 0;
  };
  wf::AttnBwdParams p{};
  p.q = q; p.k = k; p.v = v; p.dout = dout; p.idx = idx; p.dq = dq; p.dk = dk; p.dv = dv;
  p.qsb = q_strides[0]; p.qsh = q_strides[1]; p.qst = q_strides[2];
  p.ksb = k_strides[0]; p.ksh = k_strides[1]; p.kst = k_strides[2];
  p.vsb = v_strides[0]; p.vsh = v_strides[1]; p.vst = v_strides[2];
  p.osb = dout_strides[0]; p.osh = dout_strides[1]; p.ost = dout_strides[2];
  p.dqsb = dq_strides[0]; p.dqsh = dq_strides[1]; p.dqst = dq_strides[2];
  p.dksb = dk_strides[0]; p.dksh = dk_strides[1]; p.dkst = dk_strides[2];
  p.dvsb = dv_strides[0]; p.dvsh = dv_strides[1]; p.dvst = dv_strides[2];
  p.isb = idx_strides[0]; p.ist = idx_strides[1]; p.iss = idx_strides[2];
  p.B = (int)B; p.H = (int)H; p.Tq = (int)Tq; p.Tk = (int)Tk; p.D = D; p.K = K;
  p.scale = scale;
  p.mask_negative = (flags & WF_ATTN_MASK_NEGATIVE) ? 1 : 0;
  p.dq_vec_ok = vec_ok(dq, dq_strides);
  p.dk_vec_ok = vec_ok(dk, dk_strides);
  p.dv_vec_ok = vec_ok(dv, dv_strides);
  if (!(drop_rate >= 0.f && drop_rate < 1.f))
    return fail(WF_ERR_INVALID_ARGUMENT, "drop_rate must be in [0, 1), got %g", (double)drop_rate);
  p.drop_rate = drop_rate;
  p.drop_seed = drop_seed;
  p.status = status;
  rc = wf::launch_sparse_attention_backward(p, workspace, workspace_bytes, dtype, grad_dtype,
                                            static_cast<cudaStream_t>(stream));
  if (rc) return cuda_fail(rc, "wf_sparse_attention_backward");
  return ok();
}


size_t wf_causal_topk_key_mask_workspace_bytes(int64_t B, int64_t T, int32_t R, int32_t top_k, int32_t dtype) {
  if (B <= 0 || T <= 0 || top_k <= 0 || R < 1 || !valid_dtype(dtype)) return 0;
  const size_t inner = (wf_causal_topk_workspace_bytes(B, T, T, R, top_k, dtype) + 255) / 256 * 256;
  return wf::topk_key_mask_prep_bytes(B, T, R, dtype_size(dtype)) + inner;
}

int wf_causal_topk_key_mask(const void* q_addr, const void* k_addr, int32_t dtype, int64_t B, int64_t T, int32_t R,
                            const int64_t* q_strides, const int64_t* k_strides, const uint8_t* key_mask,
                            const int64_t* mask_strides, int32_t top_k, int32_t* idx_out, void* workspace,
                            size_t workspace_bytes, int32_t* status, void* stream) {
  int32_t k_eff = 0, rt = 0, rs = 1, r0 = 0;
  int rc = check_topk(q_addr, k_addr, dtype, B, T, T, R, q_strides, k_strides, top_k, WF_PAD_MASKED, rt, rs, r0,
                      idx_out, &k_eff);
  if (rc) return rc;
  if (k_eff == 0 || B == 0 || T == 0) return ok();
  if (!key_mask || !mask_strides) return fail(WF_ERR_INVALID_ARGUMENT, "key_mask: null pointer");
  const size_t need = wf_causal_topk_key_mask_workspace_bytes(B, T, R, top_k, dtype);
  if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(WF_ERR_INVALID_ARGUMENT, "wf_causal_topk_key_mask: workspace missing, not 256-byte aligned or "
                "smaller than %zu bytes (wf_causal_topk_key_mask_workspace_bytes)", need);
  const size_t prep = wf::topk_key_mask_prep_bytes(B, T, R, dtype_size(dtype));
  wf::TopkParams p{};
  p.q = q_addr;
  p.k = k_addr;
  p.qsb = q_strides[0]; p.qst = q_strides[1]; p.qsr = q_strides[2];
  p.ksb = k_strides[0]; p.kst = k_strides[1]; p.ksr = k_strides[2];
  p.B = (int)B; p.Tq = (int)T; p.Tk = (int)T; p.R = R; p.K = k_eff;
  p.pad_mode = WF_PAD_MASKED;
  p.rt = rt; p.rs = rs; p.r0 = r0;
  p.idx = idx_out;
  p.status = status;
  p.ws = static_cast<unsigned char*>(workspace) + prep;
  p.ws_bytes = workspace_bytes - prep;
  rc = wf::launch_topk_key_mask(p, dtype, key_mask, mask_strides[0], mask_strides[1], workspace,
                                static_cast<cudaStream_t>(stream));
  if (rc) return cuda_fail(rc, "wf_causal_topk_key_mask");
  return ok();
}

}  // extern "C"
