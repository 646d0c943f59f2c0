// Exact causal top-K retrieval with tcgen05 tensor-core scoring (bf16 / fp16 addresses).
//
// Same contract as the CUDA-core kernel in wf_topk.cu (and the reference's
// routing_attention/kernels/causal_topk.py:133-171 + :37-57): for every query
// row g, the K keys j <= g with the largest fp32 score <q_g, k_j> (ties to the
// lower index), pad slots for short rows.  The order of the selected keys within
// a row is unspecified (here: the candidate lists' order), as it is for the
// reference's topk(sorted=False); the CUDA-core kernel happens to sort.
//
// Work split.  A tile of 128 query rows (the 128 TMEM lanes) is handled by a
// cluster of two CTAs on two SMs; CTA rank r streams the key chunks c = r, r+2,
// ... (128 keys each), so the long rows at the end of the causal triangle are
// shared by two SMs.  Each CTA has 9 warps: warp 8 TMA-loads the q tile and the
// key chunks into a shared-memory ring and one of its lanes issues tcgen05.mma
// (M=128, N=128, K=16 per instruction, fp32 accumulate) into a 2-deep TMEM
// accumulator ring; warps 0-7 are two per TMEM lane quadrant: thread t of warp w
// owns query row 32*(w%4)+t and the column half w/4 of every chunk.
//
// Selection is two passes over the CTA's chunks (the MMAs are recomputed; they
// are nearly free):
//   pass 1  each thread keeps, in 256 TMEM columns of its lane, the maximum
//           tensor-core score of each of 256 key groups (column x parity of the
//           chunk in the CTA's stream).  The K-th largest of the pair's 512 group
//           maxima is the score of K distinct keys, so it lower-bounds the row's
//           K-th best score; the two CTAs bisect it together (7 steps, counts
//           exchanged through distributed shared memory with asynchronous
//           stores that complete on the receiver's barrier).
//   pass 2  a key is admitted when its tensor-core score reaches
//           (bound - margin); about 75 keys per row and CTA at K = 128.  The
//           lane that owns the row appends the key's index to its own list in a
//           caller-provided workspace, one list of KW slots per (row, CTA, warp)
//           with the count in a register (KW = 256 for K <= 128, 384 for
//           K <= 256).  A list within 64 of full is compacted to its exact top-K
//           (its entries rescored exactly from the address rows in global
//           memory, then a warp radix select), which raises the row's admission
//           threshold.  Nothing else is rescored here: that work would sit on
//           this kernel's critical chain of chunks.
//   output  topk_rescore_kernel (one warp per list, full occupancy) computes the
//           exact fp32 score of every candidate of rows holding more than K
//           (sequential FMA over d: the CUDA-core kernel's arithmetic), and
//           topk_finalize_kernel (one warp per row) selects the exact top-K of
//           the four lists and writes the indices and pads.  Batches larger
//           than about 65536 query rows run in slices that reuse the workspace.
// The selection warps also take max|k| over the chunks they score (for the
// margin), so the producer warp only loads and issues MMAs.
// The margin, 2^-13 * sum_d |q_d| * max|k|, exceeds any plausible accumulation
// error of a 32-term fp32 dot product with exact bf16/fp16 products, so every
// key whose exact score reaches the K-th best is admitted: the result is exact
// with respect to the fp32 scores.  Every wait is bounded; a timeout sets bit 1
// of the status word (plus one bit, 4..2048, naming the wait site) instead of hanging.
#include "wf_common.cuh"
#include "wf_kernels.h"
#include "wf_select.cuh"
#include "wf_sm100.cuh"

#include <atomic>
#include <mutex>
#include <type_traits>

namespace wf {
namespace {

using namespace sm100;
using select::merge_row;
using select::select_compact;

constexpr int kM = 128;   // query rows per tile = TMEM lanes
constexpr int kN = 128;   // keys per chunk = MMA N
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant
constexpr int kThreads = (kEpiWarps + 1) * 32;
constexpr int kGroups = 256;  // pass-1 key groups per row (TMEM columns 256..511)
// Workspace list capacity KW per (row, CTA, warp) is a template parameter: 256 for
// K <= 128 and 384 for K <= 256 (a list within 64 of full is compacted to its top-K,
// which leaves room for the next chunk).
constexpr int kRowsPerPass = 65536;  // query rows per launch pair; larger batches run in slices
constexpr int kLists = 4;     // candidate lists per row: 2 CTAs x 2 selection warps
constexpr unsigned kFullMask = 0xffffffffu;
constexpr uint64_t kWaitLimitNs = 1000000000ull;
constexpr float kEpsScale = 1.0f / 8192.0f;
constexpr int kMaxDevices = 64;
constexpr size_t kMaxSmem = 232448;

// Address rows in their input type (fp32 addresses: the original fp32 rows, not
// the bf16 copies the tensor cores read), element strides.
struct ScoreSrc {
  const void* q;
  const void* k;
  int64_t qsb, qst, ksb, kst;
};

struct TcParams {
  const void* q;
  int64_t qsb, qst;
  int B, Tq, Tk, K;
  int pad_mode;
  int rt, rs, r0;
  int32_t* idx;
  int32_t* status;
  int32_t* ws;       // [B*Tq][kLists][KW] candidate key indices
  int32_t* ws_cnt;   // [B*Tq][kLists] candidate counts
  const int32_t* lim;  // optional [B][Tq] per-row key limits (see TopkParams)
  // Test hook, set by wf_testing_withhold_pair_arrive (0 = off): CTA 1 of every pair
  // skips its send to the peer in bisection exchange (withhold - 1), and
  // the waits of the exchanges give up after xwait_ns, so CTA 0's wait runs out.
  int withhold;
  uint64_t xwait_ns;
  // fp32 addresses: the MMAs read bf16 copies; admitted keys are rescored from these
  const float* qf;
  const float* kf;
  int64_t fqsb, fqst, fksb, fkst;
  ScoreSrc src;  // address rows for exact rescoring
};

__host__ __device__ constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

constexpr int kXRounds = 8;  // pair exchanges for the bound: extrema + 7 bisection steps

template <int R, int KW>
struct Layout {
  static constexpr int KB = KW - 128;  // merge buffer entries per warp (>= K)
  static constexpr int ROWB = R * 2;
  static constexpr int S = R >= 64 ? 2 : 3;  // shared-memory stages
  static constexpr size_t Q_BYTES = (size_t)kM * ROWB;
  static constexpr size_t STAGE_BYTES = (size_t)kN * ROWB;
  static constexpr size_t STAGE_STRIDE = align_up(STAGE_BYTES, 1024);
  static constexpr size_t off_q = 0;
  static constexpr size_t off_k = align_up(Q_BYTES, 1024);
  static constexpr size_t off_kmax = off_k + S * STAGE_STRIDE;
  static constexpr size_t off_bar = align_up(off_kmax + sizeof(float) * S, 8);
  static constexpr size_t n_bar = 3 * S + 3 + kXRounds;  // full, mdone, done, qbar, kbar, xbar[rounds], drain
  static constexpr size_t off_misc = off_bar + 8 * n_bar;  // tmem base, kmax own, kmax peer, abort
  static constexpr size_t off_xslot = align_up(off_misc + 16, 16);  // [2 parities][kM rows][4] bisection exchange
  static constexpr size_t off_xpair = off_xslot + 4 * 2 * kM * 4;  // [2 parities][2 warps][kM][4] pair sums
  static constexpr size_t off_merge = off_xpair + 4 * 2 * 2 * kM * 4;  // per warp: KB keys + KB indices
  static constexpr size_t bytes = off_merge + (size_t)kEpiWarps * KB * (4 + 4);
  // Slack to align the dynamic base to 1024, and at least 116 KB in total: two of
  // these CTAs must never share an SM (each allocates all 512 TMEM columns), while
  // sparse-attention blocks (37 KB) may run beside one.
  static constexpr size_t smem = bytes + 1024 > 116 * 1024 ? bytes + 1024 : 116 * 1024;
};

// Exact fp32 score of q-tile row qr and stage row kr, both stored with the TMA
// swizzle of `ROWB`-byte rows: 16-byte chunk c of row j sits at c ^ ((j*ROWB >> 7) & (ROWB/16 - 1)).
// A wait that every lane of the warp performs; the verdict is made warp-uniform
// so a timeout never leaves the warp diverged in front of warp-synchronous code.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, kWaitLimitNs));
}
// Named barrier of all selection warps.
__device__ __forceinline__ void sel_sync() {
  asm volatile("bar.sync 5, %0;" ::"n"(kEpiWarps * 32) : "memory");
}
// Named barrier of the 64 threads of one quadrant's two warps.
__device__ __forceinline__ void pair_sync(int id) {
  asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
}

__device__ __forceinline__ bool warp_wait_cluster(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
  return __all_sync(0xffffffffu, mbar_wait_cluster(bar, parity, limit_ns));
}

// Exact fp32 score of two bf16 / fp16 rows: sequential FMA over d in order, with
// both operands converted to fp32 (the CUDA-core kernel's arithmetic).
template <typename TI, int R>
__device__ __forceinline__ float dot_rows(const TI* qrow, const TI* krow) {
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < R / 8; ++c) {
    float a[8], b[8];
    Vec16<TI>::unpack(ldg16(qrow + c * 8), a);
    Vec16<TI>::unpack(ldg16(krow + c * 8), b);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc = fmaf(a[e], b[e], acc);
  }
  return acc;
}

// Exact fp32 score from the original fp32 rows (sequential FMA over d, as the
// CUDA-core kernel and dot_swizzled compute it).
template <int R>
__device__ __forceinline__ float dot_f32_rows(const float* qrow, const float* krow) {
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < R / 4; ++c) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(qrow) + c);
    const float4 b = __ldg(reinterpret_cast<const float4*>(krow) + c);
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    acc = fmaf(a.w, b.w, acc);
  }
  return acc;
}

// Exact fp32 score of query row `qrow` and key `key` of batch element b.
template <typename TI, int R, bool F32>
__device__ __forceinline__ float exact_score(const ScoreSrc& s, int b, int qrow, int key) {
  if constexpr (F32)
    return dot_f32_rows<R>(static_cast<const float*>(s.q) + (int64_t)b * s.qsb + (int64_t)qrow * s.qst,
                           static_cast<const float*>(s.k) + (int64_t)b * s.ksb + (int64_t)key * s.kst);
  else
    return dot_rows<TI, R>(static_cast<const TI*>(s.q) + (int64_t)b * s.qsb + (int64_t)qrow * s.qst,
                           static_cast<const TI*>(s.k) + (int64_t)b * s.ksb + (int64_t)key * s.kst);
}

// F32: fp32 addresses.  The tensor cores score bf16 copies (TI = bf16); every
// product is then off by at most 2^-8 |q_d k_d| (two bf16 roundings), so the
// admission margin widens to 2^-6 sum|q| max|k| (twice the worst-case score error,
// with slack for max|k| being taken from the rounded keys), and admitted keys are
// rescored from the fp32 rows: the result is exact with respect to fp32 scores.
template <typename TI, int R, int KW, bool F32>
__global__ void __launch_bounds__(kThreads, 1)
    causal_topk_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                          const TcParams p) {
  using L = Layout<R, KW>;
  constexpr int KB = L::KB;
  constexpr int S = L::S;
  constexpr int ROWB = L::ROWB;
  constexpr int KSTEPS = R / 16;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr bool kBf16 = !std::is_same<TI, __half>::value;
  constexpr uint32_t IDESC = idesc_f16(kBf16, kM, kN);

  extern __shared__ unsigned char smem_raw[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* qs = base + L::off_q;
  unsigned char* ks = base + L::off_k;
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L::off_bar);
  uint64_t* mdone = full + S;
  uint64_t* done = mdone + S;
  uint64_t* qbar = done + S;
  uint64_t* kbar = qbar + 1;  // peer posted its key magnitude
  // One single-use barrier per bisection exchange: a fast warp of the peer may post
  // step i+1 before a slow one has posted step i, so the steps cannot share phases.
  uint64_t* xbar = qbar + 2;
  uint64_t* drain = xbar + kXRounds;  // the producer's last tcgen05.commit (nothing in flight at exit)
  uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(base + L::off_misc);
  uint32_t* kmax_own_s = tmem_base_s + 1;
  uint32_t* kmax_in_s = tmem_base_s + 2;
  uint32_t* xslot = reinterpret_cast<uint32_t*>(base + L::off_xslot);
  uint32_t* xpair = reinterpret_cast<uint32_t*>(base + L::off_xpair);
  uint32_t* mkey = reinterpret_cast<uint32_t*>(base + L::off_merge);       // [warp][KB]
  int* midx = reinterpret_cast<int*>(mkey + kEpiWarps * KB);               // [warp][KB]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  const int ntile = (p.Tq + kM - 1) / kM;
  const int tile = ntile - 1 - (int)(blockIdx.x >> 1);  // heaviest tiles first
  const int b = blockIdx.y;
  const int l0 = tile * kM;
  const int nrows = min(kM, p.Tq - l0);
  const int g0 = p.lim ? 0 : ((l0 / p.rt) * p.rs + p.r0) * p.rt + (l0 % p.rt);
  const int32_t* lrow = p.lim ? p.lim + (int64_t)b * p.Tq + l0 : nullptr;  // per-row key limits
  const int key_end = min(lrow ? lrow[nrows - 1] : g0 + nrows, p.Tk);
  const int nchunks = (key_end + kN - 1) / kN;
  const int n_own = nchunks > (int)rank ? (nchunks - (int)rank + 1) / 2 : 0;
  const int n_work = 2 * n_own;  // pass 1 + pass 2 items

  if (warp == kEpiWarps && lane == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&mdone[s], 2);
      mbar_init(&done[s], kEpiWarps);
    }
    mbar_init(qbar, 1);
    // exchange barriers complete on bytes: one local expect_tx arrive each, and the
    // peer's asynchronous stores (16 bytes per row per round; 4 bytes of key magnitude)
    for (int i = 0; i < kXRounds; ++i) mbar_init(&xbar[i], 1);
    mbar_init(kbar, 1);
    mbar_init(drain, 1);
    *kmax_own_s = 0u;
    fence_mbarrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_base_s, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before any peer arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_s;
  bool ok = true;
  uint32_t why = 0;  // wait sites that timed out (status bits 4..)

  auto chunk_of = [&](int w) { return (int)rank + 2 * (w % n_own); };

  if (warp == kEpiWarps) {
    // ============================================================ producer
    // pend[s]: item whose key load into stage s was issued and not yet waited for (-1: none)
    int pend[S];
#pragma unroll
    for (int s = 0; s < S; ++s) pend[s] = s < n_work ? s : -1;
    if (lane == 0) {
      prefetch_tmap(&qmap);
      prefetch_tmap(&kmap);
      mbar_arrive_expect_tx(qbar, (uint32_t)L::Q_BYTES);
      tma_load_3d(qs, &qmap, qbar, 0, l0, b);
      for (int w = 0; w < min(S, n_work); ++w) {
        mbar_arrive_expect_tx(&full[w], (uint32_t)L::STAGE_BYTES);
        tma_load_3d(ks + w * L::STAGE_STRIDE, &kmap, &full[w], 0, chunk_of(w) * kN, b);
      }
    }
    ok = warp_wait(qbar, 0);
    const bool q_landed = ok;
    if (!ok) why |= 4;
    for (int w = 0; w < n_work && ok; ++w) {
      const int s = w % S;
      unsigned char* stage = ks + s * L::STAGE_STRIDE;
      if (!warp_wait(&full[s], (uint32_t)(w / S) & 1u)) { ok = false; why |= 8; break; }
      pend[s] = -1;
      // accumulator (w & 1) was last read by item w-2
      if (w >= 2 && !warp_wait(&done[(w - 2) % S], (uint32_t)((w - 2) / S) & 1u)) { ok = false; why |= 16; break; }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t d = tmem_base + (uint32_t)((w & 1) * kN);
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
          const uint64_t a = smem_desc_kmajor(smem_u32(qs) + kk * 32, ROWB);
          const uint64_t bd = smem_desc_kmajor(smem_u32(stage) + kk * 32, ROWB);
          mma_f16(d, a, bd, IDESC, kk > 0);
        }
        mma_commit(&mdone[s]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&mdone[s]);
      const int wn = w - 1 + S;  // refill the stage item w-1 used
      if (w >= 1 && wn < n_work) {
        const int s1 = (w - 1) % S;
        if (!warp_wait(&done[s1], (uint32_t)((w - 1) / S) & 1u)) { ok = false; why |= 32; break; }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[s1], (uint32_t)L::STAGE_BYTES);
          tma_load_3d(ks + s1 * L::STAGE_STRIDE, &kmap, &full[s1], 0, chunk_of(wn) * kN, b);
        }
        pend[s1] = wn;
      }
      __syncwarp();
    }
    // Drain before the CTA may exit: every MMA this thread issued has completed when
    // the commit below arrives, and every key or q load that no wait consumed has
    // landed (all waits bounded; on a timeout the status word already says so).
    if (lane == 0) {
      mma_commit(drain);
      mbar_wait(drain, 0, kWaitLimitNs);
      if (!q_landed) mbar_wait(qbar, 0, kWaitLimitNs);
#pragma unroll
      for (int s = 0; s < S; ++s)
        if (pend[s] >= 0) mbar_wait(&full[s], (uint32_t)(pend[s] / S) & 1u, kWaitLimitNs);
    }
    __syncwarp();
  } else {
    // ============================================================ selection
    // Two warps per TMEM lane quadrant: warp w owns rows 32*(w%4) .. +31 and the
    // column half w/4 of every chunk (slices 2*(w/4) and 2*(w/4)+1).
    const int qd = warp & 3, hf = warp >> 2;
    const int r = 32 * qd + lane;  // query row in the tile = TMEM lane
    const bool row_ok = r < nrows;
    const int g = lrow ? (row_ok ? lrow[r] - 1 : -1) : g0 + r;
    const uint32_t lane_base = (uint32_t)(32 * qd) << 16;
    const int pair_bar = 1 + qd;   // named barrier of the two warps of this quadrant
    float qabs = 0.f;
    if (row_ok) {
      if constexpr (F32) {
        const float* qrow = p.qf + (int64_t)b * p.fqsb + (int64_t)(l0 + r) * p.fqst;
#pragma unroll
        for (int c = 0; c < R; ++c) qabs += fabsf(qrow[c]);
      } else {
        const TI* qrow = reinterpret_cast<const TI*>(p.q) + (int64_t)b * p.qsb + (int64_t)(l0 + r) * p.qst;
#pragma unroll
        for (int c = 0; c < R / 8; ++c) {
          float f[8];
          Vec16<TI>::unpack(ldg16(qrow + c * 8), f);
#pragma unroll
          for (int e = 0; e < 8; ++e) qabs += fabsf(f[e]);
        }
      }
    }
    {
      uint32_t ninf[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) ninf[j] = 0xff800000u;
#pragma unroll
      for (int par = 0; par < 2; ++par)
#pragma unroll
        for (int i = 0; i < 2; ++i)
          tmem_st_32x32b_x32(tmem_base + lane_base + 256 + par * kN + (2 * hf + i) * 32, ninf);
      tmem_st_wait();
    }
    ok = warp_wait(qbar, 0);
    if (!ok) why |= 64;

    // ---------------- pass 1: group maxima of tensor-core scores (this warp's slices)
    // The selection warps also take max|k| over the CTA's chunks (bit patterns of
    // non-negative floats order like their values), each warp over 1/8 of a stage.
    uint32_t kbits = 0;
    for (int w = 0; w < n_own && ok; ++w) {
      const int s = w % S;
      const uint32_t ph = (uint32_t)(w / S) & 1u;
      if (!warp_wait(&mdone[s], ph) || !warp_wait(&full[s], ph)) { ok = false; why |= 128; break; }
      tc_fence_after();
      {
        const uint4* kv = reinterpret_cast<const uint4*>(ks + s * L::STAGE_STRIDE);
        uint32_t m2 = 0;
        for (int i = warp * 32 + lane; i < (int)(L::STAGE_BYTES / 16); i += kEpiWarps * 32) {
          const uint4 x = kv[i];
          m2 = __vmaxu2(m2, x.x & 0x7fff7fffu);
          m2 = __vmaxu2(m2, x.y & 0x7fff7fffu);
          m2 = __vmaxu2(m2, x.z & 0x7fff7fffu);
          m2 = __vmaxu2(m2, x.w & 0x7fff7fffu);
        }
        kbits = max(kbits, max(m2 & 0xffffu, m2 >> 16));
      }
      const int c = chunk_of(w);
      const uint32_t acc = tmem_base + lane_base + (uint32_t)((w & 1) * kN);
      const uint32_t gcol = tmem_base + lane_base + 256 + (uint32_t)((w & 1) * kN);
      {
        // both of this warp's slices in flight before a single wait
        uint32_t v[2][32], gm[2][32];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          tmem_ld_32x32b_x32(acc + (2 * hf + i) * 32, v[i]);
          tmem_ld_32x32b_x32(gcol + (2 * hf + i) * 32, gm[i]);
        }
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int sl = 2 * hf + i;
          const int room = g - (c * kN + sl * 32);
          if (row_ok && room >= 31) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              gm[i][j] = __float_as_uint(fmaxf(__uint_as_float(gm[i][j]), __uint_as_float(v[i][j])));
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float x = (row_ok && j <= room) ? __uint_as_float(v[i][j]) : -INFINITY;
              gm[i][j] = __float_as_uint(fmaxf(__uint_as_float(gm[i][j]), x));
            }
          }
          tmem_st_32x32b_x32(gcol + sl * 32, gm[i]);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&done[s]);
    }
    // both warps' group maxima are complete and visible to the pair
    tmem_st_wait();
    kbits = __reduce_max_sync(kFullMask, kbits);
    if (lane == 0) atomicMax(kmax_own_s, kbits);
    tc_fence_before();
    pair_sync(pair_bar);
    tc_fence_after();

    // ---------------- lower bound on the K-th best score from the pair's 512 group maxima
    // Both CTAs bisect the same value range over the union of their maxima: each
    // step counts its own maxima >= mid, swaps the count with the peer thread of the
    // same row through DSMEM (remote store + remote mbarrier arrive), and applies
    // the same decision, so both end with the same bound.  The K-th largest of the
    // union is the score of K distinct keys, so it lower-bounds the row's K-th score.
    // The two warps of a quadrant split each count (warp hf reads the column half
    // hf of the row's maxima) and add their halves through shared memory first.
    const uint32_t gbase = tmem_base + lane_base + 256 + (uint32_t)(hf * (kGroups / 2));
    int nf = 0;
    float mn = INFINITY, mx = -INFINITY;
#pragma unroll 1
    for (int blk = 0; blk < kGroups / 64; blk += 2) {
      uint32_t v[2][32];
      tmem_ld_32x32b_x32(gbase + blk * 32, v[0]);
      tmem_ld_32x32b_x32(gbase + blk * 32 + 32, v[1]);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float x = __uint_as_float(v[i][j]);
          nf += x > -INFINITY ? 1 : 0;
          mn = fminf(mn, x > -INFINITY ? x : INFINITY);
          mx = fmaxf(mx, x);
        }
    }
    // add the pair's halves: [round parity][hf][row][3]; two parities because the
    // partner may still read step i-1 while this warp writes step i+1
    auto pair_sum3 = [&](int round, uint32_t (&x)[3]) {
      uint32_t* mine = xpair + (((round & 1) * 2 + hf) * kM + r) * 4;
      const uint32_t* other = xpair + (((round & 1) * 2 + (hf ^ 1)) * kM + r) * 4;
      mine[0] = x[0];
      mine[1] = x[1];
      mine[2] = x[2];
      pair_sync(pair_bar);
      x[0] += other[0];
      x[1] = __float_as_uint(fminf(__uint_as_float(x[1]), __uint_as_float(other[1])));
      x[2] = __float_as_uint(fmaxf(__uint_as_float(x[2]), __uint_as_float(other[2])));
    };
    // one exchange with the peer CTA: the quadrant's first warp sends (a, b, c) to the
    // peer's thread of this row with one asynchronous 16-byte store that completes on
    // the peer's barrier of this round (both warps hold the same triple); both warps
    // wait for and read the peer's triple
    auto swap3 = [&](int round, const uint32_t (&x)[3], uint32_t (&got)[3]) {
      uint32_t* slot = xslot + ((round & 1) * kM + r) * 4;
      if (warp == 0 && lane == 0) mbar_arrive_expect_tx(&xbar[round], (uint32_t)(kM * 16));
      if (hf == 0 && !(p.withhold == round + 1 && rank == 1))
        st_async_v4(map_peer(slot, peer), x[0], x[1], x[2], 0u, map_peer(&xbar[round], peer));
      if (!warp_wait_cluster(&xbar[round], 0, p.xwait_ns)) { ok = false; why |= 256; }
      got[0] = slot[0];
      got[1] = slot[1];
      got[2] = slot[2];
    };
    uint32_t mine3[3] = {(uint32_t)nf, __float_as_uint(mn), __float_as_uint(mx)}, got[3];
    pair_sum3(0, mine3);
    swap3(0, mine3, got);
    const int nf_t = (int)(mine3[0] + got[0]);
    float lo = fminf(__uint_as_float(mine3[1]), __uint_as_float(got[1]));
    float hi = fmaxf(__uint_as_float(mine3[2]), __uint_as_float(got[2]));
    const bool bis = nf_t >= p.K;
    if (!bis) lo = hi = 0.f;
    // every thread runs every step (tcgen05.ld is warp-collective and every step is
    // an exchange the peer waits for); rows with fewer than K maxima ignore the result
#pragma unroll 1
    for (int it = 0; it < kXRounds - 1; ++it) {
      const float mid = lo + 0.5f * (hi - lo);
      int c = 0;
#pragma unroll 1
      for (int blk = 0; blk < kGroups / 64; blk += 2) {
        uint32_t v[2][32];
        tmem_ld_32x32b_x32(gbase + blk * 32, v[0]);
        tmem_ld_32x32b_x32(gbase + blk * 32 + 32, v[1]);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int j = 0; j < 32; ++j) c += __uint_as_float(v[i][j]) >= mid ? 1 : 0;
      }
      uint32_t x3[3] = {(uint32_t)c, 0u, 0u};
      pair_sum3(1 + it, x3);
      swap3(1 + it, x3, got);
      if ((int)(x3[0] + got[0]) >= p.K) lo = mid;
      else hi = mid;
    }
    const float theta = bis ? lo : -INFINITY;

    // key magnitudes for the margin (16-bit patterns; the barrier spans every
    // selection warp, so all their parts are in)
    sel_sync();
    if (r == 0 && hf == 0) {
      mbar_arrive_expect_tx(kbar, 4u);
      st_async_u32(map_peer(kmax_in_s, peer), *kmax_own_s, map_peer(kbar, peer));
    }
    if (!warp_wait_cluster(kbar, 0)) { ok = false; why |= 1024; }
    const uint32_t kb = max(*kmax_own_s, *kmax_in_s);
    const float kpair = kBf16 ? __uint_as_float(kb << 16) : __half2float(__ushort_as_half((unsigned short)kb));
    const float eps = (F32 ? 1.0f / 64.0f : kEpsScale) * qabs * kpair;
    float lim = theta > -INFINITY ? theta - eps : -INFINITY;

    // ---------------- pass 2: admit candidates into the workspace lists
    // A key is admitted when its tensor-core score reaches lim.  Only its index is
    // stored; the exact fp32 scores are computed by the finalisation kernel, which
    // runs at full occupancy, so this kernel's critical chain holds no rescoring.
    const int64_t row0 = (int64_t)b * p.Tq + l0 + 32 * qd;  // first row of this quadrant

    // This warp's candidates of row r go to its own list (CTA rank, column half hf):
    // the count lives in the lane's register, so no slot is shared with another warp.
    int cnt = 0;
    int32_t* mylist = p.ws + (((row0 + lane) * 2 + rank) * 2 + hf) * KW;

    bool alive = ok;
    for (int w = n_own; w < n_work; ++w) {
      const int s = w % S;
      const uint32_t ph = (uint32_t)(w / S) & 1u;
      if (alive && !warp_wait(&mdone[s], ph)) {
        alive = false;
        ok = false;
        why |= 512;
      }
      tc_fence_after();
      const int c = chunk_of(w);
      const uint32_t acc = tmem_base + lane_base + (uint32_t)((w & 1) * kN);
      // admission masks of both slices (loads in flight together)
      uint32_t v[2][32];
      if (alive) {
        tmem_ld_32x32b_x32(acc + (2 * hf) * 32, v[0]);
        tmem_ld_32x32b_x32(acc + (2 * hf + 1) * 32, v[1]);
        tmem_ld_wait();
      }
      // the scores are in registers: the accumulator and the stage are free
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&done[s]);
      uint32_t masks[2] = {0u, 0u};
      if (alive) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          uint32_t m = 0;
#pragma unroll
          for (int j = 0; j < 32; ++j) m |= (__uint_as_float(v[i][j]) >= lim ? 1u : 0u) << j;
          const int room = g - (c * kN + (2 * hf + i) * 32);
          if (!row_ok || room < 0) m = 0;
          else if (room < 31) m &= (2u << room) - 1u;
          masks[i] = m;
        }
      }
      const int np = __popc(masks[0]) + __popc(masks[1]);
      // A list that this chunk could overflow is compacted to its exact top-K first
      // (its entries rescored exactly from the address rows in global memory); that
      // also raises the row's threshold.  Rare: a row admits ~1.2 K keys in all.
      unsigned need = __ballot_sync(kFullMask, cnt + np > KW);
      while (need) {
        const int ln = __ffs(need) - 1;
        need &= need - 1;
        const int n = __shfl_sync(kFullMask, cnt, ln);
        int32_t* wrow = p.ws + (((row0 + ln) * 2 + rank) * 2 + hf) * KW;
        const int qrow = l0 + 32 * qd + ln;
        uint32_t kk[KW / 32];
        int ii[KW / 32];
#pragma unroll
        for (int t = 0; t < KW / 32; ++t) {
          const int e = t * 32 + lane;
          const int j = e < n ? wrow[e] : 0;
          kk[t] = e < n ? ordered_key(exact_score<TI, R, F32>(p.src, b, qrow, j)) : 0u;
          ii[t] = e < n ? j : INT_MAX;
        }
        uint32_t* bk = mkey + warp * KB;
        int* bi = midx + warp * KB;
        const uint32_t tau = select_compact<KW / 32>(kk, ii, n, p.K, lane, bk, bi);
        for (int e = lane; e < p.K; e += 32) wrow[e] = bi[e];
        __syncwarp();
        if (lane == ln) {
          cnt = p.K;
          lim = fmaxf(lim, key_to_float(tau) - eps);
        }
      }
      // this lane's admitted keys go to its own list
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        uint32_t m = masks[i];
        while (m) {
          const int j = __ffs(m) - 1;
          m &= m - 1;
          mylist[cnt++] = c * kN + (2 * hf + i) * 32 + j;
        }
      }
    }
    if (row_ok) p.ws_cnt[((row0 + lane) * 2 + rank) * 2 + hf] = cnt;
  }
  if (!ok && p.status) atomicOr(p.status, 2 | (int)why);

  tc_fence_before();
  cluster_sync();  // neither CTA leaves while its peer may still touch its shared memory
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- finalisation
// One warp per query row: the exact top-K of the two CTAs' candidate lists
// (composites key << 32 | ~index, so larger = better and ties favour the lower
// index), in list order, plus pad slots.  Runs at full occupancy; the
// selection is the same warp radix select the streaming kernels use.
struct FinParams {
  const int32_t* ws;
  uint32_t* ws_key;  // exact keys of the candidates, written by topk_rescore_kernel
  const int32_t* ws_cnt;
  int32_t* idx;
  int B, Tq, Tk, K, cap;
  int pad_mode;
  int rt, rs, r0;
  const int32_t* lim;
  ScoreSrc src;
};

constexpr int kFinWarps = 8;

template <int EPLF, int SE>
__device__ __forceinline__ void finalize_row(const FinParams& p, int64_t row, const int (&nl)[kLists], int lane,
                                             uint32_t* bk, int* bi) {
  const int l = (int)(row % p.Tq);
  const int g = p.lim ? p.lim[row] - 1 : ((l / p.rt) * p.rs + p.r0) * p.rt + (l % p.rt);
  const int e1 = nl[0], e2 = e1 + nl[1], e3 = e2 + nl[2], n = e3 + nl[3];
  const int32_t* a = p.ws + row * kLists * p.cap;
  const uint32_t* ak = p.ws_key + row * kLists * p.cap;
  // The row's concatenated lists are consumed in blocks of up to 32*EPLF entries
  // together with the running top-K kept in bk/bi (one block in the usual case).
  int m = 0;   // entries held in bk/bi
  int e0 = 0;  // next unconsumed list element
  do {
    const int take = min(n - e0, EPLF * 32 - m);
    const int cnt = m + take;
    uint32_t kk[EPLF];
    int ii[EPLF];
#pragma unroll
    for (int t = 0; t < EPLF; ++t) {
      const int e = t * 32 + lane;
      uint32_t key = 0;
      int j = INT_MAX;
      if (e < m) {
        key = bk[e];
        j = bi[e];
      } else if (e < cnt) {
        const int x = e0 + e - m;
        const int li = (x >= e1) + (x >= e2) + (x >= e3);
        const int off = li == 0 ? 0 : li == 1 ? e1 : li == 2 ? e2 : e3;
        j = a[li * p.cap + (x - off)];
        key = ak[li * p.cap + (x - off)];
      }
      kk[t] = key;
      ii[t] = j;
    }
    __syncwarp();
    if (cnt > p.K) {
      select_compact<EPLF>(kk, ii, cnt, p.K, lane, bk, bi);
      m = p.K;
    } else {
#pragma unroll
      for (int t = 0; t < EPLF; ++t) {
        const int e = t * 32 + lane;
        if (e < cnt) {
          bk[e] = kk[t];
          bi[e] = ii[t];
        }
      }
      __syncwarp();
      m = cnt;
    }
    e0 += take;
  } while (e0 < n);
  // The selected keys go out in the order the lists hold them (admission order,
  // compaction keeps it), not sorted by score: the reference leaves the slot order
  // open too (topk(sorted=False)), and sorting cost a tenth of the retrieval.  The
  // order is still a deterministic function of the inputs; pads take the trailing slots.
  __syncwarp();
  int32_t* out = p.idx + row * p.K;
#pragma unroll
  for (int t = 0; t < SE; ++t) {
    const int s = t * 32 + lane;
    if (s < p.K) {
      int val;
      if (s < m) val = bi[s];
      else val = p.pad_mode == 0 ? (int)(((int64_t)g + p.K + s + 1) % p.Tk) : -1;
      out[s] = val;
    }
  }
}

template <int SE, int KB>
__global__ void __launch_bounds__(kFinWarps * 32, 2) topk_finalize_kernel(const FinParams p) {
  pdl_wait();
  __shared__ uint32_t skey[kFinWarps][KB];
  __shared__ int sidx[kFinWarps][KB];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kFinWarps + warp;
  if (row >= (int64_t)p.B * p.Tq) return;
  const int4 c4 = *reinterpret_cast<const int4*>(p.ws_cnt + row * kLists);
  const int nl[kLists] = {c4.x, c4.y, c4.z, c4.w};
  const int n = c4.x + c4.y + c4.z + c4.w;
  // with the pair's shared bound a row typically holds 1.1-1.5 K candidates; the wider
  // form merges larger rows in blocks (it must hold more than KB entries to progress)
  constexpr int E1 = KB <= 128 ? 6 : 12, E2 = KB <= 128 ? 12 : 16;
  if (n <= E1 * 32) finalize_row<E1, SE>(p, row, nl, lane, skey[warp], sidx[warp]);
  else finalize_row<E2, SE>(p, row, nl, lane, skey[warp], sidx[warp]);
}

// Exact fp32 keys of every candidate: one warp per (row, list), full occupancy.
// Rows whose lists hold K candidates or fewer need no selection and are skipped.
template <typename TI, int R, bool F32>
__global__ void __launch_bounds__(256) topk_rescore_kernel(const FinParams p) {
  pdl_wait();
  const int64_t wl = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);  // (row, list)
  const int lane = threadIdx.x & 31;
  if (wl >= (int64_t)p.B * p.Tq * kLists) return;
  const int64_t row = wl / kLists;
  const int4 c4 = *reinterpret_cast<const int4*>(p.ws_cnt + row * kLists);
  if (c4.x + c4.y + c4.z + c4.w <= p.K) return;
  const int n = p.ws_cnt[wl];
  const int l = (int)(row % p.Tq), bb = (int)(row / p.Tq);
  const int32_t* a = p.ws + wl * p.cap;
  uint32_t* ak = p.ws_key + wl * p.cap;
  // two entries per lane in flight: both indices, then both key rows, then the FMAs
  for (int e0 = 0; e0 < n; e0 += 64) {
    const int e1 = e0 + lane, e2 = e1 + 32;
    const int j1 = e1 < n ? a[e1] : -1;
    const int j2 = e2 < n ? a[e2] : -1;
    if constexpr (F32 || R > 32) {
      if (j1 >= 0) ak[e1] = ordered_key(exact_score<TI, R, F32>(p.src, bb, l, j1));
      if (j2 >= 0) ak[e2] = ordered_key(exact_score<TI, R, F32>(p.src, bb, l, j2));
    } else {
      constexpr int NC = R / 8;
      const TI* qrow = static_cast<const TI*>(p.src.q) + (int64_t)bb * p.src.qsb + (int64_t)l * p.src.qst;
      const TI* kb = static_cast<const TI*>(p.src.k) + (int64_t)bb * p.src.ksb;
      uint4 qv[NC], k1[NC], k2[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        qv[c] = ldg16(qrow + c * 8);
        k1[c] = j1 >= 0 ? ldg16(kb + (int64_t)j1 * p.src.kst + c * 8) : make_uint4(0, 0, 0, 0);
        k2[c] = j2 >= 0 ? ldg16(kb + (int64_t)j2 * p.src.kst + c * 8) : make_uint4(0, 0, 0, 0);
      }
      float d1 = 0.f, d2 = 0.f;
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        float x[8], y1[8], y2[8];
        Vec16<TI>::unpack(qv[c], x);
        Vec16<TI>::unpack(k1[c], y1);
        Vec16<TI>::unpack(k2[c], y2);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          d1 = fmaf(x[t], y1[t], d1);
          d2 = fmaf(x[t], y2[t], d2);
        }
      }
      if (j1 >= 0) ak[e1] = ordered_key(d1);
      if (j2 >= 0) ak[e2] = ordered_key(d2);
    }
  }
}

// ---------------------------------------------------------------- host side
// Test hook (wf_testing_withhold_pair_arrive): consumed by the next launch.
std::atomic<int> g_test_withhold{0};
std::atomic<uint64_t> g_test_xwait_ns{kWaitLimitNs};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

bool make_map(CUtensorMap* map, const void* ptr, bool bf16, int R, int64_t T, int64_t B, int64_t st, int64_t sb,
              int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)R, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)(st * 2), (cuuint64_t)(sb * 2)};
  const cuuint32_t box[3] = {(cuuint32_t)R, (cuuint32_t)box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = R == 64   ? CU_TENSOR_MAP_SWIZZLE_128B
                                : R == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                          : CU_TENSOR_MAP_SWIZZLE_32B;
  CUresult rc = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return rc == CUDA_SUCCESS;
}

template <int R>
size_t smem_for_k(int K) {
  return K <= 128 ? Layout<R, 256>::smem : K <= 256 ? Layout<R, 384>::smem : 0;
}

size_t tc_smem(int R, int K) {
  switch (R) {
    case 16: return smem_for_k<16>(K);
    case 32: return smem_for_k<32>(K);
    case 64: return smem_for_k<64>(K);
    default: return 0;
  }
}

int list_capacity(int K) { return K <= 128 ? 256 : 384; }

// Batch elements per launch pair: the workspace holds about kRowsPerPass query rows.
int64_t batch_per_pass(int64_t B, int64_t Tq) {
  const int64_t bpp = Tq >= kRowsPerPass ? 1 : kRowsPerPass / Tq;
  return bpp < B ? bpp : B;
}

// per row: kLists lists of candidate indices and their exact keys, and the list counts
size_t ws_bytes_per_row(int K) { return (size_t)kLists * list_capacity(K) * 2 * sizeof(int32_t) + kLists * sizeof(int32_t); }

// bf16 copies of fp32 address rows (F32 path): dst[b][t][r] contiguous.
__global__ void shadow_bf16_kernel(const float* src, int64_t sb, int64_t st, int nb, int T, int R,
                                   __nv_bfloat16* dst) {
  const int64_t n = (int64_t)nb * T * R;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(e % R);
    const int64_t bt = e / R;
    const int t = (int)(bt % T), b = (int)(bt / T);
    dst[e] = __float2bfloat16_rn(src[(int64_t)b * sb + (int64_t)t * st + r]);
  }
}

size_t shadow_bytes_pass(int64_t bpp, int64_t Tq, int64_t Tk, int R) {
  return (size_t)bpp * (Tq + Tk) * R * 2 + 256;
}

template <typename TI, int R, int KW, int SE, bool F32>
int launch_t(const TopkParams& p, cudaStream_t stream) {
  using L = Layout<R, KW>;
  if (L::smem > kMaxSmem) return -1;
  auto kern = causal_topk_tc_kernel<TI, R, KW, F32>;
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev >= kMaxDevices || !configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::smem);
    if (e != cudaSuccess) return (int)e;
    if (dev < kMaxDevices) configured[dev] = true;
  }
  const bool bf16 = !std::is_same<TI, __half>::value;
  const int64_t bpp = batch_per_pass(p.B, p.Tq);
  const size_t rows_pass = (size_t)bpp * p.Tq;
  const size_t lists = rows_pass * ws_bytes_per_row(p.K);
  const size_t need = lists + (F32 ? shadow_bytes_pass(bpp, p.Tq, p.Tk, R) : 0);
  if (!p.ws || p.ws_bytes < need || reinterpret_cast<uintptr_t>(p.ws) % 16) return -3;
  int32_t* ws = reinterpret_cast<int32_t*>(p.ws);
  uint32_t* ws_key = reinterpret_cast<uint32_t*>(ws + rows_pass * kLists * KW);
  int32_t* ws_cnt = reinterpret_cast<int32_t*>(ws_key + rows_pass * kLists * KW);
  __nv_bfloat16* shq = reinterpret_cast<__nv_bfloat16*>(
      (reinterpret_cast<uintptr_t>(static_cast<char*>(p.ws) + lists) + 255) & ~uintptr_t(255));
  __nv_bfloat16* shk = shq + (size_t)bpp * p.Tq * R;
  const size_t esz = F32 ? 4 : 2;
  // Batch slices run one after the other on the stream and reuse the workspace.
  for (int64_t b0 = 0; b0 < p.B; b0 += bpp) {
    const int nb = (int)(p.B - b0 < bpp ? p.B - b0 : bpp);
    const void* q = static_cast<const char*>(p.q) + (size_t)(b0 * p.qsb) * esz;
    const void* k = static_cast<const char*>(p.k) + (size_t)(b0 * p.ksb) * esz;
    CUtensorMap qmap, kmap;
    TcParams t{};
    if constexpr (F32) {
      const unsigned gq = (unsigned)(((int64_t)nb * p.Tq * R + 255) / 256 < 148 * 8 ? ((int64_t)nb * p.Tq * R + 255) / 256 : 148 * 8);
      const unsigned gk = (unsigned)(((int64_t)nb * p.Tk * R + 255) / 256 < 148 * 8 ? ((int64_t)nb * p.Tk * R + 255) / 256 : 148 * 8);
      shadow_bf16_kernel<<<gq, 256, 0, stream>>>(static_cast<const float*>(q), p.qsb, p.qst, nb, p.Tq, R, shq);
      shadow_bf16_kernel<<<gk, 256, 0, stream>>>(static_cast<const float*>(k), p.ksb, p.kst, nb, p.Tk, R, shk);
      if (!make_map(&qmap, shq, true, R, p.Tq, nb, R, (int64_t)p.Tq * R, kM)) return -1;
      if (!make_map(&kmap, shk, true, R, p.Tk, nb, R, (int64_t)p.Tk * R, kN)) return -1;
      t.qf = static_cast<const float*>(q);
      t.kf = static_cast<const float*>(k);
      t.fqsb = p.qsb; t.fqst = p.qst; t.fksb = p.ksb; t.fkst = p.kst;
      t.q = shq;
      t.qsb = (int64_t)p.Tq * R;
      t.qst = R;
    } else {
      if (!make_map(&qmap, q, bf16, R, p.Tq, nb, p.qst, p.qsb, kM)) return -1;
      if (!make_map(&kmap, k, bf16, R, p.Tk, nb, p.kst, p.ksb, kN)) return -1;
      t.q = q;
      t.qsb = p.qsb;
      t.qst = p.qst;
    }
    t.B = nb; t.Tq = p.Tq; t.Tk = p.Tk; t.K = p.K;
    t.pad_mode = p.pad_mode;
    t.rt = p.rt; t.rs = p.rs; t.r0 = p.r0;
    t.lim = p.lim ? p.lim + (size_t)b0 * p.Tq : nullptr;
    t.idx = p.idx + (size_t)b0 * p.Tq * p.K;
    t.status = p.status;
    t.ws = ws;
    t.ws_cnt = ws_cnt;
    t.src = ScoreSrc{q, k, p.qsb, p.qst, p.ksb, p.kst};
    t.withhold = g_test_withhold.exchange(0);
    t.xwait_ns = t.withhold ? g_test_xwait_ns.load() : kWaitLimitNs;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * ((p.Tq + kM - 1) / kM), nb);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, qmap, kmap, t);
    if (e != cudaSuccess) return (int)e;
    FinParams f{};
    f.ws = ws;
    f.ws_cnt = ws_cnt;
    f.ws_key = ws_key;
    f.idx = t.idx;
    f.B = nb; f.Tq = p.Tq; f.Tk = p.Tk; f.K = p.K; f.cap = KW;
    f.pad_mode = p.pad_mode;
    f.rt = p.rt; f.rs = p.rs; f.r0 = p.r0;
    f.lim = t.lim;
    f.src = t.src;
    const size_t rows = (size_t)nb * p.Tq;
    e = launch_pdl(topk_rescore_kernel<TI, R, F32>, dim3((unsigned)((rows * kLists + 7) / 8)), dim3(256), 0, stream, f);
    if (e != cudaSuccess) return (int)e;
    e = launch_pdl(topk_finalize_kernel<SE, KW - 128>, dim3((unsigned)((rows + kFinWarps - 1) / kFinWarps)),
                   dim3(kFinWarps * 32), 0, stream, f);
    e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

template <typename TI, int R, bool F32>
int launch_r(const TopkParams& p, cudaStream_t s) {
  if (p.K <= 32) return launch_t<TI, R, 256, 1, F32>(p, s);
  if (p.K <= 64) return launch_t<TI, R, 256, 2, F32>(p, s);
  if (p.K <= 128) return launch_t<TI, R, 256, 4, F32>(p, s);
  if (p.K <= 256) return launch_t<TI, R, 384, 8, F32>(p, s);
  return -1;
}

template <typename TI, bool F32>
int launch_ti(const TopkParams& p, cudaStream_t s) {
  switch (p.R) {
    case 16: return launch_r<TI, 16, F32>(p, s);
    case 32: return launch_r<TI, 32, F32>(p, s);
    case 64: return launch_r<TI, 64, F32>(p, s);
    default: return -1;
  }
}

}  // namespace

bool topk_tc_supported(const TopkParams& p, int dtype) {
  if (dtype != kBF16 && dtype != kF16 && dtype != kF32) return false;
  if (p.R != 16 && p.R != 32 && p.R != 64) return false;
  if (p.K > 256 || p.Tk > 65536 || p.B > 65535) return false;
  const size_t sm = tc_smem(p.R, p.K);
  if (sm == 0 || sm > kMaxSmem) return false;
  if (p.qsr != 1 || p.ksr != 1) return false;
  if ((reinterpret_cast<uintptr_t>(p.q) | reinterpret_cast<uintptr_t>(p.k)) % 16) return false;
  const int esz = dtype == kF32 ? 4 : 2;  // fp32: rows read as float4 for the rescoring
  if ((p.qst * esz) % 16 || (p.kst * esz) % 16 || (p.qsb * esz) % 16 || (p.ksb * esz) % 16) return false;
  const bool identity = p.rs == 1 && p.r0 == 0;
  if (!identity && p.rt % kM) return false;
  return encode_fn() != nullptr;
}

size_t topk_tc_workspace_bytes(int64_t B, int64_t Tq, int64_t Tk, int R, int K, int dtype) {
  if (K > 256 || B <= 0 || Tq <= 0) return 0;
  const int64_t bpp = batch_per_pass(B, Tq);
  const size_t lists = (size_t)bpp * Tq * ws_bytes_per_row(K);
  return dtype == kF32 ? lists + shadow_bytes_pass(bpp, Tq, Tk, R) : lists;
}

void topk_tc_test_withhold(int round, uint64_t wait_ns) {
  g_test_xwait_ns.store(wait_ns);
  g_test_withhold.store(round >= 0 && round < kXRounds ? round + 1 : 0);
}

int launch_causal_topk_tc(const TopkParams& p, int dtype, cudaStream_t stream) {
  if (dtype == kBF16) return launch_ti<__nv_bfloat16, false>(p, stream);
  if (dtype == kF16) return launch_ti<__half, false>(p, stream);
  if (dtype == kF32) return launch_ti<__nv_bfloat16, true>(p, stream);
  return -1;
}

// ---------------------------------------------------------------- allocation-free scratch
// Retrieval scratch for callers that cannot allocate device memory at all.  This
// array is part of the library image: every GPU that loads the library reserves
// kNoAllocScratchBytes for it until the process exits.  All calls share it and it
// keeps the previous call's contents; nothing in it needs to start at zero,
// because the retrieval kernel writes every count and candidate it later reads.
constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB: B*Tq <= 2044 query rows (8208 bytes each) for K <= 128; fp32 addresses add bf16 copies of the rows
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
}  // namespace

size_t noalloc_scratch_capacity() { return kNoAllocScratchBytes; }

// Device address of the scratch array on the current device.  In host code the
// array's name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, queried once per device with that device current.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace wf
