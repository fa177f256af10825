// tc_scan.cu -- large-batch exact flat search on the tensor cores.
//
// For query batches the exact CUDA-core scan (scan.cu) becomes FP32-issue
// bound, so batches run as the dense contraction they are: a tcgen05 bf16 GEMM
// produces approximate distances, a certified error bound turns them into a
// candidate set that provably contains the exact top-k, and the candidates are
// re-scored with the exact fp32 arithmetic of the reference CPU path
// (sequential dot, dots.c:40-47; host-tier finalize, ParallelFlatScan.swift
// :237-258).  Results therefore equal the exact scan's bit for bit.
//
// Per query q and row r let s = dot(q, r) (real), s~ the bf16 tensor-core dot.
//   |s~ - s| <= |q - q~| |r| + |q~| |r - r~| + c_acc |q~| |r~|      (Cauchy-Schwarz)
// with q~, r~ the bf16 roundings and c_acc bounding the fp32 accumulation.
// The distance is affine in s per (q, r) -- IP: -s; L2: |q|^2 - 2s + |r|^2;
// cosine: 1 - s / (|q| |r|) -- so with corpus-wide maxima the approximate
// distance d~ and the exact fp32 distance d obey |d~ - d| <= eps_q.  If T_k is
// the k-th smallest d~ over all rows, a row with d~ > T_k + 2 eps_q has
// d > T_k + eps_q >= (k-th smallest d): it cannot be in the exact top-k, ties
// included.
//
// Pipeline per batch:
//   1. query prep: bf16 queries, exact |q|^2 (sequential), eps_q, affine terms;
//   2. sample pass: GEMM over the first S rows writing d~ densely;
//   3. per query: thr_q = (k-th smallest d~ of the sample) + 2 eps_q, which
//      is >= T_k + 2 eps_q because the sample is a subset;
//   4. full pass: GEMM over all rows, the epilogue appends (d~, row) when
//      d~ <= thr_q;
//   5. per query: T_k from the candidates, exact re-score of those with
//      d~ <= T_k + 2 eps_q, (distance, id) top-k.  A query whose candidate
//      list overflowed or whose certificate fails is re-scanned exactly by
//      its block (slow, rare, still exact).
//
// GEMM layout (tcgen05 kind::f16, one CTA per SM, persistent over tiles):
//   A = 128 corpus rows x 64 bf16 (K-major, 128-byte swizzle), B = 256 queries
//   x 64 bf16, D = 128 x 256 fp32 in TMEM, two accumulators (512 columns) so
//   the epilogue of one tile overlaps the MMAs of the next.  Warp 0 lane 0
//   issues TMA, warp 1 lane 0 issues MMAs and commits, warps 4-7 read TMEM
//   (TMEM lane = corpus row) in the epilogue.  No multicast anywhere.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"
#include "tc.h"

namespace mans {
namespace {

constexpr int kQM = 128;  // queries per block (MMA M, TMEM lanes)
constexpr int kRN = 256;  // corpus rows per tile (MMA N, TMEM columns)
constexpr int kBK = 64;   // bf16 per 128-byte swizzle row
constexpr int kQBytes = kQM * kBK * 2;  // 16 KiB per k-block of queries
constexpr int kRBytes = kRN * kBK * 2;  // 32 KiB per k-block of rows
constexpr int kTcThreads = 640;         // warps 0-3 control, 4-19 epilogue
constexpr int kEpiWarps = 16;
constexpr int kTmemCols = 512;          // two 256-column accumulators
constexpr size_t kResidentMax = 96 * 1024;
constexpr size_t kPipeBudget = 196 * 1024;
constexpr int kRerankThreads = 128;
constexpr int kRtSlots = 4;       // row-term ring depth (tiles)

// Shared scratch of block_kth_smallest.
struct KthSmem {
  uint32_t hist[2048];
  float list[1024];
  float red[64];
  uint32_t wsum[32];
  float lo[4], scale[4];
  int sel[4];
  uint32_t sh[4];
  // dynamic tail of the fused pass: the producer's claimed tiles (-1: none
  // left), each published to the MMA issuer and the epilogue by ufull[slot]
  uint64_t ufull[16];
  int64_t uq[16];
};

// Shared-memory plan of tc_scan_kernel for a given width: the query block is
// kept resident when its nk k-blocks fit in 96 KiB (dim <= 384), otherwise
// it is streamed beside the rows in every stage.
struct TcLayout {
  int nk;
  bool resident;
  int stages;
  size_t a_bytes;
  size_t stage_bytes;
  size_t rt_off;  // ring of per-row terms (kRtSlots x [row factor | |r|^2] x kRN floats)
  size_t bar_off;
  size_t kth_off;
  size_t total;
};

// k-blocks of 128 bytes per row: 64 bf16 or 128 int8 elements
__host__ __device__ inline int tc_kblocks(int dim, bool i8) {
  return i8 ? (dim + 127) / 128 : (dim + kBK - 1) / kBK;
}

// With `pair` (a CTA pair sharing M = 256 MMAs) a stage holds this CTA's
// half of the row tile, 128 rows, so the same budget keeps twice the stages.
// `lean` (the bf16 filtered pass without per-row terms or fused sampling:
// cosine and inner product) has neither the row-term ring nor the k-th
// selection scratch, and gives the freed shared memory to the stage ring:
// every stage that fits in kLeanBudget (one more 32 KiB stage at d = 384).
constexpr size_t kLeanBudget = 227 * 1024;
__host__ __device__ inline TcLayout tc_layout(int nk, int stream_queries, bool pair = false,
                                              bool lean = false) {
  TcLayout L;
  L.nk = nk;
  L.resident = !stream_queries && static_cast<size_t>(L.nk) * kQBytes <= kResidentMax;
  L.a_bytes = L.resident ? static_cast<size_t>(L.nk) * kQBytes : 0;
  L.stage_bytes = (pair ? kRBytes / 2 : kRBytes) + (L.resident ? 0 : kQBytes);
  // barriers: full/empty per stage, acc_full/acc_empty x2, a_full, a_empty,
  // drain, rt_full/rt_empty per row-term slot (at most 8 stages)
  const size_t bars_max = 8 * (2 * 8 + 7 + 2 * kRtSlots);
  const size_t budget = lean ? kLeanBudget - 1024 - bars_max - 16 : kPipeBudget;
  size_t st = budget > L.a_bytes ? (budget - L.a_bytes) / L.stage_bytes : 0;
  L.stages = static_cast<int>(st > 8 ? 8 : st);
  L.rt_off = L.a_bytes + static_cast<size_t>(L.stages) * L.stage_bytes;  // 1 KiB aligned
  L.bar_off = L.rt_off + (lean ? 0 : static_cast<size_t>(kRtSlots) * 2 * kRN * sizeof(float));
  const size_t bars = 8 * (2 * static_cast<size_t>(L.stages) + 7 + 2 * kRtSlots);
  // + tmem slot / abort (16 B) + the k-th selection scratch of the fused sampling
  L.kth_off = L.bar_off + bars + 16;
  L.total = 1024 + L.kth_off + (lean ? 0 : sizeof(KthSmem));
  return L;
}

// ---- tcgen05 wrappers (inline PTX) ------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 in, fp32 accumulate)
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8 (s8 in, s32 accumulate)
__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
// arrive on `bar` once every MMA previously issued by this thread completed
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- CTA pairs (cta_group::2): two CTAs of a cluster share one MMA --------
// The leader (cluster rank 0) issues M = 256 MMAs whose A rows 0-127 and B
// rows 0-127 come from its own shared memory and rows 128-255 from its
// peer's, at the same offsets; each CTA's TMEM receives its own 128 A rows x
// all N columns.  Every tcgen05 instruction of such a kernel uses
// cta_group::2.  Loads carry no multicast: each CTA copies its own half.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// shared::cluster address of the variable at `local`'s offset in CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
// arrive on an mbarrier given by its shared::cluster address (any CTA of the cluster)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}
// 2-D TMA load into this CTA's shared memory completing on an mbarrier of
// either CTA of the pair (shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int32_t x,
                                                 int32_t y, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, int ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, int ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
// D[tmem of both CTAs] (+)= A[smem, both] * B[smem, both]^T, kind::f16, M = 256
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// arrive on the mbarrier at `bar`'s offset in every CTA of `cta_mask` once
// every pair MMA previously issued by this thread completed
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand with 128-byte swizzle:
// rows of 128 B, 8-row core groups 1024 B apart (SBO = 64 x 16 B), LBO field 1,
// descriptor version 1 (bits 46-47), layout type 2 = SWIZZLE_128B (bits 61-63).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A bf16 (7-9 = 1),
// B bf16 (10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A and B signed
// 8-bit (bits 7-9 = 1, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at 24.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int* err,
                                        volatile int* abort) {
  if (*abort) return false;
  if (mbar_wait_bounded(bar, parity, err)) return true;
  *abort = 1;
  return false;
}

// 16-byte shared load the compiler may not merge with an earlier one (keeping
// 32 row terms live between two loops of the epilogue would spill).
__device__ __forceinline__ float4 lds4(const float* p) {
  float4 r;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "r"(smem_u32(p)));
  return r;
}

// Approximate distance from the bf16 dot v (rows are pre-normalised for
// cosine, so no per-row factor remains); one expression shared by the dense
// and the filtered pass so both produce the same value for a pair.
__device__ __forceinline__ float approx_distance(float alpha, float gamma, float beta, float v) {
  return (alpha + beta) - gamma * v;
}


__device__ __forceinline__ int kth_bin(float v, float lo, float scale) {
  return min(2047, max(0, static_cast<int>((v - lo) * scale)));
}

// k-th smallest of n finite values (counting repeats), by `nthreads` threads
// (thread ids 0..nthreads-1) that meet at `sync`.  Each level takes the values still in play, reduces their min and
// max, builds a 2048-bin linear histogram over [min, max] (the bin is a
// monotone function of the value, so order is preserved) and scans to the bin
// holding the k-th value.  A bin of at most 1024 values is sorted exactly;
// a larger one becomes the set in play of the next level (membership = the
// same bin at every earlier level).  Equal min and max end the search.  The
// result is exact, or after four levels an upper bound (see below).
template <typename Get, typename Sync>
__device__ float block_kth_smallest(Get get, int64_t n, int k, KthSmem& S, int tid, int nthreads,
                                    Sync sync) {
  const int nw = nthreads >> 5;
  const float inf = __int_as_float(0x7F800000);
  uint32_t kk = static_cast<uint32_t>(k);
  // only finite values take part (+inf marks an empty sample slot); with
  // fewer than k of them the result is +inf
  auto member = [&](float v, int level) {
    if (!(v < inf) || !(v > -inf)) return false;
    for (int l = 0; l < level; ++l)
      if (kth_bin(v, S.lo[l], S.scale[l]) != S.sel[l]) return false;
    return true;
  };
  for (int level = 0; level < 4; ++level) {
    float lo = inf, hi = -inf;
    uint32_t nfin = 0;
    for (int64_t i = tid; i < n; i += nthreads) {
      const float v = get(i);
      if (member(v, level)) {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
        ++nfin;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xFFFFFFFFu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xFFFFFFFFu, hi, o));
      nfin += __shfl_xor_sync(0xFFFFFFFFu, nfin, o);
    }
    if ((tid & 31) == 0) {
      S.red[tid >> 5] = lo;
      S.red[32 + (tid >> 5)] = hi;
      S.wsum[tid >> 5] = nfin;
    }
    sync();
    if (tid == 0) {
      for (int w = 1; w < nw; ++w) {
        S.red[0] = fminf(S.red[0], S.red[w]);
        S.red[32] = fmaxf(S.red[32], S.red[32 + w]);
        S.wsum[0] += S.wsum[w];
      }
    }
    sync();
    lo = S.red[0];
    hi = S.red[32];
    const uint32_t total = S.wsum[0];
    sync();
    if (total < kk) return inf;  // (level 0 only: deeper levels hold >= kk)
    if (!(hi > lo)) return lo;   // every value in play is equal
    const float scale = 2047.0f / (hi - lo);
    for (int i = tid; i < 2048; i += nthreads) S.hist[i] = 0;
    sync();
    for (int64_t i = tid; i < n; i += nthreads) {
      const float v = get(i);
      if (member(v, level)) atomicAdd(&S.hist[kth_bin(v, lo, scale)], 1u);
    }
    sync();
    {
      // bin of the kk-th value: each thread sums a run of bins, a block-wide
      // exclusive scan of the runs locates the crossing, whose owner scans it
      const int per = 2048 / nthreads;
      uint32_t run = 0;
      for (int j = 0; j < per; ++j) run += S.hist[tid * per + j];
      uint32_t inc = run;
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if ((tid & 31) >= o) inc += y;
      }
      if ((tid & 31) == 31) S.wsum[tid >> 5] = inc;
      sync();
      uint32_t before = 0;
      for (int w = 0; w < (tid >> 5); ++w) before += S.wsum[w];
      const uint32_t excl = before + inc - run;
      if (excl < kk && excl + run >= kk) {
        uint32_t cum = excl;
        int b = tid * per;
        for (int j = 0; j < per - 1; ++j, ++b) {
          if (cum + S.hist[b] >= kk) break;
          cum += S.hist[b];
        }
        S.lo[level] = lo;
        S.scale[level] = scale;
        S.sel[level] = b;
        S.sh[1] = kk - cum;
        S.sh[2] = S.hist[b];
        S.sh[3] = 0;
      }
      sync();
    }
    kk = S.sh[1];
    const uint32_t cnt = S.sh[2];
    // four levels without isolating 1024 values (only for value sets of
    // extreme dynamic range): the largest value in play bounds the k-th from
    // above, which both callers accept (a looser threshold, a wider band)
    if (cnt > 1024 && level == 3) return hi;
    if (cnt <= 1024) {
      for (int64_t i = tid; i < n; i += nthreads) {
        const float v = get(i);
        if (member(v, level + 1)) {
          const uint32_t at = atomicAdd(&S.sh[3], 1u);
          if (at < 1024) S.list[at] = v;
        }
      }
      sync();
      const int c = static_cast<int>(min(cnt, 1024u));
      int m = 1;
      while (m < c) m <<= 1;
      for (int i = c + tid; i < m; i += nthreads) S.list[i] = __int_as_float(0x7F800000);
      sync();
      for (int a = 2; a <= m; a <<= 1) {
        for (int j = a >> 1; j > 0; j >>= 1) {
          for (int i = tid; i < m; i += nthreads) {
            const int ixj = i ^ j;
            if (ixj > i) {
              const float x = S.list[i], y = S.list[ixj];
              const bool up = (i & a) == 0;
              if ((x > y) == up) {
                S.list[i] = y;
                S.list[ixj] = x;
              }
            }
          }
          sync();
        }
      }
      const float r = S.list[min(kk, static_cast<uint32_t>(c)) - 1];
      sync();
      return r;
    }
  }
  return 0.0f;  // not reached
}


// 16-byte global -> shared copy without a register round trip (cp.async);
// cp_async_wait_all waits for every copy the thread issued.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// Ascending sort of 32 floats, one per lane, by shuffles (bitonic network).
__device__ __forceinline__ float warp_sort32_f(float x, int lane) {
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const float y = __shfl_xor_sync(0xFFFFFFFFu, x, stride);
      const bool up = (lane & size) == 0;
      const bool lower = (lane & stride) == 0;
      x = (lower == up) ? fminf(x, y) : fmaxf(x, y);
    }
  }
  return x;
}

// k-th smallest of n finite values (counting repeats) by one warp, with the
// levels of block_kth_smallest at warp scale: the values in play (finite, and
// in the selected bin of every earlier level) are reduced to their min and
// max, binned into 256 linear bins over [min, max] (distances of one search
// spread over the bins, so the shared atomics rarely collide), and the bin of
// the k-th value becomes the set in play of the next level.  At most 32
// values in play are gathered and sorted by shuffles.  Equal min and max end
// the search; after four levels without isolating 32 values (extreme dynamic
// range only) the largest value in play bounds the k-th from above, which the
// callers accept as block_kth_smallest's.  Non-finite values take no part;
// with fewer than k finite values the result is +inf.  `hist` is the warp's
// own 256 words of shared memory; no block barrier.
template <typename Get>
__device__ float warp_kth_smallest(Get get, int64_t n, int k, uint32_t* hist, int lane) {
  const float inf = __int_as_float(0x7F800000);
  float lo_at[4], sc_at[4];
  int sel_at[4];
  uint32_t kk = static_cast<uint32_t>(k);
  auto member = [&](float v, int level) {
    if (!(fabsf(v) < inf)) return false;
#pragma unroll
    for (int l = 0; l < 4; ++l)
      if (l < level && min(255, max(0, static_cast<int>((v - lo_at[l]) * sc_at[l]))) != sel_at[l])
        return false;
    return true;
  };
#pragma unroll
  for (int level = 0; level < 4; ++level) {
    float lo = inf, hi = -inf;
    uint32_t cnt = 0;
    for (int64_t i = lane; i < n; i += 32) {
      const float v = get(i);
      if (member(v, level)) {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
        ++cnt;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xFFFFFFFFu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xFFFFFFFFu, hi, o));
      cnt += __shfl_xor_sync(0xFFFFFFFFu, cnt, o);
    }
    if (cnt < kk) return inf;  // (level 0 only: deeper levels hold >= kk)
    if (!(hi > lo)) return lo;  // every value in play is equal
    if (cnt <= 32) {
      // gather the values in play (ballot compaction) and sort them
      float* list = reinterpret_cast<float*>(hist);
      uint32_t at = 0;
      for (int64_t i0 = 0; i0 < n; i0 += 32) {
        const int64_t i = i0 + lane;
        const float v = i < n ? get(i) : inf;
        const bool m = i < n && member(v, level);
        const unsigned bal = __ballot_sync(0xFFFFFFFFu, m);
        if (m) list[at + __popc(bal & ((1u << lane) - 1u))] = v;
        at += __popc(bal);
      }
      __syncwarp();
      const float x = warp_sort32_f(lane < static_cast<int>(cnt) ? list[lane] : inf, lane);
      __syncwarp();
      return __shfl_sync(0xFFFFFFFFu, x, static_cast<int>(kk) - 1);
    }
    if (level == 3) return hi;
    const float scale = 255.0f / (hi - lo);
#pragma unroll
    for (int j = lane; j < 256; j += 32) hist[j] = 0u;
    __syncwarp();
    for (int64_t i = lane; i < n; i += 32) {
      const float v = get(i);
      if (member(v, level))
        atomicAdd(&hist[min(255, max(0, static_cast<int>((v - lo) * scale)))], 1u);
    }
    __syncwarp();
    // bin of the kk-th value: lane l sums bins 8l..8l+7, an inclusive scan
    // over the lanes finds the crossing, its owner walks its bins
    uint32_t c[8], s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      c[j] = hist[lane * 8 + j];
      s += c[j];
    }
    uint32_t inc = s;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, inc, o);
      if (lane >= o) inc += y;
    }
    const uint32_t excl = inc - s;
    const bool mine = excl < kk && kk <= inc;
    const int owner = __ffs(__ballot_sync(0xFFFFFFFFu, mine)) - 1;
    int d = 0;
    uint32_t before = excl;
    if (mine) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (before + c[j] >= kk) {
          d = lane * 8 + j;
          break;
        }
        before += c[j];
      }
    }
    d = __shfl_sync(0xFFFFFFFFu, d, owner);
    before = __shfl_sync(0xFFFFFFFFu, before, owner);
    lo_at[level] = lo;
    sc_at[level] = scale;
    sel_at[level] = d;
    kk -= before;
    __syncwarp();
  }
  return inf;  // not reached
}

// k-th smallest of n values (counting repeats) by one warp for k <= K:
// every lane keeps the K smallest finite values of its strided share sorted
// in registers (a value below the lane's largest kept one is inserted by a
// compare-exchange chain), then k rounds of a warp-wide minimum over the
// lanes' smallest kept values pop one value each (the lowest lane holding the
// minimum pops); the k-th popped value is the answer.  A lane contributes at
// most k of the k smallest, so K kept values per lane suffice.  Exact, with
// no shared memory and no barrier; non-finite values take no part (+inf when
// fewer than k are finite), as in warp_kth_smallest.
constexpr int kSmallK = 16;  // k up to which the register selection is used

template <int K, typename Get>
__device__ float warp_kth_small(Get get, int64_t n, int k, int lane) {
  const float inf = __int_as_float(0x7F800000);
  float a[K];
#pragma unroll
  for (int j = 0; j < K; ++j) a[j] = inf;
  for (int64_t i = lane; i < n; i += 32) {
    float x = get(i);
    if (!(fabsf(x) < inf) || !(x < a[K - 1])) continue;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const float lo = fminf(a[j], x);
      x = fmaxf(a[j], x);
      a[j] = lo;
    }
  }
  float res = inf;
  for (int r = 0; r < k; ++r) {
    float m = a[0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fminf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
    if (!(m < inf)) return inf;  // fewer than k finite values (warp-uniform)
    const int w = __ffs(__ballot_sync(0xFFFFFFFFu, a[0] == m)) - 1;
    if (lane == w) {
#pragma unroll
      for (int j = 0; j < K - 1; ++j) a[j] = a[j + 1];
      a[K - 1] = inf;
    }
    res = m;
  }
  return res;
}

// Filter threshold of one query from the k-th smallest sampled value `kth`
// (+inf when the sample holds fewer than k values): t = kth + 2 eps (rounded
// up) and the score-domain constant c.  With d~ = alpha + beta - gamma v the
// filter keeps x = v - beta/gamma >= c = (alpha - t)/gamma (beta = 0 for
// cosine / IP; alpha = 1 for cosine, 0 for IP), lowered by a margin far above
// the rounding of either side, so the kept set contains every row with
// d~ <= t (a few extra rows are harmless).  "Keep everything" is -FLT_MAX,
// not -inf: padding rows carry x = -inf.
__device__ __forceinline__ void threshold_from_kth(float kth, float eps, float alpha, float gamma,
                                                   float scale, float* t_out, float* c_out) {
  const float inf = __int_as_float(0x7F800000);
  float t = inf;
  if (kth != inf) {
    // same rounding-safe widening as the band in tc_rerank_kernel, so that
    // band <= thr whenever T_k <= the sample's k-th distance
    t = kth + 2.0f * eps;
    t = t + fabsf(t) * 1e-6f;
  }
  const float keep_all = -3.40282347e+38f;
  float c;
  if (t == inf) {
    c = keep_all;
  } else if (gamma > 0.0f) {
    c = (alpha - t) / gamma;
  } else {
    c = alpha <= t ? keep_all : inf;
  }
  if (c != inf && c != keep_all) c = fmaxf(c - (fabsf(c) + scale) * 6.103515625e-05f, keep_all);
  *t_out = t;
  *c_out = c;
}

// Fused sampling, between the two grid barriers: the thresholds of the
// queries qb*128 + l, l = grp, grp + groups, ... (this block's share of its
// query block), from the sample minima all blocks wrote.  The 512 epilogue
// threads (`et`) meet at named barrier 1.  Out of line, so that its registers
// do not weigh on the epilogue's main loop.
__device__ __noinline__ void fused_thresholds(const float* samp, int64_t samp_ld, int32_t k,
                                              int64_t nq, int64_t gstep, const float* eps,
                                              const float* alpha, const float* gamma,
                                              const float* scale, float* thr_out, float* c_out,
                                              KthSmem* ks, int et, int64_t qb, int64_t grp) {
  for (int64_t l = grp; l < kQM; l += gstep) {
    const int64_t qq = qb * kQM + l;
    if (qq >= nq) break;
    const float* vals = samp + qq * samp_ld;
    float kth = __int_as_float(0x7F800000);
    if (samp_ld >= k)
      kth = block_kth_smallest([&](int64_t i) { return __ldcg(vals + i); }, samp_ld, k, *ks, et,
                               kEpiWarps * 32, [] { named_sync(1, kEpiWarps * 32); });
    if (et == 0)
      threshold_from_kth(kth, eps[qq], alpha[qq], gamma[qq], scale[qq], thr_out + qq, c_out + qq);
  }
}

// Per-query terms of the tensor-core pass from the query's sums (double):
// |q|^2 (nq2), |q - q'|^2 (nres), |q'|^2 (nt) for the rounded query q', its
// scale qs (int8; 1 for bf16) and the exact path's sequential fp32 |q|^2
// (acc): the affine map d~ = alpha + beta - gamma s, the certified bound eps of
// |d~ - d| and the magnitude bound `scale` of the score-domain value.
struct QueryTerms {
  float qn, alpha, gamma, eps, scale;
};

__device__ __forceinline__ QueryTerms query_terms(const TcCorpusStats& cs, int metric, int dim,
                                                  float acc, double nq2, double nres, double nt,
                                                  double qs) {
  const double qnorm = sqrt(nq2), qres = sqrt(nres), qt = sqrt(nt);
  // |dot(q, r) - dot(q', r')| <= |q - q'||r| + |q'||r - r'| plus the fp32
  // accumulation of the tensor core (bf16) and of the exact sequential path:
  // generously dim * 2^-22 of the magnitude sum each.  (For cosine the row
  // terms are relative to |r|.)
  const double cacc = static_cast<double>(dim) * 2.384185791015625e-07;
  const double es = qres * cs.max_norm + qt * cs.max_resid + cacc * qt * cs.max_norm_bf16 +
                    cacc * qnorm * cs.max_norm;
  double alpha = 0.0, gamma = 1.0, lip = 1.0, mag, extra = 0.0;
  if (metric == kL2) {
    // alpha and the row terms are the exact path's own fp32 |q|^2, |r|^2
    alpha = acc;
    gamma = 2.0;
    lip = 2.0;
    mag = acc + cs.max_sqnorm + 2.0 * (qnorm * cs.max_norm + es);
  } else if (metric == kCosine) {
    // the tensor-core dot approximates dot(q, r)/|r| (bf16: rows normalised
    // before rounding; int8: the row factor is u/|r|)
    alpha = 1.0;
    gamma = qnorm > 0.0 ? 1.0 / qnorm : 0.0;
    lip = gamma;
    mag = 1.0 + lip * (qnorm * cs.max_norm + es);
    // the exact path divides by sqrt(fp32 |q|^2 * fp32 |r|^2); each sequential
    // sum of squares is off by at most dim*2^-24 relatively, and |cos| <= 1
    extra = (2.0 * dim + 16.0) * 5.960464477539063e-08;
  } else {
    mag = qnorm * cs.max_norm + es;
  }
  // rounding of both distance formulas (and, for int8, of the row factor and
  // the product with the converted integer dot): 64 ulps of the largest magnitude
  const double slack = mag * 64.0 * 5.960464477539063e-08 + extra + 1e-30;
  QueryTerms t;
  t.qn = acc;
  t.alpha = static_cast<float>(alpha);
  // the integer dot counts in units of the query scale
  t.gamma = static_cast<float>(gamma * qs);
  t.eps = static_cast<float>((lip * es + slack) * (1.0 + 1e-6));
  // magnitude bound of the score-domain value x = v - beta / gamma
  double sc = qt / qs * cs.max_norm_bf16;
  if (metric == kL2) sc += cs.max_sqnorm / (gamma * qs);
  t.scale = static_cast<float>(sc);
  return t;
}

// Epilogue variants: the dense sample pass, the filter on the raw dot
// (cosine on normalised rows, IP) and the filter with a per-row bias (L2).
enum TcMode : int { kDense = 0, kFilterPlain = 1, kFilterBias = 2 };

// I8: signed 8-bit codes with a per-row factor (TcParams::row_w) instead of
// bf16 rows; the s32 accumulator is converted and scaled in the epilogue.
// PAIR: the filtered pass as CTA pairs (clusters of two): the pair holds two
// query blocks (256 queries, one per CTA, resident), each CTA streams its
// half of every 256-row tile (`map_r` with 128-row boxes), the leader issues
// the M = 256 MMAs, and each CTA's epilogue reads its own queries' scores
// for all 256 rows.  Each CTA then feeds half the row bytes per MMA, so its
// stage ring covers twice the load latency.  Requires `groups` > 0.
template <int MODE, bool I8, bool FUSED = false, bool PAIR = false>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_scan_kernel(const __grid_constant__ CUtensorMap map_q,
                   const __grid_constant__ CUtensorMap map_r, const TcParams p) {
  static_assert(!PAIR || (!I8 && !FUSED && MODE != kDense), "pairs run the bf16 filtered pass");
  // no per-row terms and no fused sampling: the lean layout (more stages)
  constexpr bool kLean = MODE == kFilterPlain && !I8 && !FUSED && !PAIR;
  extern __shared__ uint8_t smem_raw[];
  const TcLayout L = tc_layout(tc_kblocks(p.dim, I8), p.stream_queries, PAIR, kLean);
  uint8_t* base =
      reinterpret_cast<uint8_t*>((reinterpret_cast<size_t>(smem_raw) + 1023) / 1024 * 1024);
  uint8_t* qres = base;                  // resident query block (nk x 16 KiB)
  uint8_t* stages = base + L.a_bytes;    // ring of (rows [| queries]) stages
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.bar_off);
  uint64_t* empty = full + L.stages;
  uint64_t* acc_full = empty + L.stages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* a_full = acc_empty + 2;
  uint64_t* a_empty = a_full + 1;
  uint64_t* drain = a_empty + 1;
  uint64_t* rt_full = drain + 1;
  uint64_t* rt_empty = rt_full + kRtSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rt_empty + kRtSlots);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // per tile: [kRN] row factor of the integer dot (int8), [kRN] |r|^2 (L2)
  float* rowpar = reinterpret_cast<float*>(base + L.rt_off);
  // Per-row terms come with the tile: the producer bulk-copies them into the
  // ring slot of virtual unit v (v % kRtSlots), the epilogue warps release it.
  constexpr bool kRowTerms = I8 || MODE == kFilterBias || MODE == kDense;
  const bool row_terms = kRowTerms && (I8 || p.row_beta != nullptr);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nk = L.nk;
  constexpr int kKElems = I8 ? 128 : kBK;  // elements per 128-byte k-block (TMA x step)
  const int64_t rtiles = (p.rows + kRN - 1) / kRN;
  const int64_t units = rtiles * p.qblocks;
  // Work split.  With `groups` > 0 block c owns query block c % qblocks and
  // the row tiles of group c / qblocks: the qblocks blocks of a group walk
  // the same rows in step, so each row tile comes from HBM once and from L2
  // for the others.  Otherwise blocks take contiguous query-block-major
  // ranges of (query block, row tile) units.
  // Pairs: pair c / 2 owns query blocks 2 s and 2 s + 1 (s = pair % pair
  // superblocks; CTA rank r takes block 2 s + r, which may lie past the last
  // block: zero queries, no results) and the row tiles of group pair / s.
  const uint32_t crank = PAIR ? cluster_rank() : 0u;
  int64_t u_begin, u_end;
  if (PAIR) {
    const int64_t qsb = (p.qblocks + 1) / 2;
    const int64_t pr = blockIdx.x / 2;
    const int64_t qb = 2 * (pr % qsb) + crank;
    const int64_t g = pr / qsb;
    u_begin = qb * rtiles + rtiles * g / p.groups;
    u_end = qb * rtiles + rtiles * (g + 1) / p.groups;
  } else if (FUSED && p.pool) {
    u_begin = blockIdx.x * p.static_tiles;
    u_end = u_begin + p.static_tiles;
  } else if (p.groups > 0) {
    const int64_t qb = blockIdx.x % p.qblocks;
    const int64_t g = blockIdx.x / p.qblocks;
    u_begin = qb * rtiles + rtiles * g / p.groups;
    u_end = qb * rtiles + rtiles * (g + 1) / p.groups;
  } else {
    u_begin = units * blockIdx.x / gridDim.x;
    u_end = units * (blockIdx.x + 1) / gridDim.x;
  }
  // Fused sampling: the block's first s_c units run twice, first as the
  // sample, then again with the filter (virtual unit v -> unit_of(v)).
  const int64_t nown = u_end - u_begin;
  const int64_t s_c =
      FUSED ? (nown < p.sample_tiles ? nown : static_cast<int64_t>(p.sample_tiles)) : 0;
  const int64_t nvirt = s_c + nown;
  auto unit_of = [&](int64_t v) { return u_begin + (v < s_c ? v : v - s_c); };
  // Dynamic tail: virtual units from nvirt on come from the pool, in the
  // order this block's producer claimed them (slot (v - nvirt) % 16 of the
  // ring, phase ((v - nvirt) / 16) & 1).  The producer runs at most a few
  // units ahead of the epilogue (two accumulators and a ring of less than two
  // tiles), so a slot is read by both consumers before it is written again.
  const bool dyn = FUSED && p.pool != nullptr;
  KthSmem* kss = reinterpret_cast<KthSmem*>(base + L.kth_off);


  if (tid == 0) {
    for (int s = 0; s < L.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    if (dyn)
      for (int s = 0; s < 16; ++s) mbar_init(&kss->ufull[s], 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      // pairs: both CTAs' epilogue warps release the leader's accumulator
      mbar_init(&acc_empty[b], PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    mbar_init(drain, 1);
    for (int r = 0; r < kRtSlots; ++r) {
      mbar_init(&rt_full[r], 1);
      mbar_init(&rt_empty[r], kEpiWarps);
    }
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  if (tid == 64) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_r);
  }
  tc_fence_before();
  __syncthreads();
  // pairs: the peer's barriers are initialised before any copy or arrival
  // reaches them
  if (PAIR) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // launched while the query prep (or the sample pass) may still run: the
  // barriers and TMEM are set up; wait for its queries, bounds and counters
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      int64_t cur_qb = -1;
      uint32_t a_round = 0;
      int64_t issued = 0;
      int64_t rt_issued = 0;
      bool a_pending = false;
      // the claim of the next pool tile is issued one unit ahead, so its
      // round trip overlaps the current unit's copies
      unsigned long long claim = dyn ? atomicAdd(p.pool, 1ull) : 0ull;
      for (int64_t v = 0; (v < nvirt || dyn) && !*abort; ++v) {
        int64_t u;
        if (v < nvirt) {
          u = unit_of(v);
        } else {
          const int64_t t = static_cast<int64_t>(claim);
          u = t < p.pool_tiles ? p.pool_first + t : -1;
          const int slot = static_cast<int>((v - nvirt) % 16);
          kss->uq[slot] = u;
          mbar_arrive(&kss->ufull[slot]);
          if (u < 0) break;
          claim = atomicAdd(p.pool, 1ull);
        }
        const int64_t qb = u / rtiles;
        const int64_t rt = u - qb * rtiles;
        if (L.resident && qb != cur_qb) {
          // refill the resident query block once the MMAs on the old one finished
          if (cur_qb >= 0 && !tc_wait(a_empty, (a_round - 1) & 1u, p.err, abort)) break;
          if (PAIR) {
            // both halves complete on the leader's barrier (loaded once: pairs
            // keep their query blocks for the whole pass)
            if (crank == 0) mbar_arrive_expect_tx(a_full, static_cast<uint32_t>(2 * nk * kQBytes));
            const uint32_t lead = map_to_rank(a_full, 0);
            for (int kb = 0; kb < nk; ++kb)
              tma_load_2d_pair(qres + kb * kQBytes, &map_q, kb * kKElems,
                               static_cast<int32_t>(qb * kQM), lead);
          } else {
            mbar_arrive_expect_tx(a_full, static_cast<uint32_t>(nk * kQBytes));
            for (int kb = 0; kb < nk; ++kb)
              tma_load_2d(qres + kb * kQBytes, &map_q, kb * kKElems, static_cast<int32_t>(qb * kQM),
                          a_full);
          }
          a_pending = true;
          cur_qb = qb;
          ++a_round;
        }
        const int32_t y = static_cast<int32_t>(p.row0 + rt * kRN);
        if (row_terms) {
          const int r = static_cast<int>(v % kRtSlots);
          if (!tc_wait(&rt_empty[r], static_cast<uint32_t>((v / kRtSlots) & 1) ^ 1u, p.err, abort))
            break;
          // rows of the tile rounded up to 16 bytes: the arrays are allocated
          // in multiples of 64 floats, and rows past the pass are masked
          const int64_t left = p.rows - rt * kRN;
          const uint32_t bytes =
              static_cast<uint32_t>(((left < kRN ? left : kRN) + 3) / 4 * 16);
          float* slot = rowpar + r * 2 * kRN;
          mbar_arrive_expect_tx(&rt_full[r], bytes * ((I8 ? 1u : 0u) + (p.row_beta ? 1u : 0u)));
          if (I8) bulk_load(slot, p.row_w + p.row0 + rt * kRN, bytes, &rt_full[r]);
          if (p.row_beta) bulk_load(slot + kRN, p.row_beta + p.row0 + rt * kRN, bytes, &rt_full[r]);
          rt_issued = v + 1;
        }
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!tc_wait(&empty[stage], phase ^ 1u, p.err, abort)) {
            ok = false;
            break;
          }
          uint8_t* st = stages + stage * L.stage_bytes;
          if (PAIR) {
            // this CTA's 128 rows of the tile, completing on the leader's barrier
            if (crank == 0)
              mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(2 * L.stage_bytes));
            tma_load_2d_pair(st, &map_r, kb * kKElems, y + static_cast<int32_t>(crank) * (kRN / 2),
                             map_to_rank(&full[stage], 0));
          } else {
            mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(L.stage_bytes));
            tma_load_2d(st, &map_r, kb * kKElems, y, &full[stage]);
            if (!L.resident)
              tma_load_2d(st + kRBytes, &map_q, kb * kKElems, static_cast<int32_t>(qb * kQM),
                          &full[stage]);
          }
          ++issued;
          if (++stage == L.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
      // after an abort, wait (bounded) for the copies still in flight
      if (PAIR && *abort) {
        // a pair's stage and query copies complete on the leader's barriers,
        // which this CTA cannot wait on: give them a bounded moment to land
        const unsigned long long t0 = global_ns();
        while (global_ns() - t0 < 200000ull) {
        }
      } else if (*abort) {
        for (int64_t i = issued > L.stages ? issued - L.stages : 0; i < issued; ++i)
          mbar_wait_bounded(&full[i % L.stages], static_cast<uint32_t>((i / L.stages) & 1), nullptr);
        if (a_pending) mbar_wait_bounded(a_full, (a_round - 1) & 1u, nullptr);
        for (int64_t i = rt_issued > kRtSlots ? rt_issued - kRtSlots : 0; i < rt_issued; ++i)
          mbar_wait_bounded(&rt_full[i % kRtSlots], static_cast<uint32_t>((i / kRtSlots) & 1),
                            nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && crank == 0) {
      // ---------------- MMA issuer (a pair's leader alone) ----------------
      const uint32_t idesc =
          I8 ? idesc_i8(kQM, kRN) : idesc_bf16(PAIR ? 2 * kQM : kQM, kRN);
      int stage = 0;
      uint32_t phase = 0;
      int64_t cur_qb = -1;
      uint32_t a_round = 0;
      int local = 0;
      for (int64_t v = 0; (v < nvirt || dyn) && !*abort; ++v, ++local) {
        int64_t u;
        if (v < nvirt) {
          u = unit_of(v);
        } else {
          const int slot = static_cast<int>((v - nvirt) % 16);
          if (!tc_wait(&kss->ufull[slot], static_cast<uint32_t>(((v - nvirt) / 16) & 1), p.err,
                       abort))
            break;
          u = kss->uq[slot];
          if (u < 0) break;
        }
        const int64_t qb = u / rtiles;
        if (L.resident && qb != cur_qb) {
          // old query block free once prior MMAs finish (pairs keep theirs)
          if constexpr (!PAIR) {
            if (cur_qb >= 0) tc_commit(a_empty);
          }
          if (!tc_wait(a_full, a_round & 1u, p.err, abort)) break;
          cur_qb = qb;
          ++a_round;
        }
        const int b = local & 1;
        const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
        if (!tc_wait(&acc_empty[b], acc_phase ^ 1u, p.err, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(b * kRN);
        bool ok = true;
        for (int kb = 0; kb < nk; ++kb) {
          if (!tc_wait(&full[stage], phase, p.err, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sr = smem_u32(stages + stage * L.stage_bytes);
          const uint32_t sq = L.resident ? smem_u32(qres + kb * kQBytes) : sr + kRBytes;
          const uint64_t adesc = smem_desc_sw128(sq);
          const uint64_t bdesc = smem_desc_sw128(sr);
          // four MMAs of 32 bytes of K per 128-byte stage (16 bf16 / 32 int8)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            if constexpr (PAIR)
              tc_mma_pair(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
            else if constexpr (I8)
              tc_mma_i8(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
            else
              tc_mma(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
          }
          // frees the smem stage (of both CTAs of a pair) once these MMAs finish
          if constexpr (PAIR)
            tc_commit_pair(&empty[stage], 3);
          else
            tc_commit(&empty[stage]);
          if (++stage == L.stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        // accumulator ready for the epilogue (of both CTAs of a pair)
        if constexpr (PAIR)
          tc_commit_pair(&acc_full[b], 3);
        else
          tc_commit(&acc_full[b]);
      }
      // every MMA issued by this thread has completed once `drain` flips
      if constexpr (PAIR)
        tc_commit_pair(drain, 1);
      else
        tc_commit(drain);
      mbar_wait_bounded(drain, 0, nullptr);
    }
  } else if (warp >= 4) {
    // ---------------- epilogue: TMEM -> candidates / distances ----------------
    // Thread = one query (TMEM lane) over a quarter of the tile's 256 rows
    // (four warps per TMEM lane quarter).  With per-row terms (L2) the sixteen
    // warps stage them and meet at a named barrier every tile, so they must not
    // poll the abort flag; they all stop when their bounded accumulator wait
    // gives up.
    const int ew = warp - 4;
    const int quarter = warp & 3;
    const int part = ew >> 2;          // columns part*64 .. +63
    const int et = tid - 128;          // 0..511
    int local = 0;
    int64_t cur_qb = -1;
    float alpha = 0.0f, gamma = 0.0f, hq = 0.0f, cq = __int_as_float(0x7F800000);
    int64_t q = 0;
    bool qvalid = false;
    const int64_t grp = p.groups > 0 ? blockIdx.x / p.qblocks : 0;
    KthSmem* ks = reinterpret_cast<KthSmem*>(base + L.kth_off);
    volatile int* bar_ok = reinterpret_cast<volatile int*>(&ks->sh[0]);
    bool synced = !FUSED;
    // Candidate slots: a thread reserves p.cand_reserve slots of its query's
    // list at a time (one returning atomic, an L2 round trip that stalls the
    // warp) and fills them without atomics; slots it does not use are padded
    // with kKeyMax, whose NaN distance the re-rank skips.  One atomic per
    // passing row bounded the batched pass at ~2 round trips per warp and tile.
    int rbase = 0, rleft = 0;
    uint64_t* cdst = nullptr;
    auto cand_pad = [&]() {
      for (int i = 0; i < rleft; ++i)
        if (rbase + i < p.cand_cap) cdst[rbase + i] = kKeyMax;
      rleft = 0;
    };
    // grid barrier n (1 or 2) of this call: arrive, then wait (bounded)
    auto grid_barrier = [&](unsigned long long n) -> bool {
      named_sync(1, kEpiWarps * 32);
      if (et == 0) {
        __threadfence();
        atomicAdd(p.bar, 1ull);
        const unsigned long long target = p.bar_base + n * gridDim.x;
        const unsigned long long t0 = global_ns();
        int ok = 1;
        for (uint32_t it = 0;; ++it) {
          unsigned long long cur;
          asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(cur) : "l"(p.bar) : "memory");
          if (cur >= target) break;
          if ((it & 63u) == 63u && global_ns() - t0 > kWaitLimitNs) {
            atomicExch(p.err, kErrTimeout);
            ok = 0;
            break;
          }
        }
        *bar_ok = ok;
      }
      named_sync(1, kEpiWarps * 32);
      return *bar_ok != 0;
    };
    // after the sample tiles: thresholds of this block's share of its query
    // block's queries (query qb*128 + l for l = grp, grp + groups, ...), then
    // every block reads its queries' constants
    // A single query: every block derives its threshold from the sample
    // itself (the same inputs and steps in every block, so the same value,
    // which every block also stores for the re-rank), and the second barrier
    // is only arrived at, keeping the counter's per-call advance.
    auto fused_sync = [&](int64_t qb) -> bool {
      if (!grid_barrier(1)) return false;
      if (p.nq == 1) {
        fused_thresholds(p.samp_out, p.samp_ld, p.k, p.nq, 1, p.q_eps, p.q_alpha, p.q_gamma,
                         p.q_scale, p.thr_out, p.c_out, ks, et, qb, 0);
        named_sync(1, kEpiWarps * 32);  // thread 0's stores of thr / c are seen by the block
        if (et == 0) atomicAdd(p.bar, 1ull);
      } else {
        fused_thresholds(p.samp_out, p.samp_ld, p.k, p.nq, p.groups > 0 ? p.groups : 1, p.q_eps,
                         p.q_alpha, p.q_gamma, p.q_scale, p.thr_out, p.c_out, ks, et, qb, grp);
        if (!grid_barrier(2)) return false;
      }
      cq = qvalid ? __ldcg(p.c_out + q) : __int_as_float(0x7F800000);
      return true;
    };
    for (int64_t vu = 0; vu < nvirt || dyn; ++vu, ++local) {
      int64_t u;
      if (vu < nvirt) {
        u = unit_of(vu);
      } else {
        const int slot = static_cast<int>((vu - nvirt) % 16);
        if (!mbar_wait_bounded(&kss->ufull[slot], static_cast<uint32_t>(((vu - nvirt) / 16) & 1),
                               p.err)) {
          *abort = 1;
          break;
        }
        u = kss->uq[slot];
        if (u < 0) break;
      }
      const int64_t qb = u / rtiles;
      const int64_t rt = u - qb * rtiles;
      if (qb != cur_qb) {
        cand_pad();  // the reserved slots belong to the previous query
        cur_qb = qb;
        q = qb * kQM + quarter * 32 + lane;
        cdst = p.cand + q * p.cand_cap;
        qvalid = q < p.nq;
        alpha = qvalid ? p.q_alpha[q] : 0.0f;
        gamma = qvalid ? p.q_gamma[q] : 0.0f;
        hq = gamma > 0.0f ? 1.0f / gamma : 0.0f;
        cq = (qvalid && MODE != kDense && synced) ? p.q_c[q] : __int_as_float(0x7F800000);
        if (FUSED && !synced && qvalid) {
          // sample slots this block has no tile for stay +inf
          for (int64_t w = s_c; w < p.sample_tiles; ++w)
            for (int c = 0; c < 2; ++c)
              p.samp_out[q * p.samp_ld + (grp * p.sample_tiles + w) * 8 + part * 2 + c] =
                  __int_as_float(0x7F800000);
        }
      }
      const bool sampling = FUSED && vu < s_c;
      if (FUSED && !synced && !sampling) {
        synced = true;
        if (!fused_sync(qb)) {
          *abort = 1;
          break;
        }
      }
      const int b = local & 1;
      const uint32_t acc_phase = static_cast<uint32_t>((local >> 1) & 1);
      const int rslot = static_cast<int>(vu % kRtSlots);
      const float* rp = rowpar + rslot * 2 * kRN;
      if (row_terms &&
          !mbar_wait_bounded(&rt_full[rslot], static_cast<uint32_t>((vu / kRtSlots) & 1), p.err)) {
        *abort = 1;
        break;
      }
      if (!mbar_wait_bounded(&acc_full[b], acc_phase, p.err)) {
        *abort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) +
                             static_cast<uint32_t>(b * kRN + part * 64);
      const int64_t lrow0 = rt * kRN + part * 64;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float v[32];
        tmem_ld32(taddr + c * 32, v);
        const int j0 = part * 64 + c * 32;
        if (I8) {
          // s32 dot x row factor, four factors per 16-byte shared load
          const float4* w4 = reinterpret_cast<const float4*>(rp + j0);
#pragma unroll
          for (int t4 = 0; t4 < 8; ++t4) {
            const float4 w = w4[t4];
            v[4 * t4] = __int2float_rn(__float_as_int(v[4 * t4])) * w.x;
            v[4 * t4 + 1] = __int2float_rn(__float_as_int(v[4 * t4 + 1])) * w.y;
            v[4 * t4 + 2] = __int2float_rn(__float_as_int(v[4 * t4 + 2])) * w.z;
            v[4 * t4 + 3] = __int2float_rn(__float_as_int(v[4 * t4 + 3])) * w.w;
          }
        }
        const int64_t lr = lrow0 + c * 32;
        if (sampling) {
          // fused sample tile: one minimum per 32 rows (as the dense pass below)
          const int64_t rem = p.rows - lr;
          const int tmax = rem >= 32 ? 32 : (rem < 0 ? 0 : static_cast<int>(rem));
          if (qvalid) {
            float m = __int_as_float(0x7F800000);
#pragma unroll
            for (int t = 0; t < 32; ++t)
              if (t < tmax)
                m = fminf(m, approx_distance(alpha, gamma,
                                             p.row_beta ? rp[kRN + j0 + t] : 0.0f, v[t]));
            p.samp_out[q * p.samp_ld + (grp * p.sample_tiles + vu) * 8 + part * 2 + c] = m;
          }
        } else if (MODE == kDense && p.dense_group == 32) {
          // minimum of each 32-row group: the k-th smallest group minimum bounds
          // the sample's k-th smallest distance from above (k distinct rows lie
          // at or below it), at 1/32 of the output
          const int64_t rem = p.rows - lr;
          const int tmax = rem >= 32 ? 32 : (rem < 0 ? 0 : static_cast<int>(rem));
          if (qvalid && tmax > 0) {
            float m = __int_as_float(0x7F800000);
#pragma unroll
            for (int t = 0; t < 32; ++t)
              if (t < tmax)
                m = fminf(m, approx_distance(alpha, gamma,
                                             p.row_beta ? rp[kRN + j0 + t] : 0.0f, v[t]));
            p.dense_out[q * p.dense_ld + (lr >> 5)] = m;
          }
        } else if (MODE == kDense) {
          if (qvalid) {
#pragma unroll
            for (int t = 0; t < 32; t += 4) {
              float o[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                o[i] = approx_distance(alpha, gamma,
                                       p.row_beta ? rp[kRN + j0 + t + i] : 0.0f, v[t + i]);
              if (lr + t + 3 < p.rows) {
                *reinterpret_cast<float4*>(p.dense_out + q * p.dense_ld + lr + t) =
                    make_float4(o[0], o[1], o[2], o[3]);
              } else {
                for (int i = 0; i < 4; ++i)
                  if (lr + t + i < p.rows) p.dense_out[q * p.dense_ld + lr + t + i] = o[i];
              }
            }
          }
        } else {
          // Filtered score of rows 4 t4 .. 4 t4 + 3: v (plain) or v less the
          // row's bias (L2), from one 16-byte shared load of |r|^2 (the same
          // address in every lane: a broadcast).  Recomputed where needed
          // rather than kept beside v, which would cost 32 registers.
          auto score4 = [&](int t4, float* sc) {
            if (MODE != kFilterBias) {
#pragma unroll
              for (int i = 0; i < 4; ++i) sc[i] = v[4 * t4 + i];
            } else {
              const float4 bb = lds4(rp + kRN + j0 + 4 * t4);
              const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
              for (int i = 0; i < 4; ++i)
                sc[i] = I8 ? fmaf(-bv[i], hq, v[4 * t4 + i]) : fmaf(-0.5f, bv[i], v[4 * t4 + i]);
            }
          };
          // only rows of the pass: the tail of the last tile reads zero rows
          const int64_t rem = p.rows - lr;
          const int tmax = rem >= 32 ? 32 : (rem < 0 ? 0 : static_cast<int>(rem));
          float m = -__int_as_float(0x7F800000);
          if (MODE != kFilterBias && tmax == 32) {  // full chunk: no row predicates
#pragma unroll
            for (int t4 = 0; t4 < 8; ++t4) {
              float sc[4];
              score4(t4, sc);
              m = fmaxf(fmaxf(m, fmaxf(sc[0], sc[1])), fmaxf(sc[2], sc[3]));
            }
          } else {
#pragma unroll
            for (int t4 = 0; t4 < 8; ++t4) {
              float sc[4];
              score4(t4, sc);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (4 * t4 + i < tmax) m = fmaxf(m, sc[i]);
            }
          }
          if (__any_sync(0xFFFFFFFFu, m >= cq)) {
            uint32_t pass = 0;
#pragma unroll
            for (int t4 = 0; t4 < 8; ++t4) {
              float sc[4];
              score4(t4, sc);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (4 * t4 + i < tmax && sc[i] >= cq) pass |= 1u << (4 * t4 + i);
            }
            const int np = __popc(pass);
            if (np > rleft) {
              cand_pad();
              rleft = np > p.cand_reserve ? np : p.cand_reserve;
              rbase = atomicAdd(p.cand_count + q, rleft);
            }
            // rows that pass for some lane of the warp: a warp-uniform branch
            // per row keeps the write loop at the cost of the rows found
            const uint32_t wpass = __reduce_or_sync(0xFFFFFFFFu, pass);
            int w = rbase;
#pragma unroll
            for (int t = 0; t < 32; ++t) {
              if (((wpass >> t) & 1u) && ((pass >> t) & 1u)) {
                const float beta = MODE == kFilterBias ? rp[kRN + j0 + t] : 0.0f;
                if (w < p.cand_cap)
                  cdst[w] = make_key(approx_distance(alpha, gamma, beta, v[t]),
                                     static_cast<uint32_t>(p.row0 + lr + t));
                ++w;
              }
            }
            rbase = w;
            rleft -= np;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          mbar_arrive_cluster(map_to_rank(&acc_empty[b], 0));  // the leader issues the MMAs
        else
          mbar_arrive(&acc_empty[b]);
        if (row_terms) mbar_arrive(&rt_empty[rslot]);
      }
    }
    cand_pad();
    // a block whose range held only sample tiles (or none) still takes its
    // part in both grid barriers
    if (FUSED && !synced && !*abort) {
      synced = true;
      if (!fused_sync(cur_qb >= 0 ? cur_qb : static_cast<int64_t>(blockIdx.x % p.qblocks)))
        *abort = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  // pairs: neither CTA leaves (or frees TMEM) while the other may still
  // signal its barriers or the leader's MMAs read its shared memory
  if (PAIR) cluster_sync_all();
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem, kTmemCols);
    else
      tmem_dealloc(tmem, kTmemCols);
  }
}

// fp32 rows -> bf16 rows (round to nearest even), one warp per row.  With
// `normalise` (cosine) each row is first divided by its norm (in double), so
// the tensor-core dot approximates dot(q, r)/|r|.  Per-row error-bound terms
// (double sums, rounded up): |r'|, |r' - bf16(r')|, |bf16(r')| for the row r'
// that is rounded, and |r| rounded down.
__global__ void to_bf16_rows_kernel(const float* __restrict__ rows, int64_t n, int32_t dim,
                                    int64_t ld, __nv_bfloat16* __restrict__ out, int64_t ld16,
                                    float* __restrict__ stats, int normalise) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  double n0 = 0.0;
  for (int c = lane; c < dim; c += 32) {
    const double xx = rows[r * ld + c];
    n0 += xx * xx;
  }
  for (int o = 16; o > 0; o >>= 1) n0 += __shfl_xor_sync(0xFFFFFFFFu, n0, o);
  const double norm = sqrt(n0);
  const double scale = (normalise && norm > 0.0) ? 1.0 / norm : 1.0;
  double nr = 0.0, nres = 0.0, nt = 0.0;
  for (int c = lane; c < ld16; c += 32) {
    const double xx = c < dim ? static_cast<double>(rows[r * ld + c]) * scale : 0.0;
    const __nv_bfloat16 b = __double2bfloat16(xx);
    out[r * ld16 + c] = b;
    const double xb = static_cast<double>(__bfloat162float(b));
    nr += xx * xx;
    nres += (xx - xb) * (xx - xb);
    nt += xb * xb;
  }
  for (int o = 16; o > 0; o >>= 1) {
    nr += __shfl_xor_sync(0xFFFFFFFFu, nr, o);
    nres += __shfl_xor_sync(0xFFFFFFFFu, nres, o);
    nt += __shfl_xor_sync(0xFFFFFFFFu, nt, o);
  }
  if (lane == 0) {
    stats[r * 4 + 0] = __double2float_ru(sqrt(nr) * (1.0 + 1e-9));
    stats[r * 4 + 1] = __double2float_ru(sqrt(nres) * (1.0 + 1e-9));
    stats[r * 4 + 2] = __double2float_ru(sqrt(nt) * (1.0 + 1e-9));
    stats[r * 4 + 3] = __double2float_rd(norm * (1.0 - 1e-9));
  }
}

// Signed 8-bit codes of each row as Int8CodeBuffer.fill quantises them
// (Sources/MetalANNSCore/Int8CodeCache.swift:64-99): scale u = maxAbs / 127
// (1 for a zero row), inverse 1 / u, code = trunc(v * inverse +- 0.5) (half
// away from zero) clamped to +-127, all in fp32.  One warp per row.  Also the
// per-row factor of the integer dot (u, and u / |r| for cosine) and the bound
// terms (double, rounded up): |r|, |r - u code|, |u code|, and |r| rounded
// down.
__global__ void to_i8_rows_kernel(const float* __restrict__ rows, int64_t n, int32_t dim,
                                  int64_t ld, int8_t* __restrict__ out, int64_t ld8,
                                  float* __restrict__ u_out, float* __restrict__ wcos_out,
                                  float* __restrict__ stats) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= n) return;
  const float* v = rows + r * ld;
  float mx = 0.0f;
  for (int c = lane; c < dim; c += 32) mx = fmaxf(mx, fabsf(v[c]));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  const float inverse = __fdiv_rn(1.0f, scale);
  double n0 = 0.0, nres = 0.0, nt = 0.0;
  for (int c = lane; c < ld8; c += 32) {
    int code = 0;
    double xx = 0.0;
    if (c < dim) {
      const float x = v[c];
      const float scaled = __fmul_rn(x, inverse);
      code = __float2int_rz(scaled >= 0.0f ? __fadd_rn(scaled, 0.5f) : __fsub_rn(scaled, 0.5f));
      code = code > 127 ? 127 : (code < -127 ? -127 : code);
      xx = x;
    }
    out[r * ld8 + c] = static_cast<int8_t>(code);
    const double xb = static_cast<double>(scale) * code;
    n0 += xx * xx;
    nres += (xx - xb) * (xx - xb);
    nt += xb * xb;
  }
  for (int o = 16; o > 0; o >>= 1) {
    n0 += __shfl_xor_sync(0xFFFFFFFFu, n0, o);
    nres += __shfl_xor_sync(0xFFFFFFFFu, nres, o);
    nt += __shfl_xor_sync(0xFFFFFFFFu, nt, o);
  }
  if (lane == 0) {
    const double norm = sqrt(n0);
    u_out[r] = scale;
    wcos_out[r] = norm > 0.0 ? static_cast<float>(static_cast<double>(scale) / norm) : 0.0f;
    stats[r * 4 + 0] = __double2float_ru(norm * (1.0 + 1e-9));
    stats[r * 4 + 1] = __double2float_ru(sqrt(nres) * (1.0 + 1e-9));
    stats[r * 4 + 2] = __double2float_ru(sqrt(nt) * (1.0 + 1e-9));
    stats[r * 4 + 3] = __double2float_rd(norm * (1.0 - 1e-9));
  }
}

struct TcQueryParams {
  const float* queries;  // nq x dim fp32
  int64_t nq;
  int32_t dim;
  int64_t ld16;
  int metric;
  TcCorpusStats cs;
  __nv_bfloat16* qbf;  // nq_pad x ld16 (bf16 pass)
  int8_t* q8;          // nq_pad x ld16 (int8 pass; ld16 is then the int8 pitch)
  float* qn_exact;     // nq, sequential |q|^2
  float* alpha;
  float* gamma;
  float* eps;
  float* scale;  // magnitude bound of the score-domain value x
  int64_t nq_pad;      // query rows of the bf16 block (multiple of 128); rows >= nq are zeroed
  int32_t* ccount;     // candidate counters (nq + 1, the last one counts fallbacks), zeroed
  unsigned long long* pool;  // tile counter of the fused pass's dynamic tail (or null), zeroed
};

// One warp per query: the bf16 copy (or the int8 codes with their scale
// s_q, quantised in double as BoundedExactScan.swift:52-64 does), the exact
// squared norm in index order, the affine terms and the certified bound eps_q
// of |d~ - d|.
constexpr int kPrepWarps = 8;   // queries per block
constexpr int kPrepSq = 512;    // squares per warp buffered before lane 0 sums them

template <bool I8>
__global__ void __launch_bounds__(kPrepWarps * 32) tc_query_prep_kernel(const TcQueryParams p) {
  pdl_trigger();  // the pass may launch and set up while the queries are prepared
  const int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= p.nq_pad) return;
  if (q >= p.nq) {  // padding row of the last query block
    for (int c = lane; c < p.ld16; c += 32) {
      if (I8)
        p.q8[q * p.ld16 + c] = 0;
      else
        p.qbf[q * p.ld16 + c] = __float2bfloat16_rn(0.0f);
    }
    return;
  }
  if (lane == 0) {
    p.ccount[q] = 0;
    if (q == 0) {
      p.ccount[p.nq] = 0;
      if (p.pool) *p.pool = 0;
    }
  }
  const float* v = p.queries + q * p.dim;
  double qs = 1.0;  // query scale (int8)
  if (I8) {
    float mx = 0.0f;
    for (int c = lane; c < p.dim; c += 32) mx = fmaxf(mx, fabsf(v[c]));
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    qs = mx > 0.0f ? static_cast<double>(mx) / 127.0 : 1.0;
  }
  double nq2 = 0.0, nres = 0.0, nt = 0.0;
  // |q|^2 of the exact path: sequential fp32 sum in index order.  The lanes
  // square their elements into the warp's shared slice (up to 512 at a time)
  // and lane 0 adds them in index order: a short loop instead of a long
  // unrolled shuffle chain, which matters for a kernel whose run time is its
  // latency.  Lanes past `dim` store +0, which leaves a sum of non-negative
  // squares (never -0) unchanged.
  __shared__ __align__(16) float sqbuf[kPrepWarps][kPrepSq];
  float* sb = sqbuf[threadIdx.x >> 5];
  int filled = 0;
  float acc = 0.0f;
  auto drain = [&]() {
    __syncwarp();
    if (lane == 0) {
#pragma unroll 4
      for (int j = 0; j < filled; j += 4) {
        const float4 t = *reinterpret_cast<const float4*>(sb + j);
        acc = __fadd_rn(acc, t.x);
        acc = __fadd_rn(acc, t.y);
        acc = __fadd_rn(acc, t.z);
        acc = __fadd_rn(acc, t.w);
      }
    }
    __syncwarp();
    filled = 0;
  };
  // Up to 384 columns (the usual widths) the query's elements are loaded in
  // one round trip and held in registers; wider queries load 32 at a time.
  constexpr int kHeld = 12;
  float held[kHeld];
  const bool in_regs = p.ld16 <= 32 * kHeld;
  if (in_regs) {
#pragma unroll
    for (int j = 0; j < kHeld; ++j) {
      const int c = 32 * j + lane;
      held[j] = c < p.dim ? __ldg(v + c) : 0.0f;
    }
  }
  // one 32-column chunk: the exact |q|^2 steps, the rounded copy, the sums
  auto column = [&](int c0, float x) {
    const int c = c0 + lane;
    if (c0 < p.dim) {
      sb[filled + lane] = __fmul_rn(x, x);  // x = 0 past dim
      filled += 32;
      if (filled == kPrepSq) drain();
    }
    if (c < p.ld16) {
      double xb;
      if (I8) {
        const double sc = static_cast<double>(x) / qs;
        int code = static_cast<int>(sc >= 0.0 ? sc + 0.5 : sc - 0.5);
        code = code > 127 ? 127 : (code < -127 ? -127 : code);
        p.q8[q * p.ld16 + c] = static_cast<int8_t>(code);
        xb = qs * code;
      } else {
        const __nv_bfloat16 b = __float2bfloat16_rn(x);
        p.qbf[q * p.ld16 + c] = b;
        xb = __bfloat162float(b);
      }
      const double xx = x;
      nq2 += xx * xx;
      nres += (xx - xb) * (xx - xb);
      nt += xb * xb;
    }
  };
  if (in_regs) {
#pragma unroll
    for (int j = 0; j < kHeld; ++j)
      if (32 * j < p.ld16) column(32 * j, held[j]);
  } else {
    // read-only loads (no aliasing with the stores), four in flight
#pragma unroll 4
    for (int c0 = 0; c0 < p.ld16; c0 += 32)
      column(c0, c0 + lane < p.dim ? __ldg(v + c0 + lane) : 0.0f);
  }
  if (filled > 0) drain();
  for (int o = 16; o > 0; o >>= 1) {
    nq2 += __shfl_xor_sync(0xFFFFFFFFu, nq2, o);
    nres += __shfl_xor_sync(0xFFFFFFFFu, nres, o);
    nt += __shfl_xor_sync(0xFFFFFFFFu, nt, o);
  }
  if (lane != 0) return;
  const QueryTerms t = query_terms(p.cs, p.metric, p.dim, acc, nq2, nres, nt, qs);
  p.qn_exact[q] = t.qn;
  p.alpha[q] = t.alpha;
  p.gamma[q] = t.gamma;
  p.eps[q] = t.eps;
  p.scale[q] = t.scale;
}

// Per query: thr_q = (k-th smallest value of the dense sample: row distances
// or 32-row group minima, either at or above the sample's k-th smallest
// distance) + 2 eps_q (+inf when the sample has fewer than k values) and the
// matching score-domain filter constant.
constexpr int kThresholdThreads = 1024;
constexpr int kThresholdStageMax = 160 * 1024;  // bytes of a staged sample row

__global__ void __launch_bounds__(kThresholdThreads) tc_threshold_kernel(
    const float* __restrict__ dense, int64_t ld, int64_t rows, int32_t k, int staged,
    const float* __restrict__ eps, const float* __restrict__ alpha,
    const float* __restrict__ gamma, const float* __restrict__ scale, int metric,
    float* __restrict__ thr_out, float* __restrict__ c_out) {
  __shared__ KthSmem ks;
  extern __shared__ __align__(16) float stage[];  // the sample row, when staged
  pdl_trigger();
  pdl_wait();  // the sample pass's values
  const int64_t q = blockIdx.x;
  const float* row = dense + q * ld;
  const float inf = __int_as_float(0x7F800000);
  if (staged) {
    // every pass of the selection then reads shared memory
#pragma unroll 4
    for (int64_t i = threadIdx.x; i < rows / 4; i += blockDim.x)
      reinterpret_cast<float4*>(stage)[i] = __ldg(reinterpret_cast<const float4*>(row) + i);
    for (int64_t i = rows / 4 * 4 + threadIdx.x; i < rows; i += blockDim.x) stage[i] = row[i];
    __syncthreads();
    row = stage;
  }
  float kth = inf;
  if (rows >= k)
    kth = block_kth_smallest([&](int64_t i) { return row[i]; }, rows, k, ks,
                             static_cast<int>(threadIdx.x), static_cast<int>(blockDim.x),
                             [] { __syncthreads(); });
  (void)metric;
  if (threadIdx.x == 0)
    threshold_from_kth(kth, eps[q], alpha[q], gamma[q], scale[q], thr_out + q, c_out + q);
}

// The same thresholds for batches of more queries than SMs, one warp per
// query: the query's sample values (at most kThrWarpMax) are staged in the
// warp's shared slice and its k-th smallest taken by warp_kth_smallest, so
// the whole batch fits in one wave of small blocks with no block barrier.
constexpr int kThrWarps = 4;
constexpr int kThrWarpMax = 2048;

__global__ void __launch_bounds__(kThrWarps * 32) tc_threshold_warp_kernel(
    const float* __restrict__ dense, int64_t ld, int64_t rows, int32_t k, int64_t nq,
    const float* __restrict__ eps, const float* __restrict__ alpha,
    const float* __restrict__ gamma, const float* __restrict__ scale,
    float* __restrict__ thr_out, float* __restrict__ c_out) {
  __shared__ uint32_t hist[kThrWarps][256];
  __shared__ __align__(16) float vals[kThrWarps][kThrWarpMax];
  pdl_trigger();
  pdl_wait();  // the sample pass's values
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * kThrWarps + w;
  if (q >= nq) return;
  // `ld` is a multiple of 4 and the sample block 256-byte aligned: 16-byte
  // asynchronous copies, all in flight at once (one memory round trip)
  const float* row = dense + q * ld;
  float* sv = vals[w];
  for (int64_t i = lane; i < (rows + 3) / 4; i += 32) cp_async16(sv + 4 * i, row + 4 * i);
  cp_async_wait_all();
  __syncwarp();
  float kth = __int_as_float(0x7F800000);
  if (rows >= k) {
    auto get = [&](int64_t i) { return sv[i]; };
    kth = k <= kSmallK ? warp_kth_small<kSmallK>(get, rows, k, lane)
                       : warp_kth_smallest(get, rows, k, hist[w], lane);
  }
  if (lane == 0)
    threshold_from_kth(kth, eps[q], alpha[q], gamma[q], scale[q], thr_out + q, c_out + q);
}

struct RerankParams {
  const uint64_t* cand;
  const int32_t* cand_count;
  int32_t cand_cap;
  const float* thr;
  const float* eps;
  const float* qn_exact;
  const float* queries;  // fp32 nq x dim
  const float* rows;     // fp32 corpus, ld pitch
  int64_t ld;
  const float* norms;
  int64_t n;
  int32_t dim;
  int32_t metric;
  uint32_t id_offset;
  int32_t k;   // effective k
  int32_t kp;
  int32_t kout;
  float* out_dist;
  uint32_t* out_ids;
  int32_t* out_counts;
  int32_t* fallbacks;  // count of queries re-scanned exactly
  int32_t region;      // bytes of the shared staging region
  int32_t max_band;    // entries of the band buffer (>= kSortN, a power of two)
};

// Exact distance of one corpus row in the reference order.
__device__ __forceinline__ float exact_distance(const RerankParams& p, const float* q, float qn,
                                                int64_t row) {
  // rows have a 16-byte pitch: 32 columns per batch of eight 16-byte loads,
  // accumulated strictly in index order
  const float* r = p.rows + row * p.ld;
  float acc = 0.0f;
  int c = 0;
  for (; c + 32 <= p.dim; c += 32) {
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldg(reinterpret_cast<const float4*>(r + c) + j);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      acc = __fadd_rn(acc, __fmul_rn(v[j].x, q[c + 4 * j]));
      acc = __fadd_rn(acc, __fmul_rn(v[j].y, q[c + 4 * j + 1]));
      acc = __fadd_rn(acc, __fmul_rn(v[j].z, q[c + 4 * j + 2]));
      acc = __fadd_rn(acc, __fmul_rn(v[j].w, q[c + 4 * j + 3]));
    }
  }
  for (; c < p.dim; ++c) acc = __fadd_rn(acc, __fmul_rn(__ldg(r + c), q[c]));
  return finalize_distance(p.metric, acc, qn, p.metric == kIP ? 0.0f : __ldg(p.norms + row));
}


// Dynamic shared memory of tc_rerank_kernel: the query (dim floats, 16-byte
// rounded), the band buffer (max_band 64-bit entries: first the band's row
// ids, then their exact keys; the exact fallback's running top-k), then one
// region that first holds the candidate keys and later the staged corpus rows
// of the exact re-score.
// The region is large (64 KB) and the band buffer 2048 entries while the
// queries fit on the SMs in one wave.  For larger batches the region holds
// 16 staged rows (at least 16 KB, at most 32 KB) and the band buffer 512
// entries: the usual band (k plus a few rows) is re-scored in one round, and
// at d = 384 seven blocks share an SM, so 1,024 queries still run in one
// wave.  A band wider than the buffer takes the exact re-scan.
inline int rerank_region_bytes(int64_t nq, int num_sms, int64_t dim) {
  if (nq <= num_sms) return 64 * 1024;
  const int64_t r16 = 16 * ((dim + 3) / 4 * 4 + 4) * 4;
  return static_cast<int>(std::max<int64_t>(16 * 1024, std::min<int64_t>(r16, 32 * 1024)));
}
inline int rerank_max_band(int64_t nq, int num_sms) { return nq <= num_sms ? 2048 : 512; }
inline size_t rerank_smem_bytes(int64_t dim, int max_band, int region) {
  return static_cast<size_t>((dim + 3) / 4 * 4) * sizeof(float) +
         static_cast<size_t>(max_band) * sizeof(uint64_t) + region;
}

// Exact distance of a row staged in shared memory, in the reference order;
// `q` (shared, 16-byte aligned) is the query, `vn` the row's |r|^2 (0 for IP).
__device__ __forceinline__ float exact_distance_smem(const RerankParams& p, const float* q,
                                                     float qn, const float* r, float vn) {
  float acc = 0.0f;
  int c = 0;
  for (; c + 4 <= p.dim; c += 4) {
    const float4 v = *reinterpret_cast<const float4*>(r + c);
    const float4 w = *reinterpret_cast<const float4*>(q + c);
    acc = __fadd_rn(acc, __fmul_rn(v.x, w.x));
    acc = __fadd_rn(acc, __fmul_rn(v.y, w.y));
    acc = __fadd_rn(acc, __fmul_rn(v.z, w.z));
    acc = __fadd_rn(acc, __fmul_rn(v.w, w.w));
  }
  for (; c < p.dim; ++c) acc = __fadd_rn(acc, __fmul_rn(r[c], q[c]));
  return finalize_distance(p.metric, acc, qn, vn);
}

// Per query: certify the candidate list, then re-score the band exactly.
//   T_k  = k-th smallest approximate distance among the candidates
//   band = T_k + 2 eps (rounded up); every row of the exact top-k has an
//          approximate distance <= band, so the exact top-k of the band rows
//          is the exact top-k of the corpus, provided the filter kept every
//          row up to band (band <= thr) and the list did not overflow.
// Otherwise the query is re-scanned exactly over all rows by this block.
__global__ void __launch_bounds__(kRerankThreads, 8) tc_rerank_kernel(const RerankParams p) {
  extern __shared__ __align__(16) unsigned char rsm[];
  float* qsm = reinterpret_cast<float*>(rsm);
  // band row ids (phase 1), then the band's exact keys (phase 2)
  uint64_t* ekeys = reinterpret_cast<uint64_t*>(rsm + static_cast<size_t>((p.dim + 3) / 4 * 4) *
                                                          sizeof(float));
  unsigned char* region = reinterpret_cast<unsigned char*>(ekeys + p.max_band);
  uint64_t* skeys = reinterpret_cast<uint64_t*>(region);  // candidate keys (phase 1)
  float* srows = reinterpret_cast<float*>(region);         // staged rows (phase 2)
  __shared__ uint32_t hist[256];                            // k-th selection (warp 0)
  __shared__ uint64_t thr;
  __shared__ int qc, nb, fail_flag, nlist;
  __shared__ float band_sh;
  const int tid = threadIdx.x;
  const int64_t q = blockIdx.x;
  pdl_wait();  // the pass's candidates
#pragma unroll 2
  for (int c = tid; c < p.dim; c += kRerankThreads) qsm[c] = __ldg(p.queries + q * p.dim + c);
  const int total = p.cand_count[q];
  const int cnt = min(total, p.cand_cap);
  const float e = p.eps[q];
  const float qn = p.qn_exact[q];
  const float thr_q = p.thr[q];  // loaded with the others, read after the k-th selection
  if (tid == 0) {
    nlist = 0;
    fail_flag = (total > p.cand_cap || cnt < p.k) ? 1 : 0;
  }
  const uint64_t* cq = p.cand + q * p.cand_cap;
  const bool stage_keys = cnt * 8 <= p.region;
  if (stage_keys) {
    // pairs of keys by 16-byte asynchronous copies, all in flight at once
    // (the list capacity is even and each list 16-byte aligned)
    for (int i = tid; i < (cnt + 1) / 2; i += kRerankThreads) cp_async16(skeys + 2 * i, cq + 2 * i);
    cp_async_wait_all();
  }
  const uint64_t* keys = stage_keys ? skeys : cq;
  __syncthreads();
  if (!fail_flag) {
    if (tid < 32) {
      // the k-th smallest candidate distance, by warp 0 alone
      auto get = [&](int64_t i) { return key_distance(keys[i]); };
      const float tk = p.k <= kSmallK ? warp_kth_small<kSmallK>(get, cnt, p.k, tid)
                                      : warp_kth_smallest(get, cnt, p.k, hist, tid);
      if (tid == 0) {
        float band = tk + 2.0f * e;
        band = band + fabsf(band) * 1e-6f;
        if (!(band <= thr_q)) fail_flag = 1;  // the filter did not cover the band
        band_sh = band;
      }
    }
    __syncthreads();
    if (!fail_flag) {
      const float band = band_sh;
      for (int i = tid; i < cnt; i += kRerankThreads) {
        const uint64_t key = keys[i];
        if (key_distance(key) <= band) {
          const int pos = atomicAdd(&nlist, 1);
          if (pos < p.max_band) ekeys[pos] = key_id(key);
        }
      }
      __syncthreads();
      if (tid == 0 && nlist > p.max_band) fail_flag = 1;
      __syncthreads();
    }
  }
  if (!fail_flag) {
    // exact re-score of the band: rows staged in shared memory by cp.async
    // (all loads of a round in flight), one thread per row.  Entry i of the
    // band buffer holds row id i until thread i - b of its round replaces it
    // by the exact key, after every read of the round's ids.
    const int m = nlist;
    const int pitch = (p.dim + 3) / 4 * 4 + 4;  // floats; +4 spreads rows over the banks
    const int per_round = max(1, min(kRerankThreads, p.region / (pitch * 4)));
    const int chunks = (p.dim + 3) / 4;  // 16-byte pieces of one row
    for (int b = 0; b < m; b += per_round) {
      const int rn = min(per_round, m - b);
      const int64_t my_row = tid < rn ? static_cast<int64_t>(ekeys[b + tid]) : 0;
      // the row's |r|^2, loaded while its row is in flight
      const float vn = (tid < rn && p.metric != kIP) ? __ldg(p.norms + my_row) : 0.0f;
      for (int t = tid; t < rn * chunks; t += kRerankThreads) {
        const int r = t / chunks, c = t - r * chunks;
        cp_async16(srows + r * pitch + 4 * c,
                   p.rows + static_cast<int64_t>(ekeys[b + r]) * p.ld + 4 * c);
      }
      cp_async_wait_all();
      __syncthreads();
      if (tid < rn)
        ekeys[b + tid] = make_key(exact_distance_smem(p, qsm, qn, srows + tid * pitch, vn),
                                  static_cast<uint32_t>(my_row + p.id_offset));
      __syncthreads();
    }
    if (m <= 32) {
      // the usual band (about k rows): one warp sorts it by shuffles
      if (tid < 32) {
        const uint64_t x = warp_sort32(tid < m ? ekeys[tid] : kKeyMax, tid);
        __syncwarp();
        ekeys[tid] = x;
      }
      __syncthreads();
    } else {
      int mp = 1;
      while (mp < m) mp <<= 1;
      for (int i = m + tid; i < mp; i += kRerankThreads) ekeys[i] = kKeyMax;
      __syncthreads();
      bitonic_sort_keys<kRerankThreads>(ekeys, mp, tid, 0);
    }
    const int have = min(m, p.k);
    for (int i = tid; i < p.kout; i += kRerankThreads) {
      p.out_dist[q * p.kout + i] = i < have ? key_distance(ekeys[i]) : __int_as_float(0x7F800000);
      p.out_ids[q * p.kout + i] = i < have ? key_id(ekeys[i]) : kEmptyId;
    }
    if (tid == 0) p.out_counts[q] = have;
    return;
  }
  // certificate failed: exact scan of every row by this block
  if (tid == 0) {
    atomicAdd(p.fallbacks, 1);
    thr = kKeyMax;
    qc = 0;
    nb = 0;
  }
  __syncthreads();
  TopKState st{ekeys, &qc, &nb, &thr};
  for (int64_t b = 0; b < p.n; b += kRerankThreads) {
    const int64_t row = b + tid;
    const bool valid = row < p.n;
    uint64_t key = kKeyMax;
    if (valid) key = make_key(exact_distance(p, qsm, qn, row), static_cast<uint32_t>(row + p.id_offset));
    topk_offer(st, p.kp, key, valid);
    __syncthreads();
    if (qc > kSortN - p.kp - kRerankThreads) topk_merge<kRerankThreads>(st, p.k, p.kp, kSortN, tid, 0);
  }
  if (qc > 0) topk_merge<kRerankThreads>(st, p.k, p.kp, kSortN, tid, 0);
  for (int i = tid; i < p.kout; i += kRerankThreads) {
    const bool have = i < nb;
    p.out_dist[q * p.kout + i] = have ? key_distance(ekeys[i]) : __int_as_float(0x7F800000);
    p.out_ids[q * p.kout + i] = have ? key_id(ekeys[i]) : kEmptyId;
  }
  if (tid == 0) p.out_counts[q] = nb;
}


// 2-D tensor map of a row-major matrix with a 128-byte inner box (64 bf16 or
// 128 int8 elements) and 128-byte swizzle; `ld` in elements.
int32_t encode_tc_map(CUtensorMap* map, const void* base, int64_t rows, int64_t dim, int64_t ld,
                      int box_rows, bool i8) {
  auto enc_ptr = [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<void*>(nullptr);
    return fn;
  };
  static void* fn = enc_ptr();
  if (!fn) return fail(MANS_ERR_PIPELINE, "cuTensorMapEncodeTiled is unavailable");
  using Enc = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                           const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                           CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                           CUtensorMapFloatOOBfill);
  cuuint64_t gdim[2] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(std::max<int64_t>(rows, 1))};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(ld) * (i8 ? 1 : 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(i8 ? 128 : kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = reinterpret_cast<Enc>(fn)(map, i8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                         const_cast<void*>(base), gdim, gstride, box, estride,
                                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MANS_ERR_PIPELINE, "tensor-core map encoding failed");
  return MANS_OK;
}

}  // namespace

// Builds (once per corpus and row scaling) the bf16 copy and the bound terms:
// cosine rounds the normalised rows, L2 and IP the rows as stored.
static int32_t tc_prepare_bf16(mans_corpus* c, int metric) {
  const int norm_mode = metric == kCosine ? 1 : 0;
  if (c->tc_ready && c->tc_metric == norm_mode) return MANS_OK;
  DeviceGuard g(c->ctx->device);
  const int64_t n = c->n;
  const int64_t ld16 = (c->dim + 7) / 8 * 8;
  cudaError_t e = cudaSuccess;
  if (!c->tc_rows) {
    e = cudaMalloc(&c->tc_rows, std::max<int64_t>(n, 1) * ld16 * sizeof(__nv_bfloat16));
    if (e == cudaSuccess) e = cudaMalloc(&c->tc_stats, std::max<int64_t>(n, 1) * 4 * sizeof(float));
    if (e != cudaSuccess) return fail_cuda(e, "cudaMalloc(bf16 corpus)");
    c->tc_ld16 = ld16;
    int32_t rc = encode_tc_map(&c->tc_map, c->tc_rows, n, c->dim, ld16, kRN, false);
    if (rc == MANS_OK)
      rc = encode_tc_map(&c->tc_map_half, c->tc_rows, n, c->dim, ld16, kRN / 2, false);
    if (rc != MANS_OK) return rc;
  }
  if (n > 0) {
    to_bf16_rows_kernel<<<static_cast<unsigned>((n + 7) / 8), 256>>>(
        c->rows, n, static_cast<int32_t>(c->dim), c->ld, static_cast<__nv_bfloat16*>(c->tc_rows),
        ld16, c->tc_stats, norm_mode);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail_cuda(e, "bf16 corpus conversion");
  }
  // corpus-wide maxima of the bound terms (host reduction, once)
  std::vector<float> st(static_cast<size_t>(std::max<int64_t>(n, 1)) * 4);
  if (n > 0) {
    e = cudaMemcpy(st.data(), c->tc_stats, n * 4 * sizeof(float), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail_cuda(e, "bf16 corpus stats");
  }
  TcCorpusStats cs{};
  cs.min_norm = n > 0 ? INFINITY : 0.0f;
  bool finite = true;
  for (int64_t r = 0; r < n; ++r) {
    for (int j = 0; j < 4; ++j) finite = finite && std::isfinite(st[r * 4 + j]);
    cs.max_norm = std::max(cs.max_norm, st[r * 4 + 0]);
    cs.max_resid = std::max(cs.max_resid, st[r * 4 + 1]);
    cs.max_norm_bf16 = std::max(cs.max_norm_bf16, st[r * 4 + 2]);
    cs.min_norm = std::min(cs.min_norm, st[r * 4 + 3]);
    // |r|^2 of the stored row, bounded above (L2 uses it; for L2 / IP the
    // rounded row is the stored one, so stats[0] is |r| rounded up)
    const double up = norm_mode ? static_cast<double>(st[r * 4 + 3]) * (1.0 + 1e-6) : st[r * 4 + 0];
    cs.max_sqnorm = std::max(cs.max_sqnorm, static_cast<float>(up * up * (1.0 + 1e-5)));
  }
  if (!finite) cs.max_norm = INFINITY;  // a NaN / infinite row: the bound does not apply
  c->tc_stats_host = cs;
  c->tc_metric = norm_mode;
  c->tc_ready = true;
  return MANS_OK;
}

// Launches `fn` with programmatic stream serialization (it may start while
// the previous kernel on `stream` runs and waits for it with pdl_wait), and
// as a cooperative launch when `coop`.  If the runtime refuses the attribute
// the kernel is launched plainly, and the context stops asking.
static cudaError_t launch_pdl(mans_ctx* ctx, const void* fn, dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, void** args, bool coop) {
  if (ctx->pdl) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeCooperative;
    at[1].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = coop ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e == cudaSuccess) return e;
    cudaGetLastError();  // clear the refusal and fall back for good
    ctx->pdl = false;
  }
  if (coop) return cudaLaunchCooperativeKernel(fn, grid, block, args, smem, stream);
  return cudaLaunchKernel(fn, grid, block, args, smem, stream);
}

// Clusters of two CTAs (one per SM) of the pair pass, launched with the
// programmatic-dependent-launch attribute like the other kernels.
static cudaError_t launch_pair(mans_ctx* ctx, const void* fn, dim3 grid, dim3 block, size_t smem,
                               cudaStream_t stream, void** args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = ctx->pdl ? 2 : 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

// How many CTA pairs of the pair pass the device runs at once (0: the
// one-CTA pass runs).  The pair pass is opt-in (MANS_TC_PAIRS=1 when the
// context first runs a multi-block batch): measured on B200 it is correct but
// slower than the one-CTA pass (1M x 384, 1024 queries: 672.6 against
// 640.6 us; 125k rows: 119.6 against 107.2 us).  Asked once per context.
static int tc_pair_capacity(mans_ctx* ctx, size_t smem) {
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (ctx->tc_pairs < 0) {
    const char* env = getenv("MANS_TC_PAIRS");
    int n = 0;
    if (env && env[0] == '1') {
      cudaLaunchConfig_t cfg{};
      cfg.gridDim = dim3(2 * (ctx->num_sms / 2));
      cfg.blockDim = dim3(kTcThreads);
      cfg.dynamicSmemBytes = smem;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 2;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      const void* fn = reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, false, false, true>);
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           ctx->max_smem);
      if (e == cudaSuccess) e = cudaOccupancyMaxActiveClusters(&n, fn, &cfg);
      if (e != cudaSuccess) {
        cudaGetLastError();
        n = 0;
      }
    }
    ctx->tc_pairs = std::min(n, ctx->num_sms / 2);
  }
  return ctx->tc_pairs;
}

static size_t carve(size_t& o, size_t bytes) {
  size_t at = (o + 255) / 256 * 256;
  o = at + bytes;
  return at;
}

// Whether the tensor-core path applies to this corpus and metric: cosine
// needs every row norm bounded away from zero so the bound stays finite.
// The int8 codes and scales (metric independent) and both sets of bound terms.
static int32_t tc_prepare_int8(mans_corpus* c) {
  if (c->tc8_ready) return MANS_OK;
  DeviceGuard g(c->ctx->device);
  const int64_t n = c->n;
  const int64_t ld8 = (c->dim + 127) / 128 * 128;
  cudaError_t e = cudaSuccess;
  if (!c->tc8_rows) {
    const int64_t nn = std::max<int64_t>(n, 1);
    const int64_t nn64 = (nn + 63) / 64 * 64;  // whole 16-byte pieces per tile (bulk copies)
    e = cudaMalloc(&c->tc8_rows, nn * ld8);
    if (e == cudaSuccess) e = cudaMalloc(&c->tc8_u, nn64 * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&c->tc8_wcos, nn64 * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&c->tc8_stats, nn * 4 * sizeof(float));
    if (e != cudaSuccess) return fail_cuda(e, "cudaMalloc(int8 corpus)");
    c->tc8_ld = ld8;
    int32_t rc = encode_tc_map(&c->tc8_map, c->tc8_rows, n, c->dim, ld8, kRN, true);
    if (rc != MANS_OK) return rc;
  }
  if (n > 0) {
    to_i8_rows_kernel<<<static_cast<unsigned>((n + 7) / 8), 256>>>(
        c->rows, n, static_cast<int32_t>(c->dim), c->ld, static_cast<int8_t*>(c->tc8_rows), ld8,
        c->tc8_u, c->tc8_wcos, c->tc8_stats);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail_cuda(e, "int8 corpus conversion");
  }
  std::vector<float> st(static_cast<size_t>(std::max<int64_t>(n, 1)) * 4);
  if (n > 0) {
    e = cudaMemcpy(st.data(), c->tc8_stats, n * 4 * sizeof(float), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail_cuda(e, "int8 corpus stats");
  }
  TcCorpusStats pl{}, co{};
  pl.min_norm = co.min_norm = n > 0 ? INFINITY : 0.0f;
  co.max_norm = static_cast<float>(1.0 + 1e-6);
  bool finite = true;
  for (int64_t r = 0; r < n; ++r) {
    const float* x = &st[r * 4];
    for (int j = 0; j < 4; ++j) finite = finite && std::isfinite(x[j]);
    pl.max_norm = std::max(pl.max_norm, x[0]);
    pl.max_resid = std::max(pl.max_resid, x[1]);
    pl.max_norm_bf16 = std::max(pl.max_norm_bf16, x[2]);
    pl.min_norm = std::min(pl.min_norm, x[3]);
    const double up = static_cast<double>(x[0]);
    pl.max_sqnorm = std::max(pl.max_sqnorm, static_cast<float>(up * up * (1.0 + 1e-5)));
    if (x[3] > 0.0f) {  // relative terms; a zero row keeps cosine off this path
      co.max_resid = std::max(co.max_resid, static_cast<float>(x[1] / static_cast<double>(x[3]) * (1.0 + 1e-6)));
      co.max_norm_bf16 = std::max(co.max_norm_bf16, static_cast<float>(x[2] / static_cast<double>(x[3]) * (1.0 + 1e-6)));
    }
    co.min_norm = std::min(co.min_norm, x[3]);
  }
  if (!finite) pl.max_norm = co.max_norm = INFINITY;
  c->tc8_plain = pl;
  c->tc8_cos = co;
  c->tc8_ready = true;
  return MANS_OK;
}

int32_t tc_prepare_corpus(mans_corpus* c, int metric, bool i8) {
  return i8 ? tc_prepare_int8(c) : tc_prepare_bf16(c, metric);
}

static const TcCorpusStats& tc_stats_for(const mans_corpus* c, int metric, bool i8) {
  if (!i8) return c->tc_stats_host;
  return metric == kCosine ? c->tc8_cos : c->tc8_plain;
}

// AUTO is bf16: on L2-normalised data the int8 bound is about 6x wider
// (|q - q'| |r| + |q'| |r - r'| with per-row scales maxAbs/127), which grows
// the candidate and re-score sets more than the halved row bytes save.
bool tc_use_int8(const mans_ctx* ctx, int64_t nq) {
  (void)nq;
  return ctx->tc_format == MANS_TC_INT8;
}

bool tc_applicable(const mans_corpus* c, int metric, bool i8) {
  if (c->n <= 0 || c->n >= (1ll << 31)) return false;
  if (!(i8 ? c->tc8_ready : c->tc_ready)) return true;
  const TcCorpusStats& cs = tc_stats_for(c, metric, i8);
  if (metric == kCosine && cs.min_norm < 1e-6f) return false;
  // a NaN or infinite row makes the bound meaningless: exact scan
  if (!(std::isfinite(cs.max_norm) && std::isfinite(cs.max_sqnorm))) return false;
  return true;
}

int32_t tc_export_int8(mans_corpus* c, int8_t* codes, float* scales) {
  int32_t rc = tc_prepare_int8(c);
  if (rc != MANS_OK) return rc;
  DeviceGuard g(c->ctx->device);
  cudaError_t e = cudaSuccess;
  if (codes && c->n > 0)
    e = cudaMemcpy2D(codes, c->dim, c->tc8_rows, c->tc8_ld, c->dim, c->n, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && scales && c->n > 0)
    e = cudaMemcpy(scales, c->tc8_u, c->n * sizeof(float), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? MANS_OK : fail_cuda(e, "int8 code download");
}

// Kernel attributes of the tensor-core path, set once per context (they are
// per device and outlive the call): every pass variant may use the device's
// whole opt-in shared memory, and the small per-query kernels prefer the
// whole carve-out as shared memory, so that seven re-rank or six threshold
// blocks share an SM.
static int32_t tc_configure(mans_ctx* ctx) {
  std::lock_guard<std::mutex> lk(ctx->mu);
  if (ctx->tc_configured) return MANS_OK;
  const void* pass[] = {
      reinterpret_cast<const void*>(tc_scan_kernel<kDense, false>),
      reinterpret_cast<const void*>(tc_scan_kernel<kDense, true>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, false>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, true>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, false>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, true>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, false, true>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, true, true>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, false, true>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, true, true>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, false, false, true>),
      reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, false, false, true>)};
  cudaError_t e = cudaSuccess;
  for (const void* fn : pass)
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, ctx->max_smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tc_threshold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kThresholdStageMax);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tc_rerank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(rerank_smem_bytes(12 * 1024, 2048, 64 * 1024)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tc_rerank_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tc_threshold_warp_kernel,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return fail_cuda(e, "tc configure");
  ctx->tc_configured = true;
  return MANS_OK;
}

int32_t run_flat_search_tc(mans_ctx* ctx, mans_corpus* corpus, mans_workspace* ws,
                           const float* d_queries, int64_t nq, int32_t k, int32_t metric,
                           float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                           cudaStream_t stream, bool i8) {
  int32_t rc = tc_prepare_corpus(corpus, metric, i8);
  if (rc != MANS_OK) return rc;
  if (!tc_applicable(corpus, metric, i8))
    return run_flat_search(ctx, corpus, ws, d_queries, nq, k, metric, d_out_dist, d_out_ids,
                           d_out_counts, stream, kModeHost, MANS_MAX_TOPK);
  const int64_t n = corpus->n;
  const int32_t kout = std::min<int32_t>(k, MANS_MAX_TOPK);
  const int32_t keff = static_cast<int32_t>(std::min<int64_t>(kout, n));
  const int32_t kp = pow2_at_least(keff);
  // row pitch of the operand copy, in elements (128-byte multiple)
  const int64_t ld16 = i8 ? corpus->tc8_ld : corpus->tc_ld16;
  const size_t esize = i8 ? 1 : sizeof(__nv_bfloat16);
  const int64_t qblocks = (nq + kQM - 1) / kQM;
  const int64_t nq_pad = qblocks * kQM;
  // Sample size.  The filter threshold (sample k-th + 2 eps) sits near rank
  // k n / S of the corpus, so the candidate lists hold about k n / S rows plus
  // the rows of the 2 eps band: S >= k n / 2048 keeps that near two thousand
  // for every k.  Several query blocks run the sample as its own GEMM costing
  // S / n of the pass; there S >= n / 16 also thins the candidates, which
  // saves more epilogue work (list appends) than the sample costs.  The int8
  // bound is about 4x wider than the bf16 one, hence its larger minimum.
  const int64_t smin = i8 ? 65536 : 16384;
  int64_t sample = std::max<int64_t>(smin, static_cast<int64_t>(keff) * n / 2048);
  if (qblocks > 1) sample = std::max<int64_t>(sample, n / 16);
  sample = std::min<int64_t>(n, (sample + kRN - 1) / kRN * kRN);
  // candidate list capacity per query, even: the re-rank stages a list by
  // 16-byte copies of key pairs, so every list must start 16-byte aligned
  const int32_t cap = static_cast<int32_t>(
      (std::min<int64_t>(std::max<int64_t>(i8 ? 32768 : 8192, 64ll * keff), n) + 1) / 2 * 2);

  static const int stream_q = [] {
    const char* e = getenv("MANS_TC_STREAM_QUERIES");
    return e && e[0] == '1' ? 1 : 0;
  }();
  const TcLayout lay = tc_layout(tc_kblocks(static_cast<int>(corpus->dim), i8), stream_q);
  // Full-pass grid: lockstep row groups when every query block gets a block.
  const int64_t rtiles_all = (n + kRN - 1) / kRN;
  int32_t groups_full =
      qblocks <= ctx->num_sms ? static_cast<int32_t>(ctx->num_sms / qblocks) : 0;
  groups_full = static_cast<int32_t>(std::min<int64_t>(groups_full, rtiles_all));
  // Fused sampling (one cooperative launch instead of sample + threshold +
  // pass): each block samples its first S tiles, S chosen so that the sample
  // holds at least max(16384, 256 k) rows per query.
  int coop = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->device);
  // (Only for one query block: with several, sampling S tiles per block
  // inside the pass and deriving thresholds between the barriers stalls the
  // MMA pipeline longer than the separate sample and threshold launches take.)
  const bool fused = qblocks == 1 && groups_full > 0 && lay.resident && coop != 0;
  int64_t samp_tiles = 0, samp_ld = 0;
  if (fused) {
    const int64_t want = sample;
    samp_tiles = (want + kRN * groups_full - 1) / (kRN * groups_full);
    samp_tiles = std::max<int64_t>(1, std::min<int64_t>(samp_tiles, rtiles_all / groups_full));
    samp_ld = groups_full * samp_tiles * 8;
  }

  size_t o = 0;
  const size_t o_qbf = carve(o, nq_pad * ld16 * esize);
  const size_t o_qn = carve(o, nq * sizeof(float));
  const size_t o_al = carve(o, nq * sizeof(float));
  const size_t o_ga = carve(o, nq * sizeof(float));
  const size_t o_ep = carve(o, nq * sizeof(float));
  const size_t o_th = carve(o, nq * sizeof(float));
  const size_t o_sc = carve(o, nq * sizeof(float));
  const size_t o_cq = carve(o, nq * sizeof(float));
  // the sample pass writes one value per 32-row group when that leaves at
  // least 4k groups, otherwise every row
  const int dgroup = (sample / 32 >= 4ll * keff) ? 32 : 1;
  const int64_t dvals = (sample + dgroup - 1) / dgroup;
  const int64_t dld = (dvals + 3) / 4 * 4;  // float4-aligned pitch of the dense sample
  const size_t o_dn = carve(o, nq * (fused ? samp_ld : dld) * sizeof(float));
  const size_t o_cc = carve(o, nq * sizeof(int32_t) + sizeof(int32_t));
  const size_t o_cd = carve(o, nq * static_cast<size_t>(cap) * sizeof(uint64_t));
  const size_t o_pl = carve(o, sizeof(unsigned long long));
  if ((rc = ws->tc_aux.reserve(o)) != MANS_OK) return rc;
  if (fused && !ws->tc_bar.ptr) {
    if ((rc = ws->tc_bar.reserve(sizeof(unsigned long long))) != MANS_OK) return rc;
    cudaError_t e0 = cudaMemsetAsync(ws->tc_bar.ptr, 0, sizeof(unsigned long long), stream);
    if (e0 != cudaSuccess) return fail_cuda(e0, "barrier clear");
    ws->tc_bar_base = 0;
  }
  if ((rc = ws->err.reserve(sizeof(int))) != MANS_OK) return rc;
  if (!ws->err_cleared) {
    cudaError_t e = cudaMemsetAsync(ws->err.ptr, 0, sizeof(int), stream);
    if (e != cudaSuccess) return fail_cuda(e, "cudaMemsetAsync(err)");
    ws->err_cleared = true;
  }
  uint8_t* A = static_cast<uint8_t*>(ws->tc_aux.ptr);
  auto F = [&](size_t off) { return reinterpret_cast<float*>(A + off); };
  __nv_bfloat16* qbf = reinterpret_cast<__nv_bfloat16*>(A + o_qbf);
  int32_t* ccount = reinterpret_cast<int32_t*>(A + o_cc);
  int32_t* fallbacks = ccount + nq;
  uint64_t* cand = reinterpret_cast<uint64_t*>(A + o_cd);

  cudaError_t e = cudaSuccess;
  TcQueryParams qp{};
  qp.queries = d_queries;
  qp.nq = nq;
  qp.dim = static_cast<int32_t>(corpus->dim);
  qp.ld16 = ld16;
  qp.metric = metric;
  qp.cs = tc_stats_for(corpus, metric, i8);
  qp.qbf = qbf;
  qp.q8 = reinterpret_cast<int8_t*>(qbf);
  qp.qn_exact = F(o_qn);
  qp.alpha = F(o_al);
  qp.gamma = F(o_ga);
  qp.eps = F(o_ep);
  qp.scale = F(o_sc);
  qp.nq_pad = nq_pad;
  qp.ccount = ccount;
  // Fused pass: each block streams a static share of about 85 % of the
  // tiles (its sample tiles first), and the tail is claimed tile by tile, so
  // that blocks whose stream runs faster take more of it: the blocks' rates
  // differ by several percent, which a static split leaves as idle SMs at
  // the end of the pass.
  int64_t static_tiles = 0;
  if (fused) {
    static_tiles = std::max<int64_t>(samp_tiles, rtiles_all * 17 / (20 * groups_full));
    if (static_tiles * groups_full > rtiles_all) static_tiles = 0;
  }
  qp.pool = static_tiles > 0 ? reinterpret_cast<unsigned long long*>(A + o_pl) : nullptr;
  cudaEvent_t st_stop = stage_begin(ws, stream, MANS_STAGE_QUERY_PREP);
  if (i8)
    tc_query_prep_kernel<true><<<static_cast<unsigned>((nq_pad + kPrepWarps - 1) / kPrepWarps),
                                   kPrepWarps * 32, 0, stream>>>(qp);
  else
    tc_query_prep_kernel<false><<<static_cast<unsigned>((nq_pad + kPrepWarps - 1) / kPrepWarps),
                                    kPrepWarps * 32, 0, stream>>>(qp);
  if ((e = cudaGetLastError()) != cudaSuccess) return fail_cuda(e, "tc query prep launch");
  timing_end(st_stop, stream);

  CUtensorMap map_q;
  if ((rc = encode_tc_map(&map_q, qbf, nq_pad, corpus->dim, ld16, kQM, i8)) != MANS_OK) return rc;
  const CUtensorMap& map_r = i8 ? corpus->tc8_map : corpus->tc_map;
  const size_t smem = lay.total;
  if (lay.stages < 2) return fail(MANS_ERR_SEARCH, "dimension too large for the tensor-core pass");
  const void* kd = i8 ? reinterpret_cast<const void*>(tc_scan_kernel<kDense, true>)
                     : reinterpret_cast<const void*>(tc_scan_kernel<kDense, false>);
  const void* kp_ = i8 ? reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, true>)
                       : reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, false>);
  const void* kb_ = i8 ? reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, true>)
                       : reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, false>);
  if (smem > static_cast<size_t>(ctx->max_smem))
    return fail(MANS_ERR_SEARCH, "tensor-core pass needs more shared memory than the device has");
  if ((rc = tc_configure(ctx)) != MANS_OK) return rc;
  if (corpus->dim * sizeof(float) > 48 * 1024)
    return fail(MANS_ERR_SEARCH, "dimension too large for the tensor-core re-rank");

  TcParams tp{};
  tp.row_beta = metric == kL2 ? corpus->norms : nullptr;  // the exact path's fp32 |r|^2
  tp.row_w = i8 ? (metric == kCosine ? corpus->tc8_wcos : corpus->tc8_u) : nullptr;
  // the row terms travel by bulk copies of 16-byte pieces from tile starts
  if ((reinterpret_cast<uintptr_t>(tp.row_beta) | reinterpret_cast<uintptr_t>(tp.row_w)) & 15u)
    return fail(MANS_ERR_SEARCH, "row terms not 16-byte aligned");
  tp.stream_queries = stream_q;
  tp.nq = nq;
  tp.dim = static_cast<int32_t>(corpus->dim);
  tp.qblocks = static_cast<int32_t>(qblocks);
  tp.q_alpha = F(o_al);
  tp.q_gamma = F(o_ga);
  tp.q_c = F(o_cq);
  tp.err = static_cast<int*>(ws->err.ptr);
  // 2. sample pass (dense) and 3. thresholds -- inside the full pass when fused
  if (!fused) {
  tp.row0 = 0;
  tp.rows = sample;
  tp.dense_out = F(o_dn);
  tp.dense_ld = dld;
  tp.dense_group = dgroup;
  // lockstep grouping when every query block gets at least one block
  tp.groups = qblocks <= ctx->num_sms ? static_cast<int32_t>(ctx->num_sms / qblocks) : 0;
  const int64_t units_s = (sample + kRN - 1) / kRN * qblocks;
  int grid_s = static_cast<int>(std::min<int64_t>(units_s, ctx->num_sms));
  if (tp.groups > 0) {
    tp.groups = static_cast<int32_t>(std::min<int64_t>(tp.groups, (sample + kRN - 1) / kRN));
    grid_s = static_cast<int>(tp.groups * qblocks);
  }
  st_stop = stage_begin(ws, stream, MANS_STAGE_SAMPLE);
  {
    void* args[] = {const_cast<CUtensorMap*>(&map_q), const_cast<CUtensorMap*>(&map_r), &tp};
    e = launch_pdl(ctx, kd, dim3(grid_s), dim3(kTcThreads), smem, stream, args, false);
  }
  if (e != cudaSuccess) return fail_cuda(e, "tc sample launch");
  timing_end(st_stop, stream);
  // 3. thresholds
  // one wave of queries: wide blocks over a staged row (latency); larger
  // batches: narrow blocks reading global memory (occupancy)
  const bool one_wave = nq <= ctx->num_sms;
  const int staged =
      one_wave && dld * sizeof(float) <= static_cast<size_t>(kThresholdStageMax) ? 1 : 0;
  const size_t th_smem = staged ? dld * sizeof(float) : 0;
  st_stop = stage_begin(ws, stream, MANS_STAGE_THRESHOLD);
  {
    float* a_dn = F(o_dn);
    int64_t a_ld = dld, a_rows = dvals, a_nq = nq;
    int32_t a_k = keff;
    int a_staged = staged, a_metric = metric;
    float *a_ep = F(o_ep), *a_al = F(o_al), *a_ga = F(o_ga), *a_sc = F(o_sc), *a_th = F(o_th),
          *a_cq = F(o_cq);
    if (!one_wave && dld <= kThrWarpMax) {
      // many queries, short samples: one warp per query
      void* args[] = {&a_dn, &a_ld, &a_rows, &a_k, &a_nq, &a_ep, &a_al, &a_ga, &a_sc, &a_th, &a_cq};
      e = launch_pdl(ctx, reinterpret_cast<const void*>(tc_threshold_warp_kernel),
                     dim3(static_cast<unsigned>((nq + kThrWarps - 1) / kThrWarps)),
                     dim3(kThrWarps * 32), 0, stream, args, false);
    } else {
      void* args[] = {&a_dn, &a_ld, &a_rows, &a_k, &a_staged, &a_ep, &a_al, &a_ga, &a_sc,
                      &a_metric, &a_th, &a_cq};
      e = launch_pdl(ctx, reinterpret_cast<const void*>(tc_threshold_kernel),
                     dim3(static_cast<unsigned>(nq)), dim3(one_wave ? kThresholdThreads : 256),
                     th_smem, stream, args, false);
    }
  }
  if (e != cudaSuccess) return fail_cuda(e, "tc threshold launch");
  timing_end(st_stop, stream);
  }
  // 4. full filtered pass
  tp.rows = n;
  tp.dense_out = nullptr;
  tp.cand = cand;
  tp.cand_count = ccount;
  tp.cand_cap = cap;
  const int64_t units = (n + kRN - 1) / kRN * qblocks;
  int grid = static_cast<int>(std::min<int64_t>(units, ctx->num_sms));
  tp.groups = qblocks <= ctx->num_sms ? static_cast<int32_t>(ctx->num_sms / qblocks) : 0;
  if (tp.groups > 0) {
    tp.groups = static_cast<int32_t>(std::min<int64_t>(tp.groups, (n + kRN - 1) / kRN));
    grid = static_cast<int>(tp.groups * qblocks);
  }
  // CTA pairs (bf16, two or more query blocks, the query block resident):
  // pairs of query blocks walk row groups in step, `groups` pairs per pair
  // of query blocks, as many pairs as fit on the device at once.
  const TcLayout lay2 = tc_layout(lay.nk, stream_q, true);
  const int64_t qsb = (qblocks + 1) / 2;
  const int max_pairs = (!i8 && !fused && qblocks >= 2 && lay2.resident && !stream_q)
                            ? tc_pair_capacity(ctx, lay2.total)
                            : 0;
  const bool pair = max_pairs > 0 && qsb <= max_pairs;
  if (pair) {
    tp.groups = static_cast<int32_t>(std::min<int64_t>(max_pairs / qsb, (n + kRN - 1) / kRN));
    grid = static_cast<int>(2 * tp.groups * qsb);
  }
  tp.row0 = 0;
  {
    // Reservation size: padding may take at most 1/8 of the list over the
    // (block, column part) writers of one query.  The fused pass (at most 128
    // queries, HBM bound) reserves exactly what each chunk needs: no padding
    // for the re-rank to read past.
    const int64_t writers = 4 * (tp.groups > 0 ? tp.groups : grid / qblocks + 1);
    tp.cand_reserve = fused ? 1
                            : static_cast<int32_t>(std::max<int64_t>(
                                  1, std::min<int64_t>(8, cap / (8 * writers))));
  }
  if (fused) {
    tp.sample_tiles = static_cast<int32_t>(samp_tiles);
    tp.samp_out = F(o_dn);
    tp.samp_ld = samp_ld;
    tp.bar = static_cast<unsigned long long*>(ws->tc_bar.ptr);
    tp.bar_base = ws->tc_bar_base;
    tp.pool = qp.pool;
    tp.static_tiles = static_tiles;
    tp.pool_first = static_tiles * grid;
    tp.pool_tiles = rtiles_all - static_tiles * grid;
    tp.k = keff;
    tp.q_eps = F(o_ep);
    tp.q_scale = F(o_sc);
    tp.thr_out = F(o_th);
    tp.c_out = F(o_cq);
  }
  st_stop = stage_begin(ws, stream, MANS_STAGE_PASS);
  cudaEvent_t stop = timing_begin(ws, stream);
  if (fused) {
    // co-resident blocks (one per SM) meet at two grid barriers
    const void* fn =
        metric == kL2 ? (i8 ? reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, true, true>)
                            : reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, false, true>))
                      : (i8 ? reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, true, true>)
                            : reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, false, true>));
    void* args[] = {const_cast<CUtensorMap*>(&map_q), const_cast<CUtensorMap*>(&map_r), &tp};
    e = launch_pdl(ctx, fn, dim3(grid), dim3(kTcThreads), smem, stream, args, true);
    if (e == cudaSuccess) ws->tc_bar_base += 2ull * static_cast<unsigned long long>(grid);
  } else if (pair) {
    const void* fn = metric == kL2
                         ? reinterpret_cast<const void*>(tc_scan_kernel<kFilterBias, false, false, true>)
                         : reinterpret_cast<const void*>(tc_scan_kernel<kFilterPlain, false, false, true>);
    void* args[] = {const_cast<CUtensorMap*>(&map_q), &corpus->tc_map_half, &tp};
    e = launch_pair(ctx, fn, dim3(grid), dim3(kTcThreads), lay2.total, stream, args);
  } else {
    // the bf16 plain filter (cosine, inner product) runs the lean layout
    const size_t smem_pass =
        (metric != kL2 && !i8) ? tc_layout(lay.nk, stream_q, false, true).total : smem;
    void* args[] = {const_cast<CUtensorMap*>(&map_q), const_cast<CUtensorMap*>(&map_r), &tp};
    e = launch_pdl(ctx, metric == kL2 ? kb_ : kp_, dim3(grid), dim3(kTcThreads), smem_pass, stream,
                   args, false);
  }
  if (e != cudaSuccess) return fail_cuda(e, "tc scan launch");
  timing_end(stop, stream);
  timing_end(st_stop, stream);
  // 5. certify + exact re-rank
  RerankParams rp{};
  rp.cand = cand;
  rp.cand_count = ccount;
  rp.cand_cap = cap;
  rp.thr = F(o_th);
  rp.eps = F(o_ep);
  rp.qn_exact = F(o_qn);
  rp.queries = d_queries;
  rp.rows = corpus->rows;
  rp.ld = corpus->ld;
  rp.norms = corpus->norms;
  rp.n = n;
  rp.dim = static_cast<int32_t>(corpus->dim);
  rp.metric = metric;
  rp.id_offset = corpus->id_offset;
  rp.k = keff;
  rp.kp = kp;
  rp.kout = kout;
  rp.out_dist = d_out_dist;
  rp.out_ids = d_out_ids;
  rp.out_counts = d_out_counts;
  rp.fallbacks = fallbacks;
  rp.region = rerank_region_bytes(nq, ctx->num_sms, corpus->dim);
  rp.max_band = rerank_max_band(nq, ctx->num_sms);
  st_stop = stage_begin(ws, stream, MANS_STAGE_RERANK);
  {
    void* args[] = {&rp};
    e = launch_pdl(ctx, reinterpret_cast<const void*>(tc_rerank_kernel),
                   dim3(static_cast<unsigned>(nq)), dim3(kRerankThreads),
                   rerank_smem_bytes(corpus->dim, rp.max_band, rp.region), stream, args, false);
  }
  if (e != cudaSuccess) return fail_cuda(e, "tc rerank launch");
  timing_end(st_stop, stream);
  ws->tc_fallbacks = fallbacks;
  ws->launches += fused ? 3 : 5;
  ws->last_path = i8 ? 2 : 1;
  return MANS_OK;
}

void tc_free_corpus(mans_corpus* c) {
  if (c->tc_rows) cudaFree(c->tc_rows);
  if (c->tc_stats) cudaFree(c->tc_stats);
  c->tc_rows = nullptr;
  c->tc_stats = nullptr;
  c->tc_ready = false;
  if (c->tc8_rows) cudaFree(c->tc8_rows);
  if (c->tc8_u) cudaFree(c->tc8_u);
  if (c->tc8_wcos) cudaFree(c->tc8_wcos);
  if (c->tc8_stats) cudaFree(c->tc8_stats);
  c->tc8_rows = nullptr;
  c->tc8_u = nullptr;
  c->tc8_wcos = nullptr;
  c->tc8_stats = nullptr;
  c->tc8_ready = false;
}

}  // namespace mans
