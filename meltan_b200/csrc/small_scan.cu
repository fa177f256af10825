// small_scan.cu -- exact search of a query batch over a small corpus.
//
// The centroid steps of the index searches (IVF-flat top-nprobe,
// IVFFlatSearch.swift:214-291; IVF-PQ coarse selection, IVFPQIndex.swift
// :484-512) and of the device builds (assignRows, IVFFlatSearch.swift
// :633-703; nearestCoarseCentroid, IVFPQIndex.swift:514-550) scan a few
// thousand centroids for hundreds to millions of queries.  The streaming scan
// (scan.cu) parallelises over corpus tiles and so leaves most SMs idle on a
// corpus of 16 tiles; here a block takes a 32-query x 64-row tile of the
// score matrix, every thread a 2 x 4 register block, with both operands
// staged in shared memory 64 dimensions at a time.  Each score is the same
// sequential fp32 sum in index order as the streaming scan (separately
// rounded products and sums; SIMDDistance L2 as the sum of (q - r)^2), and the
// same finalize, so the results are bit-equal.  A second kernel sorts each
// query's (distance, id) keys in shared memory and writes the k smallest.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"

namespace mans {
namespace {

constexpr int kSsThreads = 256;
constexpr int kSsQ = 32;       // queries per block
constexpr int kSsR = 64;       // corpus rows per block
constexpr int kSsD = 64;       // dimensions staged per step
constexpr int kSsQPitch = kSsQ + 2;  // even: 8-byte aligned pairs, 2-way staging conflicts
constexpr int kSsRPitch = kSsR + 4;  // multiple of 4: 16-byte aligned quads
constexpr int kSelThreads = 512;
constexpr size_t kScoreBudget = 64ull << 20;  // bytes of one chunk of the score matrix

struct SsParams {
  const float* queries;  // nq x dim (dense)
  int64_t nq;
  int32_t dim;
  const float* rows;  // n x ld
  int64_t ld;
  int64_t n;
  const float* norms;  // |r|^2 per row, null for IP
  int32_t metric;
  int32_t mode;   // kModeHost / kModeSimd
  float* scores;  // nq x sld
  int64_t sld;
  int32_t need_qn;  // the finalize reads |q|^2 (cosine; L2 of the host formula)
};

// Scores of queries [32 y, 32 y + 32) x rows [64 x, 64 x + 64).  Thread t
// owns queries 2 (t / 16) + {0, 1} and rows 4 (t % 16) + {0..3}.
template <bool DIFFSQ>
__global__ void __launch_bounds__(kSsThreads) small_scores_kernel(const SsParams p) {
  __shared__ __align__(16) float qs[kSsD * kSsQPitch];  // [d][query]
  __shared__ __align__(16) float rs[kSsD * kSsRPitch];  // [d][row]
  __shared__ float qn_s[kSsQ];
  const int tid = threadIdx.x;
  const int tq = tid >> 4;
  const int tr = tid & 15;
  const int64_t q0 = static_cast<int64_t>(blockIdx.y) * kSsQ;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kSsR;
  float acc[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  float qn = 0.0f;  // threads 0..31: |q|^2 of query q0 + tid, index order across the steps
  for (int d0 = 0; d0 < p.dim; d0 += kSsD) {
    const int dn = min(kSsD, p.dim - d0);
    __syncthreads();  // the previous step's operands are consumed
    for (int i = tid; i < kSsQ * kSsD; i += kSsThreads) {
      const int qi = i / kSsD, d = i - qi * kSsD;
      const int64_t q = q0 + qi;
      qs[d * kSsQPitch + qi] = (q < p.nq && d < dn) ? __ldg(p.queries + q * p.dim + d0 + d) : 0.0f;
    }
    for (int i = tid; i < kSsR * kSsD; i += kSsThreads) {
      const int ri = i / kSsD, d = i - ri * kSsD;
      const int64_t r = r0 + ri;
      rs[d * kSsRPitch + ri] = (r < p.n && d < dn) ? __ldg(p.rows + r * p.ld + d0 + d) : 0.0f;
    }
    __syncthreads();
    if (p.need_qn && tid < kSsQ)
      for (int d = 0; d < dn; ++d) {
        const float x = qs[d * kSsQPitch + tid];
        qn = __fadd_rn(qn, __fmul_rn(x, x));
      }
    // only the dimensions of the step: an extra +0 term could turn a -0 dot into +0
#pragma unroll 4
    for (int d = 0; d < dn; ++d) {
      const float2 qv = *reinterpret_cast<const float2*>(qs + d * kSsQPitch + 2 * tq);
      const float4 rv = *reinterpret_cast<const float4*>(rs + d * kSsRPitch + 4 * tr);
      const float qq[2] = {qv.x, qv.y};
      const float rr[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (DIFFSQ) {
            const float t = __fsub_rn(qq[i], rr[j]);
            acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(t, t));
          } else {
            acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(rr[j], qq[i]));
          }
        }
    }
  }
  if (tid < kSsQ) qn_s[tid] = qn;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int64_t q = q0 + 2 * tq + i;
    if (q >= p.nq) continue;
    const float qnv = qn_s[2 * tq + i];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t r = r0 + 4 * tr + j;
      if (r >= p.n) continue;
      const float vn = p.norms ? __ldg(p.norms + r) : 0.0f;
      p.scores[q * p.sld + r] = p.mode == kModeSimd ? finalize_simd(p.metric, acc[i][j], qnv, vn)
                                                    : finalize_distance(p.metric, acc[i][j], qnv, vn);
    }
  }
}

// Per query (block): the keff smallest (distance, id) keys of its n scores,
// ascending; slots keff .. kout - 1 empty.  keff = 1 is a block minimum.
// Otherwise a radix select (four 8-bit passes over the order-preserving
// 32-bit image of the distances, staged in shared memory) finds T, the
// keff-th smallest distance; the keys of distance <= T -- every key below T
// and all keys tied at T, whose ids decide -- are sorted and the first keff
// written.  Far more ties at T than the staging room leaves (duplicate rows)
// fall back to sorting all n keys.
__global__ void __launch_bounds__(kSelThreads) small_select_kernel(
    const float* __restrict__ scores, int64_t sld, int64_t n, const uint32_t* __restrict__ ids,
    uint32_t id_offset, int32_t keff, int32_t kout, int np2, float* __restrict__ out_dist,
    uint32_t* __restrict__ out_ids, int32_t* __restrict__ out_counts) {
  extern __shared__ uint64_t keys[];  // np2 keys; the radix select uses it as
                                      // [n ordered distances | np2/2 candidate keys]
  __shared__ uint64_t wmin[kSelThreads / 32];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel_prefix, sel_rank, ncand;
  const int tid = threadIdx.x;
  const int64_t q = blockIdx.x;
  const float* row = scores + q * sld;
  auto id_of = [&](int64_t i) {
    return ids ? __ldg(ids + i) : static_cast<uint32_t>(i + id_offset);
  };
  int sorted_n = 0;  // keys[0 .. keff) hold the result once set
  if (keff == 1) {
    uint64_t m = kKeyMax;
    for (int64_t i = tid; i < n; i += kSelThreads) {
      const uint64_t x = make_key(__ldcg(row + i), id_of(i));
      m = x < m ? x : m;
    }
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t x = __shfl_xor_sync(0xFFFFFFFFu, m, o);
      m = x < m ? x : m;
    }
    if ((tid & 31) == 0) wmin[tid >> 5] = m;
    __syncthreads();
    if (tid < 32) {
      m = tid < kSelThreads / 32 ? wmin[tid] : kKeyMax;
      for (int o = 16; o > 0; o >>= 1) {
        const uint64_t x = __shfl_xor_sync(0xFFFFFFFFu, m, o);
        m = x < m ? x : m;
      }
      if (tid == 0) keys[0] = m;
    }
    __syncthreads();
    sorted_n = 1;
  } else {
    uint32_t* u = reinterpret_cast<uint32_t*>(keys);  // n ordered distances
    uint64_t* cand = keys + np2 / 2;                  // np2 / 2 candidate keys
    const int cap = np2 / 2;
    for (int64_t i = tid; i < n; i += kSelThreads) u[i] = float_to_ordered(__ldcg(row + i));
    if (tid == 0) {
      sel_prefix = 0;
      sel_rank = static_cast<uint32_t>(keff);
      ncand = 0;
    }
    uint32_t mask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
      __syncthreads();
      const uint32_t prefix = sel_prefix;
      for (int64_t i = tid; i < n; i += kSelThreads)
        if ((u[i] & mask) == prefix) atomicAdd(&hist[(u[i] >> shift) & 255u], 1u);
      __syncthreads();
      if (tid < 32) {
        // digit holding the rank-th value: lane l sums bins 8l .. 8l + 7
        uint32_t c[8], run = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          c[j] = hist[tid * 8 + j];
          run += c[j];
        }
        uint32_t incl = run;
        for (int o = 1; o < 32; o <<= 1) {
          const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (tid >= o) incl += y;
        }
        const uint32_t rank = sel_rank;
        uint32_t before = incl - run;
        if (before < rank && incl >= rank) {
          int d = 0;
          while (before + c[d] < rank) before += c[d++];
          sel_prefix = prefix | (static_cast<uint32_t>(tid * 8 + d) << shift);
          sel_rank = rank - before;
        }
      }
      mask |= 255u << shift;
      __syncthreads();
    }
    const uint32_t t = sel_prefix;  // keff-th smallest ordered distance
    for (int64_t i = tid; i < n; i += kSelThreads) {
      if (u[i] <= t) {
        const uint32_t at = atomicAdd(&ncand, 1u);
        if (at < static_cast<uint32_t>(cap))
          cand[at] = (static_cast<uint64_t>(u[i]) << 32) | id_of(i);
      }
    }
    __syncthreads();
    const int c = static_cast<int>(ncand);
    if (c <= cap) {
      int m = 1;
      while (m < c) m <<= 1;
      for (int i = c + tid; i < m; i += kSelThreads) cand[i] = kKeyMax;
      __syncthreads();
      bitonic_sort_keys<kSelThreads>(cand, m, tid, 0);
      for (int i = tid; i < keff; i += kSelThreads) keys[i] = cand[i];  // keff <= c < np2 / 2
      __syncthreads();
      sorted_n = keff;
    }
  }
  if (sorted_n == 0) {
    // heavy ties: sort every key
    for (int i = tid; i < np2; i += kSelThreads)
      keys[i] = i < n ? make_key(__ldcg(row + i), id_of(i)) : kKeyMax;
    __syncthreads();
    bitonic_sort_keys<kSelThreads>(keys, np2, tid, 0);
  }
  for (int i = tid; i < kout; i += kSelThreads) {
    const bool have = i < keff;
    out_dist[q * kout + i] = have ? key_distance(keys[i]) : __int_as_float(0x7F800000);
    out_ids[q * kout + i] = have ? key_id(keys[i]) : kEmptyId;
  }
  if (tid == 0) out_counts[q] = keff;
}

}  // namespace

bool small_batch_applies(const mans_corpus* corpus, int64_t nq) {
  return nq >= kSmallBatchMinQueries && corpus->n > 0 && corpus->n <= kSmallBatchMaxRows;
}

int32_t run_small_batch_search(mans_ctx* ctx, const mans_corpus* corpus, mans_workspace* ws,
                               const float* d_queries, int64_t nq, int32_t kout, int32_t metric,
                               float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                               cudaStream_t stream, int mode) {
  const int64_t n = corpus->n;
  const int32_t keff = static_cast<int32_t>(std::min<int64_t>(kout, n));
  const int64_t sld = (n + 3) / 4 * 4;
  int64_t chunk = static_cast<int64_t>(kScoreBudget / (static_cast<size_t>(sld) * sizeof(float)));
  chunk = std::max<int64_t>(kSsQ, chunk / kSsQ * kSsQ);
  chunk = std::min<int64_t>(chunk, 65535ll * kSsQ);  // query tiles fit grid.y
  chunk = std::min<int64_t>(chunk, (nq + kSsQ - 1) / kSsQ * kSsQ);
  int32_t rc = ws->small_scores.reserve(static_cast<size_t>(chunk) * sld * sizeof(float));
  if (rc != MANS_OK) return rc;
  const int np2 = pow2_at_least(static_cast<int>(n));
  const size_t sel_smem = keff == 1 ? sizeof(uint64_t) : static_cast<size_t>(np2) * sizeof(uint64_t);
  cudaError_t e = cudaFuncSetAttribute(small_select_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(std::max<size_t>(sel_smem, 1)));
  if (e != cudaSuccess) return fail_cuda(e, "small-corpus select configure");
  const bool diffsq = mode == kModeSimd && metric == MANS_METRIC_L2;
  SsParams p{};
  p.dim = static_cast<int32_t>(corpus->dim);
  p.rows = corpus->rows;
  p.ld = corpus->ld;
  p.n = n;
  p.norms = metric == MANS_METRIC_IP ? nullptr : corpus->norms;
  p.metric = metric;
  p.mode = mode;
  p.scores = static_cast<float*>(ws->small_scores.ptr);
  p.sld = sld;
  p.need_qn = metric != MANS_METRIC_IP && !diffsq;
  for (int64_t c0 = 0; c0 < nq; c0 += chunk) {
    const int64_t cq = std::min(chunk, nq - c0);
    p.queries = d_queries + c0 * corpus->dim;
    p.nq = cq;
    const dim3 grid(static_cast<unsigned>((n + kSsR - 1) / kSsR),
                    static_cast<unsigned>((cq + kSsQ - 1) / kSsQ));
    cudaEvent_t stop = timing_begin(ws, stream);
    if (diffsq)
      small_scores_kernel<true><<<grid, kSsThreads, 0, stream>>>(p);
    else
      small_scores_kernel<false><<<grid, kSsThreads, 0, stream>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "small-corpus score launch");
    timing_end(stop, stream);
    small_select_kernel<<<static_cast<unsigned>(cq), kSelThreads, sel_smem, stream>>>(
        p.scores, sld, n, corpus->ids, corpus->id_offset, keff, kout, np2,
        d_out_dist + c0 * kout, d_out_ids + c0 * kout, d_out_counts + c0);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "small-corpus select launch");
    ws->launches += 2;
  }
  return MANS_OK;
}

}  // namespace mans
