// pq.cu -- IVF-PQ search (coarse probe, per-list LUT + ADC, newest-first merge)
// and the single-list ADC of GPUADCSearch.
//
// Restates _IVFPQIndex.search (Sources/MetalANNS/IVFPQIndex.swift:177-226):
//   1. coarse scores SIMDDistance.distance(q, c) for every coarse centroid,
//      ranked in a BoundedSortedList of capacity nprobe (:484-512);
//   2. for each probed cluster in that order: residual q - c (:366-368), the
//      LUT of ProductQuantizer.distanceTableFlattened over the residual
//      (ProductQuantizer.swift:223-253) and the sequential ADC sum of
//      cpuADCDistances (IVFPQIndex.swift:418-452);
//   3. every candidate inserted, in probe order then list order, into a
//      BoundedSortedList of capacity k (BoundedSelection.swift:158-214).
//
// BoundedSortedList keeps the list sorted by score with equal scores newest
// first, rejects an equal-score newcomer when full and evicts the last entry
// on overflow.  Its final content has a closed form that the device computes
// from the 2K smallest candidates by (score, insertion sequence):
//   w = K-th smallest score, L = candidates with score < w (always kept,
//   |L| = l < K), E = candidates with score == w in insertion order.  Once the
//   list first holds K entries it stays full, so only E entries that arrive
//   while it is filling are inserted -- the E entries among the first K
//   arrivals of L u E -- and later L arrivals evict the oldest of them.  The
//   kept E entries are the newest K - l inserted ones.  Those first K
//   arrivals contain at most K E entries, which are the K earliest E entries,
//   and all of L u {K earliest E} lies within the 2K smallest (score, seq)
//   keys.  Output order: score ascending, newest first among equal scores.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"

#include <cub/cub.cuh>

using namespace mans;

struct mans_ivfpq {
  mans_ctx* ctx = nullptr;
  int32_t nlist = 0;
  int64_t n = 0;
  int64_t dim = 0;
  int32_t m = 0;
  int32_t ks = 256;
  int32_t sub = 0;
  int32_t metric = 1;
  int64_t max_len = 0;
  int64_t max_pos = 0;  // largest list position an entry reports
  mans_corpus* coarse = nullptr;  // coarse centroids (SIMDDistance scoring)
  float* codebooks = nullptr;     // m x ks x sub
  uint8_t* codes = nullptr;       // list-contiguous, n x m
  uint32_t* ids = nullptr;        // list-contiguous internal ids
  uint32_t* pos = nullptr;        // global position of each entry in its list (shards)
  int64_t* offsets = nullptr;     // nlist + 1
};

namespace mans {

// One distance-table entry of W queries side by side (the grouped ADC reads
// all W with one shared-memory load).
template <int W>
struct LutVec;
template <>
struct LutVec<1> {
  using T = float;
  __device__ static float get(const T& v, int j) { return v; }
  __device__ static T make(const float* v) { return v[0]; }
};
template <>
struct LutVec<2> {
  using T = float2;
  __device__ static float get(const T& v, int j) { return j == 0 ? v.x : v.y; }
  __device__ static T make(const float* v) { return make_float2(v[0], v[1]); }
};
template <>
struct LutVec<4> {
  using T = float4;
  __device__ static float get(const T& v, int j) {
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
  }
  __device__ static T make(const float* v) { return make_float4(v[0], v[1], v[2], v[3]); }
};

namespace {

// Insertion sequence of a candidate: probe rank << pos_bits | list position,
// with pos_bits = 32 - ceil(log2(nprobe)) capped at 31 (a search needs every
// list position below 2^pos_bits: lists of up to 2^27 entries at nprobe 32).
inline int32_t seq_pos_bits(int32_t probe) {
  int rank_bits = 0;
  while ((1 << rank_bits) < probe) ++rank_bits;
  return std::min(31, 32 - rank_bits);
}
constexpr int kAdcThreads = 128;

struct ResolveParams {
  const float* in_score;
  const uint32_t* in_seq;
  const uint32_t* in_payload;  // null: payload derived from seq
  const int32_t* in_count;
  int32_t kin;
  int64_t nq;
  int32_t cap;  // K
  int32_t pos_bits;  // insertion sequence layout (see seq_pos_bits)
  // seq -> internal id mapping (IVF-PQ candidates); null: payload = seq
  const uint32_t* probe_lists;  // [nq][probe_stride]
  int32_t probe_stride;
  const int64_t* offsets;
  const uint32_t* ids;
  const uint32_t* pos;  // optional: each entry's position in its global list
  float* out_score;
  uint32_t* out_id;
  int32_t* out_count;
  int32_t kout;
};

__device__ __forceinline__ uint32_t seq_payload(const ResolveParams& p, int64_t q, uint32_t seq);

__device__ __forceinline__ uint32_t resolve_payload(const ResolveParams& p, int64_t q, int i) {
  uint32_t seq = p.in_seq[q * p.kin + i];
  if (p.in_payload) return p.in_payload[q * p.kin + i];
  return seq_payload(p, q, seq);
}

// Internal id of the entry with insertion sequence `seq` (probe rank, list
// position) among query q's probed lists.
__device__ __forceinline__ uint32_t seq_payload(const ResolveParams& p, int64_t q, uint32_t seq) {
  if (!p.probe_lists) return seq;
  uint32_t rank = seq >> p.pos_bits;
  uint32_t pos = seq & ((1u << p.pos_bits) - 1u);
  uint32_t list = p.probe_lists[q * p.probe_stride + rank];
  const int64_t off = p.offsets[list];
  if (!p.pos) return p.ids[off + pos];
  // entries that report positions in a larger (global) list: the entry with
  // that position, found by binary search (positions ascend within a list)
  int64_t lo = 0, hi = p.offsets[list + 1] - off;
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (p.pos[off + mid] < pos)
      lo = mid + 1;
    else
      hi = mid;
  }
  return p.ids[off + lo];
}

// One block per query.  Input rows are sorted by (score, seq) ascending.
__global__ void __launch_bounds__(256) bsl_resolve_kernel(const ResolveParams p) {
  __shared__ uint64_t keys[1024];
  __shared__ int sh_l, sh_e, sh_ins;
  const int64_t q = blockIdx.x;
  const int tid = threadIdx.x;
  const int c = p.in_count[q];
  const int K = p.cap;
  const float* sc = p.in_score + q * p.kin;
  const uint32_t* sq = p.in_seq + q * p.kin;
  int nout;
  int l = 0, e_first = 0, e_keep = 0;  // kept E entries: E[e_first, e_first + e_keep)
  if (c <= K) {
    nout = c;
    l = c;  // everything kept; output = input with equal-score runs reversed
  } else {
    const float w = sc[K - 1];
    if (tid == 0) {
      int a = 0;
      while (a < c && sc[a] < w) ++a;
      int b = a;
      while (b < c && sc[b] == w) ++b;
      sh_l = a;
      sh_e = b - a;
    }
    __syncthreads();
    l = sh_l;
    const int ecount = min(sh_e, K);  // the K earliest E entries (seq ascending)
    // first K arrivals among L u E': sort their sequences, tag E entries
    const int total = l + ecount;
    int n2 = 1;
    while (n2 < total) n2 <<= 1;
    for (int i = tid; i < n2; i += blockDim.x) {
      uint64_t key = kKeyMax;
      if (i < l) key = (static_cast<uint64_t>(sq[i]) << 1);
      else if (i < total) key = (static_cast<uint64_t>(sq[i]) << 1) | 1u;
      keys[i] = key;
    }
    __syncthreads();
    bitonic_sort_keys<256>(keys, n2, tid, 0);
    if (tid == 0) {
      int ins = 0;
      for (int i = 0; i < K && i < total; ++i) ins += static_cast<int>(keys[i] & 1u);
      sh_ins = ins;
    }
    __syncthreads();
    const int ins = sh_ins;
    e_keep = K - l;
    e_first = l + ins - e_keep;  // newest K - l of the inserted E entries
    nout = K;
  }
  // write: L with equal-score runs reversed (newest first), then kept E newest first
  for (int i = tid; i < l; i += blockDim.x) {
    // find the equal-score run [a, b) that holds i; position inside it reversed
    int a = i, b = i + 1;
    while (a > 0 && sc[a - 1] == sc[i]) --a;
    while (b < l && sc[b] == sc[i]) ++b;
    int src = a + (b - 1 - i);
    p.out_score[q * p.kout + i] = sc[src];
    p.out_id[q * p.kout + i] = resolve_payload(p, q, src);
  }
  for (int j = tid; j < e_keep; j += blockDim.x) {
    int src = e_first + (e_keep - 1 - j);
    p.out_score[q * p.kout + l + j] = sc[src];
    p.out_id[q * p.kout + l + j] = resolve_payload(p, q, src);
  }
  for (int i = nout + tid; i < p.kout; i += blockDim.x) {
    p.out_score[q * p.kout + i] = __int_as_float(0x7F800000);
    p.out_id[q * p.kout + i] = kEmptyId;
  }
  if (tid == 0) p.out_count[q] = nout;
}

struct AdcParams {
  const float* queries;     // nq x dim
  const float* coarse;      // coarse rows (ld pitch)
  int64_t coarse_ld;
  const float* codebooks;   // m x ks x sub
  const uint8_t* codes;     // packed n x m
  const uint32_t* pos;      // optional global list positions
  const int64_t* offsets;
  const uint32_t* probe_lists;  // [nq][probe]
  const int32_t* probe_counts;
  int32_t probe;
  int32_t pos_bits;         // insertion sequence layout (see seq_pos_bits)
  int64_t nq;
  int32_t dim, m, ks, sub, metric;
  int32_t k;   // candidates kept per (query, list)
  int32_t kp;
  int32_t sortn;            // running top-k buffer (power of two >= kp + block)
  uint64_t* slot_keys;      // [q*probe + p][kp]
  int32_t* slot_counts;
};

__device__ __forceinline__ float lut_entry(int metric, const float* r, const float* cb, int sub) {
  if (metric == kL2) {
    float s = 0.0f;
    for (int d = 0; d < sub; ++d) {
      float t = __fsub_rn(r[d], cb[d]);
      s = __fadd_rn(s, __fmul_rn(t, t));
    }
    return s;
  }
  float dot = 0.0f;
  for (int d = 0; d < sub; ++d) dot = __fadd_rn(dot, __fmul_rn(r[d], cb[d]));
  if (metric == kIP) return -dot;
  float na = 0.0f, nb = 0.0f;
  for (int d = 0; d < sub; ++d) na = __fadd_rn(na, __fmul_rn(r[d], r[d]));
  for (int d = 0; d < sub; ++d) nb = __fadd_rn(nb, __fmul_rn(cb[d], cb[d]));
  float denom = __fmul_rn(__fsqrt_rn(na), __fsqrt_rn(nb));
  if (denom < 1e-10f) return 1.0f;
  return __fsub_rn(1.0f, __fdiv_rn(dot, denom));
}

// The distance tables of W queries for one list (the index has ks == 256):
// entry (s, c) of query j at lut[s * 256 + c], component j.  Thread t of T
// fills the columns c = t, t + T, ... of every subspace s, so a subspace's
// residuals are loaded once per thread (broadcast reads) and no index is
// divided; each entry is lut_entry's sequential sum, in the same order.
template <int W, int T>
__device__ __forceinline__ void build_tables(const AdcParams& p,
                                             typename LutVec<W>::T* __restrict__ lut,
                                             const float* __restrict__ resid) {
  const int tid = threadIdx.x;
  const float* cb = p.codebooks;
  if (p.metric == kL2 && p.sub == 8) {
    for (int s = 0; s < p.m; ++s) {
      float r[W][8];
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const float4* r4 = reinterpret_cast<const float4*>(resid + j * p.dim + s * 8);
        const float4 a = r4[0], b = r4[1];
        r[j][0] = a.x; r[j][1] = a.y; r[j][2] = a.z; r[j][3] = a.w;
        r[j][4] = b.x; r[j][5] = b.y; r[j][6] = b.z; r[j][7] = b.w;
      }
#pragma unroll 2
      for (int c = tid; c < 256; c += T) {
        const float4* c4 =
            reinterpret_cast<const float4*>(cb + (static_cast<int64_t>(s) * 256 + c) * 8);
        const float4 a = __ldg(c4), b = __ldg(c4 + 1);
        const float cw[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        float v[W];
#pragma unroll
        for (int j = 0; j < W; ++j) {
          float sum = 0.0f;
#pragma unroll
          for (int d = 0; d < 8; ++d) {
            const float t = __fsub_rn(r[j][d], cw[d]);
            sum = __fadd_rn(sum, __fmul_rn(t, t));
          }
          v[j] = sum;
        }
        lut[s * 256 + c] = LutVec<W>::make(v);
      }
    }
  } else {
    for (int s = 0; s < p.m; ++s)
      for (int c = tid; c < 256; c += T) {
        float v[W];
#pragma unroll
        for (int j = 0; j < W; ++j)
          v[j] = lut_entry(p.metric, resid + j * p.dim + s * p.sub,
                           cb + (static_cast<int64_t>(s) * 256 + c) * p.sub, p.sub);
        lut[s * 256 + c] = LutVec<W>::make(v);
      }
  }
}

// Persistent: block b handles items b, b + grid, ... ; item = (query, probe rank).
// One code row: its m bytes as 16-, 4- or 1-byte loads (the row stride is m
// bytes, so the wide loads are aligned whenever m is a multiple of the width).
__device__ __forceinline__ float adc_sum(const float* lut, int ks, const uint8_t* code, int m) {
  float total = 0.0f;
  if ((m & 15) == 0) {
    for (int s0 = 0; s0 < m; s0 += 16) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(code + s0));
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const uint32_t c = (words[j >> 2] >> (8 * (j & 3))) & 0xFFu;
        total = __fadd_rn(total, lut[(s0 + j) * ks + c]);
      }
    }
  } else if ((m & 3) == 0) {
    for (int s0 = 0; s0 < m; s0 += 4) {
      const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(code + s0));
#pragma unroll
      for (int j = 0; j < 4; ++j)
        total = __fadd_rn(total, lut[(s0 + j) * ks + ((w >> (8 * j)) & 0xFFu)]);
    }
  } else {
    for (int s = 0; s < m; ++s) total = __fadd_rn(total, lut[s * ks + __ldg(code + s)]);
  }
  return total;
}

// Block b handles items b, b + grid, ... ; item = (query, probe rank).  Small
// blocks (several resident per SM) hide the latency of the per-item steps:
// residual, LUT in shared memory, sequential ADC per code, the item's k
// smallest (score, seq) keys.  WARP_TOPK (k <= 32): every warp keeps its own
// 32 smallest keys in registers (one per lane; a batch of 32 codes that beats
// the k-th is sorted by shuffles and merged in), and warp 0 merges the four
// lists at the end -- no block barrier while scanning.  Otherwise a running
// top-k in shared memory (append queue + block bitonic merges).
template <bool WARP_TOPK>
__global__ void __launch_bounds__(kAdcThreads) pq_adc_kernel(const AdcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<size_t>(smem_raw) + 15) / 16 * 16);
  uint64_t* topbuf = reinterpret_cast<uint64_t*>(base);
  float* lut = reinterpret_cast<float*>(base + (WARP_TOPK ? 0 : static_cast<size_t>(p.sortn) * 8));
  float* resid = lut + p.m * p.ks;
  __shared__ uint64_t thr;
  __shared__ int qc, nb;
  __shared__ uint64_t wlist[kAdcThreads / 32][32];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t items = p.nq * p.probe;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t q = it / p.probe;
    const int pr = static_cast<int>(it - q * p.probe);
    __syncthreads();  // previous item fully done with the shared buffers
    if (pr >= p.probe_counts[q]) {
      if (tid == 0) p.slot_counts[it] = 0;
      continue;
    }
    const uint32_t list = p.probe_lists[q * p.probe + pr];
    const int64_t off = p.offsets[list];
    const int64_t len = p.offsets[list + 1] - off;
    if (len == 0) {  // an empty list (a shard holding other lists): no table to build
      if (tid == 0) p.slot_counts[it] = 0;
      continue;
    }
    for (int d = tid; d < p.dim; d += kAdcThreads)
      resid[d] = __fsub_rn(p.queries[q * p.dim + d], p.coarse[list * p.coarse_ld + d]);
    if (!WARP_TOPK && tid == 0) {
      thr = kKeyMax;
      qc = 0;
      nb = 0;
    }
    __syncthreads();
    build_tables<1, kAdcThreads>(p, lut, resid);
    __syncthreads();
    if (WARP_TOPK) {
      uint64_t best = kKeyMax;  // lane i: this warp's (i+1)-th smallest key
      uint64_t kth = kKeyMax;   // this warp's k-th smallest key
      // m = 16: one 16-byte code row per lane, the next batch's row (and list
      // position) loaded before the current one is scored
      const bool wide = p.m == 16;
      const uint4* crow = reinterpret_cast<const uint4*>(p.codes + off * 16);
      auto fetch = [&](int64_t e, uint4& w, uint32_t& ps) {
        if (wide && e < len) {
          w = __ldg(crow + e);
          ps = p.pos ? __ldg(p.pos + off + e) : static_cast<uint32_t>(e);
        }
      };
      uint4 w = make_uint4(0u, 0u, 0u, 0u);
      uint32_t ps = 0;
      fetch(static_cast<int64_t>(warp) * 32 + lane, w, ps);
      for (int64_t b = static_cast<int64_t>(warp) * 32; b < len; b += kAdcThreads) {
        const int64_t e = b + lane;
        uint4 wn = w;
        uint32_t psn = ps;
        fetch(e + kAdcThreads, wn, psn);
        uint64_t key = kKeyMax;
        if (e < len) {
          float total;
          uint32_t pos;
          if (wide) {
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
            total = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j)
              total = __fadd_rn(total, lut[j * 256 + ((words[j >> 2] >> (8 * (j & 3))) & 0xFFu)]);
            pos = ps;
          } else {
            total = adc_sum(lut, p.ks, p.codes + (off + e) * p.m, p.m);
            pos = p.pos ? p.pos[off + e] : static_cast<uint32_t>(e);
          }
          key = make_key(total, (static_cast<uint32_t>(pr) << p.pos_bits) | pos);
        }
        w = wn;
        ps = psn;
        warp_topk_offer(best, kth, key, p.k, lane);
      }
      wlist[warp][lane] = best;
      __syncthreads();
      if (warp == 0) {
#pragma unroll
        for (int ow = 1; ow < kAdcThreads / 32; ++ow)
          best = warp_merge32(best, wlist[ow][lane], lane);
        const int have = static_cast<int>(len < p.k ? len : p.k);
        if (lane < have) p.slot_keys[it * p.kp + lane] = best;
        if (lane == 0) p.slot_counts[it] = have;
      }
      continue;
    }
    TopKState st{topbuf, &qc, &nb, &thr};
    for (int64_t b = 0; b < len; b += kAdcThreads) {
      const int64_t e = b + tid;
      const bool valid = e < len;
      uint64_t key = kKeyMax;
      if (valid) {
        const float total = adc_sum(lut, p.ks, p.codes + (off + e) * p.m, p.m);
        const uint32_t pos = p.pos ? p.pos[off + e] : static_cast<uint32_t>(e);
        key = make_key(total, (static_cast<uint32_t>(pr) << p.pos_bits) | pos);
      }
      topk_offer(st, p.kp, key, valid);
      __syncthreads();
      if (qc > p.sortn - p.kp - kAdcThreads)
        topk_merge<kAdcThreads>(st, p.k, p.kp, p.sortn, tid, 0);
    }
    if (qc > 0) topk_merge<kAdcThreads>(st, p.k, p.kp, p.sortn, tid, 0);
    for (int i = tid; i < nb; i += kAdcThreads) p.slot_keys[it * p.kp + i] = topbuf[i];
    if (tid == 0) p.slot_counts[it] = nb;
  }
}

// ---- grouped ADC: the queries that probe one list share its code reads -----
//
// For a batch, most lists are probed by several queries (C4: 32,768 (query,
// list) pairs over 4,096 lists).  adc_group_plan_kernel groups the pairs by
// list and cuts each group into tiles of up to kAdcGroup queries; a tile is
// one item of pq_adc_group_kernel, which builds the tile's tables interleaved
// (entry (s, c) of its W queries side by side, W = 1, 2 or 4 by the tile's
// query count) and reads every code row once for all of them: one 16-byte
// code load and one W-wide table load per subspace serve W queries, and a
// W-wide load of random entries costs fewer shared-memory wavefronts per
// entry than W single loads.  Each query keeps its own sequential fp32 sum
// and its own warp-resident top-k, so every (query, list) slot gets exactly
// the keys of pq_adc_kernel.

constexpr int kAdcGroup = 2;          // queries per tile at most
constexpr int kAdcGroupThreads = 128;  // threads of a grouped ADC block
constexpr int kAdcLutBytes = kAdcGroup >= 4 ? 16 : 4 * kAdcGroup;  // one interleaved entry
constexpr int kAdcPlanThreads = 1024;
constexpr int64_t kAdcGroupMinQueries = 16;  // smaller batches share few lists

struct AdcGroupPlan {
  const uint32_t* probe_lists;  // [nq][probe]
  const int32_t* probe_counts;  // [nq]
  int64_t nq;
  int32_t probe;
  int32_t nlist;
  int32_t* list_cnt;    // [nlist] scratch
  int32_t* list_off;    // [nlist + 1]: the pairs of list l at grouped[list_off[l] ..)
  int32_t* tile_off;    // [nlist + 1]
  int32_t* grouped;     // [nq * probe] pair (item) indices q * probe + rank, by list
  int32_t* tile_list;   // [nq * probe]
  int32_t* tile_first;  // [nq * probe]
  int32_t* ntiles;      // [1]
  int32_t* slot_counts; // pairs without a list (rank >= probe count) get 0 here
};

// One block: counting sort of the (query, rank) pairs by list (the order
// inside a list does not matter: every pair owns its output slot) and the
// tile table.
__global__ void __launch_bounds__(kAdcPlanThreads) adc_group_plan_kernel(const AdcGroupPlan g) {
  __shared__ int32_t part[64];
  const int t = threadIdx.x, nt = blockDim.x;
  const int64_t items = g.nq * g.probe;
  for (int l = t; l < g.nlist; l += nt) g.list_cnt[l] = 0;
  __syncthreads();
  for (int64_t i = t; i < items; i += nt) {
    const int64_t q = i / g.probe;
    const int r = static_cast<int>(i - q * g.probe);
    if (r < g.probe_counts[q])
      atomicAdd(&g.list_cnt[g.probe_lists[i]], 1);
    else
      g.slot_counts[i] = 0;
  }
  __syncthreads();
  block_exclusive_scan(g.list_cnt, g.nlist, g.list_off, part);
  for (int l = t; l < g.nlist; l += nt) g.list_cnt[l] = (g.list_cnt[l] + kAdcGroup - 1) / kAdcGroup;
  __syncthreads();
  block_exclusive_scan(g.list_cnt, g.nlist, g.tile_off, part);
  for (int l = t; l < g.nlist; l += nt) g.list_cnt[l] = 0;
  __syncthreads();
  for (int64_t i = t; i < items; i += nt) {
    const int64_t q = i / g.probe;
    const int r = static_cast<int>(i - q * g.probe);
    if (r < g.probe_counts[q]) {
      const uint32_t l = g.probe_lists[i];
      const int at = atomicAdd(&g.list_cnt[l], 1);
      g.grouped[g.list_off[l] + at] = static_cast<int32_t>(i);
    }
  }
  for (int l = t; l < g.nlist; l += nt) {
    const int t0 = g.tile_off[l], t1 = g.tile_off[l + 1];
    for (int j = t0; j < t1; ++j) {
      g.tile_list[j] = l;
      g.tile_first[j] = g.list_off[l] + (j - t0) * kAdcGroup;
    }
  }
  if (t == 0) *g.ntiles = g.tile_off[g.nlist];
}

// One tile: W-wide tables for its `cnt` queries (cnt <= W), then the scan of
// the list's m = 16 code rows with W sequential sums per row.  The caller
// has the residuals in shared memory and synchronises before and after.
template <int W>
__device__ __forceinline__ void adc_group_tile(const AdcParams& p, uint8_t* lut_raw,
                                               const float* resid, const int32_t* s_item,
                                               int cnt, int64_t off, int64_t len,
                                               uint64_t (*wlist)[kAdcGroup][32]) {
  using V = typename LutVec<W>::T;
  V* lut = reinterpret_cast<V*>(lut_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  build_tables<W, kAdcGroupThreads>(p, lut, resid);
  __syncthreads();
  uint32_t seqhi[W];
#pragma unroll
  for (int j = 0; j < W; ++j) {
    const int32_t it = s_item[j < cnt ? j : 0];
    seqhi[j] = static_cast<uint32_t>(it - (it / p.probe) * p.probe) << p.pos_bits;
  }
  uint64_t best[W], kth[W];
#pragma unroll
  for (int j = 0; j < W; ++j) best[j] = kth[j] = kKeyMax;
  const uint4* crow = reinterpret_cast<const uint4*>(p.codes + off * 16);
  auto fetch = [&](int64_t e, uint4& w, uint32_t& ps) {
    if (e < len) {
      w = __ldg(crow + e);
      ps = p.pos ? __ldg(p.pos + off + e) : static_cast<uint32_t>(e);
    }
  };
  uint4 w = make_uint4(0u, 0u, 0u, 0u);
  uint32_t ps = 0;
  fetch(static_cast<int64_t>(warp) * 32 + lane, w, ps);
  for (int64_t b = static_cast<int64_t>(warp) * 32; b < len; b += kAdcGroupThreads) {
    const int64_t e = b + lane;
    uint4 wn = w;
    uint32_t psn = ps;
    fetch(e + kAdcGroupThreads, wn, psn);
    float acc[W];
#pragma unroll
    for (int j = 0; j < W; ++j) acc[j] = 0.0f;
    if (e < len) {
      const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const V x = lut[jj * 256 + ((words[jj >> 2] >> (8 * (jj & 3))) & 0xFFu)];
#pragma unroll
        for (int j = 0; j < W; ++j) acc[j] = __fadd_rn(acc[j], LutVec<W>::get(x, j));
      }
    }
#pragma unroll
    for (int j = 0; j < W; ++j) {
      if (j < cnt) {
        const uint64_t key = e < len ? make_key(acc[j], seqhi[j] | ps) : kKeyMax;
        warp_topk_offer(best[j], kth[j], key, p.k, lane);
      }
    }
    w = wn;
    ps = psn;
  }
#pragma unroll
  for (int j = 0; j < W; ++j) wlist[warp][j][lane] = best[j];
  __syncthreads();
  for (int j = warp; j < cnt; j += kAdcGroupThreads / 32) {
    uint64_t bb = wlist[0][j][lane];
#pragma unroll
    for (int ow = 1; ow < kAdcGroupThreads / 32; ++ow) bb = warp_merge32(bb, wlist[ow][j][lane], lane);
    const int have = static_cast<int>(len < p.k ? len : p.k);
    const int64_t it = s_item[j];
    if (lane < have) p.slot_keys[it * p.kp + lane] = bb;
    if (lane == 0) p.slot_counts[it] = have;
  }
}

// Persistent over the tiles of adc_group_plan_kernel (m = 16, k <= 32 kept
// per (query, list)).
__global__ void __launch_bounds__(kAdcGroupThreads) pq_adc_group_kernel(
    const AdcParams p, const int32_t* __restrict__ grouped, const int32_t* __restrict__ list_off,
    const int32_t* __restrict__ tile_list, const int32_t* __restrict__ tile_first,
    const int32_t* __restrict__ ntiles_ptr) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* lut_raw =
      reinterpret_cast<uint8_t*>((reinterpret_cast<size_t>(smem_raw) + 15) / 16 * 16);
  float* resid = reinterpret_cast<float*>(lut_raw + static_cast<size_t>(p.m) * p.ks * kAdcLutBytes);
  __shared__ uint64_t wlist[kAdcGroupThreads / 32][kAdcGroup][32];
  __shared__ int32_t s_item[kAdcGroup];
  const int tid = threadIdx.x;
  const int ntiles = *ntiles_ptr;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
    __syncthreads();  // the previous tile is done with the shared buffers
    const int list = tile_list[t];
    const int first = tile_first[t];
    const int cnt = min(kAdcGroup, list_off[list + 1] - first);
    if (tid < kAdcGroup) s_item[tid] = grouped[first + min(tid, cnt - 1)];
    const int64_t off = p.offsets[list];
    const int64_t len = p.offsets[list + 1] - off;
    __syncthreads();
    if (len == 0) {  // an empty list (a shard holding other lists): no table to build
      if (tid < cnt) p.slot_counts[s_item[tid]] = 0;
      continue;
    }
    const int wq = cnt == 1 ? 1 : cnt == 2 ? 2 : 4;  // table width (<= kAdcGroup)
    for (int idx = tid; idx < wq * p.dim; idx += kAdcGroupThreads) {
      const int j = idx / p.dim, d = idx - j * p.dim;
      const int64_t q = s_item[j < cnt ? j : 0] / p.probe;
      resid[idx] = __fsub_rn(p.queries[q * p.dim + d], p.coarse[list * p.coarse_ld + d]);
    }
    __syncthreads();
    if (wq == 1) {
      adc_group_tile<1>(p, lut_raw, resid, s_item, cnt, off, len, wlist);
    } else if (wq == 2) {
      adc_group_tile<2>(p, lut_raw, resid, s_item, cnt, off, len, wlist);
    } else {
      if constexpr (kAdcGroup >= 4) adc_group_tile<4>(p, lut_raw, resid, s_item, cnt, off, len, wlist);
    }
  }
}

// GPUADCSearch.computeDistances for one list (GPUADCSearch.swift:35-173 with
// pq_compute_distance_table + pq_adc_scan, PQDistance.metal:4-66): a squared
// L2 LUT over the query, then the sequential sum per code.  Every block
// rebuilds the LUT in shared memory and scores a stripe of codes.
__global__ void __launch_bounds__(kAdcThreads) pq_adc_list_kernel(
    const float* __restrict__ query, const float* __restrict__ codebooks, int m, int ks, int sub,
    const uint8_t* __restrict__ codes, int64_t count, float* __restrict__ out) {
  extern __shared__ float lut[];
  for (int e = threadIdx.x; e < m * ks; e += blockDim.x) {
    const int s = e / ks;
    lut[e] = lut_entry(kL2, query + s * sub, codebooks + static_cast<int64_t>(e) * sub, sub);
  }
  __syncthreads();
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint8_t* code = codes + i * m;
    float total = 0.0f;
    for (int s = 0; s < m; ++s) {
      const int c = code[s];
      if (c >= ks) {
        total = 3.40282347e+38f;  // FLT_MAX, as pq_adc_scan
        break;
      }
      total = __fadd_rn(total, lut[s * ks + c]);
    }
    out[i] = total;
  }
}

}  // namespace

namespace {

// Shard output of the IVF-PQ search: the (score, seq) 2k-lists of the merge
// step with each entry's internal id.  seq = probe rank << pos_bits | the
// entry's position in its global list; a shard's list holds a subset of the global
// entries with their global positions (`pos`, ascending), found by binary
// search.
__global__ void ivfpq_payload_kernel(int64_t nq, int32_t kin, const float* __restrict__ md,
                                     const uint32_t* __restrict__ mi,
                                     const int32_t* __restrict__ mc,
                                     const uint32_t* __restrict__ probe_lists, int32_t probe,
                                     const int64_t* __restrict__ offsets,
                                     const uint32_t* __restrict__ ids,
                                     const uint32_t* __restrict__ pos, int32_t pos_bits,
                                     float* out_score, uint32_t* out_seq, uint32_t* out_id,
                                     int32_t* out_count) {
  const int64_t q = blockIdx.x;
  const int cnt = mc[q];
  for (int i = threadIdx.x; i < kin; i += blockDim.x) {
    const int64_t at = q * kin + i;
    if (i < cnt) {
      const uint32_t seq = mi[at];
      const uint32_t rank = seq >> pos_bits, gpos = seq & ((1u << pos_bits) - 1u);
      const uint32_t list = probe_lists[q * probe + rank];
      const int64_t off = offsets[list], len = offsets[list + 1] - off;
      int64_t idx = gpos;
      if (pos) {
        int64_t lo = 0, hi = len;
        while (lo < hi) {
          const int64_t mid = (lo + hi) >> 1;
          if (pos[off + mid] < gpos) lo = mid + 1;
          else hi = mid;
        }
        idx = lo;
      }
      out_score[at] = md[at];
      out_seq[at] = seq;
      out_id[at] = ids[off + idx];
    } else {
      out_score[at] = __int_as_float(0x7F800000);
      out_seq[at] = 0xFFFFFFFFu;
      out_id[at] = kEmptyId;
    }
  }
  if (threadIdx.x == 0) out_count[q] = cnt;
}

// Per query: the (score, seq) smallest kin entries over the shard blocks
// (block r at blocks + r * stride words: score | seq | id | count), with
// their ids.  Sequences are unique per query (each global entry lives in
// one shard), so (score, seq) orders them totally.
__global__ void __launch_bounds__(256) ivfpq_shard_merge_kernel(
    const int32_t* __restrict__ blocks, int32_t n_blocks, int64_t stride, int64_t nq, int32_t kin,
    float* m_score, uint32_t* m_seq, uint32_t* m_id, int32_t* m_count) {
  extern __shared__ uint64_t mk[];  // n2 keys, then n2 ids (uint32)
  const int64_t q = blockIdx.x;
  int n2 = 1;
  while (n2 < n_blocks * kin) n2 <<= 1;
  uint32_t* mv = reinterpret_cast<uint32_t*>(mk + n2);
  for (int i = threadIdx.x; i < n2; i += blockDim.x) {
    const int r = i / kin, j = i - r * kin;
    uint64_t key = kKeyMax;
    uint32_t id = kEmptyId;
    if (r < n_blocks) {
      const int32_t* b = blocks + r * stride;
      const int32_t cnt = b[3 * nq * kin + q];
      if (j < cnt) {
        const float sc = __int_as_float(b[q * kin + j]);
        const uint32_t seq = static_cast<uint32_t>(b[nq * kin + q * kin + j]);
        key = (static_cast<uint64_t>(float_to_ordered(sc)) << 32) | seq;
        id = static_cast<uint32_t>(b[2 * nq * kin + q * kin + j]);
      }
    }
    mk[i] = key;
    mv[i] = id;
  }
  __syncthreads();
  for (int a = 2; a <= n2; a <<= 1) {
    for (int jj = a >> 1; jj > 0; jj >>= 1) {
      for (int i = threadIdx.x; i < n2; i += blockDim.x) {
        const int ixj = i ^ jj;
        if (ixj > i) {
          const uint64_t x = mk[i], y = mk[ixj];
          const bool up = (i & a) == 0;
          if ((x > y) == up) {
            mk[i] = y;
            mk[ixj] = x;
            const uint32_t t = mv[i];
            mv[i] = mv[ixj];
            mv[ixj] = t;
          }
        }
      }
      __syncthreads();
    }
  }
  __shared__ int valid;
  if (threadIdx.x == 0) valid = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < kin; i += blockDim.x) {
    const uint64_t key = mk[i];
    const bool ok = key != kKeyMax;
    m_score[q * kin + i] = ok ? ordered_to_float(static_cast<uint32_t>(key >> 32)) : __int_as_float(0x7F800000);
    m_seq[q * kin + i] = ok ? static_cast<uint32_t>(key) : 0xFFFFFFFFu;
    m_id[q * kin + i] = ok ? mv[i] : kEmptyId;
    if (ok) atomicAdd(&valid, 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) m_count[q] = valid;
}

// ---- k above 256: every probed entry's key, sorted per query ------------------
//
// The shared-memory top-k lists of the batch kernels hold at most 512 keys,
// while _IVFPQIndex.search keeps BoundedSortedList(capacity: k) for any k
// (IVFPQIndex.swift:197).  For k > 256 every probed entry's (score, insertion
// sequence) key is written out, the keys are sorted per query (CUB
// segmented radix sort), and the list's outcome is read off the sorted keys.

// Per query: the entries of each probed list (rank order) and their running
// offsets within the query's key segment; counts[q] = the query's total.
__global__ void __launch_bounds__(256) lk_offsets_kernel(const uint32_t* __restrict__ probe_lists,
                                                         const int32_t* __restrict__ probe_counts,
                                                         const int64_t* __restrict__ offsets,
                                                         int32_t probe, int64_t* __restrict__ qoff,
                                                         int64_t* __restrict__ counts) {
  __shared__ int64_t wsum[8];
  const int64_t q = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  int64_t len = 0;
  if (t < probe && t < probe_counts[q]) {
    const uint32_t l = probe_lists[q * probe + t];
    len = offsets[l + 1] - offsets[l];
  }
  int64_t incl = len;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  int64_t add = 0;
  for (int i = 0; i < w; ++i) add += wsum[i];
  if (t < probe) qoff[q * probe + t] = incl + add - len;
  if (t == 255) counts[q] = incl + add;
}

// Exclusive running sum of counts[0, n) into seg[0, n] by one block.
__global__ void __launch_bounds__(1024) lk_scan_kernel(const int64_t* __restrict__ counts, int64_t n,
                                                       int64_t* __restrict__ seg) {
  __shared__ int64_t part[32];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int64_t per = (n + 1023) / 1024;
  const int64_t b = t * per, e = b + per < n ? b + per : n;
  int64_t sum = 0;
  for (int64_t i = b; i < e; ++i) sum += counts[i];
  int64_t incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += u;
  }
  if (lane == 31) part[w] = incl;
  __syncthreads();
  int64_t add = 0;
  for (int i = 0; i < w; ++i) add += part[i];
  int64_t acc = incl - sum + add;
  for (int64_t i = b; i < e; ++i) {
    seg[i] = acc;
    acc += counts[i];
  }
  if (t == 1023) seg[n] = acc;
}

// One block per (query, probe rank) item: the residual, the distance table,
// and the key of every entry of the list at its place in the query's segment.
__global__ void __launch_bounds__(kAdcThreads) pq_adc_all_kernel(const AdcParams p,
                                                                 const int64_t* __restrict__ seg,
                                                                 const int64_t* __restrict__ qoff,
                                                                 uint64_t* __restrict__ keys) {
  extern __shared__ uint8_t smem_raw[];
  float* lut = reinterpret_cast<float*>((reinterpret_cast<size_t>(smem_raw) + 15) / 16 * 16);
  float* resid = lut + p.m * p.ks;
  const int tid = threadIdx.x;
  const int64_t items = p.nq * p.probe;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    const int64_t q = it / p.probe;
    const int pr = static_cast<int>(it - q * p.probe);
    __syncthreads();  // the previous item is done with the table
    if (pr >= p.probe_counts[q]) continue;
    const uint32_t list = p.probe_lists[q * p.probe + pr];
    const int64_t off = p.offsets[list];
    const int64_t len = p.offsets[list + 1] - off;
    if (len == 0) continue;
    for (int d = tid; d < p.dim; d += kAdcThreads)
      resid[d] = __fsub_rn(p.queries[q * p.dim + d], p.coarse[list * p.coarse_ld + d]);
    __syncthreads();
    build_tables<1, kAdcThreads>(p, lut, resid);
    __syncthreads();
    uint64_t* out = keys + seg[q] + qoff[it];
    for (int64_t e = tid; e < len; e += kAdcThreads) {
      const float total = adc_sum(lut, p.ks, p.codes + (off + e) * p.m, p.m);
      const uint32_t pos = p.pos ? __ldg(p.pos + off + e) : static_cast<uint32_t>(e);
      out[e] = make_key(total, (static_cast<uint32_t>(pr) << p.pos_bits) | pos);
    }
  }
}

// The k-th smallest (1-based) of n 32-bit words by a block of 256 threads:
// four 8-bit radix passes over get(i).
template <typename Get>
__device__ uint32_t block_kth_u32(Get get, int64_t n, int64_t k, int* hist, int* ctl) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  uint32_t prefix = 0, mask = 0;
  int64_t rank = k;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    hist[t] = 0;
    __syncthreads();
    for (int64_t i = t; i < n; i += 256) {
      const uint32_t v = get(i);
      if ((v & mask) == prefix) atomicAdd(&hist[(v >> shift) & 255u], 1);
    }
    __syncthreads();
    if (w == 0) {
      int h[8];
      int64_t s = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        h[i] = hist[lane * 8 + i];
        s += h[i];
      }
      int64_t incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int64_t u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (lane >= o) incl += u;
      }
      const int64_t excl = incl - s;
      if (excl < rank && rank <= incl) {
        int64_t c = excl;
        int bin = lane * 8 + 7;
        for (int i = 0; i < 8; ++i) {
          if (c + h[i] >= rank) {
            bin = lane * 8 + i;
            break;
          }
          c += h[i];
        }
        ctl[0] = bin;
        ctl[1] = static_cast<int>(rank - c);
      }
    }
    __syncthreads();
    prefix |= static_cast<uint32_t>(ctl[0]) << shift;
    mask |= 0xFFu << shift;
    rank = ctl[1];
  }
  return prefix;
}

// BoundedSortedList(capacity K) over one query's keys sorted by (score, seq)
// (the closed form of bsl_resolve_kernel, read off the full sorted segment).
// Keys below the K-th key's score are all kept (runs of equal scores newest
// first); of the keys equal to it, those among the first K arrivals (by
// sequence) of the ones below and the K earliest equal ones were inserted,
// and the newest K - l of them survive.
__global__ void __launch_bounds__(256) bsl_resolve_large_kernel(const ResolveParams p,
                                                                const uint64_t* __restrict__ sorted,
                                                                const int64_t* __restrict__ seg) {
  __shared__ int hist[256];
  __shared__ int ctl[2];
  __shared__ uint32_t skth;
  const int64_t q = blockIdx.x;
  const int tid = threadIdx.x;
  const uint64_t* ks = sorted + seg[q];
  const int64_t c = seg[q + 1] - seg[q];
  const int64_t K = p.cap;
  auto hi = [&](int64_t i) { return static_cast<uint32_t>(ks[i] >> 32); };
  // first index in [a, b) whose score word is >= x (> x when `strict`)
  auto bound = [&](int64_t a, int64_t b, uint32_t x, bool strict) {
    while (a < b) {
      const int64_t mid = (a + b) >> 1;
      const uint32_t v = hi(mid);
      if (strict ? v <= x : v < x)
        a = mid + 1;
      else
        b = mid;
    }
    return a;
  };
  int64_t l, nout, e_keep = 0, e_first = 0;
  if (c <= K) {
    l = nout = c;
  } else {
    const uint32_t wv = hi(K - 1);
    l = bound(0, K, wv, false);
    const int64_t e_end = bound(K, c, wv, true);
    const int64_t ecount = min(e_end - l, K);
    const int64_t total = l + ecount;
    const uint32_t sk =
        block_kth_u32([&](int64_t i) { return static_cast<uint32_t>(ks[i]); }, total, K, hist, ctl);
    if (tid == 0) skth = sk;
    __syncthreads();
    // inserted equal-score entries: the E' entries with sequence <= the K-th
    // arrival (E' is sorted by sequence)
    int64_t a = l, b = l + ecount;
    while (a < b) {
      const int64_t mid = (a + b) >> 1;
      if (static_cast<uint32_t>(ks[mid]) <= skth)
        a = mid + 1;
      else
        b = mid;
    }
    const int64_t ins = a - l;
    e_keep = K - l;
    e_first = l + ins - e_keep;
    nout = K;
  }
  for (int64_t i = tid; i < l; i += 256) {
    // the equal-score run [a, b) holding i, read back to front
    const uint32_t v = hi(i);
    const int64_t a = bound(0, i + 1, v, false), b = bound(i, l, v, true);
    const int64_t src = a + (b - 1 - i);
    p.out_score[q * p.kout + i] = key_distance(ks[src]);
    p.out_id[q * p.kout + i] = seq_payload(p, q, static_cast<uint32_t>(ks[src]));
  }
  for (int64_t j = tid; j < e_keep; j += 256) {
    const int64_t src = e_first + (e_keep - 1 - j);
    p.out_score[q * p.kout + l + j] = key_distance(ks[src]);
    p.out_id[q * p.kout + l + j] = seq_payload(p, q, static_cast<uint32_t>(ks[src]));
  }
  for (int64_t i = nout + tid; i < p.kout; i += 256) {
    p.out_score[q * p.kout + i] = __int_as_float(0x7F800000);
    p.out_id[q * p.kout + i] = kEmptyId;
  }
  if (tid == 0) p.out_count[q] = static_cast<int32_t>(nout);
}

}  // namespace

static size_t carve(size_t& o, size_t bytes) {
  size_t at = (o + 255) / 256 * 256;
  o = at + bytes;
  return at;
}

// partial: null, or this shard's block [score | seq | id | count] (2k
// entries per query) instead of the resolved top-k (the row-sharded search)
// k above 256 (not for shard blocks): steps 2-4 over every probed entry.
static int32_t run_ivfpq_large_k(mans_ctx* ctx, mans_ivfpq* ix, mans_workspace* ws,
                                 const float* d_queries, int64_t nq, int32_t k, int32_t probe,
                                 int32_t pos_bits, const uint32_t* pl, const int32_t* pc,
                                 float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                                 cudaStream_t stream) {
  int32_t rc;
  // per-query offsets and segment starts (small; in `small_scores`, which the
  // coarse step no longer needs)
  const size_t o_qo = 0;
  const size_t o_ct = (nq * probe * sizeof(int64_t) + 255) / 256 * 256;
  const size_t o_sg = o_ct + (nq * sizeof(int64_t) + 255) / 256 * 256;
  const size_t small_bytes = o_sg + (nq + 1) * sizeof(int64_t);
  if ((rc = ws->small_scores.reserve(small_bytes)) != MANS_OK) return rc;
  uint8_t* S = static_cast<uint8_t*>(ws->small_scores.ptr);
  int64_t* qoff = reinterpret_cast<int64_t*>(S + o_qo);
  int64_t* counts = reinterpret_cast<int64_t*>(S + o_ct);
  int64_t* seg = reinterpret_cast<int64_t*>(S + o_sg);
  lk_offsets_kernel<<<static_cast<unsigned>(nq), 256, 0, stream>>>(pl, pc, ix->offsets, probe, qoff,
                                                                  counts);
  lk_scan_kernel<<<1, 1024, 0, stream>>>(counts, nq, seg);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "large-k offsets launch");
  // the total number of keys sizes the buffers: one host round trip
  int64_t total = 0;
  e = cudaMemcpyAsync(&total, seg + nq, sizeof(int64_t), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return fail_cuda(e, "large-k total");
  if (total > INT32_MAX) return fail(MANS_ERR_SEARCH, "too many probed entries for one batch");
  size_t tmp_bytes = 0;
  e = cub::DeviceSegmentedRadixSort::SortKeys(nullptr, tmp_bytes, static_cast<const uint64_t*>(nullptr),
                                              static_cast<uint64_t*>(nullptr), static_cast<int>(total),
                                              static_cast<int>(nq), seg, seg + 1, 0, 64, stream);
  if (e != cudaSuccess) return fail_cuda(e, "large-k sort size");
  const size_t keys_bytes = (static_cast<size_t>(std::max<int64_t>(total, 1)) * 8 + 255) / 256 * 256;
  if ((rc = ws->big.reserve(2 * keys_bytes + tmp_bytes)) != MANS_OK) return rc;
  uint64_t* kin = static_cast<uint64_t*>(ws->big.ptr);
  uint64_t* kout_keys = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(ws->big.ptr) + keys_bytes);
  void* tmp = static_cast<uint8_t*>(ws->big.ptr) + 2 * keys_bytes;
  if (total > 0) {
    AdcParams a{};
    a.queries = d_queries;
    a.coarse = ix->coarse->rows;
    a.coarse_ld = ix->coarse->ld;
    a.codebooks = ix->codebooks;
    a.codes = ix->codes;
    a.pos = ix->pos;
    a.offsets = ix->offsets;
    a.probe_lists = pl;
    a.probe_counts = pc;
    a.probe = probe;
    a.pos_bits = pos_bits;
    a.nq = nq;
    a.dim = static_cast<int32_t>(ix->dim);
    a.m = ix->m;
    a.ks = ix->ks;
    a.sub = ix->sub;
    a.metric = ix->metric;
    const size_t smem = 16 + static_cast<size_t>(ix->m) * ix->ks * 4 +
                        static_cast<size_t>((ix->dim + 3) / 4 * 4) * 4;
    if (smem > static_cast<size_t>(ctx->max_smem) - 64)
      return fail(MANS_ERR_SEARCH, "PQ distance table exceeds shared memory");
    e = cudaFuncSetAttribute(pq_adc_all_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return fail_cuda(e, "large-k adc configure");
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pq_adc_all_kernel, kAdcThreads, smem);
    if (e != cudaSuccess) return fail_cuda(e, "large-k adc occupancy");
    const int grid = static_cast<int>(std::min<int64_t>(
        nq * probe, static_cast<int64_t>(ctx->num_sms) * std::max(1, per_sm)));
    cudaEvent_t stop = timing_begin(ws, stream);
    pq_adc_all_kernel<<<grid, kAdcThreads, smem, stream>>>(a, seg, qoff, kin);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "large-k adc launch");
    timing_end(stop, stream);
    e = cub::DeviceSegmentedRadixSort::SortKeys(tmp, tmp_bytes, kin, kout_keys,
                                                static_cast<int>(total), static_cast<int>(nq), seg,
                                                seg + 1, 0, 64, stream);
    if (e != cudaSuccess) return fail_cuda(e, "large-k sort");
  }
  ResolveParams f{};
  f.nq = nq;
  f.cap = k;
  f.pos_bits = pos_bits;
  f.probe_lists = pl;
  f.probe_stride = probe;
  f.offsets = ix->offsets;
  f.ids = ix->ids;
  f.pos = ix->pos;
  f.out_score = d_out_dist;
  f.out_id = d_out_ids;
  f.out_count = d_out_counts;
  f.kout = k;
  bsl_resolve_large_kernel<<<static_cast<unsigned>(nq), 256, 0, stream>>>(f, kout_keys, seg);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "large-k resolve launch");
  ws->launches += 6;
  return MANS_OK;
}

static int32_t run_ivfpq_search(mans_ctx* ctx, mans_ivfpq* ix, mans_workspace* ws,
                                const float* d_queries, int64_t nq, int32_t k, int32_t nprobe,
                                float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                                cudaStream_t stream, int32_t* partial = nullptr) {
  // Results are k wide (BoundedSortedList(capacity: k), IVFPQIndex.swift:197);
  // the shard blocks of the partial search keep at most 256.
  const int32_t kout = partial ? std::min<int32_t>(k, MANS_MAX_TOPK) : k;
  if (nq <= 0) return MANS_OK;
  if (k <= 0 || ix->n <= 0 || ix->nlist <= 0) {
    if (kout <= 0) {
      cudaError_t e = cudaMemsetAsync(d_out_counts, 0, sizeof(int32_t) * nq, stream);
      return e == cudaSuccess ? MANS_OK : fail_cuda(e, "cudaMemsetAsync");
    }
    cudaError_t e = launch_fill_empty(d_out_dist, d_out_ids, d_out_counts, nq, kout, stream);
    return e == cudaSuccess ? MANS_OK : fail_cuda(e, "fill_empty launch");
  }
  const int32_t probe = std::max(1, std::min(nprobe, ix->nlist));
  const int32_t kc = std::min<int32_t>(2 * probe, ix->nlist);  // coarse candidates
  if (kc > 512) return fail(MANS_ERR_SEARCH, "nprobe above 256 is not supported on the GPU");
  const int32_t pos_bits = seq_pos_bits(probe);
  if (ix->max_pos >= (int64_t{1} << pos_bits)) {
    char msg[160];
    std::snprintf(msg, sizeof msg,
                  "list position %lld does not fit the insertion sequence at nprobe %d "
                  "(positions below 2^%d)",
                  static_cast<long long>(ix->max_pos), probe, pos_bits);
    return fail(MANS_ERR_SEARCH, msg);
  }
  const bool large_k = kout > MANS_MAX_TOPK;
  const int32_t k2 = 2 * std::min<int32_t>(kout, MANS_MAX_TOPK);  // ADC candidates per list and after the merge
  const int32_t kp2 = pow2_at_least(k2);

  size_t o = 0;
  const size_t o_cd = carve(o, nq * kc * sizeof(float));
  const size_t o_ci = carve(o, nq * kc * sizeof(uint32_t));
  const size_t o_cc = carve(o, nq * sizeof(int32_t));
  const size_t o_ps = carve(o, nq * probe * sizeof(float));
  const size_t o_pl = carve(o, nq * probe * sizeof(uint32_t));
  const size_t o_pc = carve(o, nq * sizeof(int32_t));
  const size_t o_md = carve(o, nq * k2 * sizeof(float));
  const size_t o_mi = carve(o, nq * k2 * sizeof(uint32_t));
  const size_t o_mc = carve(o, nq * sizeof(int32_t));
  // batches of m = 16 codes with at most 32 kept keys per list run the grouped
  // ADC (the queries probing one list share its code reads)
  const bool grouped = 2 * kout <= 32 && ix->m == 16 && nq >= kAdcGroupMinQueries &&
                       16 + static_cast<size_t>(ix->m) * ix->ks * kAdcLutBytes +
                               static_cast<size_t>(kAdcGroup) * ix->dim * 4 <=
                           static_cast<size_t>(ctx->max_smem) - 5120;
  const int64_t items_all = nq * probe;
  if (items_all > INT32_MAX) return fail(MANS_ERR_SEARCH, "query batch too large");
  const size_t o_gl = carve(o, grouped ? ix->nlist * sizeof(int32_t) : 0);
  const size_t o_go = carve(o, grouped ? (ix->nlist + 1) * sizeof(int32_t) : 0);
  const size_t o_gt = carve(o, grouped ? (ix->nlist + 1) * sizeof(int32_t) : 0);
  const size_t o_gg = carve(o, grouped ? items_all * sizeof(int32_t) : 0);
  const size_t o_gtl = carve(o, grouped ? items_all * sizeof(int32_t) : 0);
  const size_t o_gtf = carve(o, grouped ? items_all * sizeof(int32_t) : 0);
  const size_t o_gn = carve(o, grouped ? sizeof(int32_t) : 0);
  int32_t rc;
  if ((rc = ws->aux2.reserve(o)) != MANS_OK) return rc;
  // slot buffers: coarse search and ADC items, reserved once before any launch
  const int64_t cent_tiles = (ix->nlist + kTileRows - 1) / kTileRows;
  const size_t cent_slots =
      static_cast<size_t>((nq + 7) / 8 * 8) * std::min<int64_t>(ctx->num_sms, cent_tiles);
  const size_t adc_slots = static_cast<size_t>(nq) * probe;
  const size_t need_keys =
      std::max(cent_slots * pow2_at_least(kc), adc_slots * kp2) * sizeof(uint64_t);
  if ((rc = ws->slot_keys.reserve(need_keys)) != MANS_OK) return rc;
  if ((rc = ws->slot_counts.reserve(std::max(cent_slots, adc_slots) * sizeof(int32_t))) != MANS_OK)
    return rc;
  uint8_t* A = static_cast<uint8_t*>(ws->aux2.ptr);
  float* cd = reinterpret_cast<float*>(A + o_cd);
  uint32_t* ci = reinterpret_cast<uint32_t*>(A + o_ci);
  int32_t* cc = reinterpret_cast<int32_t*>(A + o_cc);
  float* ps = reinterpret_cast<float*>(A + o_ps);
  uint32_t* pl = reinterpret_cast<uint32_t*>(A + o_pl);
  int32_t* pc = reinterpret_cast<int32_t*>(A + o_pc);
  float* md = reinterpret_cast<float*>(A + o_md);
  uint32_t* mi = reinterpret_cast<uint32_t*>(A + o_mi);
  int32_t* mc = reinterpret_cast<int32_t*>(A + o_mc);

  // 1. coarse: SIMDDistance scores, 2 x nprobe smallest by (score, index)
  {
    TimingHold hold(ws);  // the coarse scan is not the timed ADC kernel
    rc = run_flat_search(ctx, ix->coarse, ws, d_queries, nq, kc, ix->metric, cd, ci, cc, stream,
                         kModeSimd, 512);
  }
  if (rc != MANS_OK) return rc;
  ResolveParams r{};
  r.in_score = cd;
  r.in_seq = ci;
  r.in_count = cc;
  r.kin = kc;
  r.nq = nq;
  r.cap = probe;
  r.out_score = ps;
  r.out_id = pl;
  r.out_count = pc;
  r.kout = probe;
  bsl_resolve_kernel<<<static_cast<unsigned>(nq), 256, 0, stream>>>(r);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "coarse resolve launch");
  if (large_k)
    return run_ivfpq_large_k(ctx, ix, ws, d_queries, nq, kout, probe, pos_bits, pl, pc,
                             d_out_dist, d_out_ids, d_out_counts, stream);

  // 2. per (query, probed list): residual LUT + ADC, 2k best per list
  AdcParams a{};
  a.queries = d_queries;
  a.coarse = ix->coarse->rows;
  a.coarse_ld = ix->coarse->ld;
  a.codebooks = ix->codebooks;
  a.codes = ix->codes;
  a.pos = ix->pos;
  a.offsets = ix->offsets;
  a.probe_lists = pl;
  a.probe_counts = pc;
  a.probe = probe;
  a.pos_bits = pos_bits;
  a.nq = nq;
  a.dim = static_cast<int32_t>(ix->dim);
  a.m = ix->m;
  a.ks = ix->ks;
  a.sub = ix->sub;
  a.metric = ix->metric;
  a.k = k2;
  a.kp = kp2;
  a.slot_keys = static_cast<uint64_t*>(ws->slot_keys.ptr);
  a.slot_counts = static_cast<int32_t*>(ws->slot_counts.ptr);
  a.sortn = std::max(512, pow2_at_least(kp2 + kAdcThreads));
  if (grouped) {
    AdcGroupPlan gp{};
    gp.probe_lists = pl;
    gp.probe_counts = pc;
    gp.nq = nq;
    gp.probe = probe;
    gp.nlist = ix->nlist;
    gp.list_cnt = reinterpret_cast<int32_t*>(A + o_gl);
    gp.list_off = reinterpret_cast<int32_t*>(A + o_go);
    gp.tile_off = reinterpret_cast<int32_t*>(A + o_gt);
    gp.grouped = reinterpret_cast<int32_t*>(A + o_gg);
    gp.tile_list = reinterpret_cast<int32_t*>(A + o_gtl);
    gp.tile_first = reinterpret_cast<int32_t*>(A + o_gtf);
    gp.ntiles = reinterpret_cast<int32_t*>(A + o_gn);
    gp.slot_counts = a.slot_counts;
    adc_group_plan_kernel<<<1, kAdcPlanThreads, 0, stream>>>(gp);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "adc plan launch");
    const size_t gsmem = 16 + static_cast<size_t>(ix->m) * ix->ks * kAdcLutBytes +
                         static_cast<size_t>(kAdcGroup) * ix->dim * 4;
    e = cudaFuncSetAttribute(pq_adc_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(gsmem));
    if (e != cudaSuccess) return fail_cuda(e, "grouped adc configure");
    int per_sm = 1;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pq_adc_group_kernel,
                                                      kAdcGroupThreads, gsmem);
    if (e != cudaSuccess) return fail_cuda(e, "grouped adc occupancy");
    const int grid = static_cast<int>(std::min<int64_t>(
        items_all, static_cast<int64_t>(ctx->num_sms) * std::max(1, per_sm)));
    cudaEvent_t stop = timing_begin(ws, stream);
    pq_adc_group_kernel<<<grid, kAdcGroupThreads, gsmem, stream>>>(a, gp.grouped, gp.list_off,
                                                              gp.tile_list, gp.tile_first,
                                                              gp.ntiles);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "grouped adc launch");
    timing_end(stop, stream);
    ws->launches += 1;
  }
  // up to 32 kept keys per item: warp-resident lists, no shared top-k buffer
  const bool warp_topk = k2 <= 32;
  const void* kfn = warp_topk ? reinterpret_cast<const void*>(pq_adc_kernel<true>)
                              : reinterpret_cast<const void*>(pq_adc_kernel<false>);
  const size_t smem = 16 + (warp_topk ? 0 : static_cast<size_t>(a.sortn) * 8) +
                      static_cast<size_t>(ix->m) * ix->ks * 4 +
                      static_cast<size_t>((ix->dim + 3) / 4 * 4) * 4;
  if (smem > static_cast<size_t>(ctx->max_smem) - 64)
    return fail(MANS_ERR_SEARCH, "PQ distance table exceeds shared memory");
  e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
  if (e != cudaSuccess) return fail_cuda(e, "adc configure");
  int per_sm = 1;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kAdcThreads, smem);
  if (e != cudaSuccess) return fail_cuda(e, "adc occupancy");
  const int64_t items = nq * probe;
  const int grid = static_cast<int>(
      std::min<int64_t>(items, static_cast<int64_t>(ctx->num_sms) * std::max(1, per_sm)));
  if (!grouped) {
    cudaEvent_t stop = timing_begin(ws, stream);
    if (warp_topk)
      pq_adc_kernel<true><<<grid, kAdcThreads, smem, stream>>>(a);
    else
      pq_adc_kernel<false><<<grid, kAdcThreads, smem, stream>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "adc launch");
    timing_end(stop, stream);
  }

  // 3. 2k smallest (score, seq) per query over its probed lists
  MergeParams m{};
  m.in_keys = a.slot_keys;
  m.in_counts = a.slot_counts;
  m.slots_per_query = probe;
  m.kp_in = kp2;
  m.nq = nq;
  m.k = k2;
  m.kp = kp2;
  m.kout = k2;
  m.out_dist = md;
  m.out_ids = mi;
  m.out_counts = mc;
  e = launch_merge(m, stream);
  if (e != cudaSuccess) return fail_cuda(e, "adc merge launch");

  if (partial) {
    float* ps_ = reinterpret_cast<float*>(partial);
    uint32_t* pq_ = reinterpret_cast<uint32_t*>(partial) + nq * k2;
    uint32_t* pi_ = reinterpret_cast<uint32_t*>(partial) + 2 * nq * k2;
    int32_t* pc_ = partial + 3 * nq * k2;
    ivfpq_payload_kernel<<<static_cast<unsigned>(nq), 128, 0, stream>>>(
        nq, k2, md, mi, mc, pl, probe, ix->offsets, ix->ids, ix->pos, pos_bits, ps_, pq_, pi_,
        pc_);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "payload launch");
    ws->launches += 4;
    return MANS_OK;
  }
  // 4. BoundedSortedList(capacity k) outcome, seq -> internal id
  ResolveParams f{};
  f.in_score = md;
  f.in_seq = mi;
  f.in_count = mc;
  f.kin = k2;
  f.nq = nq;
  f.cap = kout;
  f.pos_bits = pos_bits;
  f.probe_lists = pl;
  f.probe_stride = probe;
  f.offsets = ix->offsets;
  f.ids = ix->ids;
  f.pos = ix->pos;
  f.out_score = d_out_dist;
  f.out_id = d_out_ids;
  f.out_count = d_out_counts;
  f.kout = kout;
  bsl_resolve_kernel<<<static_cast<unsigned>(nq), 256, 0, stream>>>(f);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "resolve launch");
  ws->launches += 4;
  return MANS_OK;
}

}  // namespace mans

extern "C" {

int32_t mans_ivfpq_create(mans_ctx* ctx, const float* coarse, int32_t nlist, int64_t dim,
                          const float* codebooks, int32_t m, int32_t ks, const uint8_t* codes,
                          int64_t n, const int64_t* list_offsets, const uint32_t* lists,
                          const uint32_t* list_positions, int32_t metric, mans_ivfpq** out) {
  if (!ctx || !out) return fail(MANS_ERR_INVALID, "null context or output");
  *out = nullptr;
  if (int32_t r = reject_group(ctx, nullptr, "an IVF-PQ index")) return r;
  if (nlist <= 0 || dim <= 0 || m <= 0 || n < 0) return fail(MANS_ERR_INVALID, "bad IVF-PQ shape");
  if (ks != 256)
    return fail(MANS_ERR_INVALID, "_IVFPQIndex requires numCentroids == 256 (UInt8 codes)");
  if (dim % m != 0) return fail(MANS_ERR_INVALID, "dimension must be divisible by numSubspaces");
  if (metric < 0 || metric > 2) return fail(MANS_ERR_INVALID, "unsupported metric");
  if (!coarse || !codebooks || !list_offsets || (n > 0 && (!codes || !lists)))
    return fail(MANS_ERR_INVALID, "null IVF-PQ buffer");
  const int64_t total = list_offsets[nlist];
  if (list_offsets[0] != 0 || total < 0) return fail(MANS_ERR_INVALID, "bad list offsets");
  int64_t max_len = 0;
  for (int32_t l = 0; l < nlist; ++l) {
    int64_t len = list_offsets[l + 1] - list_offsets[l];
    if (len < 0) return fail(MANS_ERR_INVALID, "list offsets must be non-decreasing");
    max_len = std::max(max_len, len);
  }
  for (int64_t i = 0; i < total; ++i)
    if (lists[i] >= static_cast<uint64_t>(n)) return fail(MANS_ERR_INVALID, "list id out of range");
  int64_t max_pos = max_len - 1;
  if (list_positions) {
    // the searches find an entry from its position by binary search
    for (int32_t l = 0; l < nlist; ++l)
      for (int64_t i = list_offsets[l] + 1; i < list_offsets[l + 1]; ++i)
        if (list_positions[i] <= list_positions[i - 1])
          return fail(MANS_ERR_INVALID, "list positions must ascend within each list");
    for (int64_t i = 0; i < total; ++i)
      max_pos = std::max<int64_t>(max_pos, list_positions[i]);
  }
  DeviceGuard g(ctx->device);
  mans_ivfpq* ix = new mans_ivfpq();
  ix->ctx = ctx;
  ix->nlist = nlist;
  ix->n = total;
  ix->dim = dim;
  ix->m = m;
  ix->ks = ks;
  ix->sub = static_cast<int32_t>(dim / m);
  ix->metric = metric;
  ix->max_len = max_len;
  ix->max_pos = max_pos;
  // gather codes into list order on the host (codes are stored per internal id)
  std::vector<uint8_t> packed(static_cast<size_t>(std::max<int64_t>(total, 1)) * m);
  for (int64_t i = 0; i < total; ++i)
    std::memcpy(&packed[i * m], codes + static_cast<int64_t>(lists[i]) * m, m);
  int32_t rc = corpus_upload(ctx, coarse, nlist, dim, 0, &ix->coarse);
  cudaError_t e = cudaSuccess;
  const size_t cb_count = static_cast<size_t>(m) * ks * ix->sub;
  if (rc == MANS_OK) {
    e = cudaMalloc(&ix->codebooks, cb_count * sizeof(float));
    if (e == cudaSuccess)
      e = cudaMemcpy(ix->codebooks, codebooks, cb_count * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&ix->codes, packed.size());
    if (e == cudaSuccess)
      e = cudaMemcpy(ix->codes, packed.data(), packed.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&ix->ids, std::max<int64_t>(total, 1) * sizeof(uint32_t));
    if (e == cudaSuccess && total > 0)
      e = cudaMemcpy(ix->ids, lists, total * sizeof(uint32_t), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && list_positions) {
      e = cudaMalloc(&ix->pos, std::max<int64_t>(total, 1) * sizeof(uint32_t));
      if (e == cudaSuccess && total > 0)
        e = cudaMemcpy(ix->pos, list_positions, total * sizeof(uint32_t), cudaMemcpyHostToDevice);
    }
    if (e == cudaSuccess) e = cudaMalloc(&ix->offsets, (nlist + 1) * sizeof(int64_t));
    if (e == cudaSuccess)
      e = cudaMemcpy(ix->offsets, list_offsets, (nlist + 1) * sizeof(int64_t),
                     cudaMemcpyHostToDevice);
    if (e != cudaSuccess) rc = fail_cuda(e, "IVF-PQ upload");
  }
  if (rc != MANS_OK) {
    corpus_free(ix->coarse);
    cudaFree(ix->codebooks);
    cudaFree(ix->codes);
    cudaFree(ix->ids);
    cudaFree(ix->pos);
    cudaFree(ix->offsets);
    delete ix;
    return rc;
  }
  *out = ix;
  return MANS_OK;
}

int32_t mans_ivfpq_destroy(mans_ivfpq* ix) {
  if (!ix) return MANS_OK;
  DeviceGuard g(ix->ctx->device);
  cudaDeviceSynchronize();
  corpus_free(ix->coarse);
  cudaFree(ix->codebooks);
  cudaFree(ix->codes);
  cudaFree(ix->ids);
  cudaFree(ix->pos);
  cudaFree(ix->offsets);
  delete ix;
  return MANS_OK;
}

int32_t mans_ivfpq_search_device(mans_ctx* ctx, mans_ivfpq* ix, mans_workspace* ws,
                                 const float* d_queries, int64_t nq, int32_t k, int32_t nprobe,
                                 float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                                 void* cuda_stream) {
  if (!ctx || !ix || ix->ctx != ctx) return fail(MANS_ERR_INVALID, "null or foreign IVF-PQ index");
  if (!ws || ws->ctx != ctx) return fail(MANS_ERR_INVALID, "workspace missing or foreign");
  if (nq < 0) return fail(MANS_ERR_INVALID, "negative query count");
  DeviceGuard g(ctx->device);
  return run_ivfpq_search(ctx, ix, ws, d_queries, nq, k, nprobe, d_out_dist, d_out_ids,
                          d_out_counts, static_cast<cudaStream_t>(cuda_stream));
}

int32_t mans_ivfpq_search_partial_device(mans_ctx* ctx, mans_ivfpq* ix, mans_workspace* ws,
                                         const float* d_queries, int64_t nq, int32_t k,
                                         int32_t nprobe, int32_t* d_block, void* cuda_stream) {
  if (!ctx || !ix || ix->ctx != ctx) return fail(MANS_ERR_INVALID, "null or foreign IVF-PQ index");
  if (!ws || ws->ctx != ctx) return fail(MANS_ERR_INVALID, "workspace missing or foreign");
  if (nq < 0 || k <= 0 || !d_block) return fail(MANS_ERR_INVALID, "bad partial search request");
  if (nq == 0) return MANS_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  const int64_t kin = 2 * std::min<int32_t>(k, MANS_MAX_TOPK);
  if (ix->n <= 0 || ix->nlist <= 0) {  // an empty shard contributes nothing
    cudaError_t e = cudaMemsetAsync(d_block + 3 * nq * kin, 0, nq * sizeof(int32_t), st);
    return e == cudaSuccess ? MANS_OK : fail_cuda(e, "cudaMemsetAsync");
  }
  return run_ivfpq_search(ctx, ix, ws, d_queries, nq, k, nprobe, nullptr, nullptr, nullptr, st,
                          d_block);
}

int32_t mans_ivfpq_resolve_device(mans_ctx* ctx, mans_workspace* ws, const int32_t* d_blocks,
                                  int32_t n_blocks, int64_t block_stride, int64_t nq, int32_t k,
                                  float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                                  void* cuda_stream) {
  if (!ctx || !ws || ws->ctx != ctx) return fail(MANS_ERR_INVALID, "null context or workspace");
  if (nq < 0 || k <= 0 || n_blocks < 1 || !d_blocks) return fail(MANS_ERR_INVALID, "bad resolve request");
  if (nq == 0) return MANS_OK;
  const int32_t kout = std::min<int32_t>(k, MANS_MAX_TOPK);
  const int64_t kin = 2 * kout;
  if (block_stride < nq * (3 * kin + 1)) return fail(MANS_ERR_INVALID, "block stride too small");
  int n2 = 1;
  while (n2 < n_blocks * kin) n2 <<= 1;
  const size_t smem = static_cast<size_t>(n2) * (sizeof(uint64_t) + sizeof(uint32_t));
  if (smem > static_cast<size_t>(ctx->max_smem) - 1024)
    return fail(MANS_ERR_SEARCH, "too many shards x candidates to merge in shared memory");
  DeviceGuard g(ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  size_t o = 0;
  const size_t o_s = carve(o, nq * kin * sizeof(float));
  const size_t o_q = carve(o, nq * kin * sizeof(uint32_t));
  const size_t o_i = carve(o, nq * kin * sizeof(uint32_t));
  const size_t o_c = carve(o, nq * sizeof(int32_t));
  int32_t rc;
  if ((rc = ws->aux2.reserve(o)) != MANS_OK) return rc;
  uint8_t* A = static_cast<uint8_t*>(ws->aux2.ptr);
  float* ms = reinterpret_cast<float*>(A + o_s);
  uint32_t* mq = reinterpret_cast<uint32_t*>(A + o_q);
  uint32_t* mi = reinterpret_cast<uint32_t*>(A + o_i);
  int32_t* mc = reinterpret_cast<int32_t*>(A + o_c);
  cudaError_t e = cudaFuncSetAttribute(ivfpq_shard_merge_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return fail_cuda(e, "shard merge configure");
  ivfpq_shard_merge_kernel<<<static_cast<unsigned>(nq), 256, smem, st>>>(
      d_blocks, n_blocks, block_stride, nq, static_cast<int32_t>(kin), ms, mq, mi, mc);
  if ((e = cudaGetLastError()) != cudaSuccess) return fail_cuda(e, "shard merge launch");
  ResolveParams f{};
  f.in_score = ms;
  f.in_seq = mq;
  f.in_payload = mi;
  f.in_count = mc;
  f.kin = static_cast<int32_t>(kin);
  f.nq = nq;
  f.cap = kout;
  f.out_score = d_out_dist;
  f.out_id = d_out_ids;
  f.out_count = d_out_counts;
  f.kout = kout;
  bsl_resolve_kernel<<<static_cast<unsigned>(nq), 256, 0, st>>>(f);
  if ((e = cudaGetLastError()) != cudaSuccess) return fail_cuda(e, "resolve launch");
  ws->launches += 2;
  return MANS_OK;
}

int32_t mans_ivfpq_search(mans_ctx* ctx, mans_ivfpq* ix, const float* queries, int64_t nq,
                          int64_t dim, int32_t k, int32_t nprobe, float* out_dist,
                          uint32_t* out_ids, int32_t* out_counts) {
  if (!ctx || !ix || ix->ctx != ctx) return fail(MANS_ERR_INVALID, "null or foreign IVF-PQ index");
  if (nq < 0) return fail(MANS_ERR_INVALID, "negative query count");
  if (nq == 0) return MANS_OK;
  const int32_t kout = std::max<int32_t>(0, k);  // k wide: the list has no cap beyond k
  if (dim != ix->dim) {
    // _IVFPQIndex.search returns [] for a query of the wrong width (:184-186)
    for (int64_t i = 0; i < nq * kout; ++i) {
      out_dist[i] = __builtin_inff();
      out_ids[i] = MANS_EMPTY_ID;
    }
    for (int64_t i = 0; i < nq; ++i) out_counts[i] = 0;
    return MANS_OK;
  }
  if (!queries || !out_dist || !out_ids || !out_counts) return fail(MANS_ERR_INVALID, "null buffer");
  DeviceGuard g(ctx->device);
  mans_workspace* ws = acquire_workspace(ctx);
  if (!ws) return fail(MANS_ERR_OOM, "cannot create a workspace stream");
  const int32_t rc =
      host_buffer_search(ws, queries, nq, dim, kout, out_dist, out_ids, out_counts,
                         [&](const float* dq, float* dd, uint32_t* di, int32_t* dc,
                             cudaStream_t st) {
                           return run_ivfpq_search(ctx, ix, ws, dq, nq, k, nprobe, dd, di, dc, st);
                         });
  release_workspace(ctx, ws);
  return rc;
}

int32_t mans_pq_adc_list(mans_ctx* ctx, const float* query, int64_t dim, const float* codebooks,
                         int32_t m, int32_t ks, const uint8_t* codes, int64_t count,
                         float* out_dist) {
  if (!ctx) return fail(MANS_ERR_INVALID, "null context");
  if (int32_t r = reject_group(ctx, nullptr, "mans_pq_adc_list")) return r;
  if (count < 0) return fail(MANS_ERR_SEARCH, "Vector count must be non-negative");
  if (m <= 0 || dim <= 0 || dim % m != 0) return fail(MANS_ERR_DIM, "dimensionMismatch");
  if (count == 0) return MANS_OK;
  if (ks > 256) return fail(MANS_ERR_SEARCH, "GPU ADC supports at most 256 centroids per subspace");
  if (!query || !codebooks || !codes || !out_dist) return fail(MANS_ERR_INVALID, "null buffer");
  for (int64_t i = 0; i < count * m; ++i)
    if (codes[i] >= ks) return fail(MANS_ERR_SEARCH, "PQ code value out of range");
  const size_t table = static_cast<size_t>(m) * ks * sizeof(float);
  if (table > static_cast<size_t>(ctx->max_smem))
    return fail(MANS_ERR_SEARCH, "PQ distance table exceeds device shared memory");
  const int sub = static_cast<int>(dim / m);
  DeviceGuard g(ctx->device);
  mans_workspace* ws = acquire_workspace(ctx);
  if (!ws) return fail(MANS_ERR_OOM, "cannot create a workspace stream");
  cudaStream_t st = ws->stream;
  int32_t rc = MANS_OK;
  do {
    size_t o = 0;
    const size_t o_q = carve(o, dim * sizeof(float));
    const size_t o_cb = carve(o, static_cast<size_t>(m) * ks * sub * sizeof(float));
    const size_t o_c = carve(o, count * m);
    const size_t o_d = carve(o, count * sizeof(float));
    if ((rc = ws->aux.reserve(o)) != MANS_OK) break;
    uint8_t* A = static_cast<uint8_t*>(ws->aux.ptr);
    cudaError_t e = cudaMemcpyAsync(A + o_q, query, dim * sizeof(float), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(A + o_cb, codebooks, static_cast<size_t>(m) * ks * sub * sizeof(float),
                          cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(A + o_c, codes, count * m, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(pq_adc_list_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(table));
    if (e != cudaSuccess) {
      rc = fail_cuda(e, "ADC upload");
      break;
    }
    const int64_t blocks = std::min<int64_t>((count + kAdcThreads - 1) / kAdcThreads, 4 * ctx->num_sms);
    pq_adc_list_kernel<<<static_cast<unsigned>(blocks), kAdcThreads, table, st>>>(
        reinterpret_cast<float*>(A + o_q), reinterpret_cast<float*>(A + o_cb), m, ks, sub,
        A + o_c, count, reinterpret_cast<float*>(A + o_d));
    e = cudaGetLastError();
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(out_dist, A + o_d, count * sizeof(float), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) rc = fail_cuda(e, "ADC execution");
  } while (false);
  release_workspace(ctx, ws);
  return rc;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Encoding on the device (IVFPQIndex.add: nearestCoarseCentroid,
// IVFPQIndex.swift:514-550, then ProductQuantizer.encode(vector:subtracting:),
// ProductQuantizer.swift:120-169).
// ---------------------------------------------------------------------------

namespace mans {
namespace {

// One warp per vector.  Per subspace every lane scores the codewords
// lane, lane + 32, ... with the reference's sequential sum of ((v - c) - cb)^2
// and keeps the first strict minimum; the warp then takes the smallest
// (distance, index).  No distance below FLT_MAX leaves code 0, as the
// reference's `bestDistance = greatestFiniteMagnitude` start does.
__global__ void pq_encode_kernel(const float* __restrict__ vecs, int64_t n, int32_t dim,
                                 const float* __restrict__ coarse, int64_t coarse_ld,
                                 const uint32_t* __restrict__ assign,
                                 const float* __restrict__ codebooks, int32_t m, int32_t ks,
                                 int32_t sub, int32_t cb_in_smem, uint8_t* __restrict__ out) {
  extern __shared__ float cbs[];
  if (cb_in_smem) {
    for (int64_t i = threadIdx.x; i < static_cast<int64_t>(m) * ks * sub; i += blockDim.x)
      cbs[i] = codebooks[i];
    __syncthreads();
  }
  const float* cb = cb_in_smem ? cbs : codebooks;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; i < n;
       i += warps) {
    const float* v = vecs + i * dim;
    const float* c = coarse + static_cast<int64_t>(assign[i]) * coarse_ld;
    for (int s = 0; s < m; ++s) {
      float bd = 3.40282347e+38f;
      int bi = 0x7FFFFFFF;
      for (int w = lane; w < ks; w += 32) {
        const float* code = cb + (static_cast<int64_t>(s) * ks + w) * sub;
        float sum = 0.0f;
        for (int d = 0; d < sub; ++d) {
          const float delta = __fsub_rn(__fsub_rn(v[s * sub + d], c[s * sub + d]), code[d]);
          sum = __fadd_rn(sum, __fmul_rn(delta, delta));
        }
        if (sum < bd) {
          bd = sum;
          bi = w;
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const float od = __shfl_xor_sync(0xFFFFFFFFu, bd, o);
        const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
        if (od < bd || (od == bd && oi < bi)) {
          bd = od;
          bi = oi;
        }
      }
      if (lane == 0) out[i * m + s] = static_cast<uint8_t>(bi == 0x7FFFFFFF ? 0 : bi);
    }
  }
}

}  // namespace
}  // namespace mans

extern "C" int32_t mans_pq_encode(mans_ctx* ctx, const float* vectors, int64_t n, int64_t dim,
                                  const float* coarse, int32_t nlist, const float* codebooks,
                                  int32_t m, int32_t ks, int32_t metric, uint8_t* out_codes,
                                  int32_t* out_assign) {
  using namespace mans;
  if (!ctx || (n > 0 && (!vectors || !out_codes)) || !coarse || !codebooks)
    return fail(MANS_ERR_INVALID, "null context or buffer");
  if (int32_t r = reject_group(ctx, nullptr, "mans_pq_encode")) return r;
  if (n < 0 || dim <= 0 || nlist <= 0 || m <= 0 || ks <= 0 || ks > 256 || dim % m != 0)
    return fail(MANS_ERR_INVALID, "bad PQ shape (dim must split into m subspaces, ks <= 256)");
  if (metric < 0 || metric > 2) return fail(MANS_ERR_SEARCH, "PQ encode needs cosine, l2 or ip");
  if (n == 0) return MANS_OK;
  DeviceGuard g(ctx->device);
  const int32_t sub = static_cast<int32_t>(dim / m);
  mans_corpus* cc = nullptr;
  int32_t rc = corpus_upload(ctx, coarse, nlist, dim, 0, &cc);
  if (rc != MANS_OK) return rc;
  mans_workspace* ws = acquire_workspace(ctx);
  if (!ws) {
    corpus_free(cc);
    return fail(MANS_ERR_OOM, "no workspace stream");
  }
  const size_t cb_bytes = static_cast<size_t>(m) * ks * sub * sizeof(float);
  const int cb_in_smem = cb_bytes <= static_cast<size_t>(ctx->max_smem) - 1024 ? 1 : 0;
  const int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(1 << 20, (512ll << 20) / (dim * 4)));
  float *d_v = nullptr, *d_cb = nullptr, *d_dist = nullptr;
  uint32_t* d_assign = nullptr;
  int32_t* d_cnt = nullptr;
  uint8_t* d_codes = nullptr;
  auto ck = [&](cudaError_t x, const char* what) {
    if (rc == MANS_OK && x != cudaSuccess) rc = fail_cuda(x, what);
  };
  ck(cudaMalloc(&d_v, chunk * dim * sizeof(float)), "cudaMalloc(encode)");
  ck(cudaMalloc(&d_cb, cb_bytes), "cudaMalloc(encode)");
  ck(cudaMalloc(&d_dist, chunk * sizeof(float)), "cudaMalloc(encode)");
  ck(cudaMalloc(&d_assign, chunk * sizeof(uint32_t)), "cudaMalloc(encode)");
  ck(cudaMalloc(&d_cnt, chunk * sizeof(int32_t)), "cudaMalloc(encode)");
  ck(cudaMalloc(&d_codes, chunk * m), "cudaMalloc(encode)");
  if (rc == MANS_OK) ck(cudaMemcpy(d_cb, codebooks, cb_bytes, cudaMemcpyHostToDevice), "codebooks");
  if (rc == MANS_OK && cb_in_smem)
    ck(cudaFuncSetAttribute(pq_encode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            static_cast<int>(cb_bytes)),
       "encode configure");
  for (int64_t r0 = 0; rc == MANS_OK && r0 < n; r0 += chunk) {
    const int64_t rows = std::min(chunk, n - r0);
    ck(cudaMemcpyAsync(d_v, vectors + r0 * dim, rows * dim * sizeof(float),
                       cudaMemcpyHostToDevice, ws->stream),
       "vectors upload");
    // nearestCoarseCentroid: SIMDDistance, strict '<' = (distance, index) minimum
    if (rc == MANS_OK)
      rc = run_flat_search(ctx, cc, ws, d_v, rows, 1, metric, d_dist, d_assign, d_cnt, ws->stream,
                           kModeSimd, 512);
    if (rc == MANS_OK) {
      const int grid = static_cast<int>(std::min<int64_t>((rows + 7) / 8, ctx->num_sms * 8ll));
      pq_encode_kernel<<<grid, 256, cb_in_smem ? cb_bytes : 0, ws->stream>>>(
          d_v, rows, static_cast<int32_t>(dim), cc->rows, cc->ld, d_assign, d_cb, m, ks, sub,
          cb_in_smem, d_codes);
      ck(cudaGetLastError(), "encode launch");
    }
    if (rc == MANS_OK)
      ck(cudaMemcpyAsync(out_codes + r0 * m, d_codes, rows * m, cudaMemcpyDeviceToHost, ws->stream),
         "codes download");
    if (rc == MANS_OK && out_assign)
      ck(cudaMemcpyAsync(out_assign + r0, d_assign, rows * sizeof(uint32_t),
                         cudaMemcpyDeviceToHost, ws->stream),
         "assignment download");
    if (rc == MANS_OK) ck(cudaStreamSynchronize(ws->stream), "encode");
  }
  if (rc == MANS_OK) rc = check_device_error(ws, ws->stream);
  cudaFree(d_v);
  cudaFree(d_cb);
  cudaFree(d_dist);
  cudaFree(d_assign);
  cudaFree(d_cnt);
  cudaFree(d_codes);
  release_workspace(ctx, ws);
  corpus_free(cc);
  return rc;
}
