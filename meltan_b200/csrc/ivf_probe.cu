// ivf_probe.cu -- IVF-flat search of a few queries in one cooperative launch.
//
// The batch path (ivf.cu) takes six launches -- query norms, centroid scan,
// centroid merge, planner, list scan, slot merge -- and for a single query
// each is a latency step while the list scan reaches ~20 of 148 SMs.  This
// kernel runs the whole of IVFFlatSearch.scanProbedLists
// (Sources/MetalANNSCore/IVFFlatSearch.swift:214-291) for up to kProbeMaxQ
// queries in one launch of one block per SM (rows staged by 16-byte-aligned
// bulk copies, one per row, into shared memory):
//   1. centroid keys: block b scores centroid rows [b*nlist/G, (b+1)*nlist/G)
//      against every query (the dot in index order with separately rounded
//      multiply and add, the host-tier finalize of :293-311) and writes each
//      key as an order-preserving word;
//   -- grid barrier (bounded wait on a monotonic arrival counter) --
//   2. the blocks are split between the queries; each reads its query's
//      centroid keys and finds the nprobe smallest, ties to the lower list
//      index (smallestIndices, :314-382): for nprobe <= 32 every warp keeps
//      the smallest (key, index) pairs of its slice in registers and one warp
//      merges them; above that a 4-pass radix select and an index-order
//      compaction;
//   3. the blocks of a query split the concatenated rows of its probed lists
//      evenly.  Runs of at most 32 rows (cut at list ends) go to one stage
//      per consumer warp: lane i copies row i (one contiguous bulk copy on
//      its own mbarrier), scores it in the reference's summation order, and
//      each warp keeps its 32 smallest (distance, id) keys in registers;
//   4. each block merges its warps' lists into a slot; the last block of a
//      query to arrive (an arrival counter that it resets) selects the top-k
//      among the slot keys at or below the k-th smallest slot head.
// The result equals the batch path's: TopKHeap's strict (distance, id) order
// (:384-444) makes it independent of the order in which lists are visited.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"

namespace mans {
namespace {

constexpr int kProbeThreads = 256;
constexpr int kProbeWarps = kProbeThreads / 32;
constexpr int kProbeRows = 32;  // rows per tile: one per lane of the consumer warp
constexpr int kLoadBatch = 8;   // independent global loads a thread keeps in flight

struct ProbeParams {
  const float* queries;  // nq x dim
  int32_t nq;
  int32_t dim;
  int32_t ld;      // row pitch of centroids and packed rows (dim rounded up to 4)
  int32_t qw;      // staged query width (ld rounded up to 32)
  int32_t stages;  // tile stages = consumer warps in step 3
  int32_t metric;
  int32_t nlist;
  int32_t nprobe;  // < nlist, <= 256
  int32_t k;       // effective k, <= 32
  int32_t kout;    // output row width, <= 32
  const float* cent_rows;   // nlist x ld
  const float* cent_norms;
  const float* rows;        // packed rows, n x ld
  const float* row_norms;
  const uint32_t* ids;      // packed row -> reported id
  const int64_t* offsets;   // nlist + 1
  uint32_t* ckeys;          // [nq][nlist] ordered centroid distances
  uint64_t* slot_keys;      // [grid][32]
  unsigned long long* bar;
  unsigned long long bar_base;
  int32_t* done;  // [kProbeMaxQ] arrival counters, zero between launches
  float* out_dist;
  uint32_t* out_ids;
  int32_t* out_counts;
  int* err;
};

struct ProbeLayout {
  size_t full, q, qn, kv, hist, plist, lstart, pre, wl, ctl, total;
};

__host__ __device__ inline size_t probe_align(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Shared-memory row pitch of a staged tile: ld + 4 floats, so the rows of a
// quarter-warp start 4 banks apart and their 16-byte reads hit distinct banks.
__host__ __device__ inline int probe_pitch(int ld) { return ld + 4; }

// The tile stages sit at offset 0; after the scan the last block of a query
// reuses them for the group's slot keys and the merge candidates (up to
// 2 x grid x 32 keys), so they are at least that large.  One mbarrier per row
// of every stage.
__host__ __device__ inline ProbeLayout probe_layout(int ld, int qw, int stages, int nlist, int nq,
                                                    int grid) {
  ProbeLayout L;
  size_t o = static_cast<size_t>(stages) * kProbeRows * probe_pitch(ld) * 4;
  if (o < static_cast<size_t>(grid) * 64 * 8) o = static_cast<size_t>(grid) * 64 * 8;
  L.full = o = probe_align(o, 16);
  o += static_cast<size_t>(stages) * kProbeRows * 8;
  L.q = o = probe_align(o, 16);
  o += static_cast<size_t>(nq) * qw * 4;
  L.qn = o;
  o += kProbeMaxQ * 4;
  L.kv = o = probe_align(o, 16);
  o += static_cast<size_t>(nlist) * 4;
  L.hist = o = probe_align(o, 16);
  o += 256 * 4;
  L.plist = o;
  o += 256 * 4;
  L.lstart = o = probe_align(o, 8);
  o += 256 * 8;
  L.pre = o;
  o += 257 * 8;
  L.wl = o = probe_align(o, 8);
  o += kProbeWarps * 32 * 8;
  L.ctl = o;
  o += 16 * 4;
  L.total = o;
  return L;
}

__global__ void __launch_bounds__(kProbeThreads, 1) ivf_probe_kernel(const ProbeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(probe_align(reinterpret_cast<size_t>(smem_raw), 128));
  const ProbeLayout L = probe_layout(p.ld, p.qw, p.stages, p.nlist, p.nq, gridDim.x);
  float* tiles = reinterpret_cast<float*>(base);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + L.full);
  float* qs = reinterpret_cast<float*>(base + L.q);
  float* qn = reinterpret_cast<float*>(base + L.qn);
  uint32_t* kv = reinterpret_cast<uint32_t*>(base + L.kv);
  int* hist = reinterpret_cast<int*>(base + L.hist);
  int32_t* plist = reinterpret_cast<int32_t*>(base + L.plist);
  int64_t* lstart = reinterpret_cast<int64_t*>(base + L.lstart);
  int64_t* pre = reinterpret_cast<int64_t*>(base + L.pre);
  uint64_t* wl = reinterpret_cast<uint64_t*>(base + L.wl);
  volatile int* ctl = reinterpret_cast<volatile int*>(base + L.ctl);
  // ctl: [0] abort, [1] grid barrier passed, [2] radix bin, [3] rank left,
  //      [4] probed lists, [5] last block of the query, [6..7] merge threshold

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, b = blockIdx.x;
  const int qw = p.qw, ld = p.ld, pitch = probe_pitch(ld);
  const size_t stage_floats = static_cast<size_t>(kProbeRows) * pitch;
  const int c0 = static_cast<int>(static_cast<int64_t>(p.nlist) * b / G);
  const int c1 = static_cast<int>(static_cast<int64_t>(p.nlist) * (b + 1) / G);

  // warp 0 sets up every row barrier and starts copying this block's first
  // centroid rows (one per lane) while the block loads the queries
  uint32_t ph0 = 0;  // warp 0: parity of its lane's stage-0 barrier
  if (warp == 0) {
    for (int s = lane; s < p.stages * kProbeRows; s += 32) mbar_init(&full[s], 1);
    fence_mbar_init();
    __syncwarp();
    if (lane == 0) ctl[0] = 0;
    if (c0 + lane < min(c1, c0 + kProbeRows))
      stage_row(tiles + lane * pitch, p.cent_rows + static_cast<int64_t>(c0 + lane) * ld, ld,
                &full[lane]);
  }
  {
    const int total = p.nq * qw;
    for (int i0 = tid; i0 < total; i0 += kProbeThreads * kLoadBatch) {
      float v[kLoadBatch];
#pragma unroll
      for (int u = 0; u < kLoadBatch; ++u) {
        const int i = i0 + u * kProbeThreads;
        const int qq = i / qw, c = i - qq * qw;
        v[u] = (i < total && c < p.dim) ? __ldg(p.queries + static_cast<int64_t>(qq) * p.dim + c)
                                        : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < kLoadBatch; ++u)
        if (i0 + u * kProbeThreads < total) qs[i0 + u * kProbeThreads] = v[u];
    }
  }
  if (tid < kProbeMaxQ) qn[tid] = 0.0f;
  __syncthreads();

  // ---- 1. centroid keys of this block's centroid rows ----
  if (warp == 1 && lane < p.nq && p.metric != kIP) {
    // |q|^2 in index order (IVFFlatSearch.swift:226)
    const float4* v = reinterpret_cast<const float4*>(qs + lane * qw);
    float a = 0.0f;
#pragma unroll 4
    for (int c = 0; c < ld / 4; ++c) {
      const float4 x = v[c];
      a = __fadd_rn(a, __fmul_rn(x.x, x.x));
      a = __fadd_rn(a, __fmul_rn(x.y, x.y));
      a = __fadd_rn(a, __fmul_rn(x.z, x.z));
      a = __fadd_rn(a, __fmul_rn(x.w, x.w));
    }
    qn[lane] = a;
  }
  for (int t0 = c0; t0 < c1; t0 += kProbeRows) {
    const int c = t0 + lane;
    const bool has = c < c1 && lane < kProbeRows;
    float acc[kProbeMaxQ];
    bool ok = true;
    if (warp == 0) {
      if (t0 > c0 && has)
        stage_row(tiles + lane * pitch, p.cent_rows + static_cast<int64_t>(c) * ld, ld, &full[lane]);
      ok = wait_row(&full[lane], ph0, has, p.err);
      if (has) ph0 ^= 1u;
      if (ok) row_dots<kProbeMaxQ>(tiles + lane * pitch, qs, qw, p.nq, ld, acc);
      else if (lane == 0) ctl[0] = 1;
    }
    __syncthreads();  // qn ready; an abort is seen by every warp
    if (warp == 0 && ok && has) {
      const float cn = p.metric != kIP ? __ldg(p.cent_norms + c) : 0.0f;
#pragma unroll
      for (int i = 0; i < kProbeMaxQ; ++i)
        if (i < p.nq)
          p.ckeys[static_cast<int64_t>(i) * p.nlist + c] =
              float_to_ordered(finalize_distance(p.metric, acc[i], qn[i], cn));
    }
    __syncthreads();
    if (ctl[0]) break;
  }

  // ---- grid barrier: every block's centroid keys are written (block barrier,
  // then one thread releases, arrives and acquires -- the keys written by the
  // block's other threads are ordered by the block barrier) ----
  if (tid == 0) {
    __threadfence();
    atomicAdd(p.bar, 1ull);
    const unsigned long long target = p.bar_base + static_cast<unsigned long long>(G);
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
    ctl[1] = ok;
  }
  __syncthreads();
  const bool failed = ctl[0] != 0 || ctl[1] == 0;

  // the query this block serves and its block group [gb0, gb1)
  const int q = static_cast<int>(static_cast<int64_t>(b) * p.nq / G);
  const int gb0 = static_cast<int>((static_cast<int64_t>(q) * G + p.nq - 1) / p.nq);
  const int gb1 = static_cast<int>((static_cast<int64_t>(q + 1) * G + p.nq - 1) / p.nq);
  const int gs = gb1 - gb0, j = b - gb0;
  const uint32_t* qkeys = p.ckeys + static_cast<int64_t>(q) * p.nlist;

  uint64_t best = kKeyMax, kth = kKeyMax;
  if (!failed) {
    // ---- 2. the nprobe smallest centroid keys of query q, ties to the lower
    // list index ----
    for (int i0 = tid; i0 < p.nlist; i0 += kProbeThreads * kLoadBatch) {
      uint32_t v[kLoadBatch];
#pragma unroll
      for (int u = 0; u < kLoadBatch; ++u) {
        const int i = i0 + u * kProbeThreads;
        v[u] = i < p.nlist ? __ldcg(qkeys + i) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kLoadBatch; ++u)
        if (i0 + u * kProbeThreads < p.nlist) kv[i0 + u * kProbeThreads] = v[u];
    }
    __syncthreads();
    int np = p.nprobe;
    if (p.nprobe <= 32) {
      // 64-bit keys (ordered distance, list index): every warp keeps the 32
      // smallest of its slice in registers, then warp 0 merges the eight lists
      const int per = (p.nlist + kProbeWarps - 1) / kProbeWarps;
      const int w0 = warp * per, w1 = min(p.nlist, w0 + per);
      uint64_t wb = kKeyMax, wk = kKeyMax;
      for (int i0 = w0; i0 < w1; i0 += 32) {
        const int i = i0 + lane;
        const uint64_t key =
            i < w1 ? (static_cast<uint64_t>(kv[i]) << 32) | static_cast<uint32_t>(i) : kKeyMax;
        warp_topk_offer(wb, wk, key, p.nprobe, lane);
      }
      wl[warp * 32 + lane] = wb;
      __syncthreads();
      if (warp == 0) {
        uint64_t m = wl[lane];
        for (int w = 1; w < kProbeWarps; ++w) {
          const uint64_t x = wl[w * 32 + lane];
          if (__shfl_sync(0xFFFFFFFFu, x, 0) >= __shfl_sync(0xFFFFFFFFu, m, p.nprobe - 1))
            continue;
          m = warp_merge32(m, x, lane);
        }
        if (lane < p.nprobe) plist[lane] = static_cast<int32_t>(static_cast<uint32_t>(m));
      }
      __syncthreads();
    } else {
      // 4-pass radix select of the nprobe-th smallest distance word (lanes
      // with equal digits add to the histogram once), then every word below
      // it and the lowest-index words equal to it, in ascending list order
      uint32_t prefix = 0, mask = 0;
      int rank = p.nprobe;  // 1-based rank sought among the words matching prefix
      for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        hist[tid] = 0;
        __syncthreads();
        for (int i0 = warp * 32; i0 < p.nlist; i0 += kProbeThreads) {
          const int i = i0 + lane;
          const uint32_t v = i < p.nlist ? kv[i] : 0u;
          const bool act = i < p.nlist && (v & mask) == prefix;
          const unsigned am = __ballot_sync(0xFFFFFFFFu, act);
          if (act) {
            const uint32_t bin = (v >> shift) & 255u;
            const unsigned peers = __match_any_sync(am, bin);
            if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
          }
        }
        __syncthreads();
        if (warp == 0) {
          int h[8], s = 0;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            h[i] = hist[lane * 8 + i];
            s += h[i];
          }
          int incl = s;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += u;
          }
          const int excl = incl - s;
          if (excl < rank && rank <= incl) {
            int c = excl, bin = lane * 8 + 7;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              if (c + h[i] >= rank) {
                bin = lane * 8 + i;
                break;
              }
              c += h[i];
            }
            ctl[2] = bin;
            ctl[3] = rank - c;
          }
        }
        __syncthreads();
        prefix |= static_cast<uint32_t>(ctl[2]) << shift;
        mask |= 0xFFu << shift;
        rank = ctl[3];
      }
      if (warp == 0) {
        int taken = 0, eq_seen = 0;
        for (int i0 = 0; i0 < p.nlist; i0 += 32) {
          const int i = i0 + lane;
          const uint32_t v = i < p.nlist ? kv[i] : 0u;
          const bool lt = i < p.nlist && v < prefix;
          const bool eq = i < p.nlist && v == prefix;
          const unsigned eqm = __ballot_sync(0xFFFFFFFFu, eq);
          const bool take = lt || (eq && eq_seen + __popc(eqm & ((1u << lane) - 1u)) < rank);
          const unsigned tm = __ballot_sync(0xFFFFFFFFu, take);
          if (take) plist[taken + __popc(tm & ((1u << lane) - 1u))] = i;
          taken += __popc(tm);
          eq_seen += __popc(eqm);
        }
        if (lane == 0) ctl[4] = taken;
      }
      __syncthreads();
      np = ctl[4];
    }
    // list lengths and their running sum (np <= 256 = threads)
    int64_t len = 0;
    if (tid < np) {
      const int l = plist[tid];
      const int64_t s = p.offsets[l];
      len = p.offsets[l + 1] - s;
      lstart[tid] = s;
    }
    int64_t incl = len;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += u;
    }
    int64_t* wsum = reinterpret_cast<int64_t*>(wl) + 32;  // warp totals (wl[32..40) is free)
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int64_t add = 0;
    for (int w = 0; w < warp; ++w) add += wsum[w];
    pre[tid + 1] = incl + add;
    if (tid == 0) pre[0] = 0;
    __syncthreads();
    const int64_t R = pre[np];
    const int64_t lo = R * j / gs, hi = R * (j + 1) / gs;

    // ---- 3. scan this block's share of the probed rows ----
    if (warp < p.stages) {
      int li = 0;
      int64_t pos = lo;
      // next run of at most 32 rows of [lo, hi) within one list
      auto next_tile = [&](int64_t& row, int& cnt) -> bool {
        if (pos >= hi) return false;
        while (pre[li + 1] <= pos) ++li;
        const int64_t end = pre[li + 1] < hi ? pre[li + 1] : hi;
        cnt = static_cast<int>(end - pos < kProbeRows ? end - pos : kProbeRows);
        row = lstart[li] + (pos - pre[li]);
        pos += cnt;
        return true;
      };
      int64_t row = 0;
      int cnt = 0;
      bool have = true;
      for (int s = 0; s < warp && have; ++s) have = next_tile(row, cnt);  // warp w: tiles w, w+S, ...
      have = have && next_tile(row, cnt);
      float* srow = tiles + warp * stage_floats + lane * pitch;
      uint64_t* bar = &full[warp * kProbeRows + lane];
      uint32_t ph = warp == 0 ? ph0 : 0u;
      if (have && lane < cnt) stage_row(srow, p.rows + (row + lane) * ld, ld, bar);
      const float qnq = qn[q];
      while (have) {
        const bool valid = lane < cnt;
        float vn = 0.0f;
        uint32_t id = 0;
        if (valid) {
          if (p.metric != kIP) vn = __ldg(p.row_norms + row + lane);
          id = __ldg(p.ids + row + lane);
        }
        if (!wait_row(bar, ph, valid, p.err)) {
          if (lane == 0) ctl[0] = 1;
          break;
        }
        if (valid) ph ^= 1u;
        float acc[1];
        row_dots<1>(srow, qs + q * qw, qw, 1, ld, acc);
        __syncwarp();
        int64_t row2 = 0;
        int cnt2 = 0;
        bool have2 = true;
        for (int s = 0; s < p.stages - 1 && have2; ++s) have2 = next_tile(row2, cnt2);
        have2 = have2 && next_tile(row2, cnt2);
        if (have2 && lane < cnt2) stage_row(srow, p.rows + (row2 + lane) * ld, ld, bar);
        const float d = finalize_distance(p.metric, acc[0], qnq, vn);
        warp_topk_offer(best, kth, valid ? make_key(d, id) : kKeyMax, p.k, lane);
        row = row2;
        cnt = cnt2;
        have = have2;
      }
    }
  }

  // ---- 4. block list -> slot; the last block of the query merges ----
  __syncthreads();
  wl[warp * 32 + lane] = best;
  __syncthreads();
  if (warp == 0) {
    uint64_t m = wl[lane];
    for (int w = 1; w < kProbeWarps; ++w) {
      const uint64_t x = wl[w * 32 + lane];
      if (__shfl_sync(0xFFFFFFFFu, x, 0) >= __shfl_sync(0xFFFFFFFFu, m, p.k - 1)) continue;
      m = warp_merge32(m, x, lane);
    }
    p.slot_keys[static_cast<size_t>(b) * 32 + lane] = m;
    __syncwarp();
    if (lane == 0) {
      __threadfence();
      const bool last = atomicAdd(&p.done[q], 1) == gs - 1;
      if (last) {
        __threadfence();  // the other blocks' slots are read after this
        p.done[q] = 0;    // ready for the next launch
      }
      ctl[5] = last ? 1 : 0;
    }
  }
  __syncthreads();
  if (!ctl[5]) return;
  // The k smallest of the group's slots.  A slot's keys past its k-th cannot
  // be among them (k smaller keys share its slot), and none of them lies above
  // T0, the k-th smallest slot head (the k slots with heads at or below T0
  // each hold a key at or below it).  Load the first k keys of every slot at
  // once into the idle tile stages, take T0, and select among the keys <= T0.
  uint64_t* sk = reinterpret_cast<uint64_t*>(tiles);
  const int kk = p.k;
  const int nsk = gs * kk;
  for (int i0 = tid; i0 < nsk; i0 += kProbeThreads * kLoadBatch) {
    uint64_t v[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = i0 + u * kProbeThreads;
      const int s = i / kk;
      v[u] = i < nsk ? __ldcg(p.slot_keys + static_cast<size_t>(gb0 + s) * 32 + (i - s * kk))
                     : kKeyMax;
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u)
      if (i0 + u * kProbeThreads < nsk) sk[i0 + u * kProbeThreads] = v[u];
  }
  __syncthreads();
  if (warp == 0) {
    uint64_t hb = kKeyMax, hk = kKeyMax;
    for (int s0 = 0; s0 < gs; s0 += 32) {
      const int s = s0 + lane;
      warp_topk_offer(hb, hk, s < gs ? sk[s * kk] : kKeyMax, kk, lane);
    }
    if (lane == 0) {
      ctl[6] = static_cast<int>(static_cast<uint32_t>(hk));
      ctl[7] = static_cast<int>(static_cast<uint32_t>(hk >> 32));
      hist[0] = 0;
    }
  }
  __syncthreads();
  const uint64_t t0 = (static_cast<uint64_t>(static_cast<uint32_t>(ctl[7])) << 32) |
                      static_cast<uint32_t>(ctl[6]);
  // candidates (at most k*k, or every key when fewer than k slots are filled)
  // go after the loaded keys in the same area (2 x grid x 32 keys in all)
  uint64_t* cand = sk + nsk;
  for (int i = tid; i < nsk; i += kProbeThreads) {
    const uint64_t x = sk[i];
    if (x != kKeyMax && x <= t0) cand[atomicAdd(&hist[0], 1)] = x;
  }
  __syncthreads();
  const int nc = hist[0];
  uint64_t m = kKeyMax, mk = kKeyMax;
  for (int i0 = warp * 32; i0 < nc; i0 += kProbeThreads) {
    const int i = i0 + lane;
    warp_topk_offer(m, mk, i < nc ? cand[i] : kKeyMax, kk, lane);
  }
  wl[warp * 32 + lane] = m;
  __syncthreads();
  if (warp == 0) {
    uint64_t r = wl[lane];
    for (int w = 1; w < kProbeWarps; ++w) {
      const uint64_t x = wl[w * 32 + lane];
      if (__shfl_sync(0xFFFFFFFFu, x, 0) >= __shfl_sync(0xFFFFFFFFu, r, kk - 1)) continue;
      r = warp_merge32(r, x, lane);
    }
    // a device wait that gave up anywhere leaves every result empty
    const bool bad = *reinterpret_cast<volatile int*>(p.err) != 0;
    const bool valid = !bad && lane < kk && r != kKeyMax;
    const unsigned vm = __ballot_sync(0xFFFFFFFFu, valid);
    if (lane < p.kout) {
      p.out_dist[static_cast<int64_t>(q) * p.kout + lane] =
          valid ? key_distance(r) : __int_as_float(0x7F800000);
      p.out_ids[static_cast<int64_t>(q) * p.kout + lane] = valid ? key_id(r) : kEmptyId;
    }
    if (lane == 0) p.out_counts[q] = __popc(vm);
  }
}

}  // namespace

// The most tile stages (consumer warps) that fit the shared memory.
static int probe_stages(const mans_ctx* ctx, int64_t ld, int32_t nlist, int64_t nq) {
  const int qw = static_cast<int>((ld + 31) / 32 * 32);
  int stages = 0;
  for (int s = 1; s <= kProbeWarps; ++s)
    if (probe_layout(static_cast<int>(ld), qw, s, nlist, static_cast<int>(nq), ctx->num_sms).total +
            128 <= static_cast<size_t>(ctx->max_smem))
      stages = s;
  return stages;
}

bool ivf_probe_applies(const mans_ctx* ctx, const mans_corpus* packed, int32_t nlist, int64_t nq,
                       int32_t kout, int32_t probe) {
  if (nq < 1 || nq > kProbeMaxQ || nq > ctx->num_sms) return false;
  if (kout < 1 || kout > 32 || probe < 1 || probe > 256 || probe >= nlist) return false;
  if (nlist > kProbeMaxNlist || !ctx->coop_launch || packed->n >= INT32_MAX) return false;
  return probe_stages(ctx, packed->ld, nlist, nq) >= 1;
}

int32_t run_ivf_probe(mans_ctx* ctx, const mans_corpus* cent, const mans_corpus* packed,
                      const int64_t* d_offsets, mans_workspace* ws, const float* d_queries,
                      int64_t nq, int32_t kout, int32_t keff, int32_t probe, int32_t metric,
                      float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                      cudaStream_t stream) {
  const int32_t nlist = static_cast<int32_t>(cent->n);
  const int ld = static_cast<int>(cent->ld);
  const int qw = (ld + 31) / 32 * 32;
  const int stages = probe_stages(ctx, ld, nlist, nq);
  const int grid = ctx->num_sms;
  int32_t rc;
  if ((rc = ws->aux.reserve(static_cast<size_t>(nq) * nlist * sizeof(uint32_t))) != MANS_OK)
    return rc;
  if ((rc = ws->slot_keys.reserve(static_cast<size_t>(grid) * 32 * sizeof(uint64_t))) != MANS_OK)
    return rc;
  if ((rc = ws->err.reserve(sizeof(int))) != MANS_OK) return rc;
  if (!ws->err_cleared) {
    cudaError_t e = cudaMemsetAsync(ws->err.ptr, 0, sizeof(int), stream);
    if (e != cudaSuccess) return fail_cuda(e, "cudaMemsetAsync(err)");
    ws->err_cleared = true;
  }
  if (!ws->probe_sync.ptr) {
    if ((rc = ws->probe_sync.reserve(kProbeSyncBytes)) != MANS_OK) return rc;
    cudaError_t e = cudaMemsetAsync(ws->probe_sync.ptr, 0, kProbeSyncBytes, stream);
    if (e != cudaSuccess) return fail_cuda(e, "cudaMemsetAsync(probe counters)");
    ws->probe_bar_base = 0;
  }
  ProbeParams p{};
  p.queries = d_queries;
  p.nq = static_cast<int32_t>(nq);
  p.dim = static_cast<int32_t>(cent->dim);
  p.ld = ld;
  p.qw = qw;
  p.stages = stages;
  p.metric = metric;
  p.nlist = nlist;
  p.nprobe = probe;
  p.k = keff;
  p.kout = kout;
  p.cent_rows = cent->rows;
  p.cent_norms = cent->norms;
  p.rows = packed->rows;
  p.row_norms = packed->norms;
  p.ids = packed->ids;
  p.offsets = d_offsets;
  p.ckeys = static_cast<uint32_t*>(ws->aux.ptr);
  p.slot_keys = static_cast<uint64_t*>(ws->slot_keys.ptr);
  p.bar = static_cast<unsigned long long*>(ws->probe_sync.ptr);
  p.bar_base = ws->probe_bar_base;
  p.done = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws->probe_sync.ptr) + 64);
  p.out_dist = d_out_dist;
  p.out_ids = d_out_ids;
  p.out_counts = d_out_counts;
  p.err = static_cast<int*>(ws->err.ptr);
  const size_t smem = probe_layout(ld, qw, stages, nlist, static_cast<int>(nq), grid).total + 128;
  cudaError_t e = cudaSuccess;
  if (!ctx->probe_configured) {  // the largest opt-in size, once per context (device)
    e = cudaFuncSetAttribute(ivf_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ctx->max_smem);
    if (e != cudaSuccess) return fail_cuda(e, "ivf probe configure");
    ctx->probe_configured = true;
  }
  void* args[] = {&p};
  cudaEvent_t stop = timing_begin(ws, stream);
  e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(ivf_probe_kernel), grid,
                                  kProbeThreads, args, smem, stream);
  if (e != cudaSuccess) return fail_cuda(e, "ivf probe launch");
  timing_end(stop, stream);
  ws->probe_bar_base += static_cast<unsigned long long>(grid);
  ws->launches += 1;
  return MANS_OK;
}

}  // namespace mans
