// ivf_probe.cu -- IVF-flat search of a few queries in one cooperative launch.
//
// The batch path (ivf.cu) takes six launches -- query norms, centroid scan,
// centroid merge, planner, list scan, slot merge -- and for a single query
// each is a latency step while the list scan reaches ~20 of 148 SMs.  This
// kernel runs the whole of IVFFlatSearch.scanProbedLists
// (Sources/MetalANNSCore/IVFFlatSearch.swift:214-291) for up to kProbeMaxQ
// queries in one launch of one block per SM:
//   1. centroid keys: block b scores centroid rows [b*nlist/G, (b+1)*nlist/G)
//      against every query (the dot in index order with separately rounded
//      multiply and add, the host-tier finalize of :293-311) and writes each
//      key as an order-preserving word;
//   -- grid barrier (bounded wait on a monotonic arrival counter) --
//   2. the blocks are split between the queries; each reads its query's
//      centroid keys and finds the nprobe smallest, ties to the lower list
//      index (smallestIndices, :314-382), by a 4-pass radix select followed
//      by an index-order compaction;
//   3. the blocks of a query split the concatenated rows of its probed lists
//      evenly.  Runs of at most 32 rows (cut at list ends) stream through TMA
//      into one shared-memory stage per consumer warp; lane i scores row i and
//      each warp keeps its 32 smallest (distance, id) keys in registers;
//   4. each block merges its warps' lists into a slot; the last block of a
//      query to arrive (an arrival counter that it resets) merges the slots
//      and writes the sorted top-k.
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
constexpr int kProbeRows = 32;                              // rows per tile (one box)
constexpr int kProbeBoxBytes = kProbeRows * kTileCols * 4;  // 4 KiB per 32 x 32 box

struct ProbeParams {
  const float* queries;  // nq x dim
  int32_t nq;
  int32_t dim;
  int32_t nchunks;  // ceil(dim / 32)
  int32_t stages;   // tile stages = consumer warps in step 3
  int32_t metric;
  int32_t nlist;
  int32_t nprobe;  // < nlist, <= 256
  int32_t k;       // effective k, <= 32
  int32_t kout;    // output row width, <= 32
  const float* cent_norms;
  const float* row_norms;
  const uint32_t* ids;     // packed row -> reported id
  const int64_t* offsets;  // nlist + 1
  uint32_t* ckeys;         // [nq][nlist] ordered centroid distances
  uint64_t* slot_keys;     // [grid][32]
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

// The tile stages sit at offset 0; after the scan the last block of a query
// reuses them for the group's slots (grid x 32 keys), so they are at least
// that large.
__host__ __device__ inline ProbeLayout probe_layout(int nchunks, int stages, int nlist, int nq,
                                                    int grid) {
  ProbeLayout L;
  size_t o = static_cast<size_t>(stages) * nchunks * kProbeBoxBytes;
  if (o < static_cast<size_t>(grid) * 32 * 8) o = probe_align(static_cast<size_t>(grid) * 256, 1024);
  L.full = o;
  o += 8 * 8;
  L.q = o = probe_align(o, 16);
  o += static_cast<size_t>(nq) * nchunks * kTileCols * 4;
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

// dot(q, row `lane` of a staged tile) in index order.  The tile is nchunks
// boxes of 32 rows x 32 fp32 with the 128-byte swizzle (16-byte chunk j of
// row r at chunk j ^ (r & 7)), so the eight lanes of a quarter-warp read
// eight distinct bank groups.
__device__ __forceinline__ float tile_row_dot(const uint8_t* tile, int lane, const float* q,
                                              int nchunks) {
  float a = 0.0f;
  for (int cc = 0; cc < nchunks; ++cc) {
    const uint8_t* rowp = tile + cc * kProbeBoxBytes + lane * 128;
    const float4* qv = reinterpret_cast<const float4*>(q + cc * kTileCols);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(rowp + ((j ^ (lane & 7)) << 4));
      const float4 b = qv[j];
      a = __fadd_rn(a, __fmul_rn(v.x, b.x));
      a = __fadd_rn(a, __fmul_rn(v.y, b.y));
      a = __fadd_rn(a, __fmul_rn(v.z, b.z));
      a = __fadd_rn(a, __fmul_rn(v.w, b.w));
    }
  }
  return a;
}

// The same for up to kProbeMaxQ queries at once (independent chains).
__device__ __forceinline__ void tile_row_dots(const uint8_t* tile, int lane, const float* q,
                                              int qw, int nq, int nchunks,
                                              float (&acc)[kProbeMaxQ]) {
#pragma unroll
  for (int i = 0; i < kProbeMaxQ; ++i) acc[i] = 0.0f;
  for (int cc = 0; cc < nchunks; ++cc) {
    const uint8_t* rowp = tile + cc * kProbeBoxBytes + lane * 128;
    float4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = *reinterpret_cast<const float4*>(rowp + ((j ^ (lane & 7)) << 4));
#pragma unroll
    for (int i = 0; i < kProbeMaxQ; ++i) {
      if (i >= nq) break;
      const float4* qv = reinterpret_cast<const float4*>(q + i * qw + cc * kTileCols);
      float a = acc[i];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 b = qv[j];
        a = __fadd_rn(a, __fmul_rn(v[j].x, b.x));
        a = __fadd_rn(a, __fmul_rn(v[j].y, b.y));
        a = __fadd_rn(a, __fmul_rn(v[j].z, b.z));
        a = __fadd_rn(a, __fmul_rn(v[j].w, b.w));
      }
      acc[i] = a;
    }
  }
}

__device__ __forceinline__ void load_tile(uint8_t* dst, const CUtensorMap* map, int64_t row,
                                          int nchunks, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nchunks) * kProbeBoxBytes);
  for (int cc = 0; cc < nchunks; ++cc)
    tma_load_2d(dst + cc * kProbeBoxBytes, map, cc * kTileCols, static_cast<int32_t>(row), bar);
}

__global__ void __launch_bounds__(kProbeThreads, 1)
    ivf_probe_kernel(const __grid_constant__ CUtensorMap cmap,
                     const __grid_constant__ CUtensorMap pmap, const ProbeParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(probe_align(reinterpret_cast<size_t>(smem_raw), 1024));
  const ProbeLayout L = probe_layout(p.nchunks, p.stages, p.nlist, p.nq, gridDim.x);
  uint8_t* tiles = base;
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
  //      [4] probed lists, [5] last block of the query

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x, b = blockIdx.x;
  const int qw = p.nchunks * kTileCols;
  const uint32_t tile_bytes = static_cast<uint32_t>(p.nchunks) * kProbeBoxBytes;

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    ctl[0] = 0;
  }
  if (tid == 32) {
    tma_prefetch_desc(&cmap);
    tma_prefetch_desc(&pmap);
  }
  for (int i = tid; i < p.nq * qw; i += kProbeThreads) {
    const int q = i / qw, c = i - q * qw;
    qs[i] = c < p.dim ? p.queries[static_cast<int64_t>(q) * p.dim + c] : 0.0f;
  }
  if (tid < kProbeMaxQ) qn[tid] = 0.0f;
  __syncthreads();

  // ---- 1. centroid keys of this block's centroid rows ----
  const int c0 = static_cast<int>(static_cast<int64_t>(p.nlist) * b / G);
  const int c1 = static_cast<int>(static_cast<int64_t>(p.nlist) * (b + 1) / G);
  if (tid == 0 && c1 > c0) load_tile(tiles, &cmap, c0, p.nchunks, &full[0]);
  if (warp == 1 && lane < p.nq && p.metric != kIP) {
    // |q|^2 in index order (IVFFlatSearch.swift:226); the zero padding past
    // dim adds +0, which leaves a sum that started at +0 unchanged
    const float4* v = reinterpret_cast<const float4*>(qs + lane * qw);
    float a = 0.0f;
#pragma unroll 4
    for (int c = 0; c < qw / 4; ++c) {
      const float4 x = v[c];
      a = __fadd_rn(a, __fmul_rn(x.x, x.x));
      a = __fadd_rn(a, __fmul_rn(x.y, x.y));
      a = __fadd_rn(a, __fmul_rn(x.z, x.z));
      a = __fadd_rn(a, __fmul_rn(x.w, x.w));
    }
    qn[lane] = a;
  }
  __syncthreads();
  uint32_t ph0 = 0;
  for (int t0 = c0; t0 < c1; t0 += kProbeRows) {
    if (t0 > c0 && tid == 0) load_tile(tiles, &cmap, t0, p.nchunks, &full[0]);
    if (warp == 0) {
      const bool ok = mbar_wait_bounded(&full[0], ph0, p.err);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        mbar_wait_bounded(&full[0], ph0, nullptr);  // the copy in flight: once more, bounded
        if (lane == 0) ctl[0] = 1;
      } else {
        float acc[kProbeMaxQ];
        tile_row_dots(tiles, lane, qs, qw, p.nq, p.nchunks, acc);
        const int c = t0 + lane;
        if (c < c1) {
          const float cn = p.metric != kIP ? __ldg(p.cent_norms + c) : 0.0f;
#pragma unroll
          for (int i = 0; i < kProbeMaxQ; ++i)
            if (i < p.nq)
              p.ckeys[static_cast<int64_t>(i) * p.nlist + c] =
                  float_to_ordered(finalize_distance(p.metric, acc[i], qn[i], cn));
        }
        __threadfence();  // the keys are read by other blocks after the grid barrier
      }
    }
    ph0 ^= 1u;
    __syncthreads();
    if (ctl[0]) break;
  }

  // ---- grid barrier: every block's centroid keys are written ----
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

  uint64_t best = kKeyMax, kth = kKeyMax;
  if (!failed) {
    // ---- 2. the nprobe smallest centroid keys of query q ----
    for (int i = tid; i < p.nlist; i += kProbeThreads)
      kv[i] = __ldcg(p.ckeys + static_cast<int64_t>(q) * p.nlist + i);
    uint32_t prefix = 0, mask = 0;
    int rank = p.nprobe;  // 1-based rank of the word sought among those matching prefix
    for (int pass = 0; pass < 4; ++pass) {
      const int shift = 24 - 8 * pass;
      hist[tid] = 0;
      __syncthreads();
      for (int i = tid; i < p.nlist; i += kProbeThreads) {
        const uint32_t v = kv[i];
        if ((v & mask) == prefix) atomicAdd(&hist[(v >> shift) & 255u], 1);
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
    // every word below `prefix`, then the `rank` lowest-index words equal to
    // it, in ascending list order
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
    const int np = ctl[4];
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
    int64_t* wsum = reinterpret_cast<int64_t*>(wl);  // warp totals (wl is free until step 4)
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
      uint8_t* st = tiles + static_cast<size_t>(warp) * tile_bytes;
      uint32_t ph = warp == 0 ? ph0 : 0u;
      if (have && lane == 0) load_tile(st, &pmap, row, p.nchunks, &full[warp]);
      const float qnq = qn[q];
      while (have) {
        const bool valid = lane < cnt;
        float vn = 0.0f;
        uint32_t id = 0;
        if (valid) {
          if (p.metric != kIP) vn = __ldg(p.row_norms + row + lane);
          id = __ldg(p.ids + row + lane);
        }
        const bool ok = mbar_wait_bounded(&full[warp], ph, p.err);
        if (__any_sync(0xFFFFFFFFu, !ok)) {
          mbar_wait_bounded(&full[warp], ph, nullptr);  // the copy in flight: once more, bounded
          if (lane == 0) ctl[0] = 1;
          break;
        }
        ph ^= 1u;
        const float acc = tile_row_dot(st, lane, qs + q * qw, p.nchunks);
        __syncwarp();
        int64_t row2 = 0;
        int cnt2 = 0;
        bool have2 = true;
        for (int s = 0; s < p.stages - 1 && have2; ++s) have2 = next_tile(row2, cnt2);
        have2 = have2 && next_tile(row2, cnt2);
        if (have2 && lane == 0) load_tile(st, &pmap, row2, p.nchunks, &full[warp]);
        const float d = finalize_distance(p.metric, acc, qnq, vn);
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
    for (int w = 1; w < kProbeWarps; ++w) m = warp_merge32(m, wl[w * 32 + lane], lane);
    p.slot_keys[static_cast<size_t>(b) * 32 + lane] = m;
    __threadfence();
    __syncwarp();
    if (lane == 0) ctl[5] = atomicAdd(&p.done[q], 1) == gs - 1 ? 1 : 0;
    __syncwarp();
  }
  __syncthreads();
  if (!ctl[5]) return;
  __threadfence();
  if (tid == 0) p.done[q] = 0;  // ready for the next launch
  // the group's slots, all loads in flight at once (the tile stages are idle:
  // every copy issued into them has been waited for)
  uint64_t* sk = reinterpret_cast<uint64_t*>(tiles);
  for (int i = tid; i < gs * 32; i += kProbeThreads)
    sk[i] = __ldcg(p.slot_keys + static_cast<size_t>(gb0) * 32 + i);
  __syncthreads();
  uint64_t m = kKeyMax, mk = kKeyMax;
  for (int s = warp; s < gs; s += kProbeWarps) {
    const uint64_t x = sk[s * 32 + lane];
    if (__shfl_sync(0xFFFFFFFFu, x, 0) >= mk) continue;
    m = warp_merge32(m, x, lane);
    mk = __shfl_sync(0xFFFFFFFFu, m, p.k - 1);
  }
  wl[warp * 32 + lane] = m;
  __syncthreads();
  if (warp == 0) {
    uint64_t r = wl[lane];
    for (int w = 1; w < kProbeWarps; ++w) r = warp_merge32(r, wl[w * 32 + lane], lane);
    // a device wait that gave up anywhere leaves every result empty
    const bool bad = *reinterpret_cast<volatile int*>(p.err) != 0;
    const bool valid = !bad && lane < p.k && r != kKeyMax;
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
static int probe_stages(const mans_ctx* ctx, int64_t dim, int32_t nlist, int64_t nq) {
  const int nchunks = static_cast<int>((dim + kTileCols - 1) / kTileCols);
  int stages = 0;
  for (int s = 1; s <= kProbeWarps; ++s)
    if (probe_layout(nchunks, s, nlist, static_cast<int>(nq), ctx->num_sms).total + 1024 <=
        static_cast<size_t>(ctx->max_smem))
      stages = s;
  return stages;
}

bool ivf_probe_applies(const mans_ctx* ctx, const mans_corpus* packed, int32_t nlist, int64_t nq,
                       int32_t kout, int32_t probe) {
  if (nq < 1 || nq > kProbeMaxQ || nq > ctx->num_sms) return false;
  if (kout < 1 || kout > 32 || probe < 1 || probe > 256 || probe >= nlist) return false;
  if (nlist > kProbeMaxNlist || !ctx->coop_launch || packed->n >= INT32_MAX) return false;
  return probe_stages(ctx, packed->dim, nlist, nq) >= 1;
}

int32_t run_ivf_probe(mans_ctx* ctx, const mans_corpus* cent, const mans_corpus* packed,
                      const int64_t* d_offsets, mans_workspace* ws, const float* d_queries,
                      int64_t nq, int32_t kout, int32_t keff, int32_t probe, int32_t metric,
                      float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                      cudaStream_t stream) {
  const int32_t nlist = static_cast<int32_t>(cent->n);
  const int nchunks = static_cast<int>((cent->dim + kTileCols - 1) / kTileCols);
  const int stages = probe_stages(ctx, cent->dim, nlist, nq);
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
  p.nchunks = nchunks;
  p.stages = stages;
  p.metric = metric;
  p.nlist = nlist;
  p.nprobe = probe;
  p.k = keff;
  p.kout = kout;
  p.cent_norms = cent->norms;
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
  const size_t smem =
      probe_layout(nchunks, stages, nlist, static_cast<int>(nq), grid).total + 1024;
  cudaError_t e = cudaSuccess;
  if (!ctx->probe_configured) {  // the largest opt-in size, once per context (device)
    e = cudaFuncSetAttribute(ivf_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             ctx->max_smem);
    if (e != cudaSuccess) return fail_cuda(e, "ivf probe configure");
    ctx->probe_configured = true;
  }
  void* args[] = {const_cast<CUtensorMap*>(&cent->map_probe),
                  const_cast<CUtensorMap*>(&packed->map_probe), &p};
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
