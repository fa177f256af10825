// ivf.cu -- IVF-flat probe-and-scan on the device.
//
// Restates IVFFlatSearch.scanProbedLists (Sources/MetalANNSCore/
// IVFFlatSearch.swift:214-291) for a batch of queries:
//   1. centroid keys with the host-tier metric (same formula as the flat scan)
//      and the nprobe smallest, ties to the lower list index
//      (smallestIndices, :314-382) -- the flat scan kernel over the centroid
//      matrix with k = nprobe;
//   2. a one-block planner groups the (query, probed list) pairs by list, so
//      every probed list is streamed once for all queries that probe it, and
//      cuts lists into row chunks (work units for the persistent scan);
//   3. the flat scan kernel over the packed list rows (the Partition layout,
//      :39-95: packed[p] = corpus[listIDs[p]]) reporting listIDs[p] as ids;
//   4. the slot merge per query.  The strict (distance, id) order of TopKHeap
//      (:384-444) makes the result independent of the visiting order.
// The planner runs on the device, so a search needs no host round trip.
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"

using namespace mans;

struct mans_ivf {
  mans_ctx* ctx = nullptr;
  int32_t nlist = 0;
  int64_t n = 0;
  int64_t dim = 0;
  int64_t max_len = 0;
  mans_corpus* cent = nullptr;    // centroids (ids = list index)
  mans_corpus* packed = nullptr;  // list-contiguous rows, ids = listIDs
  int64_t* offsets = nullptr;     // device, nlist + 1
  std::vector<int64_t> h_offsets;
};

namespace mans {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kChunkRows = 512;  // rows per scan work unit (two TMA boxes)

struct PlanParams {
  const uint32_t* probe_ids;
  const int32_t* probe_counts;
  int32_t pk;
  int32_t nq;
  int32_t nlist;
  const int64_t* offsets;
  int32_t qb;
  int32_t chunk;
  int32_t* list_cnt;   // [nlist]
  int32_t* list_tmp;   // [nlist]
  int32_t* list_qoff;  // [nlist + 1]
  int32_t* list_soff;  // [nlist + 1]
  int32_t* qidx;       // [nq * pk]
  ScanSegment* segs;   // [max_segs]
  int32_t* nseg;       // [1]
  int32_t* q_cnt;      // [nq]
  int32_t* q_soff;     // [nq + 1]
  int32_t* q_slots;    // [max_refs]
  int32_t max_segs;
  int32_t max_refs;
  int* err;
};

__device__ __forceinline__ int list_chunks(const int64_t* off, int l, int chunk) {
  int64_t len = off[l + 1] - off[l];
  return static_cast<int>((len + chunk - 1) / chunk);
}

// Bytes of shared memory the planner needs to keep its counters and the list
// offsets on chip (0: they do not fit, the global arrays of PlanParams are used).
inline size_t plan_smem_bytes(int nlist, int64_t nq, int max_smem) {
  const size_t b = (static_cast<size_t>(nlist) + 1) * 8 + 4 * (static_cast<size_t>(nlist) + 1) * 4 +
                   2 * (static_cast<size_t>(nq) + 1) * 4 + 64;
  return b <= static_cast<size_t>(max_smem) - 1024 ? b : 0;
}

__global__ void __launch_bounds__(kPlanThreads) ivf_plan_kernel(PlanParams p, int on_chip) {
  __shared__ int32_t part[64];
  extern __shared__ __align__(16) uint8_t plan_smem[];
  const int t = threadIdx.x, nt = blockDim.x;
  const int64_t pairs = static_cast<int64_t>(p.nq) * p.pk;
  int32_t* q_soff_out = p.q_soff;
  if (on_chip) {
    // counters, running sums and the list offsets in shared memory: the
    // atomics and scans below stay on chip; q_soff is copied out at the end
    int64_t* off_s = reinterpret_cast<int64_t*>(plan_smem);
    int32_t* w = reinterpret_cast<int32_t*>(off_s + p.nlist + 1);
    for (int i = t; i <= p.nlist; i += nt) off_s[i] = p.offsets[i];
    p.offsets = off_s;
    p.list_cnt = w;
    p.list_tmp = w + (p.nlist + 1);
    p.list_qoff = w + 2 * (p.nlist + 1);
    p.list_soff = w + 3 * (p.nlist + 1);
    p.q_cnt = w + 4 * (p.nlist + 1);
    p.q_soff = p.q_cnt + (p.nq + 1);
  }
  for (int i = t; i < p.nlist; i += nt) p.list_cnt[i] = 0;
  for (int i = t; i < p.nq; i += nt) p.q_cnt[i] = 0;
  __syncthreads();
  for (int64_t i = t; i < pairs; i += nt) {
    int q = static_cast<int>(i / p.pk), j = static_cast<int>(i - static_cast<int64_t>(q) * p.pk);
    if (j < p.probe_counts[q]) {
      int l = static_cast<int>(p.probe_ids[i]);
      atomicAdd(&p.list_cnt[l], 1);
      atomicAdd(&p.q_cnt[q], list_chunks(p.offsets, l, p.chunk));
    }
  }
  __syncthreads();
  block_exclusive_scan(p.list_cnt, p.nlist, p.list_qoff, part);
  for (int l = t; l < p.nlist; l += nt) {
    int c = p.list_cnt[l];
    p.list_tmp[l] = c > 0 ? ((c + p.qb - 1) / p.qb) * list_chunks(p.offsets, l, p.chunk) : 0;
  }
  __syncthreads();
  block_exclusive_scan(p.list_tmp, p.nlist, p.list_soff, part);
  block_exclusive_scan(p.q_cnt, p.nq, p.q_soff, part);
  for (int i = t; i < p.nlist; i += nt) p.list_cnt[i] = 0;
  for (int i = t; i < p.nq; i += nt) p.q_cnt[i] = 0;
  __syncthreads();
  for (int64_t i = t; i < pairs; i += nt) {
    int q = static_cast<int>(i / p.pk), j = static_cast<int>(i - static_cast<int64_t>(q) * p.pk);
    if (j < p.probe_counts[q]) {
      int l = static_cast<int>(p.probe_ids[i]);
      int pos = atomicAdd(&p.list_cnt[l], 1);
      p.qidx[p.list_qoff[l] + pos] = q;
    }
  }
  const int total = p.list_soff[p.nlist];
  const int nseg = min(total, p.max_segs);
  if (t == 0) {
    *p.nseg = nseg;
    if (total > p.max_segs || p.q_soff[p.nq] > p.max_refs) atomicExch(p.err, kErrBadArg);
  }
  for (int l = t; l < p.nlist; l += nt) {
    int cnt = p.list_qoff[l + 1] - p.list_qoff[l];
    if (cnt == 0) continue;
    int ch = list_chunks(p.offsets, l, p.chunk);
    int groups = (cnt + p.qb - 1) / p.qb;
    int64_t base = p.offsets[l];
    int64_t len = p.offsets[l + 1] - base;
    for (int g = 0; g < groups; ++g)
      for (int c = 0; c < ch; ++c) {
        int s = p.list_soff[l] + g * ch + c;
        if (s >= nseg) continue;
        ScanSegment sg;
        sg.row_begin = base + static_cast<int64_t>(c) * p.chunk;
        int64_t rem = len - static_cast<int64_t>(c) * p.chunk;
        sg.row_count = static_cast<int32_t>(rem < p.chunk ? rem : p.chunk);
        sg.qbase = p.list_qoff[l] + g * p.qb;
        sg.qcount = min(p.qb, cnt - g * p.qb);
        sg.slot_base = s * p.qb;
        sg.slot_stride = 1;
        sg.reserved = 0;
        p.segs[s] = sg;
      }
  }
  __syncthreads();
  for (int s = t; s < nseg; s += nt) {
    ScanSegment sg = p.segs[s];
    for (int j = 0; j < sg.qcount; ++j) {
      int q = p.qidx[sg.qbase + j];
      int pos = atomicAdd(&p.q_cnt[q], 1);
      int at = p.q_soff[q] + pos;
      if (at < p.max_refs) p.q_slots[at] = s * p.qb + j;
    }
  }
  if (on_chip)
    for (int i = t; i <= p.nq; i += nt) q_soff_out[i] = p.q_soff[i];
}

// Squared query norms in index order, one warp per query: the lanes load 32
// consecutive elements at a time (eight such loads in flight), and the chunk's
// squares are added lane by lane through shuffles, so every lane carries the
// same sequential sum (lanes past dim add +0, which leaves it unchanged).
__global__ void query_norms_warp_kernel(const float* __restrict__ q, int64_t nq, int32_t dim,
                                        float* __restrict__ out) {
  int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (w >= nq) return;
  const float* v = q + w * dim;
  float acc = 0.0f;
  for (int c0 = 0; c0 < dim; c0 += 32 * 8) {
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = c0 + u * 32 + lane;
      x[u] = c < dim ? __ldg(v + c) : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (c0 + u * 32 >= dim) break;
      const float sq = __fmul_rn(x[u], x[u]);
#pragma unroll
      for (int j = 0; j < 32; ++j) acc = __fadd_rn(acc, __shfl_sync(0xFFFFFFFFu, sq, j));
    }
  }
  if (lane == 0) out[w] = acc;
}

// List scan of query batches: one warp per block, as many blocks per SM as
// the shared memory holds.  A block walks planned segments (a run of rows of
// one probed list and up to kSegQ of the queries that probe it): 32-row
// tiles arrive as TMA boxes of 32 rows x 32 fp32 (128-byte swizzle: 16-byte
// chunk j of row r at chunk j ^ (r & 7), so the eight lanes of a
// quarter-warp read distinct bank groups), lane i scores row i against every
// query of the segment (independent chains, each the reference's summation
// order) and keeps each query's 32 smallest (distance, id) keys in
// registers; the next tile's boxes fly while the keys are ranked.  Each
// query of the segment then writes its sorted keys to its slot.  Rows are
// read once for all queries of the segment, and no block-wide barrier is
// needed anywhere.
constexpr int kSegQ = 4;
constexpr int kSegBox = 32 * kTileCols * 4;  // one 32 x 32 fp32 box

struct SegScanParams {
  const ScanSegment* segs;
  const int32_t* nseg;
  const float* queries;  // nq x dim
  const int32_t* qidx;
  const float* qnorms;   // null for IP
  const float* norms;    // null for IP
  const uint32_t* ids;
  int32_t dim;
  int32_t nchunks;  // ceil(dim / 32)
  int32_t metric;
  int32_t k;   // <= 32
  int32_t kp;  // slot width
  uint64_t* slot_keys;
  int32_t* slot_counts;
  int* err;
};

__host__ __device__ inline size_t seg_scan_smem(int nchunks) {
  return 1024 + static_cast<size_t>(nchunks) * kSegBox +
         static_cast<size_t>(kSegQ) * nchunks * kTileCols * 4 + 16 + kSegQ * 4;
}

__device__ __forceinline__ void seg_load_tile(uint8_t* stage, const CUtensorMap* map, int64_t row,
                                              int nchunks, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nchunks) * kSegBox);
  for (int cc = 0; cc < nchunks; ++cc)
    tma_load_2d(stage + cc * kSegBox, map, cc * kTileCols, static_cast<int32_t>(row), bar);
}

__global__ void __launch_bounds__(32) ivf_seg_scan_kernel(const __grid_constant__ CUtensorMap map,
                                                          const SegScanParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stage =
      reinterpret_cast<uint8_t*>((reinterpret_cast<size_t>(smem_raw) + 1023) / 1024 * 1024);
  const int nch = p.nchunks, qw = nch * kTileCols;
  float* qs = reinterpret_cast<float*>(stage + nch * kSegBox);  // kSegQ x qw
  uint64_t* bar = reinterpret_cast<uint64_t*>(qs + kSegQ * qw);
  float* qn = reinterpret_cast<float*>(bar + 1);
  const int lane = threadIdx.x;
  if (lane == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&map);
  }
  __syncwarp();
  uint32_t ph = 0;
  const int nseg = *p.nseg;
  const bool q4 = (p.dim & 3) == 0;
  for (int s = blockIdx.x; s < nseg; s += gridDim.x) {
    const ScanSegment seg = p.segs[s];
    const int nqs = seg.qcount;
    // the first tile is in flight while the queries load
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      seg_load_tile(stage, &map, seg.row_begin, nch, bar);
    }
    int qid[kSegQ];
#pragma unroll
    for (int j = 0; j < kSegQ; ++j) qid[j] = j < nqs ? __ldg(p.qidx + seg.qbase + j) : 0;
    if (q4) {
      // 16-byte loads: query rows start 16-byte aligned when dim % 4 == 0
      const int qw4 = qw / 4, d4 = p.dim / 4;
      for (int i = lane; i < kSegQ * qw4; i += 32) {
        const int j = i / qw4, c = i - j * qw4;
        int qj = qid[0];
#pragma unroll
        for (int jj = 1; jj < kSegQ; ++jj)
          if (j == jj) qj = qid[jj];
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (j < nqs && c < d4)
          v = __ldg(reinterpret_cast<const float4*>(p.queries + static_cast<int64_t>(qj) * p.dim) +
                    c);
        reinterpret_cast<float4*>(qs)[i] = v;
      }
    }
    for (int i0 = lane; !q4 && i0 < kSegQ * qw; i0 += 32 * 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * 32;
        const int j = i / qw, c = i - j * qw;
        int qj = qid[0];
#pragma unroll
        for (int jj = 1; jj < kSegQ; ++jj)
          if (j == jj) qj = qid[jj];
        v[u] = (i < kSegQ * qw && j < nqs && c < p.dim)
                   ? __ldg(p.queries + static_cast<int64_t>(qj) * p.dim + c)
                   : 0.0f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (i0 + u * 32 < kSegQ * qw) qs[i0 + u * 32] = v[u];
    }
    if (lane < kSegQ) {
      int qj = qid[0];
#pragma unroll
      for (int jj = 1; jj < kSegQ; ++jj)
        if (lane == jj) qj = qid[jj];
      qn[lane] = (p.qnorms && lane < nqs) ? __ldg(p.qnorms + qj) : 0.0f;
    }
    __syncwarp();
    float qnj[kSegQ];
#pragma unroll
    for (int j = 0; j < kSegQ; ++j) qnj[j] = qn[j];
    uint64_t best[kSegQ], kth[kSegQ];
#pragma unroll
    for (int j = 0; j < kSegQ; ++j) best[j] = kth[j] = kKeyMax;
    bool aborted = false;
    for (int t0 = 0; t0 < seg.row_count; t0 += 32) {
      const int64_t row = seg.row_begin + t0 + lane;
      const bool valid = t0 + lane < seg.row_count;
      float vn = 0.0f;
      uint32_t id = 0;
      if (valid) {
        if (p.norms) vn = __ldg(p.norms + row);
        id = __ldg(p.ids + row);
      }
      const bool ok = mbar_wait_bounded(bar, ph, p.err);
      if (__any_sync(0xFFFFFFFFu, !ok)) {
        mbar_wait_bounded(bar, ph, nullptr);  // the copies in flight: once more, bounded
        aborted = true;
        break;
      }
      ph ^= 1u;
      float acc[kSegQ];
#pragma unroll
      for (int j = 0; j < kSegQ; ++j) acc[j] = 0.0f;
      for (int cc = 0; cc < nch; ++cc) {
        const uint8_t* rowp = stage + cc * kSegBox + lane * 128;
        float4 v[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
          v[jj] = *reinterpret_cast<const float4*>(rowp + ((jj ^ (lane & 7)) << 4));
#pragma unroll
        for (int j = 0; j < kSegQ; ++j) {
          if (j >= nqs) break;
          const float4* qv = reinterpret_cast<const float4*>(qs + j * qw + cc * kTileCols);
          float a = acc[j];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const float4 b = qv[jj];
            a = __fadd_rn(a, __fmul_rn(v[jj].x, b.x));
            a = __fadd_rn(a, __fmul_rn(v[jj].y, b.y));
            a = __fadd_rn(a, __fmul_rn(v[jj].z, b.z));
            a = __fadd_rn(a, __fmul_rn(v[jj].w, b.w));
          }
          acc[j] = a;
        }
      }
      __syncwarp();
      if (t0 + 32 < seg.row_count && lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        seg_load_tile(stage, &map, seg.row_begin + t0 + 32, nch, bar);
      }
#pragma unroll
      for (int j = 0; j < kSegQ; ++j) {
        if (j >= nqs) break;
        const float d = finalize_distance(p.metric, acc[j], qnj[j], vn);
        warp_topk_offer(best[j], kth[j], valid ? make_key(d, id) : kKeyMax, p.k, lane);
      }
    }
    if (aborted) break;
#pragma unroll
    for (int j = 0; j < kSegQ; ++j) {
      if (j >= nqs) break;
      const int slot = seg.slot_base + j * seg.slot_stride;
      const bool ok = lane < p.k && best[j] != kKeyMax;
      if (lane < p.kp) p.slot_keys[static_cast<size_t>(slot) * p.kp + lane] = ok ? best[j] : kKeyMax;
      const unsigned vm = __ballot_sync(0xFFFFFFFFu, ok);
      if (lane == 0) p.slot_counts[slot] = __popc(vm);
    }
    __syncwarp();  // every lane is done with this segment's queries
  }
}

}  // namespace

// Byte layout of the per-call scratch carved from one device buffer.
struct IvfScratch {
  size_t off[16];
  size_t total;
};

static size_t carve(size_t& o, size_t bytes) {
  size_t at = (o + 255) / 256 * 256;
  o = at + bytes;
  return at;
}

static int32_t run_ivf_search(mans_ctx* ctx, mans_ivf* ivf, mans_workspace* ws,
                              const float* d_queries, int64_t nq, int32_t k, int32_t nprobe,
                              int32_t metric, float* d_out_dist, uint32_t* d_out_ids,
                              int32_t* d_out_counts, cudaStream_t stream) {
  const int32_t kout = std::min<int32_t>(k, MANS_MAX_TOPK);
  if (nq <= 0) return MANS_OK;
  if (k <= 0 || ivf->n <= 0) {
    if (kout <= 0) {
      cudaError_t e = cudaMemsetAsync(d_out_counts, 0, sizeof(int32_t) * nq, stream);
      return e == cudaSuccess ? MANS_OK : fail_cuda(e, "cudaMemsetAsync");
    }
    cudaError_t e = launch_fill_empty(d_out_dist, d_out_ids, d_out_counts, nq, kout, stream);
    return e == cudaSuccess ? MANS_OK : fail_cuda(e, "fill_empty launch");
  }
  const int32_t probe = std::max(1, std::min(nprobe, ivf->nlist));
  if (probe >= ivf->nlist) {
    // every list is probed: an exact scan of the packed rows (IVFFlatSearch
    // .swift:161-165 hands this case to the exact host scan)
    return run_flat_search(ctx, ivf->packed, ws, d_queries, nq, k, metric, d_out_dist, d_out_ids,
                           d_out_counts, stream);
  }
  if (probe > MANS_MAX_TOPK)
    return fail(MANS_ERR_SEARCH, "nprobe above 256 (and below nlist) is not supported on the GPU");
  if (nq > INT32_MAX / std::max(probe, 1)) return fail(MANS_ERR_SEARCH, "query batch too large");

  const int32_t keff = static_cast<int32_t>(std::min<int64_t>(kout, ivf->n));
  // a few queries: the whole search in one cooperative launch (ivf_probe.cu)
  if (ivf_probe_applies(ctx, ivf->packed, ivf->nlist, nq, kout, probe))
    return run_ivf_probe(ctx, ivf->cent, ivf->packed, ivf->offsets, ws, d_queries, nq, kout, keff,
                         probe, metric, d_out_dist, d_out_ids, d_out_counts, stream);
  const int32_t kp = pow2_at_least(keff);
  const int64_t pairs = nq * probe;
  const int64_t avg_len = (ivf->n + ivf->nlist - 1) / ivf->nlist;
  // Batches with k <= 32 whose rows fit a warp's stage: the warp-per-segment
  // scan (segments of up to kSegQ queries and 32..256 rows: the largest run
  // that still gives every resident warp a few segments).
  const int seg_nch = static_cast<int>((ivf->dim + kTileCols - 1) / kTileCols);
  const size_t seg_smem = seg_scan_smem(seg_nch);
  const void* seg_fn = reinterpret_cast<const void*>(ivf_seg_scan_kernel);
  int seg_blocks = 0;
  if (keff <= 32 && seg_smem <= static_cast<size_t>(ctx->max_smem)) {
    static_cast<void>(cudaFuncSetAttribute(seg_fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(seg_smem)));
    static_cast<void>(cudaFuncSetAttribute(seg_fn,
                                           cudaFuncAttributePreferredSharedMemoryCarveout,
                                           cudaSharedmemCarveoutMaxShared));
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&seg_blocks, seg_fn, 32, seg_smem) !=
        cudaSuccess)
      seg_blocks = 0;
  }
  const bool seg_scan = seg_blocks > 0;
  const int qb = seg_scan ? kSegQ : choose_qb((pairs + ivf->nlist - 1) / ivf->nlist);
  // Work units of the streaming scan: list chunks of 64 rows (64-row tiles)
  // or 256 / 512 rows (256-row tiles) -- the smallest chunk whose unit count
  // still fits in one wave of CTAs, so a short probe spreads over many SMs
  // without giving one CTA several units in a row.
  auto units_for = [&](int64_t chunk) { return pairs * ((avg_len + chunk - 1) / chunk); };
  int chunk_rows = kChunkRows;
  if (seg_scan) {
    const int64_t warps = static_cast<int64_t>(seg_blocks) * ctx->num_sms;
    chunk_rows = 256;
    while (chunk_rows > 32 && units_for(chunk_rows) < 4 * warps) chunk_rows /= 2;
  } else if (units_for(kSmallTileRows) <= ctx->num_sms) {
    chunk_rows = kSmallTileRows;
  } else if (units_for(kTileRows) <= ctx->num_sms) {
    chunk_rows = kTileRows;
  }
  const bool small = chunk_rows == kSmallTileRows;
  const int64_t max_chunks = std::max<int64_t>(1, (ivf->max_len + chunk_rows - 1) / chunk_rows);
  const int64_t max_refs = pairs * max_chunks;
  const int64_t max_segs = max_refs;
  if (max_refs * qb > INT32_MAX / 2) return fail(MANS_ERR_SEARCH, "query batch too large");
  const int nchunks = static_cast<int>((ivf->dim + kTileCols - 1) / kTileCols);
  const int stages = scan_max_stages(qb, nchunks);
  if (!seg_scan && stages < 2) return fail(MANS_ERR_SEARCH, "dimension too large for the scan kernel");

  // scratch: centroid top-k + planner arrays + slots
  size_t o = 0;
  const size_t o_pd = carve(o, pairs * sizeof(float));
  const size_t o_pi = carve(o, pairs * sizeof(uint32_t));
  const size_t o_pc = carve(o, nq * sizeof(int32_t));
  const size_t o_qn = carve(o, nq * sizeof(float));
  const size_t o_lc = carve(o, ivf->nlist * sizeof(int32_t));
  const size_t o_lt = carve(o, ivf->nlist * sizeof(int32_t));
  const size_t o_lq = carve(o, (ivf->nlist + 1) * sizeof(int32_t));
  const size_t o_ls = carve(o, (ivf->nlist + 1) * sizeof(int32_t));
  const size_t o_qi = carve(o, pairs * sizeof(int32_t));
  const size_t o_sg = carve(o, max_segs * sizeof(ScanSegment));
  const size_t o_ns = carve(o, sizeof(int32_t));
  const size_t o_qc = carve(o, nq * sizeof(int32_t));
  const size_t o_qs = carve(o, (nq + 1) * sizeof(int32_t));
  const size_t o_qr = carve(o, max_refs * sizeof(int32_t));
  int32_t rc;
  if ((rc = ws->aux.reserve(o)) != MANS_OK) return rc;
  // slot buffers sized for both the centroid search and the list scan, so
  // nothing is reallocated between launches
  const int64_t cent_tiles = (ivf->nlist + kTileRows - 1) / kTileRows;
  const size_t cent_slots = static_cast<size_t>((nq + 7) / 8 * 8) * std::min<int64_t>(ctx->num_sms, cent_tiles);
  const size_t list_slots = static_cast<size_t>(max_segs) * qb;
  const int kp_cent = pow2_at_least(probe);
  const size_t need_keys = std::max(cent_slots * kp_cent, list_slots * kp) * sizeof(uint64_t);
  const size_t need_cnts = std::max(cent_slots, list_slots) * sizeof(int32_t);
  if ((rc = ws->slot_keys.reserve(need_keys)) != MANS_OK) return rc;
  if ((rc = ws->slot_counts.reserve(need_cnts)) != MANS_OK) return rc;
  if ((rc = ws->err.reserve(sizeof(int))) != MANS_OK) return rc;
  if (!ws->err_cleared) {
    cudaError_t e = cudaMemsetAsync(ws->err.ptr, 0, sizeof(int), stream);
    if (e != cudaSuccess) return fail_cuda(e, "cudaMemsetAsync(err)");
    ws->err_cleared = true;
  }
  uint8_t* A = static_cast<uint8_t*>(ws->aux.ptr);
  float* probe_d = reinterpret_cast<float*>(A + o_pd);
  uint32_t* probe_i = reinterpret_cast<uint32_t*>(A + o_pi);
  int32_t* probe_c = reinterpret_cast<int32_t*>(A + o_pc);
  float* qn = reinterpret_cast<float*>(A + o_qn);

  // 1. centroid keys + nprobe smallest (ties -> lower list index)
  {
    TimingHold hold(ws);  // the centroid scan is not the timed list scan
    rc = run_flat_search(ctx, ivf->cent, ws, d_queries, nq, probe, metric, probe_d, probe_i,
                         probe_c, stream, kModeHost, MANS_MAX_TOPK, true);
  }
  if (rc != MANS_OK) return rc;

  // 2. plan
  PlanParams pp{};
  pp.probe_ids = probe_i;
  pp.probe_counts = probe_c;
  pp.pk = probe;
  pp.nq = static_cast<int32_t>(nq);
  pp.nlist = ivf->nlist;
  pp.offsets = ivf->offsets;
  pp.qb = qb;
  pp.chunk = chunk_rows;
  pp.list_cnt = reinterpret_cast<int32_t*>(A + o_lc);
  pp.list_tmp = reinterpret_cast<int32_t*>(A + o_lt);
  pp.list_qoff = reinterpret_cast<int32_t*>(A + o_lq);
  pp.list_soff = reinterpret_cast<int32_t*>(A + o_ls);
  pp.qidx = reinterpret_cast<int32_t*>(A + o_qi);
  pp.segs = reinterpret_cast<ScanSegment*>(A + o_sg);
  pp.nseg = reinterpret_cast<int32_t*>(A + o_ns);
  pp.q_cnt = reinterpret_cast<int32_t*>(A + o_qc);
  pp.q_soff = reinterpret_cast<int32_t*>(A + o_qs);
  pp.q_slots = reinterpret_cast<int32_t*>(A + o_qr);
  pp.max_segs = static_cast<int32_t>(max_segs);
  pp.max_refs = static_cast<int32_t>(max_refs);
  pp.err = static_cast<int*>(ws->err.ptr);
  if (metric != MANS_METRIC_IP) {
    const int64_t threads = nq * 32;
    query_norms_warp_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
        d_queries, nq, static_cast<int32_t>(ivf->dim), qn);
  }
  const size_t plan_smem = plan_smem_bytes(ivf->nlist, nq, ctx->max_smem);
  if (plan_smem > 48 * 1024) {
    cudaError_t ea = cudaFuncSetAttribute(ivf_plan_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(plan_smem));
    if (ea != cudaSuccess) return fail_cuda(ea, "ivf plan configure");
  }
  ivf_plan_kernel<<<1, kPlanThreads, plan_smem, stream>>>(pp, plan_smem > 0 ? 1 : 0);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "ivf plan launch");

  // 3. scan the probed lists
  if (seg_scan) {
    SegScanParams sp{};
    sp.segs = pp.segs;
    sp.nseg = pp.nseg;
    sp.queries = d_queries;
    sp.qidx = pp.qidx;
    sp.qnorms = metric != MANS_METRIC_IP ? qn : nullptr;
    sp.norms = metric != MANS_METRIC_IP ? ivf->packed->norms : nullptr;
    sp.ids = ivf->packed->ids;
    sp.dim = static_cast<int32_t>(ivf->dim);
    sp.nchunks = seg_nch;
    sp.metric = metric;
    sp.k = keff;
    sp.kp = kp;
    sp.slot_keys = static_cast<uint64_t*>(ws->slot_keys.ptr);
    sp.slot_counts = static_cast<int32_t*>(ws->slot_counts.ptr);
    sp.err = pp.err;
    const int64_t grid = std::min<int64_t>(static_cast<int64_t>(seg_blocks) * ctx->num_sms,
                                           std::max<int64_t>(1, max_segs));
    cudaEvent_t stop = timing_begin(ws, stream);
    ivf_seg_scan_kernel<<<static_cast<unsigned>(grid), 32, seg_smem, stream>>>(
        ivf->packed->map_seg, sp);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_cuda(e, "ivf segment scan launch");
    timing_end(stop, stream);
  }
  ScanParams p{};
  p.segs = pp.segs;
  p.nseg = static_cast<int32_t>(max_segs);
  p.nseg_dev = pp.nseg;
  p.stages = stages;
  p.n = ivf->n;
  p.nq = nq;
  p.queries = d_queries;
  p.qidx = pp.qidx;
  p.qnorms = metric != MANS_METRIC_IP ? qn : nullptr;
  p.norms = metric != MANS_METRIC_IP ? ivf->packed->norms : nullptr;
  p.ids = ivf->packed->ids;
  p.id_offset = 0;
  p.dim = static_cast<int32_t>(ivf->dim);
  p.nchunks = nchunks;
  p.metric = metric;
  p.k = keff;
  p.kp = kp;
  p.tile_rows = small ? kSmallTileRows : kTileRows;
  p.slot_keys = static_cast<uint64_t*>(ws->slot_keys.ptr);
  p.slot_counts = static_cast<int32_t*>(ws->slot_counts.ptr);
  p.err = pp.err;
  if (!seg_scan) {
    cudaEvent_t stop = timing_begin(ws, stream);
    e = launch_scan(qb, small ? ivf->packed->map_small : ivf->packed->map, p, ctx->num_sms,
                    stream);
    if (e != cudaSuccess) return fail_cuda(e, "ivf scan launch");
    timing_end(stop, stream);
  }

  // 4. merge per query
  MergeParams m{};
  m.in_keys = p.slot_keys;
  m.in_counts = p.slot_counts;
  m.q_slot_offsets = pp.q_soff;
  m.q_slot_list = pp.q_slots;
  m.kp_in = kp;
  m.nq = nq;
  m.k = keff;
  m.kp = kp;
  m.kout = kout;
  m.out_dist = d_out_dist;
  m.out_ids = d_out_ids;
  m.out_counts = d_out_counts;
  m.err = p.err;
  e = launch_merge(m, stream);
  if (e != cudaSuccess) return fail_cuda(e, "ivf merge launch");
  ws->launches += (metric != MANS_METRIC_IP ? 1 : 0) + 3;
  return MANS_OK;
}

}  // namespace mans

extern "C" {

int32_t mans_ivf_create(mans_ctx* ctx, const float* centroids, int32_t nlist, int64_t dim,
                        const float* packed_rows, const uint32_t* list_ids,
                        const int64_t* list_offsets, int64_t n, mans_ivf** out_ivf) {
  if (!ctx || !out_ivf) return fail(MANS_ERR_INVALID, "null context or output");
  *out_ivf = nullptr;
  if (int32_t r = reject_group(ctx, nullptr, "an IVF-flat index")) return r;
  if (nlist <= 0 || dim <= 0 || n < 0) return fail(MANS_ERR_INVALID, "bad IVF shape");
  if (!centroids || !list_offsets || (n > 0 && (!packed_rows || !list_ids)))
    return fail(MANS_ERR_INVALID, "null IVF buffer");
  if (list_offsets[0] != 0 || list_offsets[nlist] != n)
    return fail(MANS_ERR_INVALID, "list offsets must run from 0 to n");
  int64_t max_len = 0;
  for (int32_t l = 0; l < nlist; ++l) {
    int64_t len = list_offsets[l + 1] - list_offsets[l];
    if (len < 0) return fail(MANS_ERR_INVALID, "list offsets must be non-decreasing");
    max_len = std::max(max_len, len);
  }
  DeviceGuard g(ctx->device);
  mans_ivf* ivf = new mans_ivf();
  ivf->ctx = ctx;
  ivf->nlist = nlist;
  ivf->n = n;
  ivf->dim = dim;
  ivf->max_len = max_len;
  ivf->h_offsets.assign(list_offsets, list_offsets + nlist + 1);
  int32_t rc = corpus_upload(ctx, centroids, nlist, dim, 0, &ivf->cent);
  if (rc == MANS_OK) rc = corpus_upload(ctx, packed_rows, n, dim, 0, &ivf->packed);
  if (rc == MANS_OK) {
    cudaError_t e = cudaMalloc(&ivf->packed->ids, std::max<int64_t>(n, 1) * sizeof(uint32_t));
    if (e == cudaSuccess && n > 0)
      e = cudaMemcpy(ivf->packed->ids, list_ids, n * sizeof(uint32_t), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&ivf->offsets, (nlist + 1) * sizeof(int64_t));
    if (e == cudaSuccess)
      e = cudaMemcpy(ivf->offsets, list_offsets, (nlist + 1) * sizeof(int64_t),
                     cudaMemcpyHostToDevice);
    if (e != cudaSuccess) rc = fail_cuda(e, "IVF upload");
  }
  if (rc != MANS_OK) {
    corpus_free(ivf->cent);
    corpus_free(ivf->packed);
    if (ivf->offsets) cudaFree(ivf->offsets);
    delete ivf;
    return rc;
  }
  *out_ivf = ivf;
  return MANS_OK;
}

int32_t mans_ivf_destroy(mans_ivf* ivf) {
  if (!ivf) return MANS_OK;
  DeviceGuard g(ivf->ctx->device);
  cudaDeviceSynchronize();
  corpus_free(ivf->cent);
  corpus_free(ivf->packed);
  if (ivf->offsets) cudaFree(ivf->offsets);
  delete ivf;
  return MANS_OK;
}

static int32_t validate_ivf(const mans_ctx* ctx, const mans_ivf* ivf, int64_t nq, int32_t metric) {
  if (!ctx || !ivf) return fail(MANS_ERR_INVALID, "null context or IVF index");
  if (ivf->ctx != ctx) return fail(MANS_ERR_INVALID, "IVF index belongs to another context");
  if (nq < 0) return fail(MANS_ERR_INVALID, "negative query count");
  if (metric == MANS_METRIC_HAMMING)
    return fail(MANS_ERR_SEARCH, "IVF-flat does not support metric .hamming");
  if (metric < 0 || metric > MANS_METRIC_HAMMING) return fail(MANS_ERR_INVALID, "unknown metric");
  return MANS_OK;
}

int32_t mans_ivf_search(mans_ctx* ctx, mans_ivf* ivf, const float* queries, int64_t nq,
                        int64_t dim, int32_t k, int32_t nprobe, int32_t metric, float* out_dist,
                        uint32_t* out_ids, int32_t* out_counts) {
  int32_t rc = validate_ivf(ctx, ivf, nq, metric);
  if (rc != MANS_OK) return rc;
  if (nq == 0) return MANS_OK;
  const int32_t kout = std::max<int32_t>(0, std::min<int32_t>(k, MANS_MAX_TOPK));
  if (k <= 0 || ivf->n <= 0) {
    for (int64_t i = 0; i < nq * kout; ++i) {
      out_dist[i] = __builtin_inff();
      out_ids[i] = MANS_EMPTY_ID;
    }
    for (int64_t i = 0; i < nq; ++i) out_counts[i] = 0;
    return MANS_OK;
  }
  if (dim != ivf->dim) return fail(MANS_ERR_DIM, "dimensionMismatch");
  if (!queries || !out_dist || !out_ids || !out_counts) return fail(MANS_ERR_INVALID, "null buffer");
  DeviceGuard g(ctx->device);
  mans_workspace* ws = acquire_workspace(ctx);
  if (!ws) return fail(MANS_ERR_OOM, "cannot create a workspace stream");
  rc = host_buffer_search(ws, queries, nq, dim, kout, out_dist, out_ids, out_counts,
                          [&](const float* dq, float* dd, uint32_t* di, int32_t* dc,
                              cudaStream_t st) {
                            return run_ivf_search(ctx, ivf, ws, dq, nq, k, nprobe, metric, dd,
                                                  di, dc, st);
                          });
  release_workspace(ctx, ws);
  return rc;
}

int32_t mans_ivf_search_device(mans_ctx* ctx, mans_ivf* ivf, mans_workspace* ws,
                               const float* d_queries, int64_t nq, int32_t k, int32_t nprobe,
                               int32_t metric, float* d_out_dist, uint32_t* d_out_ids,
                               int32_t* d_out_counts, void* cuda_stream) {
  int32_t rc = validate_ivf(ctx, ivf, nq, metric);
  if (rc != MANS_OK) return rc;
  if (!ws || ws->ctx != ctx) return fail(MANS_ERR_INVALID, "workspace missing or foreign");
  DeviceGuard g(ctx->device);
  return run_ivf_search(ctx, ivf, ws, d_queries, nq, k, nprobe, metric, d_out_dist, d_out_ids,
                        d_out_counts, static_cast<cudaStream_t>(cuda_stream));
}

int64_t mans_ivf_list_count(const mans_ivf* ivf) { return ivf ? ivf->nlist : 0; }

}  // extern "C"

// ---------------------------------------------------------------------------
// Partition build on the device (IVFFlatSearch.buildPartition after the
// k-means, IVFFlatSearch.swift:559-631, and assignRows, :633-703).
// ---------------------------------------------------------------------------

namespace mans {
namespace {

__global__ void iota_u32_kernel(uint32_t* __restrict__ out, int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) out[i] = static_cast<uint32_t>(i);
}

__global__ void list_histogram_kernel(const uint32_t* __restrict__ assign, int64_t n,
                                      int64_t* __restrict__ counts) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) atomicAdd(reinterpret_cast<unsigned long long*>(counts + assign[i]), 1ull);
}

// offsets[0] = 0, offsets[l + 1] = offsets[l] + counts[l] (one block; nlist
// lists scanned in chunks of the block width, carried in shared memory)
__global__ void list_offsets_kernel(const int64_t* __restrict__ counts, int32_t nlist,
                                    int64_t* __restrict__ offsets) {
  __shared__ int64_t part[1024];
  __shared__ int64_t carry;
  const int tid = threadIdx.x;
  if (tid == 0) {
    carry = 0;
    offsets[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < nlist; base += blockDim.x) {
    const int l = base + tid;
    part[tid] = l < nlist ? counts[l] : 0;
    __syncthreads();
    for (int o = 1; o < static_cast<int>(blockDim.x); o <<= 1) {
      const int64_t y = tid >= o ? part[tid - o] : 0;
      __syncthreads();
      part[tid] += y;
      __syncthreads();
    }
    if (l < nlist) offsets[l + 1] = carry + part[tid];
    __syncthreads();
    if (tid == blockDim.x - 1) carry += part[tid];
    __syncthreads();
  }
}

// packed[p] = rows[list_ids[p]], one warp per packed row
__global__ void gather_rows_kernel(const float* __restrict__ rows, int64_t ld,
                                   const uint32_t* __restrict__ ids, int64_t n, int32_t dim,
                                   float* __restrict__ packed, uint32_t* __restrict__ out_ids,
                                   uint32_t id_offset) {
  const int64_t p = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (p >= n) return;
  // reported ids: the corpus's own (a row shard's rows carry its first row)
  if (lane == 0) out_ids[p] = ids[p] + id_offset;
  const float* src = rows + static_cast<int64_t>(ids[p]) * ld;
  float* dst = packed + p * dim;
  for (int c = lane; c < dim; c += 32) dst[c] = src[c];
}

}  // namespace

// assign[r] = the list whose centroid has the smallest key for row r, ties
// to the lower list: assignRows' key is the host-tier distance of the row
// (as query) to each centroid, so this is the exact flat search with k = 1
// over the centroids, run in row chunks.
static int32_t assign_rows_device(mans_ctx* ctx, const mans_corpus* corpus,
                                  const mans_corpus* cent, int32_t metric, uint32_t* d_assign) {
  const int64_t n = corpus->n, dim = corpus->dim;
  if (n == 0) return MANS_OK;
  mans_workspace* ws = acquire_workspace(ctx);
  if (!ws) return fail(MANS_ERR_OOM, "no workspace stream");
  const int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(65536, (256ll << 20) / (dim * 4)));
  float* d_q = nullptr;
  float* d_dist = nullptr;
  int32_t* d_cnt = nullptr;
  cudaError_t e = cudaMalloc(&d_q, chunk * dim * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&d_dist, chunk * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&d_cnt, chunk * sizeof(int32_t));
  int32_t rc = e == cudaSuccess ? MANS_OK : fail_cuda(e, "cudaMalloc(assignment)");
  for (int64_t r0 = 0; rc == MANS_OK && r0 < n; r0 += chunk) {
    const int64_t m = std::min(chunk, n - r0);
    e = cudaMemcpy2DAsync(d_q, dim * sizeof(float), corpus->rows + r0 * corpus->ld,
                          corpus->ld * sizeof(float), dim * sizeof(float), m,
                          cudaMemcpyDeviceToDevice, ws->stream);
    if (e != cudaSuccess) {
      rc = fail_cuda(e, "assignment rows");
      break;
    }
    rc = run_flat_search(ctx, cent, ws, d_q, m, 1, metric, d_dist, d_assign + r0, d_cnt,
                         ws->stream, kModeHost, MANS_MAX_TOPK, true);
  }
  if (rc == MANS_OK) {
    e = cudaStreamSynchronize(ws->stream);
    if (e != cudaSuccess) rc = fail_cuda(e, "assignment");
  }
  if (rc == MANS_OK) rc = check_device_error(ws, ws->stream);
  cudaFree(d_q);
  cudaFree(d_dist);
  cudaFree(d_cnt);
  release_workspace(ctx, ws);
  return rc;
}

}  // namespace mans

#include <cub/cub.cuh>

extern "C" {

int32_t mans_ivf_assign(mans_ctx* ctx, mans_corpus* corpus, const float* centroids,
                        int32_t nlist, int32_t metric, int32_t* out_assign) {
  if (!ctx || !corpus || !centroids || !out_assign)
    return fail(MANS_ERR_INVALID, "null context, corpus or buffer");
  if (int32_t r = reject_group(ctx, corpus, "mans_ivf_assign")) return r;
  if (nlist <= 0) return fail(MANS_ERR_INVALID, "nlist must be positive");
  if (metric < 0 || metric > 2) return fail(MANS_ERR_SEARCH, "IVF assignment needs cosine, l2 or ip");
  DeviceGuard g(ctx->device);
  mans_corpus* cent = nullptr;
  int32_t rc = corpus_upload(ctx, centroids, nlist, corpus->dim, 0, &cent);
  if (rc != MANS_OK) return rc;
  uint32_t* d_assign = nullptr;
  cudaError_t e = cudaMalloc(&d_assign, std::max<int64_t>(corpus->n, 1) * sizeof(uint32_t));
  if (e != cudaSuccess) rc = fail_cuda(e, "cudaMalloc(assignment)");
  if (rc == MANS_OK) rc = assign_rows_device(ctx, corpus, cent, metric, d_assign);
  if (rc == MANS_OK && corpus->n > 0) {
    e = cudaMemcpy(out_assign, d_assign, corpus->n * sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) rc = fail_cuda(e, "assignment download");
  }
  cudaFree(d_assign);
  corpus_free(cent);
  return rc;
}

int32_t mans_ivf_build(mans_ctx* ctx, mans_corpus* corpus, const float* centroids,
                       int32_t nlist, int32_t metric, mans_ivf** out_ivf) {
  if (!ctx || !corpus || !centroids || !out_ivf)
    return fail(MANS_ERR_INVALID, "null context, corpus or output");
  *out_ivf = nullptr;
  if (int32_t r = reject_group(ctx, corpus, "mans_ivf_build")) return r;
  if (nlist <= 0) return fail(MANS_ERR_INVALID, "nlist must be positive");
  if (metric < 0 || metric > 2) return fail(MANS_ERR_SEARCH, "IVF build needs cosine, l2 or ip");
  DeviceGuard g(ctx->device);
  const int64_t n = corpus->n, dim = corpus->dim;
  mans_ivf* ivf = new mans_ivf();
  ivf->ctx = ctx;
  ivf->nlist = nlist;
  ivf->n = n;
  ivf->dim = dim;
  int32_t rc = corpus_upload(ctx, centroids, nlist, dim, 0, &ivf->cent);
  uint32_t *d_assign = nullptr, *d_keys = nullptr, *d_iota = nullptr, *d_ids = nullptr;
  int64_t* d_counts = nullptr;
  float* d_packed = nullptr;
  void* d_tmp = nullptr;
  const int64_t nn = std::max<int64_t>(n, 1);
  cudaError_t e = cudaSuccess;
  auto ck = [&](cudaError_t x, const char* what) {
    if (rc == MANS_OK && x != cudaSuccess) rc = fail_cuda(x, what);
  };
  if (rc == MANS_OK) {
    ck(cudaMalloc(&d_assign, nn * sizeof(uint32_t)), "cudaMalloc(build)");
    ck(cudaMalloc(&d_keys, nn * sizeof(uint32_t)), "cudaMalloc(build)");
    ck(cudaMalloc(&d_iota, nn * sizeof(uint32_t)), "cudaMalloc(build)");
    ck(cudaMalloc(&d_ids, nn * sizeof(uint32_t)), "cudaMalloc(build)");
    ck(cudaMalloc(&d_counts, nlist * sizeof(int64_t)), "cudaMalloc(build)");
    ck(cudaMalloc(&ivf->offsets, (nlist + 1) * sizeof(int64_t)), "cudaMalloc(build)");
    ck(cudaMalloc(&d_packed, nn * dim * sizeof(float)), "cudaMalloc(build)");
  }
  // 1. assignment (exact, ties to the lower list)
  if (rc == MANS_OK) rc = assign_rows_device(ctx, corpus, ivf->cent, metric, d_assign);
  // 2. stable counting sort of the rows by list: list ids ascend by row
  if (rc == MANS_OK && n > 0) {
    int bits = 1;
    while ((1ll << bits) < nlist) ++bits;
    size_t tmp_bytes = 0;
    ck(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, d_assign, d_keys, d_iota, d_ids,
                                       static_cast<int>(n), 0, bits),
       "radix sort size");
    if (rc == MANS_OK) ck(cudaMalloc(&d_tmp, tmp_bytes), "cudaMalloc(sort)");
    if (rc == MANS_OK) {
      iota_u32_kernel<<<static_cast<unsigned>((n + 255) / 256), 256>>>(d_iota, n);
      ck(cudaGetLastError(), "iota");
      ck(cub::DeviceRadixSort::SortPairs(d_tmp, tmp_bytes, d_assign, d_keys, d_iota, d_ids,
                                         static_cast<int>(n), 0, bits),
         "radix sort");
    }
  }
  // 3. offsets from the list sizes
  if (rc == MANS_OK) {
    ck(cudaMemset(d_counts, 0, nlist * sizeof(int64_t)), "counts clear");
    if (rc == MANS_OK && n > 0) {
      list_histogram_kernel<<<static_cast<unsigned>((n + 255) / 256), 256>>>(d_assign, n, d_counts);
      ck(cudaGetLastError(), "list sizes");
    }
    if (rc == MANS_OK) {
      list_offsets_kernel<<<1, 1024>>>(d_counts, nlist, ivf->offsets);
      ck(cudaGetLastError(), "list offsets");
    }
  }
  // 4. packed rows in list order
  if (rc == MANS_OK && n > 0) {
    gather_rows_kernel<<<static_cast<unsigned>((n * 32 + 255) / 256), 256>>>(
        corpus->rows, corpus->ld, d_ids, n, static_cast<int32_t>(dim), d_packed, d_keys,
        corpus->id_offset);
    ck(cudaGetLastError(), "gather rows");
  }
  if (rc == MANS_OK) ck(cudaDeviceSynchronize(), "partition build");
  if (rc == MANS_OK) rc = corpus_upload(ctx, d_packed, n, dim, 0, &ivf->packed);
  if (rc == MANS_OK) {
    ivf->packed->ids = d_keys;  // (global) ids, owned by the packed corpus from here on
    d_keys = nullptr;
    ivf->h_offsets.resize(nlist + 1);
    ck(cudaMemcpy(ivf->h_offsets.data(), ivf->offsets, (nlist + 1) * sizeof(int64_t),
                  cudaMemcpyDeviceToHost),
       "offsets download");
  }
  if (rc == MANS_OK) {
    for (int32_t l = 0; l < nlist; ++l)
      ivf->max_len = std::max(ivf->max_len, ivf->h_offsets[l + 1] - ivf->h_offsets[l]);
  }
  cudaFree(d_assign);
  if (d_keys) cudaFree(d_keys);
  cudaFree(d_iota);
  cudaFree(d_ids);
  cudaFree(d_counts);
  cudaFree(d_packed);
  if (d_tmp) cudaFree(d_tmp);
  (void)e;
  if (rc != MANS_OK) {
    corpus_free(ivf->cent);
    corpus_free(ivf->packed);
    if (ivf->offsets) cudaFree(ivf->offsets);
    delete ivf;
    return rc;
  }
  *out_ivf = ivf;
  return MANS_OK;
}

int32_t mans_ivf_layout(const mans_ivf* ivf, int64_t* list_offsets, uint32_t* list_ids) {
  if (!ivf) return fail(MANS_ERR_INVALID, "null IVF index");
  DeviceGuard g(ivf->ctx->device);
  if (list_offsets)
    std::memcpy(list_offsets, ivf->h_offsets.data(), (ivf->nlist + 1) * sizeof(int64_t));
  if (list_ids && ivf->n > 0) {
    cudaError_t e = cudaMemcpy(list_ids, ivf->packed->ids, ivf->n * sizeof(uint32_t),
                               cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return fail_cuda(e, "list id download");
  }
  return MANS_OK;
}

}  // extern "C"
