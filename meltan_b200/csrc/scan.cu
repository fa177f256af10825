// scan.cu -- exact fused distance scan + running top-k (the flat exact tier).
//
// Replaces `flat_scan_distances` + `flat_finalize_metric`
// (Sources/MetalANNSCore/Shaders/FlatSearch.metal:17-77) and the host top-k
// that followed it (FlatGPUSearch.selectTopK / boundedTopK,
// FlatGPUSearch.swift:786-933).  Unlike the Metal kernel no n x nq distance
// matrix is written: each block keeps a running top-k per query in shared
// memory and emits only k keys per (segment, query).
//
// Layout and pipeline (one block per SM, persistent over segments):
//   warp 8       TMA producer: 2-D tensor-map boxes of 256 rows x 32 fp32
//                columns (32 KiB, 128-byte swizzle) into a ring of stages,
//                completion signalled on per-stage mbarriers;
//   warps 0..7   consumers: thread t owns row t of the box and accumulates
//                dot(q, row) for up to QB queries, column by column in index
//                order with separately rounded multiply and add -- the exact
//                summation order of Sources/MetalANNSC/dots.c:40-47 -- then the
//                host-tier metric finalize (ParallelFlatScan.swift:237-258).
// The 128-byte swizzle places 16-byte chunk j of box row r at chunk j^(r&7),
// so the eight threads of a quarter-warp read eight distinct bank groups.
#include "common.cuh"
#include "kernels.h"

namespace mans {

namespace {

struct ScanSmem {
  float* tiles;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* topbuf;
  uint64_t* thr;
  int* qcnt;
  int* nbest;
  int* ctrl;  // [0] abort flag, [1] consumed stage count
  float* qn;
  float* q;   // QB x (nchunks*32)
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <int QB>
__host__ __device__ inline size_t scan_layout(int nchunks, int stages, size_t* offs) {
  size_t o = 0;
  offs[0] = o;  // tiles
  o += static_cast<size_t>(stages) * kTileBytes;
  offs[1] = o;  // full
  o += stages * 8;
  offs[2] = o;  // empty
  o += stages * 8;
  offs[3] = o;  // topbuf
  o += static_cast<size_t>(QB) * kSortN * 8;
  offs[4] = o;  // thr
  o += QB * 8;
  offs[5] = o;  // qcnt
  o += QB * 4;
  offs[6] = o;  // nbest
  o += QB * 4;
  offs[7] = o;  // ctrl
  o += 16;
  offs[8] = o;  // qn
  o += QB * 4;
  o = align_up(o, 16);
  offs[9] = o;  // q
  o += static_cast<size_t>(QB) * nchunks * kTileCols * 4;
  return o;
}

__device__ inline void flat_segment(const ScanParams& p, int s, int qb, ScanSegment& seg) {
  if (p.segs) {
    seg = p.segs[s];
    return;
  }
  int g = s / p.flat_splits;
  int r = s - g * p.flat_splits;
  int64_t t0 = static_cast<int64_t>(p.flat_tiles) * r / p.flat_splits;
  int64_t t1 = static_cast<int64_t>(p.flat_tiles) * (r + 1) / p.flat_splits;
  int64_t row0 = t0 * p.tile_rows;
  int64_t row1 = t1 * p.tile_rows < p.n ? t1 * p.tile_rows : p.n;
  seg.row_begin = row0;
  seg.row_count = static_cast<int32_t>(row1 > row0 ? row1 - row0 : 0);
  seg.qbase = g * qb;
  int64_t left = p.nq - static_cast<int64_t>(g) * qb;
  seg.qcount = static_cast<int32_t>(left < qb ? left : qb);
  seg.slot_base = g * qb * p.flat_splits + r;
  seg.slot_stride = p.flat_splits;
  seg.reserved = 0;
}

template <int QB, bool DIFFSQ>
__global__ void __launch_bounds__(kScanThreads, 1)
    scan_topk_kernel(const __grid_constant__ CUtensorMap map, const ScanParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(align_up(reinterpret_cast<size_t>(smem_raw), 1024));
  size_t offs[10];
  scan_layout<QB>(p.nchunks, p.stages, offs);
  ScanSmem sm;
  sm.tiles = reinterpret_cast<float*>(base + offs[0]);
  sm.full = reinterpret_cast<uint64_t*>(base + offs[1]);
  sm.empty = reinterpret_cast<uint64_t*>(base + offs[2]);
  sm.topbuf = reinterpret_cast<uint64_t*>(base + offs[3]);
  sm.thr = reinterpret_cast<uint64_t*>(base + offs[4]);
  sm.qcnt = reinterpret_cast<int*>(base + offs[5]);
  sm.nbest = reinterpret_cast<int*>(base + offs[6]);
  sm.ctrl = reinterpret_cast<int*>(base + offs[7]);
  sm.qn = reinterpret_cast<float*>(base + offs[8]);
  sm.q = reinterpret_cast<float*>(base + offs[9]);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int stages = p.stages;

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.ctrl[0] = 0;
    sm.ctrl[1] = 0;
    fence_mbar_init();
  }
  if (tid == kConsumers) tma_prefetch_desc(&map);
  __syncthreads();

  const int qw = p.nchunks * kTileCols;
  const int nseg = p.nseg_dev ? *p.nseg_dev : p.nseg;

  if (warp == kConsumerWarps) {
    // ---------------- TMA producer ----------------
    int issued = 0;
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int s = blockIdx.x; s < nseg; s += gridDim.x) {
        ScanSegment seg;
        flat_segment(p, s, QB, seg);
        int ntiles = (seg.row_count + p.tile_rows - 1) / p.tile_rows;
        for (int rt = 0; rt < ntiles; ++rt) {
          int32_t y = static_cast<int32_t>(seg.row_begin + static_cast<int64_t>(rt) * p.tile_rows);
          for (int cc = 0; cc < p.nchunks; ++cc) {
            bool ok = mbar_wait_bounded(&sm.empty[stage], phase ^ 1u, p.err);
            if (!ok || *(volatile int*)&sm.ctrl[0]) {
              *(volatile int*)&sm.ctrl[0] = 1;
              goto producer_done;
            }
            mbar_arrive_expect_tx(&sm.full[stage], static_cast<uint32_t>(p.tile_rows) * kTileCols * 4);
            tma_load_2d(sm.tiles + static_cast<size_t>(stage) * (kTileBytes / 4), &map,
                        cc * kTileCols, y, &sm.full[stage]);
            ++issued;
            if (++stage == stages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
    producer_done:;
      // Drain: every issued copy must land before the block may exit.  In the
      // normal flow the consumers have waited on all of them; after an abort
      // wait (bounded) for the ones nobody consumed.
      __threadfence_block();
      int consumed = *(volatile int*)&sm.ctrl[1];
      if (*(volatile int*)&sm.ctrl[0]) {
        for (int i = consumed; i < issued; ++i) {
          int st = i % stages;
          uint32_t ph = static_cast<uint32_t>((i / stages) & 1);
          if (!mbar_wait_bounded(&sm.full[st], ph, p.err)) break;
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  int stage = 0;
  uint32_t phase = 0;
  int consumed = 0;
  bool aborted = false;
  for (int s = blockIdx.x; s < nseg && !aborted; s += gridDim.x) {
    ScanSegment seg;
    flat_segment(p, s, QB, seg);
    for (int i = tid; i < QB * qw; i += kConsumers) {
      int j = i / qw;
      int c = i - j * qw;
      float v = 0.0f;
      if (j < seg.qcount && c < p.dim) {
        int64_t q = p.qidx ? p.qidx[seg.qbase + j] : seg.qbase + j;
        v = p.queries[q * p.dim + c];
      }
      sm.q[i] = v;
    }
    if (tid < QB) {
      float qn = 0.0f;
      if (tid < seg.qcount && p.qnorms) {
        int64_t q = p.qidx ? p.qidx[seg.qbase + tid] : seg.qbase + tid;
        qn = p.qnorms[q];
      }
      sm.qn[tid] = qn;
      sm.qcnt[tid] = 0;
      sm.nbest[tid] = 0;
      sm.thr[tid] = kKeyMax;
    }
    named_sync(1, kConsumers);
    if (!p.qnorms && p.metric != kIP && tid < seg.qcount) {
      // squared query norm in index order (FlatGPUSearch.swift:532-535), read
      // from the staged copy while the TMA ring fills
      const float* qv = sm.q + tid * qw;
      float acc = 0.0f;
      for (int c = 0; c < p.dim; ++c) acc = __fadd_rn(acc, __fmul_rn(qv[c], qv[c]));
      sm.qn[tid] = acc;
    }
    named_sync(1, kConsumers);

    int ntiles = (seg.row_count + p.tile_rows - 1) / p.tile_rows;
    for (int rt = 0; rt < ntiles; ++rt) {
      int64_t local = static_cast<int64_t>(rt) * p.tile_rows + tid;
      bool valid = tid < p.tile_rows && local < seg.row_count;
      int64_t row = seg.row_begin + local;
      float vn = 0.0f;
      uint32_t id = 0;
      if (valid) {
        if (p.norms) vn = __ldg(p.norms + row);
        id = p.ids ? __ldg(p.ids + row) : static_cast<uint32_t>(row + p.id_offset);
      }
      float acc[QB];
#pragma unroll
      for (int q = 0; q < QB; ++q) acc[q] = 0.0f;

      for (int cc = 0; cc < p.nchunks; ++cc) {
        if (!mbar_wait_bounded(&sm.full[stage], phase, p.err)) {
          *(volatile int*)&sm.ctrl[0] = 1;
          aborted = true;
        }
        if (__any_sync(0xFFFFFFFFu, aborted) || *(volatile int*)&sm.ctrl[0]) {
          aborted = true;
          break;
        }
        const uint8_t* rowp = reinterpret_cast<const uint8_t*>(sm.tiles) +
                              static_cast<size_t>(stage) * kTileBytes + tid * 128;
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          v[j] = *reinterpret_cast<const float4*>(rowp + ((j ^ (tid & 7)) << 4));
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.empty[stage]);
        ++consumed;
        if (++stage == stages) {
          stage = 0;
          phase ^= 1u;
        }
        const float* qc = sm.q + cc * kTileCols;
#pragma unroll
        for (int q = 0; q < QB; ++q) {
          const float4* qv = reinterpret_cast<const float4*>(qc + q * qw);
          float a = acc[q];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 b = qv[j];
            if (DIFFSQ) {
              float t;
              t = __fsub_rn(b.x, v[j].x);
              a = __fadd_rn(a, __fmul_rn(t, t));
              t = __fsub_rn(b.y, v[j].y);
              a = __fadd_rn(a, __fmul_rn(t, t));
              t = __fsub_rn(b.z, v[j].z);
              a = __fadd_rn(a, __fmul_rn(t, t));
              t = __fsub_rn(b.w, v[j].w);
              a = __fadd_rn(a, __fmul_rn(t, t));
            } else {
              a = __fadd_rn(a, __fmul_rn(v[j].x, b.x));
              a = __fadd_rn(a, __fmul_rn(v[j].y, b.y));
              a = __fadd_rn(a, __fmul_rn(v[j].z, b.z));
              a = __fadd_rn(a, __fmul_rn(v[j].w, b.w));
            }
          }
          acc[q] = a;
        }
      }
      // all consumer warps agree on abort before touching shared barriers
      named_sync(1, kConsumers);
      if (*(volatile int*)&sm.ctrl[0]) {
        aborted = true;
        break;
      }

#pragma unroll
      for (int q = 0; q < QB; ++q) {
        if (q < seg.qcount) {
          float d = p.mode == kModeSimd ? finalize_simd(p.metric, acc[q], sm.qn[q], vn)
                                        : finalize_distance(p.metric, acc[q], sm.qn[q], vn);
          TopKState st{sm.topbuf + q * kSortN, &sm.qcnt[q], &sm.nbest[q], &sm.thr[q]};
          topk_offer(st, p.kp, make_key(d, id), valid);
        }
      }
      named_sync(1, kConsumers);
      for (int q = 0; q < seg.qcount; ++q) {
        if (sm.qcnt[q] > kSortN - p.kp - kConsumers) {
          TopKState st{sm.topbuf + q * kSortN, &sm.qcnt[q], &sm.nbest[q], &sm.thr[q]};
          topk_merge<kConsumers>(st, p.k, p.kp, kSortN, tid, 1);
        }
      }
    }
    if (aborted) break;

    for (int q = 0; q < seg.qcount; ++q) {
      TopKState st{sm.topbuf + q * kSortN, &sm.qcnt[q], &sm.nbest[q], &sm.thr[q]};
      if (sm.qcnt[q] > 0) topk_merge<kConsumers>(st, p.k, p.kp, kSortN, tid, 1);
      int slot = seg.slot_base + q * seg.slot_stride;
      int nb = sm.nbest[q];
      for (int i = tid; i < nb; i += kConsumers)
        p.slot_keys[static_cast<size_t>(slot) * p.kp + i] = st.buf[i];
      if (tid == 0) p.slot_counts[slot] = nb;
    }
    named_sync(1, kConsumers);
  }
  if (tid == 0) *(volatile int*)&sm.ctrl[1] = consumed;
}

// Squared row norms in index order (the sequential stand-in for the closed
// vDSP_vsq + cblas_sgemv order of FlatGPUSearch.swift:484-501).  A block of
// 128 threads stages 128 rows x 32 columns through shared memory so global
// reads stay coalesced; each thread then sums its own row sequentially.
__global__ void __launch_bounds__(128) row_norms_kernel(const float* __restrict__ rows,
                                                        int64_t n, int32_t dim, int64_t ld,
                                                        float* __restrict__ out) {
  __shared__ float tile[128][33];
  int64_t row0 = static_cast<int64_t>(blockIdx.x) * 128;
  int t = threadIdx.x;
  float acc = 0.0f;
  for (int c0 = 0; c0 < dim; c0 += 32) {
    for (int i = t; i < 128 * 32; i += 128) {
      int r = i >> 5, c = i & 31;
      int64_t row = row0 + r;
      tile[r][c] = (row < n && c0 + c < dim) ? rows[row * ld + c0 + c] : 0.0f;
    }
    __syncthreads();
    int cols = dim - c0 < 32 ? dim - c0 : 32;
    for (int c = 0; c < cols; ++c) {
      float x = tile[t][c];
      acc = __fadd_rn(acc, __fmul_rn(x, x));
    }
    __syncthreads();
  }
  if (row0 + t < n) out[row0 + t] = acc;
}

// Squared query norms, one thread per query, index order (FlatGPUSearch.swift
// :532-535 and :740-749).
__global__ void query_norms_kernel(const float* __restrict__ q, int64_t nq, int32_t dim,
                                   float* __restrict__ out) {
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nq) return;
  const float* v = q + i * dim;
  float acc = 0.0f;
#pragma unroll 8
  for (int d = 0; d < dim; ++d) acc = __fadd_rn(acc, __fmul_rn(v[d], v[d]));
  out[i] = acc;
}

__global__ void __launch_bounds__(kMergeThreads) merge_kernel(const MergeParams p) {
  __shared__ uint64_t buf[kSortN];
  __shared__ uint64_t thr;
  __shared__ int qc, nb, failed;
  const int tid = threadIdx.x;
  const int64_t q = blockIdx.x;
  if (tid == 0) {
    thr = kKeyMax;
    qc = 0;
    nb = 0;
    failed = 0;
  }
  if (p.wait_flags && tid < p.wait_count) {
    // peer blocks: acquire-load the flag a peer release-stored after its data
    const unsigned long long t0 = global_ns();
    for (uint32_t it = 0;; ++it) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.wait_flags + tid) : "memory");
      if (v == p.wait_epoch) break;
      if ((it & 63u) == 63u && global_ns() - t0 > kWaitLimitNs) {
        atomicExch(p.err, kErrTimeout);
        break;
      }
    }
  }
  __syncthreads();
  if (p.empty_on_error) {
    // An earlier kernel of this call (or a peer wait above) gave up: its
    // candidate lists are incomplete, so report no results instead of a
    // plausible-looking partial top-k.
    if (tid == 0) failed = atomicAdd(p.err, 0) != 0;
    __syncthreads();
    if (failed) {
      for (int i = tid; i < p.kout; i += kMergeThreads) {
        p.out_dist[q * p.kout + i] = __int_as_float(0x7F800000);
        p.out_ids[q * p.kout + i] = kEmptyId;
      }
      if (tid == 0) p.out_counts[q] = 0;
      return;
    }
  }
  TopKState st{buf, &qc, &nb, &thr};

  int64_t nslots;
  int64_t slot0 = 0;
  if (p.in_keys) {
    if (p.q_slot_offsets) {
      slot0 = p.q_slot_offsets[q];
      nslots = p.q_slot_offsets[q + 1] - slot0;
    } else {
      slot0 = q * p.slots_per_query;
      nslots = p.slots_per_query;
    }
  } else {
    nslots = p.n_lists;
  }
  // Every slot is sorted, so the k-th smallest slot head bounds the global
  // k-th key from above (k slots each hold a key <= it): start from there.
  if (nslots >= p.k && nslots <= kSortN) {
    int ns = 1;
    while (ns < nslots) ns <<= 1;
    for (int i = tid; i < ns; i += kMergeThreads) {
      uint64_t h = kKeyMax;
      if (i < nslots) {
        if (p.in_keys) {
          int64_t slot = p.q_slot_list ? p.q_slot_list[slot0 + i] : slot0 + i;
          if (p.in_counts[slot] > 0) h = p.in_keys[slot * p.kp_in];
        } else {
          const int64_t ls = p.list_stride ? p.list_stride : p.nq * p.kp_in;
          const int64_t cs = p.list_stride ? p.list_stride : p.nq;
          if (p.in_counts[static_cast<int64_t>(i) * cs + q] > 0) {
            const int64_t at = static_cast<int64_t>(i) * ls + q * p.kp_in;
            h = make_key(p.in_dist[at], p.in_ids[at]);
          }
        }
      }
      buf[i] = h;
    }
    __syncthreads();
    bitonic_sort_keys<kMergeThreads>(buf, ns, tid, 0);
    if (tid == 0 && buf[p.k - 1] != kKeyMax) thr = buf[p.k - 1] + 1;
    __syncthreads();
  }
  const int64_t total = nslots * p.kp_in;
  for (int64_t b = 0; b < total; b += kMergeThreads) {
    int64_t pos = b + tid;
    uint64_t key = kKeyMax;
    bool valid = false;
    if (pos < total) {
      int64_t sl = pos / p.kp_in;
      int i = static_cast<int>(pos - sl * p.kp_in);
      if (p.in_keys) {
        int64_t slot = p.q_slot_list ? p.q_slot_list[slot0 + sl] : slot0 + sl;
        if (i < p.in_counts[slot]) {
          key = p.in_keys[slot * p.kp_in + i];
          valid = true;
        }
      } else {
        const int64_t ls = p.list_stride ? p.list_stride : p.nq * p.kp_in;
        const int64_t cs = p.list_stride ? p.list_stride : p.nq;
        if (i < p.in_counts[sl * cs + q]) {
          const int64_t at = sl * ls + q * p.kp_in + i;
          key = make_key(p.in_dist[at], p.in_ids[at]);
          valid = true;
        }
      }
    }
    topk_offer(st, p.kp, key, valid);
    __syncthreads();
    if (qc > kSortN - p.kp - kMergeThreads) topk_merge<kMergeThreads>(st, p.k, p.kp, kSortN, tid, 0);
  }
  if (qc > 0) topk_merge<kMergeThreads>(st, p.k, p.kp, kSortN, tid, 0);
  for (int i = tid; i < p.kout; i += kMergeThreads) {
    bool have = i < nb;
    p.out_dist[q * p.kout + i] = have ? key_distance(buf[i]) : __int_as_float(0x7F800000);
    p.out_ids[q * p.kout + i] = have ? key_id(buf[i]) : kEmptyId;
  }
  if (tid == 0) p.out_counts[q] = nb;
}

__global__ void fill_empty_kernel(float* d, uint32_t* ids, int32_t* counts, int64_t nq,
                                  int32_t kout) {
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < nq * kout) {
    d[i] = __int_as_float(0x7F800000);
    ids[i] = kEmptyId;
  }
  if (i < nq) counts[i] = 0;
}

}  // namespace

size_t scan_smem_bytes(int qb, int nchunks, int stages) {
  size_t offs[10];
  size_t body = 0;
  switch (qb) {
    case 1: body = scan_layout<1>(nchunks, stages, offs); break;
    case 2: body = scan_layout<2>(nchunks, stages, offs); break;
    case 4: body = scan_layout<4>(nchunks, stages, offs); break;
    default: body = scan_layout<8>(nchunks, stages, offs); break;
  }
  return body + 1024;  // room to align the dynamic base to 1024 B
}

static int g_max_smem = 0;

int scan_max_stages(int qb, int nchunks) {
  int st = kMaxStages;
  while (st > 1 && scan_smem_bytes(qb, nchunks, st) > static_cast<size_t>(g_max_smem)) --st;
  if (scan_smem_bytes(qb, nchunks, st) > static_cast<size_t>(g_max_smem)) return 0;
  return st;
}

template <int QB, bool D>
static cudaError_t set_smem(int bytes) {
  return cudaFuncSetAttribute(scan_topk_kernel<QB, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              bytes);
}

cudaError_t scan_configure(int max_smem_optin) {
  g_max_smem = max_smem_optin;
  cudaError_t e;
  if ((e = set_smem<1, false>(max_smem_optin)) != cudaSuccess) return e;
  if ((e = set_smem<2, false>(max_smem_optin)) != cudaSuccess) return e;
  if ((e = set_smem<4, false>(max_smem_optin)) != cudaSuccess) return e;
  if ((e = set_smem<8, false>(max_smem_optin)) != cudaSuccess) return e;
  if ((e = set_smem<1, true>(max_smem_optin)) != cudaSuccess) return e;
  if ((e = set_smem<2, true>(max_smem_optin)) != cudaSuccess) return e;
  if ((e = set_smem<4, true>(max_smem_optin)) != cudaSuccess) return e;
  return set_smem<8, true>(max_smem_optin);
}

template <bool D>
static cudaError_t launch_scan_t(int qb, const CUtensorMap& map, const ScanParams& p, int grid,
                                 size_t smem, cudaStream_t stream) {
  switch (qb) {
    case 1: scan_topk_kernel<1, D><<<grid, kScanThreads, smem, stream>>>(map, p); break;
    case 2: scan_topk_kernel<2, D><<<grid, kScanThreads, smem, stream>>>(map, p); break;
    case 4: scan_topk_kernel<4, D><<<grid, kScanThreads, smem, stream>>>(map, p); break;
    case 8: scan_topk_kernel<8, D><<<grid, kScanThreads, smem, stream>>>(map, p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_scan(int qb, const CUtensorMap& map, const ScanParams& p, int grid,
                        cudaStream_t stream) {
  size_t smem = scan_smem_bytes(qb, p.nchunks, p.stages);
  // the (q - v)^2 accumulation is used only for SIMDDistance L2
  if (p.mode == kModeSimd && p.metric == kL2) return launch_scan_t<true>(qb, map, p, grid, smem, stream);
  return launch_scan_t<false>(qb, map, p, grid, smem, stream);
}

cudaError_t launch_row_norms(const float* rows, int64_t n, int32_t dim, int64_t ld, float* out,
                             cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  int64_t blocks = (n + 127) / 128;
  row_norms_kernel<<<static_cast<unsigned>(blocks), 128, 0, stream>>>(rows, n, dim, ld, out);
  return cudaGetLastError();
}

cudaError_t launch_query_norms(const float* q, int64_t nq, int32_t dim, float* out,
                               cudaStream_t stream) {
  if (nq <= 0) return cudaSuccess;
  query_norms_kernel<<<static_cast<unsigned>((nq + 127) / 128), 128, 0, stream>>>(q, nq, dim, out);
  return cudaGetLastError();
}

cudaError_t launch_merge(const MergeParams& p, cudaStream_t stream) {
  if (p.nq <= 0) return cudaSuccess;
  merge_kernel<<<static_cast<unsigned>(p.nq), kMergeThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_fill_empty(float* out_dist, uint32_t* out_ids, int32_t* out_counts, int64_t nq,
                              int32_t kout, cudaStream_t stream) {
  int64_t total = nq * (kout > 1 ? kout : 1);
  if (total < nq) total = nq;
  if (total <= 0) return cudaSuccess;
  fill_empty_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      out_dist, out_ids, out_counts, nq, kout);
  return cudaGetLastError();
}

}  // namespace mans
