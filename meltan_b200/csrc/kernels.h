// kernels.h -- host-side launch interface of the search kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mans {

constexpr int kTileRows = 256;                               // rows per TMA box (largest)
constexpr int kSmallTileRows = 64;  // box rows for small scans: more CTAs share a short scan
constexpr int kTileCols = 32;                                // fp32 columns per box (128 B)
constexpr int kTileBytes = kTileRows * kTileCols * 4;        // 32 KiB per pipeline stage
constexpr int kConsumerWarps = 8;                            // one corpus row per thread
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kScanThreads = kConsumers + 32;                // + one TMA producer warp
constexpr int kSortN = 1024;                                 // running top-k buffer per query
constexpr int kMaxStages = 6;
constexpr int kMergeThreads = 256;

// Device error words written by kernels (0 = no error).
constexpr int kErrTimeout = 1;
constexpr int kErrBadArg = 2;

// One unit of scan work: a contiguous row range of the row matrix scanned for
// up to QB queries.  Query j of the unit is query qidx[qbase + j] (or qbase + j
// when qidx is null) and its partial top-k goes to slot slot_base + j *
// slot_stride.
struct ScanSegment {
  int64_t row_begin;
  int32_t row_count;
  int32_t qbase;
  int32_t qcount;
  int32_t slot_base;
  int32_t slot_stride;
  int32_t reserved;
};

struct ScanParams {
  const ScanSegment* segs;  // null: flat mode, segments derived arithmetically
  int32_t nseg;
  const int32_t* nseg_dev;  // when set, the segment count is read on the device
  int32_t stages;
  // flat mode: nseg = groups * flat_splits; group g holds queries
  // [g*QB, min(nq, g*QB+QB)), split s holds tiles [s*T/S, (s+1)*T/S).
  int32_t flat_splits;
  int32_t flat_tiles;
  int64_t n;
  int64_t nq;
  const float* queries;  // nq x dim, row-major
  const int32_t* qidx;
  const float* qnorms;   // squared query norms; null: computed in the kernel when needed
  const float* norms;    // squared row norms (cosine / L2), else null
  const uint32_t* ids;   // row -> reported id (null: row + id_offset)
  uint32_t id_offset;
  int32_t dim;
  int32_t nchunks;       // ceil(dim / 32)
  int32_t metric;
  // 0: host-tier distance from dot(q, v) (ParallelFlatScan.swift:237-258);
  // 1: SIMDDistance semantics (SIMDDistance.swift:17-80): L2 accumulates
  //    sum((q - v)^2), cosine uses sqrt(|q|^2) * sqrt(|v|^2), IP = -dot.
  int32_t mode;
  int32_t k;             // effective k (<= kp)
  int32_t kp;            // power of two >= k, <= 512
  uint64_t* slot_keys;   // [slot][kp]
  int32_t* slot_counts;  // [slot]
  int* err;
  int32_t tile_rows;  // rows per TMA box / tile: kTileRows or kSmallTileRows
};

size_t scan_smem_bytes(int qb, int nchunks, int stages);
int scan_max_stages(int qb, int nchunks);
cudaError_t scan_configure(int max_smem_optin);
cudaError_t launch_scan(int qb, const CUtensorMap& map, const ScanParams& p, int grid,
                        cudaStream_t stream);
constexpr int kModeHost = 0;
constexpr int kModeSimd = 1;

cudaError_t launch_row_norms(const float* rows, int64_t n, int32_t dim, int64_t ld, float* out,
                             cudaStream_t stream);
cudaError_t launch_query_norms(const float* q, int64_t nq, int32_t dim, float* out,
                               cudaStream_t stream);

// Merges per-query candidate slots into the final sorted top-k.
//   keys mode  : in_keys[slot*kp_in + i], counts[slot], query q owns slots
//                [q*spq, (q+1)*spq) or [offs[q], offs[q+1]) when offs != null.
//   pairs mode : in_dist/in_ids[(l*nq + q)*kp_in + i], counts[l*nq + q],
//                l in [0, n_lists).
struct MergeParams {
  const uint64_t* in_keys;
  const float* in_dist;
  const uint32_t* in_ids;
  const int32_t* in_counts;
  const int32_t* q_slot_offsets;
  const int32_t* q_slot_list;  // with offsets: query q reads slots list[offs[q]..offs[q+1])
  int32_t slots_per_query;
  int32_t n_lists;
  int64_t list_stride;   // pairs mode: elements between shard blocks (0: nq*kp_in / nq)
  int32_t kp_in;
  int64_t nq;
  int32_t k;
  int32_t kp;
  int32_t kout;
  float* out_dist;
  uint32_t* out_ids;
  int32_t* out_counts;
  int* err;
  // optional: before merging, wait (bounded) until wait_flags[0..wait_count)
  // all hold wait_epoch (peer ranks' blocks have landed in in_* memory)
  const uint32_t* wait_flags;
  int32_t wait_count;
  uint32_t wait_epoch;
  // when set (err must then be a cleared word), a non-zero *err seen after
  // the waits makes every query's result empty (count 0)
  bool empty_on_error;
};
cudaError_t launch_merge(const MergeParams& p, cudaStream_t stream);

cudaError_t launch_fill_empty(float* out_dist, uint32_t* out_ids, int32_t* out_counts, int64_t nq,
                              int32_t kout, cudaStream_t stream);

}  // namespace mans
