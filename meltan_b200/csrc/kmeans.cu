// kmeans.cu -- KMeans.cluster's Lloyd iterations and ProductQuantizer.train on
// the device, from given initial centroids.
//
// The reference clusters the IVF-flat sample (IVFFlatSearch.buildPartition,
// Sources/MetalANNSCore/IVFFlatSearch.swift:529-551, 8 iterations), the IVF-PQ
// coarse quantiser (IVFPQIndex.train, Sources/MetalANNS/IVFPQIndex.swift:
// 54-104) and every PQ subspace (ProductQuantizer.train,
// Sources/MetalANNSCore/ProductQuantizer.swift:10-86, KMeans.clusterSubspace,
// L2, k = 256) with KMeans.cluster (Sources/MetalANNSCore/KMeans.swift:
// 53-254).  Its k-means++ seeding (:256-328) draws from Swift's random
// number API and stays with the caller; the Lloyd loop from those seeds is
// deterministic and is reproduced here bit for bit:
//
//   assignment  every row to the centroid of smallest SIMDDistance, strict
//               '<' from FLT_MAX (the first minimum wins) -- the k = 1 search
//               of run_flat_search in SIMDDistance mode, whose (distance,
//               index) minimum is the same choice;
//   stop        before the update when no row changed cluster;
//   update      sum * (1 / count) per non-empty cluster.  The reference splits
//               the rows into `workers` chunks of ceil(n / workers) rows when
//               workers > 1, n >= 512 and k >= 8 (useParallelLloyd); each
//               chunk sums its rows per cluster from 0 in row order, and the
//               chunk sums are added to the cluster total in chunk order.
//               Here a stable radix sort groups the rows by (chunk, cluster)
//               in row order, and one thread per (cluster, dimension) adds
//               exactly those terms in exactly that order, in fp32.
//
// The number of workers is the reference machine's core count
// (ProcessInfo.activeProcessorCount): it changes the summation order, so the
// caller passes the count whose result it wants to reproduce.

#include <cub/cub.cuh>

#include <algorithm>
#include <vector>

#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"

namespace mans {
namespace {

// New assignment per row, whether any row changed, and each row's
// (chunk, cluster) key with its segment size.
__global__ void lloyd_mark_kernel(const uint32_t* __restrict__ best, int32_t* __restrict__ assign,
                                  int64_t n, int64_t chunk, int32_t k,
                                  uint32_t* __restrict__ keys, uint32_t* __restrict__ rows,
                                  int32_t* __restrict__ seg_counts, int* __restrict__ changed) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t b = static_cast<int32_t>(best[i]);
  if (assign[i] != b) *changed = 1;
  assign[i] = b;
  const uint32_t key = static_cast<uint32_t>((i / chunk) * k + b);
  keys[i] = key;
  rows[i] = static_cast<uint32_t>(i);
  atomicAdd(&seg_counts[key], 1);
}

// Block c, threads over the dimensions: the new centroid c.  Empty chunks add
// nothing (a running sum that starts at +0 is never -0, so adding a chunk's
// +0 leaves it unchanged, as in the reference).
__global__ void lloyd_update_kernel(const float* __restrict__ x, int64_t dim,
                                    const uint32_t* __restrict__ rows,
                                    const int32_t* __restrict__ seg_start,
                                    const int32_t* __restrict__ seg_counts, int64_t chunks,
                                    int32_t k, float* __restrict__ cent, int64_t ld) {
  const int32_t c = blockIdx.x;
  int64_t count = 0;
  for (int64_t w = 0; w < chunks; ++w) count += seg_counts[w * k + c];
  if (count == 0) return;  // the stale centroid stays (KMeans.swift:236-243)
  const float scale = __fdiv_rn(1.0f, __ll2float_rn(count));
  for (int64_t d = threadIdx.x; d < dim; d += blockDim.x) {
    float total = 0.0f;
    for (int64_t w = 0; w < chunks; ++w) {
      const int32_t s = seg_start[w * k + c];
      const int32_t e = s + seg_counts[w * k + c];
      if (s == e) continue;
      float part = 0.0f;
      for (int32_t j = s; j < e; ++j) part = __fadd_rn(part, x[static_cast<int64_t>(rows[j]) * dim + d]);
      total = __fadd_rn(total, part);
    }
    cent[static_cast<int64_t>(c) * ld + d] = __fmul_rn(total, scale);
  }
}

struct LloydBuffers {
  uint32_t *best = nullptr, *keys = nullptr, *keys_sorted = nullptr, *rows = nullptr,
           *rows_sorted = nullptr;
  float* dist = nullptr;
  int32_t *cnt = nullptr, *assign = nullptr, *seg_counts = nullptr, *seg_start = nullptr;
  int* changed = nullptr;
  void* tmp = nullptr;
  size_t tmp_bytes = 0;
  ~LloydBuffers() {
    for (void* p : {static_cast<void*>(best), static_cast<void*>(keys),
                    static_cast<void*>(keys_sorted), static_cast<void*>(rows),
                    static_cast<void*>(rows_sorted), static_cast<void*>(dist),
                    static_cast<void*>(cnt), static_cast<void*>(assign),
                    static_cast<void*>(seg_counts), static_cast<void*>(seg_start),
                    static_cast<void*>(changed), tmp})
      if (p) cudaFree(p);
  }
};

// Lloyd iterations over the n x dim rows at d_x (device, contiguous); the
// centroids (host, k x dim) are read and overwritten.
int32_t lloyd_device(mans_ctx* ctx, mans_workspace* ws, const float* d_x, int64_t n, int64_t dim,
                     int32_t k, int32_t max_iter, int32_t metric, int32_t workers,
                     float* h_centroids, int32_t* h_assign, int32_t* h_updates) {
  int64_t w = std::max<int64_t>(1, workers);
  w = std::min<int64_t>(w, n);
  if (!(w > 1 && n >= 512 && k >= 8)) w = 1;  // KMeans.swift:89-90
  const int64_t chunk = (n + w - 1) / w;
  const int64_t chunks = (n + chunk - 1) / chunk;
  const int64_t nseg = chunks * k;
  if (nseg > static_cast<int64_t>(UINT32_MAX) / 2)
    return fail(MANS_ERR_INVALID, "too many (worker, cluster) pairs");
  cudaStream_t st = ws->stream;
  mans_corpus* cc = nullptr;
  int32_t rc = corpus_upload(ctx, h_centroids, k, dim, 0, &cc);
  if (rc != MANS_OK) return rc;
  LloydBuffers b;
  auto ck = [&](cudaError_t x, const char* what) {
    if (rc == MANS_OK && x != cudaSuccess) rc = fail_cuda(x, what);
  };
  ck(cudaMalloc(&b.best, n * sizeof(uint32_t)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.keys, n * sizeof(uint32_t)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.keys_sorted, n * sizeof(uint32_t)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.rows, n * sizeof(uint32_t)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.rows_sorted, n * sizeof(uint32_t)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.dist, n * sizeof(float)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.cnt, n * sizeof(int32_t)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.assign, n * sizeof(int32_t)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.seg_counts, nseg * sizeof(int32_t)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.seg_start, nseg * sizeof(int32_t)), "cudaMalloc(kmeans)");
  ck(cudaMalloc(&b.changed, sizeof(int)), "cudaMalloc(kmeans)");
  int bits = 1;
  while ((int64_t{1} << bits) < nseg) ++bits;
  if (rc == MANS_OK) {
    size_t sort_bytes = 0, scan_bytes = 0;
    ck(cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, b.keys, b.keys_sorted, b.rows,
                                       b.rows_sorted, static_cast<int>(n), 0, bits, st),
       "radix sort size");
    ck(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, b.seg_counts, b.seg_start,
                                     static_cast<int>(nseg), st),
       "scan size");
    b.tmp_bytes = std::max(sort_bytes, scan_bytes);
    ck(cudaMalloc(&b.tmp, b.tmp_bytes), "cudaMalloc(kmeans)");
  }
  // assignments start at -1, so the first pass always counts as a change
  ck(cudaMemsetAsync(b.assign, 0xFF, n * sizeof(int32_t), st), "assignment init");
  int32_t updates = 0;
  const unsigned grid = static_cast<unsigned>((n + 255) / 256);
  const int threads = static_cast<int>(std::min<int64_t>(256, (dim + 31) / 32 * 32));
  for (int32_t it = 0; rc == MANS_OK && it < max_iter; ++it) {
    ck(cudaMemsetAsync(b.changed, 0, sizeof(int), st), "flag clear");
    ck(cudaMemsetAsync(b.seg_counts, 0, nseg * sizeof(int32_t), st), "segment clear");
    if (rc == MANS_OK)
      rc = run_flat_search(ctx, cc, ws, d_x, n, 1, metric, b.dist, b.best, b.cnt, st, kModeSimd,
                           512);
    if (rc != MANS_OK) break;
    lloyd_mark_kernel<<<grid, 256, 0, st>>>(b.best, b.assign, n, chunk, k, b.keys, b.rows,
                                            b.seg_counts, b.changed);
    ck(cudaGetLastError(), "assignment marks");
    int changed = 0;
    ck(cudaMemcpyAsync(&changed, b.changed, sizeof(int), cudaMemcpyDeviceToHost, st),
       "flag readback");
    ck(cudaStreamSynchronize(st), "kmeans assignment");
    if (rc != MANS_OK || !changed) break;
    size_t tb = b.tmp_bytes;
    ck(cub::DeviceRadixSort::SortPairs(b.tmp, tb, b.keys, b.keys_sorted, b.rows, b.rows_sorted,
                                       static_cast<int>(n), 0, bits, st),
       "radix sort");
    tb = b.tmp_bytes;
    ck(cub::DeviceScan::ExclusiveSum(b.tmp, tb, b.seg_counts, b.seg_start,
                                     static_cast<int>(nseg), st),
       "segment offsets");
    if (rc != MANS_OK) break;
    lloyd_update_kernel<<<static_cast<unsigned>(k), threads, 0, st>>>(
        d_x, dim, b.rows_sorted, b.seg_start, b.seg_counts, chunks, k, cc->rows, cc->ld);
    ck(cudaGetLastError(), "centroid update");
    ck(launch_row_norms(cc->rows, k, static_cast<int32_t>(dim), cc->ld, cc->norms, st),
       "centroid norms");
    ++updates;
  }
  if (rc == MANS_OK)
    ck(cudaMemcpy2DAsync(h_centroids, dim * sizeof(float), cc->rows, cc->ld * sizeof(float),
                         dim * sizeof(float), k, cudaMemcpyDeviceToHost, st),
       "centroids download");
  if (rc == MANS_OK && h_assign)
    ck(cudaMemcpyAsync(h_assign, b.assign, n * sizeof(int32_t), cudaMemcpyDeviceToHost, st),
       "assignments download");
  if (rc == MANS_OK) ck(cudaStreamSynchronize(st), "kmeans");
  if (rc == MANS_OK) rc = check_device_error(ws, st);
  cudaStreamSynchronize(st);
  corpus_free(cc);
  if (rc == MANS_OK && h_updates) *h_updates = updates;
  return rc;
}

int32_t validate_lloyd(const mans_ctx* ctx, int64_t n, int64_t dim, int32_t k, int32_t max_iter,
                       int32_t metric) {
  if (!ctx) return fail(MANS_ERR_INVALID, "null context");
  if (int32_t r = reject_group(ctx, nullptr, "k-means")) return r;
  if (n <= 0) return fail(MANS_ERR_INVALID, "Cannot cluster empty vectors");
  if (k <= 0 || k > n) return fail(MANS_ERR_INVALID, "k must be between 1 and vector count");
  if (dim <= 0) return fail(MANS_ERR_DIM, "dimensionMismatch(expected: 1, got: 0)");
  if (max_iter < 0) return fail(MANS_ERR_INVALID, "negative iteration count");
  if (metric < 0 || metric > 2) return fail(MANS_ERR_SEARCH, "k-means needs cosine, l2 or ip");
  if (n > static_cast<int64_t>(INT32_MAX)) return fail(MANS_ERR_INVALID, "too many vectors");
  return MANS_OK;
}

}  // namespace
}  // namespace mans

extern "C" {

int32_t mans_kmeans_lloyd(mans_ctx* ctx, const float* vectors, int64_t n, int64_t row_stride,
                          int64_t offset, int64_t dim, int32_t k, int32_t max_iterations,
                          int32_t metric, int32_t workers, float* centroids,
                          int32_t* out_assignments, int32_t* out_iterations) {
  using namespace mans;
  int32_t rc = validate_lloyd(ctx, n, dim, k, max_iterations, metric);
  if (rc != MANS_OK) return rc;
  if (!vectors || !centroids) return fail(MANS_ERR_INVALID, "null vectors or centroids");
  if (offset < 0 || row_stride < offset + dim)
    return fail(MANS_ERR_DIM, "dimensionMismatch: rows shorter than offset + dim");
  DeviceGuard g(ctx->device);
  mans_workspace* ws = acquire_workspace(ctx);
  if (!ws) return fail(MANS_ERR_OOM, "no workspace stream");
  float* d_x = nullptr;
  cudaError_t e = cudaMalloc(&d_x, n * dim * sizeof(float));
  if (e == cudaSuccess)
    e = cudaMemcpy2DAsync(d_x, dim * sizeof(float), vectors + offset, row_stride * sizeof(float),
                          dim * sizeof(float), n, cudaMemcpyHostToDevice, ws->stream);
  if (e != cudaSuccess) {
    rc = fail_cuda(e, "k-means upload");
  } else {
    rc = lloyd_device(ctx, ws, d_x, n, dim, k, max_iterations, metric, workers, centroids,
                      out_assignments, out_iterations);
  }
  cudaStreamSynchronize(ws->stream);
  if (d_x) cudaFree(d_x);
  release_workspace(ctx, ws);
  return rc;
}

int32_t mans_pq_train(mans_ctx* ctx, const float* vectors, int64_t n, int64_t dim, int32_t m,
                      int32_t ks, int32_t max_iterations, int32_t workers, float* codebooks) {
  using namespace mans;
  if (!ctx || !vectors || !codebooks) return fail(MANS_ERR_INVALID, "null context or buffer");
  if (n <= 0) return fail(MANS_ERR_INVALID, "Cannot train ProductQuantizer with empty vectors");
  if (m <= 0) return fail(MANS_ERR_INVALID, "numSubspaces must be greater than zero");
  if (ks != 256) return fail(MANS_ERR_INVALID, "ProductQuantizer requires centroidsPerSubspace == 256");
  if (dim <= 0) return fail(MANS_ERR_DIM, "dimensionMismatch(expected: 1, got: 0)");
  if (n < ks) return fail(MANS_ERR_INVALID, "Need at least 256 vectors to train ProductQuantizer");
  if (dim % m != 0)
    return fail(MANS_ERR_INVALID, "Vector dimension must be divisible by numSubspaces");
  const int64_t sub = dim / m;
  int32_t rc = validate_lloyd(ctx, n, sub, ks, max_iterations, MANS_METRIC_L2);
  if (rc != MANS_OK) return rc;
  DeviceGuard g(ctx->device);
  mans_workspace* ws = acquire_workspace(ctx);
  if (!ws) return fail(MANS_ERR_OOM, "no workspace stream");
  float *d_all = nullptr, *d_x = nullptr;
  cudaError_t e = cudaMalloc(&d_all, n * dim * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&d_x, n * sub * sizeof(float));
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(d_all, vectors, n * dim * sizeof(float), cudaMemcpyHostToDevice,
                        ws->stream);
  if (e != cudaSuccess) rc = fail_cuda(e, "PQ training upload");
  // ProductQuantizer.train runs the subspaces concurrently, each independent
  // of the others; here they run one after another on the device.
  for (int32_t s = 0; rc == MANS_OK && s < m; ++s) {
    e = cudaMemcpy2DAsync(d_x, sub * sizeof(float), d_all + s * sub, dim * sizeof(float),
                          sub * sizeof(float), n, cudaMemcpyDeviceToDevice, ws->stream);
    if (e != cudaSuccess) {
      rc = fail_cuda(e, "subspace gather");
      break;
    }
    rc = lloyd_device(ctx, ws, d_x, n, sub, ks, max_iterations, MANS_METRIC_L2, workers,
                      codebooks + static_cast<int64_t>(s) * ks * sub, nullptr, nullptr);
  }
  cudaStreamSynchronize(ws->stream);
  if (d_all) cudaFree(d_all);
  if (d_x) cudaFree(d_x);
  release_workspace(ctx, ws);
  return rc;
}

}  // extern "C"
