// capi.cu -- the C ABI of include/mans_cuda.h: contexts, corpora, workspaces
// and the host orchestration of the flat exact search.
//
// The orchestration restates FlatGPUSearch.batchSearch's contract
// (Sources/MetalANNSCore/FlatGPUSearch.swift:103-181): empty query list ->
// nothing; k <= 0 or an empty corpus -> empty results; metric hamming ->
// searchFailed; a query of the wrong width -> dimensionMismatch; effective k =
// min(k, 256, n).  Device work replaces runChunk + selectTopK.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"

using namespace mans;

namespace mans {

thread_local std::string g_last_error;

int32_t fail(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int32_t fail_cuda(cudaError_t e, const char* what) {
  std::string msg = std::string(what) + ": " + cudaGetErrorString(e);
  if (e == cudaErrorMemoryAllocation) return fail(MANS_ERR_OOM, msg);
  return fail(MANS_ERR_EXEC, msg);
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

int32_t encode_row_map(CUtensorMap* map, const float* base, int64_t rows, int64_t dim,
                       int64_t ld, int box_rows) {
  auto enc = encoder();
  if (!enc) return fail(MANS_ERR_PIPELINE, "cuTensorMapEncodeTiled is unavailable");
  if (rows <= 0) rows = 1;
  cuuint64_t gdim[2] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(rows)};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(ld) * 4};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileCols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), gdim,
                   gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MANS_ERR_PIPELINE, "cuTensorMapEncodeTiled failed");
  return MANS_OK;
}

int32_t DeviceBuffer::reserve(size_t need) {
  if (need <= bytes) return MANS_OK;
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  bytes = 0;
  size_t want = std::max<size_t>(need, 256);
  cudaError_t e = cudaMalloc(&ptr, want);
  if (e != cudaSuccess) {
    ptr = nullptr;
    return fail_cuda(e, "cudaMalloc(workspace)");
  }
  bytes = want;
  return MANS_OK;
}

void DeviceBuffer::release() {
  if (ptr) cudaFree(ptr);
  ptr = nullptr;
  bytes = 0;
}

int32_t PinnedBuffer::reserve(size_t need) {
  if (need <= bytes) return MANS_OK;
  if (ptr) cudaFreeHost(ptr);
  ptr = nullptr;
  bytes = 0;
  size_t want = std::max<size_t>(need, 4096);
  cudaError_t e = cudaMallocHost(&ptr, want);
  if (e != cudaSuccess) {
    ptr = nullptr;
    return fail_cuda(e, "cudaMallocHost(workspace)");
  }
  bytes = want;
  return MANS_OK;
}

void PinnedBuffer::release() {
  if (ptr) cudaFreeHost(ptr);
  ptr = nullptr;
  bytes = 0;
}

DeviceGuard::DeviceGuard(int dev) {
  cudaGetDevice(&prev);
  if (prev != dev) cudaSetDevice(dev);
  cur = dev;
}
DeviceGuard::~DeviceGuard() {
  if (prev != cur) cudaSetDevice(prev);
}

mans_workspace* acquire_workspace(mans_ctx* ctx) {
  {
    std::lock_guard<std::mutex> lk(ctx->mu);
    if (!ctx->pool.empty()) {
      mans_workspace* ws = ctx->pool.back();
      ctx->pool.pop_back();
      return ws;
    }
  }
  mans_workspace* ws = new mans_workspace();
  ws->ctx = ctx;
  if (cudaStreamCreateWithFlags(&ws->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete ws;
    return nullptr;
  }
  ws->own_stream = true;
  return ws;
}

void release_workspace(mans_ctx* ctx, mans_workspace* ws) {
  std::lock_guard<std::mutex> lk(ctx->mu);
  ctx->pool.push_back(ws);
}

void destroy_workspace(mans_workspace* ws) {
  DeviceGuard g(ws->ctx->device);
  ws->err.release();
  ws->qnorms.release();
  ws->slot_keys.release();
  ws->slot_counts.release();
  ws->queries.release();
  ws->out_dist.release();
  ws->out_ids.release();
  ws->out_counts.release();
  ws->aux.release();
  ws->aux2.release();
  ws->tc_aux.release();
  ws->small_scores.release();
  ws->tc_bar.release();
  ws->probe_sync.release();
  ws->gather.release();
  ws->h_err.release();
  ws->io.release();
  ws->big.release();
  ws->h_io.release();
  if (ws->done) cudaEventDestroy(ws->done);
  for (auto& pr : ws->events) {
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  for (auto& pr : ws->stage_events) {
    cudaEventDestroy(pr.first);
    cudaEventDestroy(pr.second);
  }
  if (ws->own_stream && ws->stream) cudaStreamDestroy(ws->stream);
  delete ws;
}

// Records a start event before the dominant kernel when timing is enabled;
// returns the matching stop event (or null).
cudaEvent_t timing_begin(mans_workspace* ws, cudaStream_t stream) {
  if (!ws->timing || ws->timing_hold > 0) return nullptr;
  if (ws->events_used == ws->events.size()) {
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess) return nullptr;
    if (cudaEventCreate(&b) != cudaSuccess) {
      cudaEventDestroy(a);
      return nullptr;
    }
    ws->events.emplace_back(a, b);
  }
  auto& pr = ws->events[ws->events_used++];
  cudaEventRecord(pr.first, stream);
  return pr.second;
}

void timing_end(cudaEvent_t stop, cudaStream_t stream) {
  if (stop) cudaEventRecord(stop, stream);
}

cudaEvent_t stage_begin(mans_workspace* ws, cudaStream_t stream, int stage) {
  if (!ws || !ws->stage_timing || ws->timing_hold > 0) return nullptr;
  if (ws->stage_used == ws->stage_events.size()) {
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess) return nullptr;
    if (cudaEventCreate(&b) != cudaSuccess) {
      cudaEventDestroy(a);
      return nullptr;
    }
    ws->stage_events.emplace_back(a, b);
    ws->stage_of.push_back(0);
  }
  const size_t i = ws->stage_used++;
  ws->stage_of[i] = stage;
  cudaEventRecord(ws->stage_events[i].first, stream);
  return ws->stage_events[i].second;
}

int pow2_at_least(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

// Query-group width for a batch: the smallest power of two >= nq, at most 8.
int choose_qb(int64_t nq) {
  if (nq <= 1) return 1;
  if (nq <= 2) return 2;
  if (nq <= 4) return 4;
  return 8;
}

int32_t run_flat_search(mans_ctx* ctx, const mans_corpus* corpus, mans_workspace* ws,
                        const float* d_queries, int64_t nq, int32_t k, int32_t metric,
                        float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                        cudaStream_t stream, int mode, int32_t kcap, bool centroid_scan) {
  const int32_t kout = std::min<int32_t>(k, kcap);
  const int64_t n = corpus->n;
  if (nq <= 0) return MANS_OK;
  if (centroid_scan && k > 0 && small_batch_applies(corpus, nq)) {
    ws->last_path = 0;
    return run_small_batch_search(ctx, corpus, ws, d_queries, nq, kout, metric, d_out_dist,
                                  d_out_ids, d_out_counts, stream, mode);
  }
  // Tensor-core path: batches of at least tc_min_batch queries, and any batch
  // over a corpus of at least 2^25 elements (87k rows at d = 384): there the
  // bf16 pass over half the bytes, fused with its sampling, plus prep and
  // re-rank (~35 us) beats the fp32 scan, whose short shards also leave
  // SMs idle.
  const bool tc_size = nq >= ctx->tc_min_batch || n * corpus->dim >= (int64_t{1} << 25);
  ws->last_path = 0;
  if (mode == kModeHost && kcap == MANS_MAX_TOPK && ctx->tc_min_batch > 0 && tc_size && k > 0 &&
      n > 0 && !corpus->ids) {
    mans_corpus* c = const_cast<mans_corpus*>(corpus);
    const bool i8 = tc_use_int8(ctx, nq);
    std::unique_lock<std::mutex> lk(c->tc_mu);
    int32_t rc = tc_prepare_corpus(c, metric, i8);
    lk.unlock();
    if (rc != MANS_OK) return rc;
    if (tc_applicable(c, metric, i8))
      return run_flat_search_tc(ctx, c, ws, d_queries, nq, k, metric, d_out_dist, d_out_ids,
                                d_out_counts, stream, i8);
  }
  if (k <= 0 || n <= 0) {
    if (kout <= 0) {
      cudaError_t e = cudaMemsetAsync(d_out_counts, 0, sizeof(int32_t) * nq, stream);
      return e == cudaSuccess ? MANS_OK : fail_cuda(e, "cudaMemsetAsync");
    }
    cudaError_t e = launch_fill_empty(d_out_dist, d_out_ids, d_out_counts, nq, kout, stream);
    return e == cudaSuccess ? MANS_OK : fail_cuda(e, "fill_empty launch");
  }
  if (small_batch_applies(corpus, nq))
    return run_small_batch_search(ctx, corpus, ws, d_queries, nq, kout, metric, d_out_dist,
                                  d_out_ids, d_out_counts, stream, mode);
  const int32_t keff = static_cast<int32_t>(std::min<int64_t>(kout, n));
  const int32_t kp = pow2_at_least(keff);
  const int qb = choose_qb(nq);
  const int64_t groups = (nq + qb - 1) / qb;
  // a scan that would leave most SMs idle with 256-row tiles uses 64-row ones
  const int tile_rows =
      groups * ((n + kTileRows - 1) / kTileRows) * 2 <= ctx->num_sms ? kSmallTileRows : kTileRows;
  const int64_t tiles = (n + tile_rows - 1) / tile_rows;
  int64_t splits = std::max<int64_t>(1, ctx->num_sms / std::max<int64_t>(groups, 1));
  splits = std::min<int64_t>(splits, tiles);
  const int64_t nseg = groups * splits;
  if (nseg > INT32_MAX / 2) return fail(MANS_ERR_SEARCH, "query batch too large");
  const int nchunks = static_cast<int>((corpus->dim + kTileCols - 1) / kTileCols);
  const int stages = scan_max_stages(qb, nchunks);
  if (stages < 2) return fail(MANS_ERR_SEARCH, "dimension too large for the flat scan kernel");

  int32_t rc;
  const size_t nslots = static_cast<size_t>(groups) * qb * splits;
  if ((rc = ws->slot_keys.reserve(nslots * kp * sizeof(uint64_t))) != MANS_OK) return rc;
  if ((rc = ws->slot_counts.reserve(nslots * sizeof(int32_t))) != MANS_OK) return rc;
  if ((rc = ws->err.reserve(sizeof(int))) != MANS_OK) return rc;
  float* qn = nullptr;  // query norms are computed inside the scan kernel
  if (!ws->err_cleared) {
    cudaError_t e = cudaMemsetAsync(ws->err.ptr, 0, sizeof(int), stream);
    if (e != cudaSuccess) return fail_cuda(e, "cudaMemsetAsync(err)");
    ws->err_cleared = true;
  }

  ScanParams p{};
  p.segs = nullptr;
  p.nseg = static_cast<int32_t>(nseg);
  p.stages = stages;
  p.flat_splits = static_cast<int32_t>(splits);
  p.flat_tiles = static_cast<int32_t>(tiles);
  p.tile_rows = tile_rows;
  p.n = n;
  p.nq = nq;
  p.queries = d_queries;
  p.qidx = nullptr;
  p.qnorms = qn;
  p.norms = (metric == MANS_METRIC_IP) ? nullptr : corpus->norms;
  p.ids = corpus->ids;
  p.id_offset = corpus->id_offset;
  p.dim = static_cast<int32_t>(corpus->dim);
  p.nchunks = nchunks;
  p.metric = metric;
  p.mode = mode;
  p.k = keff;
  p.kp = kp;
  p.slot_keys = static_cast<uint64_t*>(ws->slot_keys.ptr);
  p.slot_counts = static_cast<int32_t*>(ws->slot_counts.ptr);
  p.err = static_cast<int*>(ws->err.ptr);
  int grid = static_cast<int>(std::min<int64_t>(nseg, ctx->num_sms));
  cudaEvent_t st_stop = stage_begin(ws, stream, MANS_STAGE_PASS);
  cudaEvent_t ev_stop = timing_begin(ws, stream);
  cudaError_t e =
      launch_scan(qb, tile_rows == kTileRows ? corpus->map : corpus->map_small, p, grid, stream);
  if (e != cudaSuccess) return fail_cuda(e, "scan launch");
  timing_end(ev_stop, stream);
  timing_end(st_stop, stream);
  ws->launches += (qn ? 1 : 0) + 2;

  MergeParams m{};
  m.in_keys = p.slot_keys;
  m.in_counts = p.slot_counts;
  m.q_slot_offsets = nullptr;
  m.slots_per_query = static_cast<int32_t>(splits);
  m.kp_in = kp;
  m.nq = nq;
  m.k = keff;
  m.kp = kp;
  m.kout = kout;
  m.out_dist = d_out_dist;
  m.out_ids = d_out_ids;
  m.out_counts = d_out_counts;
  m.err = p.err;
  st_stop = stage_begin(ws, stream, MANS_STAGE_MERGE);
  e = launch_merge(m, stream);
  if (e != cudaSuccess) return fail_cuda(e, "merge launch");
  timing_end(st_stop, stream);
  return MANS_OK;
}

int32_t corpus_upload(mans_ctx* ctx, const float* rows, int64_t n, int64_t dim, uint32_t id_offset,
                      mans_corpus** out, int64_t src_ld) {
  if (src_ld <= 0) src_ld = dim;
  if (n < 0 || dim <= 0) return fail(MANS_ERR_INVALID, "corpus needs n >= 0 and dim > 0");
  if (n > 0 && !rows) return fail(MANS_ERR_INVALID, "rows is null");
  if (n > static_cast<int64_t>(INT32_MAX)) return fail(MANS_ERR_INVALID, "corpus too large");
  DeviceGuard g(ctx->device);
  mans_corpus* c = new mans_corpus();
  c->ctx = ctx;
  c->n = n;
  c->dim = dim;
  c->ld = (dim + 3) / 4 * 4;  // 16-byte row pitch, required by TMA
  c->id_offset = id_offset;
  size_t rows_bytes = static_cast<size_t>(std::max<int64_t>(n, 1)) * c->ld * sizeof(float);
  cudaError_t e = cudaMalloc(&c->rows, rows_bytes);
  if (e != cudaSuccess) {
    delete c;
    return fail_cuda(e, "cudaMalloc(corpus)");
  }
  // rounded up to 64 floats: the tensor-core pass bulk-copies whole 16-byte
  // pieces of the last tile's norms
  e = cudaMalloc(&c->norms, static_cast<size_t>((std::max<int64_t>(n, 1) + 63) / 64 * 64) *
                                sizeof(float));
  if (e != cudaSuccess) {
    cudaFree(c->rows);
    delete c;
    return fail_cuda(e, "cudaMalloc(norms)");
  }
  if (n > 0) {
    if (c->ld != dim) cudaMemset(c->rows, 0, rows_bytes);
    // host or device source (unified addressing tells them apart)
    e = cudaMemcpy2D(c->rows, c->ld * sizeof(float), rows, src_ld * sizeof(float),
                     dim * sizeof(float), n, cudaMemcpyDefault);
    if (e == cudaSuccess)
      e = launch_row_norms(c->rows, n, static_cast<int32_t>(dim), c->ld, c->norms, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      corpus_free(c);
      return fail_cuda(e, "corpus upload");
    }
  }
  int32_t rc = encode_row_map(&c->map, c->rows, n, dim, c->ld);
  if (rc == MANS_OK) rc = encode_row_map(&c->map_small, c->rows, n, dim, c->ld, kSmallTileRows);
  if (rc == MANS_OK) rc = encode_row_map(&c->map_seg, c->rows, n, dim, c->ld, 32);
  if (rc != MANS_OK) {
    corpus_free(c);
    return rc;
  }
  *out = c;
  return MANS_OK;
}

void corpus_free(mans_corpus* c) {
  if (!c) return;
  tc_free_corpus(c);
  if (c->owned) {
    if (c->rows) cudaFree(c->rows);
    if (c->norms) cudaFree(c->norms);
    if (c->ids) cudaFree(c->ids);
  }
  delete c;
}

// Reads and clears the device error word of `ws` after its stream finished.
int32_t check_device_error(mans_workspace* ws, cudaStream_t stream) {
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return fail_cuda(e, "stream synchronize");
  if (!ws->err.ptr || !ws->err_cleared) return MANS_OK;
  int h = 0;
  e = cudaMemcpy(&h, ws->err.ptr, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail_cuda(e, "error word readback");
  return h != 0 ? device_error(ws, h) : MANS_OK;
}

// After a non-zero device error word `h` (stream idle): the next search
// clears the word, and the grid-barrier counters a kernel that gave up may
// have left out of step start again from zero.
int32_t device_error(mans_workspace* ws, int h) {
  ws->err_cleared = false;
  if (ws->tc_bar.ptr) {
    cudaMemset(ws->tc_bar.ptr, 0, sizeof(unsigned long long));
    ws->tc_bar_base = 0;
  }
  if (ws->probe_sync.ptr) {
    cudaMemset(ws->probe_sync.ptr, 0, kProbeSyncBytes);
    ws->probe_bar_base = 0;
  }
  return fail(MANS_ERR_EXEC, h == kErrTimeout ? "device wait timed out"
                                               : "device kernel reported an error");
}

static size_t carve_io(size_t& o, size_t bytes) {
  size_t at = (o + 255) / 256 * 256;
  o = at + bytes;
  return at;
}

int32_t host_buffer_search(mans_workspace* ws, const float* queries, int64_t nq, int64_t dim,
                           int32_t kout, float* out_dist, uint32_t* out_ids, int32_t* out_counts,
                           const DeviceSearch& search) {
  cudaStream_t st = ws->stream;
  const size_t qb = static_cast<size_t>(nq) * dim * sizeof(float);
  const size_t rb = static_cast<size_t>(nq) * kout * sizeof(float);
  const size_t cb = static_cast<size_t>(nq) * sizeof(int32_t);
  size_t o = 0;
  const size_t o_q = carve_io(o, qb);
  const size_t o_d = carve_io(o, rb);
  const size_t o_i = carve_io(o, rb);
  const size_t o_c = carve_io(o, cb);
  const size_t res_end = o;
  const size_t o_e = carve_io(o, sizeof(int));
  int32_t rc;
  if ((rc = ws->io.reserve(o)) != MANS_OK) return rc;
  if ((rc = ws->h_io.reserve(o)) != MANS_OK) return rc;
  uint8_t* d = static_cast<uint8_t*>(ws->io.ptr);
  uint8_t* h = static_cast<uint8_t*>(ws->h_io.ptr);
  std::memcpy(h + o_q, queries, qb);
  cudaError_t e = cudaMemcpyAsync(d + o_q, h + o_q, qb, cudaMemcpyHostToDevice, st);
  if (e != cudaSuccess) return fail_cuda(e, "query upload");
  rc = search(reinterpret_cast<const float*>(d + o_q), reinterpret_cast<float*>(d + o_d),
              reinterpret_cast<uint32_t*>(d + o_i), reinterpret_cast<int32_t*>(d + o_c), st);
  if (rc != MANS_OK) {
    cudaStreamSynchronize(st);
    return rc;
  }
  e = cudaMemcpyAsync(h + o_d, d + o_d, res_end - o_d, cudaMemcpyDeviceToHost, st);
  const bool word = ws->err.ptr && ws->err_cleared;
  if (e == cudaSuccess && word)
    e = cudaMemcpyAsync(h + o_e, ws->err.ptr, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e != cudaSuccess) {
    cudaStreamSynchronize(st);
    return fail_cuda(e, "result download");
  }
  e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail_cuda(e, "stream synchronize");
  if (word) {
    const int herr = *reinterpret_cast<const int*>(h + o_e);
    if (herr != 0) return device_error(ws, herr);
  }
  std::memcpy(out_dist, h + o_d, rb);
  std::memcpy(out_ids, h + o_i, rb);
  std::memcpy(out_counts, h + o_c, cb);
  return MANS_OK;
}

}  // namespace mans

// ============================================================================
// C ABI
// ============================================================================

extern "C" {

int32_t mans_last_error_message(char* buf, size_t buf_len) {
  if (!buf || buf_len == 0) return MANS_ERR_INVALID;
  size_t n = std::min(buf_len - 1, g_last_error.size());
  std::memcpy(buf, g_last_error.data(), n);
  buf[n] = '\0';
  return MANS_OK;
}

int32_t mans_ctx_create(int32_t device, mans_ctx** out_ctx) {
  if (!out_ctx) return fail(MANS_ERR_INVALID, "out_ctx is null");
  *out_ctx = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count)
    return fail(MANS_ERR_DEVICE, "no CUDA device with that index");
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
    return fail(MANS_ERR_DEVICE, "cudaGetDeviceProperties failed");
  if (prop.major != 10) return fail(MANS_ERR_DEVICE, "device is not an sm_100 (Blackwell) GPU");
  DeviceGuard g(device);
  cudaError_t e = scan_configure(static_cast<int>(prop.sharedMemPerBlockOptin));
  if (e != cudaSuccess) return fail_cuda(e, "kernel configuration");
  if (!encoder()) return fail(MANS_ERR_PIPELINE, "cuTensorMapEncodeTiled is unavailable");
  mans_ctx* ctx = new mans_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  ctx->max_smem = static_cast<int>(prop.sharedMemPerBlockOptin);
  ctx->coop_launch = prop.cooperativeLaunch != 0;
  *out_ctx = ctx;
  return MANS_OK;
}

int32_t mans_ctx_destroy(mans_ctx* ctx) {
  if (!ctx) return MANS_OK;
  if (is_group(ctx)) {
    for (mans_ctx* m : ctx->members) mans_ctx_destroy(m);
    delete ctx;
    return MANS_OK;
  }
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  for (mans_workspace* ws : ctx->pool) destroy_workspace(ws);
  ctx->pool.clear();
  delete ctx;
  return MANS_OK;
}

int32_t mans_ctx_sm_count(const mans_ctx* ctx) { return ctx ? ctx->num_sms : 0; }

int32_t mans_ctx_set_tensor_core_batch(mans_ctx* ctx, int32_t min_batch) {
  if (!ctx) return fail(MANS_ERR_INVALID, "null context");
  if (min_batch < 0) return fail(MANS_ERR_INVALID, "negative batch size");
  ctx->tc_min_batch = min_batch;
  for (mans_ctx* m : ctx->members) m->tc_min_batch = min_batch;
  return MANS_OK;
}

int32_t mans_ctx_set_tensor_core_format(mans_ctx* ctx, int32_t format) {
  if (!ctx) return fail(MANS_ERR_INVALID, "null context");
  if (format < MANS_TC_AUTO || format > MANS_TC_INT8)
    return fail(MANS_ERR_INVALID, "unknown tensor-core operand format");
  ctx->tc_format = format;
  for (mans_ctx* m : ctx->members) m->tc_format = format;
  return MANS_OK;
}

int32_t mans_corpus_int8_codes(mans_corpus* corpus, int8_t* codes, float* scales) {
  if (!corpus || (!codes && !scales)) return fail(MANS_ERR_INVALID, "null corpus or outputs");
  if (is_group(corpus)) {  // the shards' codes in row order
    for (size_t i = 0; i < corpus->shards.size(); ++i) {
      const int64_t r0 = corpus->shard_row0[i];
      int32_t rc = mans_corpus_int8_codes(corpus->shards[i], codes ? codes + r0 * corpus->dim : nullptr,
                                          scales ? scales + r0 : nullptr);
      if (rc != MANS_OK) return rc;
    }
    return MANS_OK;
  }
  std::lock_guard<std::mutex> lk(corpus->tc_mu);
  return tc_export_int8(corpus, codes, scales);
}

int32_t mans_workspace_last_path(mans_workspace* ws, int32_t* out) {
  if (!ws || !out) return fail(MANS_ERR_INVALID, "null workspace or output");
  *out = ws->last_path;
  return MANS_OK;
}

int32_t mans_workspace_fallbacks(mans_workspace* ws, int32_t* out) {
  if (!ws || !out) return fail(MANS_ERR_INVALID, "null workspace or output");
  *out = 0;
  if (!ws->tc_fallbacks) return MANS_OK;
  DeviceGuard g(ws->ctx->device);
  cudaError_t e = cudaMemcpy(out, ws->tc_fallbacks, sizeof(int32_t), cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? MANS_OK : fail_cuda(e, "fallback counter readback");
}

int32_t mans_corpus_create(mans_ctx* ctx, const float* rows, int64_t n, int64_t dim,
                           uint32_t id_offset, mans_corpus** out_corpus) {
  if (!ctx || !out_corpus) return fail(MANS_ERR_INVALID, "null context or output");
  *out_corpus = nullptr;
  return corpus_create_any(ctx, rows, n, dim, id_offset, out_corpus);
}

int32_t mans_corpus_update_rows(mans_corpus* c, int64_t start, const float* rows, int64_t count) {
  if (!c) return fail(MANS_ERR_INVALID, "corpus is null");
  if (start < 0 || count < 0 || start + count > c->n)
    return fail(MANS_ERR_INVALID, "row range outside the corpus");
  if (count == 0) return MANS_OK;
  if (!rows) return fail(MANS_ERR_INVALID, "rows is null");
  if (is_group(c)) {  // each shard overlapping the range takes its part
    for (size_t i = 0; i < c->shards.size(); ++i) {
      const int64_t s0 = std::max(start, c->shard_row0[i]);
      const int64_t s1 = std::min(start + count, c->shard_row0[i + 1]);
      if (s0 >= s1) continue;
      int32_t rc = mans_corpus_update_rows(c->shards[i], s0 - c->shard_row0[i],
                                           rows + (s0 - start) * c->dim, s1 - s0);
      if (rc != MANS_OK) return rc;
    }
    return MANS_OK;
  }
  DeviceGuard g(c->ctx->device);
  {
    std::lock_guard<std::mutex> lk(c->tc_mu);
    cudaDeviceSynchronize();
    tc_free_corpus(c);  // the bf16 copy and its bound terms are rebuilt on next use
  }
  float* dst = c->rows + start * c->ld;
  cudaError_t e = cudaMemcpy2D(dst, c->ld * sizeof(float), rows, c->dim * sizeof(float),
                               c->dim * sizeof(float), count, cudaMemcpyHostToDevice);
  if (e == cudaSuccess)
    e = launch_row_norms(dst, count, static_cast<int32_t>(c->dim), c->ld, c->norms + start, 0);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail_cuda(e, "corpus update");
  return MANS_OK;
}

int32_t mans_corpus_destroy(mans_corpus* c) {
  if (!c) return MANS_OK;
  if (is_group(c)) {
    for (mans_corpus* s : c->shards) mans_corpus_destroy(s);
    delete c;
    return MANS_OK;
  }
  DeviceGuard g(c->ctx->device);
  cudaDeviceSynchronize();
  corpus_free(c);
  return MANS_OK;
}

int64_t mans_corpus_count(const mans_corpus* c) { return c ? c->n : 0; }
int64_t mans_corpus_dim(const mans_corpus* c) { return c ? c->dim : 0; }

int32_t mans_workspace_create(mans_ctx* ctx, mans_workspace** out_ws) {
  if (!ctx || !out_ws) return fail(MANS_ERR_INVALID, "null context or output");
  if (int32_t rc = reject_group(ctx, nullptr, "a workspace")) return rc;
  mans_workspace* ws = new mans_workspace();
  ws->ctx = ctx;
  ws->stream = nullptr;
  ws->own_stream = false;
  *out_ws = ws;
  return MANS_OK;
}

int32_t mans_workspace_destroy(mans_workspace* ws) {
  if (!ws) return MANS_OK;
  {
    DeviceGuard g(ws->ctx->device);
    cudaDeviceSynchronize();
  }
  destroy_workspace(ws);
  return MANS_OK;
}

int32_t mans_workspace_set_timing(mans_workspace* ws, int32_t enable) {
  if (!ws) return fail(MANS_ERR_INVALID, "workspace is null");
  ws->timing = (enable & 1) != 0;
  ws->stage_timing = (enable & 2) != 0;
  ws->events_used = 0;
  ws->stage_used = 0;
  ws->launches = 0;
  return MANS_OK;
}

int32_t mans_workspace_stage_times(mans_workspace* ws, double* stage_ms, int64_t* stage_counts,
                                   int32_t n_stages) {
  if (!ws) return fail(MANS_ERR_INVALID, "workspace is null");
  if (n_stages < 0 || (n_stages > 0 && (!stage_ms || !stage_counts)))
    return fail(MANS_ERR_INVALID, "bad stage arrays");
  DeviceGuard g(ws->ctx->device);
  for (int32_t s = 0; s < n_stages; ++s) {
    stage_ms[s] = 0.0;
    stage_counts[s] = 0;
  }
  for (size_t i = 0; i < ws->stage_used; ++i) {
    float ms = 0.0f;
    cudaError_t e = cudaEventSynchronize(ws->stage_events[i].second);
    if (e == cudaSuccess)
      e = cudaEventElapsedTime(&ms, ws->stage_events[i].first, ws->stage_events[i].second);
    if (e != cudaSuccess) return fail_cuda(e, "stage timing");
    const int s = ws->stage_of[i];
    if (s >= 0 && s < n_stages) {
      stage_ms[s] += ms;
      ++stage_counts[s];
    }
  }
  ws->stage_used = 0;
  return MANS_OK;
}

int32_t mans_workspace_stats(mans_workspace* ws, double* kernel_ms, int64_t* kernel_launches,
                             int64_t* total_launches) {
  if (!ws) return fail(MANS_ERR_INVALID, "workspace is null");
  DeviceGuard g(ws->ctx->device);
  double total = 0.0;
  for (size_t i = 0; i < ws->events_used; ++i) {
    float ms = 0.0f;
    cudaError_t e = cudaEventSynchronize(ws->events[i].second);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, ws->events[i].first, ws->events[i].second);
    if (e != cudaSuccess) return fail_cuda(e, "kernel timing");
    total += ms;
  }
  if (kernel_ms) *kernel_ms = total;
  if (kernel_launches) *kernel_launches = static_cast<int64_t>(ws->events_used);
  if (total_launches) *total_launches = ws->launches;
  ws->events_used = 0;
  ws->launches = 0;
  return MANS_OK;
}

int32_t mans_workspace_check(mans_workspace* ws, void* cuda_stream) {
  if (!ws) return fail(MANS_ERR_INVALID, "workspace is null");
  DeviceGuard g(ws->ctx->device);
  return check_device_error(ws, static_cast<cudaStream_t>(cuda_stream));
}

static int32_t validate_flat(const mans_ctx* ctx, const mans_corpus* corpus, int64_t nq,
                             int32_t metric) {
  if (!ctx || !corpus) return fail(MANS_ERR_INVALID, "null context or corpus");
  if (corpus->ctx != ctx) return fail(MANS_ERR_INVALID, "corpus belongs to another context");
  if (nq < 0) return fail(MANS_ERR_INVALID, "negative query count");
  if (metric == MANS_METRIC_HAMMING)
    return fail(MANS_ERR_SEARCH, "FlatGPUSearch does not support metric .hamming");
  if (metric < 0 || metric > MANS_METRIC_HAMMING) return fail(MANS_ERR_INVALID, "unknown metric");
  return MANS_OK;
}

int32_t mans_flat_search(mans_ctx* ctx, const mans_corpus* corpus, const float* queries,
                         int64_t nq, int64_t dim, int32_t k, int32_t metric, float* out_dist,
                         uint32_t* out_ids, int32_t* out_counts) {
  int32_t rc = validate_flat(ctx, corpus, nq, metric);
  if (rc != MANS_OK) return rc;
  if (nq == 0) return MANS_OK;
  if (k <= 0 || corpus->n <= 0) {
    const int32_t kout = std::max<int32_t>(0, std::min<int32_t>(k, MANS_MAX_TOPK));
    for (int64_t i = 0; i < nq * kout; ++i) {
      out_dist[i] = __builtin_inff();
      out_ids[i] = MANS_EMPTY_ID;
    }
    for (int64_t i = 0; i < nq; ++i) out_counts[i] = 0;
    return MANS_OK;
  }
  if (dim != corpus->dim) {
    char msg[128];
    std::snprintf(msg, sizeof msg, "dimensionMismatch(expected: %lld, got: %lld)",
                  static_cast<long long>(corpus->dim), static_cast<long long>(dim));
    return fail(MANS_ERR_DIM, msg);
  }
  if (!queries || !out_dist || !out_ids || !out_counts)
    return fail(MANS_ERR_INVALID, "null buffer");
  if (is_group(ctx) != is_group(corpus))
    return fail(MANS_ERR_INVALID, "corpus and context disagree on the device group");
  if (is_group(ctx))
    return group_flat_search(ctx, corpus, queries, nq, dim, k, metric, out_dist, out_ids,
                             out_counts);
  DeviceGuard g(ctx->device);
  mans_workspace* ws = acquire_workspace(ctx);
  if (!ws) return fail(MANS_ERR_OOM, "cannot create a workspace stream");
  const int32_t kout = std::min<int32_t>(k, MANS_MAX_TOPK);
  rc = host_buffer_search(ws, queries, nq, dim, kout, out_dist, out_ids, out_counts,
                          [&](const float* dq, float* dd, uint32_t* di, int32_t* dc,
                              cudaStream_t st) {
                            return run_flat_search(ctx, corpus, ws, dq, nq, k, metric, dd, di,
                                                   dc, st);
                          });
  release_workspace(ctx, ws);
  return rc;
}

int32_t mans_flat_search_device(mans_ctx* ctx, const mans_corpus* corpus, mans_workspace* ws,
                                const float* d_queries, int64_t nq, int32_t k, int32_t metric,
                                float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                                void* cuda_stream) {
  int32_t rc = validate_flat(ctx, corpus, nq, metric);
  if (rc != MANS_OK) return rc;
  if ((rc = reject_group(ctx, corpus, "mans_flat_search_device")) != MANS_OK) return rc;
  if (!ws || ws->ctx != ctx) return fail(MANS_ERR_INVALID, "workspace missing or foreign");
  DeviceGuard g(ctx->device);
  return run_flat_search(ctx, corpus, ws, d_queries, nq, k, metric, d_out_dist, d_out_ids,
                         d_out_counts, static_cast<cudaStream_t>(cuda_stream));
}

int32_t mans_topk_merge_device(mans_ctx* ctx, mans_workspace* ws, const float* d_in_dist,
                               const uint32_t* d_in_ids, const int32_t* d_in_counts,
                               int32_t n_lists, int64_t list_stride, int64_t nq, int32_t kin,
                               int32_t k, float* d_out_dist, uint32_t* d_out_ids,
                               int32_t* d_out_counts, void* cuda_stream) {
  if (!ctx || !ws) return fail(MANS_ERR_INVALID, "null context or workspace");
  if (int32_t r = reject_group(ctx, nullptr, "mans_topk_merge_device")) return r;
  if (n_lists < 0 || nq < 0 || kin < 0 || list_stride < 0)
    return fail(MANS_ERR_INVALID, "negative size");
  if (nq == 0) return MANS_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  const int32_t kout = std::min<int32_t>(k, MANS_MAX_TOPK);
  if (k <= 0 || n_lists == 0 || kin == 0) {
    if (kout <= 0) {
      cudaError_t e = cudaMemsetAsync(d_out_counts, 0, sizeof(int32_t) * nq, st);
      return e == cudaSuccess ? MANS_OK : fail_cuda(e, "cudaMemsetAsync");
    }
    cudaError_t e = launch_fill_empty(d_out_dist, d_out_ids, d_out_counts, nq, kout, st);
    return e == cudaSuccess ? MANS_OK : fail_cuda(e, "fill_empty launch");
  }
  int32_t rc;
  if ((rc = ws->err.reserve(sizeof(int))) != MANS_OK) return rc;
  MergeParams m{};
  m.in_dist = d_in_dist;
  m.in_ids = d_in_ids;
  m.in_counts = d_in_counts;
  m.n_lists = n_lists;
  m.list_stride = list_stride;
  m.kp_in = kin;
  m.nq = nq;
  m.k = kout;
  m.kp = pow2_at_least(kout);
  m.kout = kout;
  m.out_dist = d_out_dist;
  m.out_ids = d_out_ids;
  m.out_counts = d_out_counts;
  m.err = static_cast<int*>(ws->err.ptr);
  cudaEvent_t st_stop = stage_begin(ws, st, MANS_STAGE_MERGE);
  cudaError_t e = launch_merge(m, st);
  if (e != cudaSuccess) return fail_cuda(e, "merge launch");
  timing_end(st_stop, st);
  ws->launches += 1;
  return MANS_OK;
}

}  // extern "C"
