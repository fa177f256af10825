// noalloc.cu -- exact flat search that performs no device or host allocation.
//
// Who needs this: code that may not allocate GPU memory at search time.  A
// search recorded inside a CUDA stream capture must not call cudaMalloc (the
// allocation is not part of the graph and breaks or invalidates the capture);
// services that hand all device memory to their own pool or caching allocator
// up front cannot let a library grab extra memory behind their back; and
// latency-critical loops cannot afford the implicit device synchronisation
// that cudaMalloc/cudaFree bring.  mans_flat_search_device needs a workspace
// whose buffers grow with cudaMalloc on first use, and mans_flat_search also
// allocates pinned staging; this entry point uses neither.
//
// Its scratch (per-block candidate lists, their counts and the device error
// word) lives in one file-scope __device__ array of kScratchBytes (4 MiB) that
// every GPU which loads this library holds until the process exits.  Host code
// cannot use the array's name as a device address, so the first call on each
// device resolves the address with cudaGetSymbolAddress while that device is
// current and caches it; make that first call before any stream capture
// starts.  Every call on a device shares the same array and leaves the last
// call's contents behind: calls whose GPU work can overlap (different streams
// without ordering, or several threads) race on it and must be serialised by
// the caller.  The error word is cleared on the stream at the start of every
// call; candidate counts are always written before they are read.  The call
// only enqueues work and returns argument and launch errors.  Reading the
// error word back would synchronise, so a device wait that timed out (which
// only a stalled GPU produces) is reported in the results instead: the merge
// kernel sees the word set and writes every query's result as empty (count 0,
// ids MANS_EMPTY_ID), never a partial top-k.
//
// Scratch use of one call, in bytes (the MANS_ERR_OOM test below):
//   256 + round256(4 * S) + 8 * S * kp,   S = G * qb * splits,
//   qb = smallest power of two >= nq capped at 8, G = ceil(nq / qb),
//   splits = min(max(1, SMs / G), ceil(n / 256)), kp = smallest power of two
//   >= min(k, 256, n).
// So k = 129 costs as much as k = 256, and below about 8 x SMs queries the
// need is near SMs x 8 x kp x 8 bytes whatever nq is.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"

using namespace mans;

namespace {

constexpr size_t kScratchBytes = size_t(4) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_flat_scratch[kScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_flat_scratch on `device` (the current device).
int32_t scratch_address(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) return fail(MANS_ERR_DEVICE, "device index too large");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_flat_scratch);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(scratch)");
    g_scratch_ptr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_ptr[device]);
  return MANS_OK;
}

size_t round256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

extern "C" int32_t mans_flat_search_noalloc(mans_ctx* ctx, const mans_corpus* corpus,
                                            const float* d_queries, int64_t nq, int32_t k,
                                            int32_t metric, float* d_out_dist,
                                            uint32_t* d_out_ids, int32_t* d_out_counts,
                                            void* cuda_stream) {
  if (!ctx || !corpus) return fail(MANS_ERR_INVALID, "null context or corpus");
  if (corpus->ctx != ctx) return fail(MANS_ERR_INVALID, "corpus belongs to another context");
  if (int32_t r = reject_group(ctx, corpus, "mans_flat_search_noalloc")) return r;
  if (nq < 0) return fail(MANS_ERR_INVALID, "negative query count");
  if (metric == MANS_METRIC_HAMMING)
    return fail(MANS_ERR_SEARCH, "FlatGPUSearch does not support metric .hamming");
  if (metric < 0 || metric > MANS_METRIC_HAMMING) return fail(MANS_ERR_INVALID, "unknown metric");
  if (nq == 0) return MANS_OK;
  DeviceGuard g(ctx->device);
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  const int32_t kout = std::min<int32_t>(k, MANS_MAX_TOPK);
  const int64_t n = corpus->n;
  if (k <= 0 || n <= 0) {
    cudaError_t e = kout <= 0
                        ? cudaMemsetAsync(d_out_counts, 0, sizeof(int32_t) * nq, stream)
                        : launch_fill_empty(d_out_dist, d_out_ids, d_out_counts, nq, kout, stream);
    return e == cudaSuccess ? MANS_OK : fail_cuda(e, "empty result");
  }
  // Same work split as the workspace-based search: query groups of up to 8,
  // corpus tiles spread over the SMs.
  const int32_t keff = static_cast<int32_t>(std::min<int64_t>(kout, n));
  int32_t kp = 1;
  while (kp < keff) kp <<= 1;
  const int qb = nq <= 1 ? 1 : nq <= 2 ? 2 : nq <= 4 ? 4 : 8;
  const int64_t groups = (nq + qb - 1) / qb;
  const int64_t tiles = (n + kTileRows - 1) / kTileRows;
  int64_t splits = std::max<int64_t>(1, ctx->num_sms / groups);
  splits = std::min<int64_t>(splits, tiles);
  const int64_t nslots = groups * qb * splits;
  const size_t counts_at = 256;
  const size_t keys_at = counts_at + round256(static_cast<size_t>(nslots) * sizeof(int32_t));
  const size_t need = keys_at + static_cast<size_t>(nslots) * kp * sizeof(uint64_t);
  if (need > kScratchBytes) {
    char msg[160];
    std::snprintf(msg, sizeof msg,
                  "request needs %zu bytes of scratch; the no-allocation search holds %zu "
                  "(use fewer queries or a smaller k)",
                  need, kScratchBytes);
    return fail(MANS_ERR_OOM, msg);
  }
  const int nchunks = static_cast<int>((corpus->dim + kTileCols - 1) / kTileCols);
  const int stages = scan_max_stages(qb, nchunks);
  if (stages < 2) return fail(MANS_ERR_SEARCH, "dimension too large for the flat scan kernel");

  unsigned char* scratch = nullptr;
  int32_t rc = scratch_address(ctx->device, &scratch);
  if (rc != MANS_OK) return rc;
  int* err = reinterpret_cast<int*>(scratch);
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(int), stream);
  if (e != cudaSuccess) return fail_cuda(e, "clear scratch error word");

  ScanParams p{};
  p.segs = nullptr;
  p.nseg = static_cast<int32_t>(groups * splits);
  p.nseg_dev = nullptr;
  p.stages = stages;
  p.tile_rows = kTileRows;
  p.flat_splits = static_cast<int32_t>(splits);
  p.flat_tiles = static_cast<int32_t>(tiles);
  p.n = n;
  p.nq = nq;
  p.queries = d_queries;
  p.qidx = nullptr;
  p.qnorms = nullptr;
  p.norms = metric == MANS_METRIC_IP ? nullptr : corpus->norms;
  p.ids = corpus->ids;
  p.id_offset = corpus->id_offset;
  p.dim = static_cast<int32_t>(corpus->dim);
  p.nchunks = nchunks;
  p.metric = metric;
  p.mode = kModeHost;
  p.k = keff;
  p.kp = kp;
  p.slot_keys = reinterpret_cast<uint64_t*>(scratch + keys_at);
  p.slot_counts = reinterpret_cast<int32_t*>(scratch + counts_at);
  p.err = err;
  e = launch_scan(qb, corpus->map, p, static_cast<int>(std::min<int64_t>(p.nseg, ctx->num_sms)),
                  stream);
  if (e != cudaSuccess) return fail_cuda(e, "scan launch");

  MergeParams m{};
  m.in_keys = p.slot_keys;
  m.in_counts = p.slot_counts;
  m.slots_per_query = static_cast<int32_t>(splits);
  m.kp_in = kp;
  m.nq = nq;
  m.k = keff;
  m.kp = kp;
  m.kout = kout;
  m.out_dist = d_out_dist;
  m.out_ids = d_out_ids;
  m.out_counts = d_out_counts;
  m.err = err;
  m.empty_on_error = true;
  e = launch_merge(m, stream);
  return e == cudaSuccess ? MANS_OK : fail_cuda(e, "merge launch");
}
