// internal.h -- library-private object layouts behind the opaque C handles.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <functional>
#include <mutex>
#include <string>
#include <vector>

#include "tc.h"

struct mans_workspace;

namespace mans {

struct DeviceBuffer {
  void* ptr = nullptr;
  size_t bytes = 0;
  int32_t reserve(size_t need);  // grows (contents not kept)
  void release();
};

struct PinnedBuffer {
  void* ptr = nullptr;
  size_t bytes = 0;
  int32_t reserve(size_t need);
  void release();
};

struct DeviceGuard {
  int prev = -1, cur = -1;
  explicit DeviceGuard(int dev);
  ~DeviceGuard();
};

int32_t fail(int32_t code, const std::string& msg);
int32_t fail_cuda(cudaError_t e, const char* what);
int32_t encode_row_map(CUtensorMap* map, const float* base, int64_t rows, int64_t dim, int64_t ld,
                       int box_rows = 256);

}  // namespace mans

struct mans_ctx {
  int device = 0;
  int num_sms = 0;
  int max_smem = 0;
  std::mutex mu;
  std::vector<mans_workspace*> pool;  // idle workspaces for host-pointer calls
  // query batches of at least this size use the tensor-core path (0: never)
  int tc_min_batch = 16;
  // operand format of that path: MANS_TC_AUTO / MANS_TC_BF16 / MANS_TC_INT8
  int tc_format = 0;
  // cooperative launches are available (the one-launch IVF-flat search)
  bool coop_launch = false;
  bool probe_configured = false;  // that kernel's shared-memory limit is set
  bool tc_configured = false;     // the tensor-core path's kernel attributes are set
  int tc_pairs = -1;              // CTA pairs of the pair pass resident at once (-1: not asked)
  // programmatic dependent launch between the tensor-core path's kernels
  // (cleared if the runtime refuses it)
  bool pdl = true;
  // A context over several GPUs (mans_ctx_create_multi): one single-device
  // context per GPU, members[0] on `device`; empty for a plain context.
  std::vector<mans_ctx*> members;
};

// Row-major fp32 rows with a 16-byte pitch (ld = dim rounded up to 4), the
// squared row norms and the TMA descriptor over them.
struct mans_corpus {
  mans_ctx* ctx = nullptr;
  int64_t n = 0;
  int64_t dim = 0;
  int64_t ld = 0;
  uint32_t id_offset = 0;
  float* rows = nullptr;
  float* norms = nullptr;
  uint32_t* ids = nullptr;  // optional row -> reported id (packed IVF lists)
  bool owned = true;        // rows/norms/ids freed with the object
  CUtensorMap map;
  CUtensorMap map_small;  // the same rows in boxes of kSmallTileRows
  CUtensorMap map_seg;    // the same rows in boxes of 32 (the IVF-flat batch list scan)
  // bf16 copy and error-bound terms for the tensor-core batch path (built on
  // first use, dropped when rows change)
  std::mutex tc_mu;
  bool tc_ready = false;
  int tc_metric = -1;  // row scaling of the bf16 copy: 1 normalised (cosine), 0 as stored
  void* tc_rows = nullptr;
  int64_t tc_ld16 = 0;
  float* tc_stats = nullptr;  // n x 4: |r'|, |r' - bf16(r')|, |bf16(r')|, |r| rounded down
  mans::TcCorpusStats tc_stats_host{};
  CUtensorMap tc_map;
  CUtensorMap tc_map_half;  // the same rows in 128-row boxes (one CTA of a pair)
  // signed 8-bit codes (Int8CodeBuffer quantisation), built on first use
  bool tc8_ready = false;
  void* tc8_rows = nullptr;  // n x tc8_ld int8
  int64_t tc8_ld = 0;
  float* tc8_u = nullptr;     // per-row scale u
  float* tc8_wcos = nullptr;  // u / |r| (cosine factor)
  float* tc8_stats = nullptr; // n x 4: |r|, |r - u code|, |u code|, |r| rounded down
  mans::TcCorpusStats tc8_plain{};  // L2 / IP bound terms
  mans::TcCorpusStats tc8_cos{};    // cosine: terms relative to |r|
  CUtensorMap tc8_map;
  // A corpus of a multi-GPU context: contiguous row shards, one per member
  // device (shard i holds rows [shard_row0[i], shard_row0[i+1])); the fields
  // above stay empty.  Empty for a single-device corpus.
  std::vector<mans_corpus*> shards;
  std::vector<int64_t> shard_row0;
};

struct mans_workspace {
  mans_ctx* ctx = nullptr;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  bool err_cleared = false;
  mans::DeviceBuffer err;
  mans::DeviceBuffer qnorms;
  mans::DeviceBuffer slot_keys;
  mans::DeviceBuffer slot_counts;
  mans::DeviceBuffer queries;
  mans::DeviceBuffer out_dist;
  mans::DeviceBuffer out_ids;
  mans::DeviceBuffer out_counts;
  mans::DeviceBuffer aux;
  mans::DeviceBuffer aux2;
  // scratch of the tensor-core batch path alone: it runs nested inside other
  // searches (the IVF centroid scan) whose own scratch lives in `aux`
  mans::DeviceBuffer tc_aux;
  // score matrix chunk of the small-corpus batch search (centroid scans)
  mans::DeviceBuffer small_scores;
  // grid-barrier counter of the fused tensor-core pass (monotonic; the host
  // keeps its expected value, both reset after a device error)
  mans::DeviceBuffer tc_bar;
  unsigned long long tc_bar_base = 0;
  // one-launch IVF-flat search: its grid-barrier counter (monotonic, the host
  // keeps the expected value) and per-query arrival counters (zero between
  // launches); both reset after a device error
  mans::DeviceBuffer probe_sync;
  unsigned long long probe_bar_base = 0;
  mans::PinnedBuffer h_err;
  // IVF-PQ searches with k above 256: every probed entry's key, twice (sort
  // input and output), and the sort's temporary storage
  mans::DeviceBuffer big;
  // host-buffer searches: queries and packed results on the device, and their
  // pinned staging copy on the host
  mans::DeviceBuffer io;
  mans::PinnedBuffer h_io;
  // optional CUDA-event timing of the dominant kernel (scan) launches
  bool timing = false;
  int timing_hold = 0;  // > 0 while an inner step (e.g. a centroid scan) runs untimed
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> events;
  size_t events_used = 0;
  // optional per-stage timing (mans_workspace_set_timing bit 1): CUDA events
  // around each stage of a search, summed per stage by mans_workspace_stage_times
  bool stage_timing = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> stage_events;
  std::vector<int> stage_of;
  size_t stage_used = 0;
  int64_t launches = 0;  // library kernels enqueued through this workspace
  int last_path = 0;     // path of the last flat search: 0 scan, 1 bf16 tensor, 2 int8 tensor
  int32_t* tc_fallbacks = nullptr;  // device counter of exact re-scans (last tc call)
  // multi-GPU searches: the packed per-device result blocks land here (on the
  // first device), and `done` marks the end of this workspace's part
  mans::DeviceBuffer gather;
  cudaEvent_t done = nullptr;
};

namespace mans {
mans_workspace* acquire_workspace(mans_ctx* ctx);
void release_workspace(mans_ctx* ctx, mans_workspace* ws);
void destroy_workspace(mans_workspace* ws);
int32_t check_device_error(mans_workspace* ws, cudaStream_t stream);
int32_t device_error(mans_workspace* ws, int h);
// A search with host buffers: the queries are staged through pinned memory
// and uploaded in one copy, `search` enqueues the device search on the
// workspace stream, the packed results and the device error word come back
// in one copy each, and the stream is synchronised once.
using DeviceSearch = std::function<int32_t(const float* d_queries, float* d_dist, uint32_t* d_ids,
                                           int32_t* d_counts, cudaStream_t stream)>;
int32_t host_buffer_search(mans_workspace* ws, const float* queries, int64_t nq, int64_t dim,
                           int32_t kout, float* out_dist, uint32_t* out_ids, int32_t* out_counts,
                           const DeviceSearch& search);
int pow2_at_least(int v);
int choose_qb(int64_t nq);
cudaEvent_t timing_begin(mans_workspace* ws, cudaStream_t stream);
// Keeps the inner steps of a search out of the dominant-kernel timing.
struct TimingHold {
  mans_workspace* ws;
  explicit TimingHold(mans_workspace* w) : ws(w) { ++ws->timing_hold; }
  ~TimingHold() { --ws->timing_hold; }
};
void timing_end(cudaEvent_t stop, cudaStream_t stream);
// Records a start event before stage `stage` (MANS_STAGE_*) when per-stage
// timing is on and no inner step holds the timing; returns the stop event to
// record after the stage with timing_end (or null).
cudaEvent_t stage_begin(mans_workspace* ws, cudaStream_t stream, int stage);
// Copies rows (host or device, n x dim with a row pitch of src_ld elements,
// 0 = dim) into a new corpus object (norms on the device).
int32_t corpus_upload(mans_ctx* ctx, const float* rows, int64_t n, int64_t dim, uint32_t id_offset,
                      mans_corpus** out, int64_t src_ld = 0);
void corpus_free(mans_corpus* c);
// Multi-GPU contexts (group.cu).
inline bool is_group(const mans_ctx* ctx) { return ctx && !ctx->members.empty(); }
inline bool is_group(const mans_corpus* c) { return c && !c->shards.empty(); }
// corpus_upload, or for a multi-GPU context one row shard per device.
int32_t corpus_create_any(mans_ctx* ctx, const float* rows, int64_t n, int64_t dim,
                          uint32_t id_offset, mans_corpus** out, int64_t src_ld = 0);
int32_t group_flat_search(mans_ctx* ctx, const mans_corpus* corpus, const float* queries,
                          int64_t nq, int64_t dim, int32_t k, int32_t metric, float* out_dist,
                          uint32_t* out_ids, int32_t* out_counts);
// MANS_ERR_INVALID for a multi-GPU context or corpus passed to an entry point
// that runs on one device.
int32_t reject_group(const mans_ctx* ctx, const mans_corpus* corpus, const char* what);
// One-launch IVF-flat search of a few queries (ivf_probe.cu).
constexpr int kProbeMaxQ = 4;            // queries per launch
constexpr int kProbeMaxNlist = 8192;     // centroid keys of a query staged in shared memory
constexpr size_t kProbeSyncBytes = 128;  // barrier counter at 0, arrival counters at 64
bool ivf_probe_applies(const mans_ctx* ctx, const mans_corpus* packed, int32_t nlist, int64_t nq,
                       int32_t kout, int32_t probe);
int32_t run_ivf_probe(mans_ctx* ctx, const mans_corpus* cent, const mans_corpus* packed,
                      const int64_t* d_offsets, mans_workspace* ws, const float* d_queries,
                      int64_t nq, int32_t kout, int32_t keff, int32_t probe, int32_t metric,
                      float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                      cudaStream_t stream);
// tensor-core batch path (tc_scan.cu)
// i8: the int8 operand format (else bf16); tc_use_int8 picks it for a batch.
bool tc_use_int8(const mans_ctx* ctx, int64_t nq);
int32_t tc_prepare_corpus(mans_corpus* c, int metric, bool i8);
bool tc_applicable(const mans_corpus* c, int metric, bool i8);
int32_t run_flat_search_tc(mans_ctx* ctx, mans_corpus* corpus, mans_workspace* ws,
                           const float* d_queries, int64_t nq, int32_t k, int32_t metric,
                           float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                           cudaStream_t stream, bool i8);
// host copy of the int8 codes and scales (prepared on demand)
int32_t tc_export_int8(mans_corpus* c, int8_t* codes, float* scales);
void tc_free_corpus(mans_corpus* c);
// Exact scan + top-k over `corpus`.  mode: kModeHost (host-tier distance) or
// kModeSimd (SIMDDistance semantics).  kcap bounds k (256 for the public
// searches; 512 for the internal 2k candidate lists of the IVF-PQ stages).
// centroid_scan: a batch over a small corpus takes the small-corpus path even
// where the tensor-core path would apply (the centroid steps of the indexes).
int32_t run_flat_search(mans_ctx* ctx, const mans_corpus* corpus, mans_workspace* ws,
                        const float* d_queries, int64_t nq, int32_t k, int32_t metric,
                        float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                        cudaStream_t stream, int mode = 0, int32_t kcap = 256,
                        bool centroid_scan = false);
// Batches of at least kSmallBatchMinQueries queries over a corpus of at most
// kSmallBatchMaxRows rows (centroid sets): score tiles + per-query sort
// (small_scan.cu), the same results as the streaming scan.
constexpr int64_t kSmallBatchMinQueries = 64;
constexpr int64_t kSmallBatchMaxRows = 8192;
bool small_batch_applies(const mans_corpus* corpus, int64_t nq);
int32_t run_small_batch_search(mans_ctx* ctx, const mans_corpus* corpus, mans_workspace* ws,
                               const float* d_queries, int64_t nq, int32_t kout, int32_t metric,
                               float* d_out_dist, uint32_t* d_out_ids, int32_t* d_out_counts,
                               cudaStream_t stream, int mode);
}  // namespace mans
