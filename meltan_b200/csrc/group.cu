// group.cu -- one context over several GPUs of this process.
//
// The reference drives one GPU through one MetalContext per index
// (Sources/MetalANNS/ANNSIndex.swift:35), and its callers are single
// processes.  A context made by mans_ctx_create_multi holds one ordinary
// context per GPU; a corpus created on it is split into contiguous row shards,
// one per GPU (the first n % G shards hold one extra row, global id = shard's
// first row + local row), and mans_flat_search with host buffers searches all
// shards at once:
//
//   every GPU i, on a stream of its own: query upload, the single-GPU search
//   of its shard (scan or tensor-core path, exactly as on one GPU), then
//   publish_block_kernel stores the shard's top-k block over NVLink into slot
//   i of a gather buffer on the first GPU, and an event marks the end;
//   the first GPU waits for every event, merge_kernel merges the G blocks by
//   (distance, id) -- ParallelFlatScan.mergeSorted (ParallelFlatScan.swift:
//   288-315) applied to row shards -- and the results come back to the host.
//
// Peer access comes from cudaDeviceEnablePeerAccess between the GPUs of the
// process; the only cross-GPU traffic is those plain stores (no IPC handle, no
// collective library, no multicast), and ordering uses CUDA events, so no
// kernel waits on another GPU.

#include <algorithm>
#include <cstdio>
#include <thread>
#include <vector>

#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"

namespace mans {
namespace {

// Shard i's top-k block [distances | ids | counts] (nq x kout, nq x kout, nq
// words) into `dst` (another GPU's memory).
__global__ void publish_block_kernel(const float* __restrict__ dist,
                                     const uint32_t* __restrict__ ids,
                                     const int32_t* __restrict__ counts, int64_t nq, int32_t kout,
                                     int32_t* __restrict__ dst) {
  const int64_t pairs = nq * kout;
  const int64_t total = 2 * pairs + nq;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int32_t w;
    if (i < pairs)
      w = __float_as_int(dist[i]);
    else if (i < 2 * pairs)
      w = static_cast<int32_t>(ids[i - pairs]);
    else
      w = counts[i - 2 * pairs];
    dst[i] = w;
  }
}

int64_t shard_begin(int64_t n, int64_t g, int64_t i) {
  const int64_t base = n / g, extra = n % g;
  return i * base + std::min(i, extra);
}

}  // namespace

int32_t reject_group(const mans_ctx* ctx, const mans_corpus* corpus, const char* what) {
  if (is_group(ctx) || is_group(corpus)) {
    std::string msg = std::string(what) +
                      " runs on one GPU: use a context from mans_ctx_create (a multi-GPU context "
                      "takes mans_flat_search and the corpus calls)";
    return fail(MANS_ERR_INVALID, msg);
  }
  return MANS_OK;
}

int32_t corpus_create_any(mans_ctx* ctx, const float* rows, int64_t n, int64_t dim,
                          uint32_t id_offset, mans_corpus** out, int64_t src_ld) {
  if (!is_group(ctx)) return corpus_upload(ctx, rows, n, dim, id_offset, out, src_ld);
  if (src_ld <= 0) src_ld = dim;
  if (n < 0 || dim <= 0) return fail(MANS_ERR_INVALID, "corpus needs n >= 0 and dim > 0");
  if (n > 0 && !rows) return fail(MANS_ERR_INVALID, "rows is null");
  if (n > static_cast<int64_t>(INT32_MAX)) return fail(MANS_ERR_INVALID, "corpus too large");
  const int64_t g = static_cast<int64_t>(ctx->members.size());
  mans_corpus* c = new mans_corpus();
  c->ctx = ctx;
  c->n = n;
  c->dim = dim;
  c->ld = (dim + 3) / 4 * 4;
  c->id_offset = id_offset;
  c->owned = false;
  c->shards.assign(g, nullptr);
  c->shard_row0.resize(g + 1);
  for (int64_t i = 0; i <= g; ++i) c->shard_row0[i] = shard_begin(n, g, i);
  // each GPU uploads its rows and computes their norms at the same time
  std::vector<int32_t> rc(g, MANS_OK);
  std::vector<std::string> msg(g);
  std::vector<std::thread> th;
  for (int64_t i = 0; i < g; ++i) {
    th.emplace_back([&, i] {
      const int64_t r0 = c->shard_row0[i], r1 = c->shard_row0[i + 1];
      rc[i] = corpus_upload(ctx->members[i], rows ? rows + r0 * src_ld : nullptr, r1 - r0, dim,
                            id_offset + static_cast<uint32_t>(r0), &c->shards[i], src_ld);
      if (rc[i] != MANS_OK) {
        char buf[1024];
        mans_last_error_message(buf, sizeof buf);
        msg[i] = buf;
      }
    });
  }
  for (auto& t : th) t.join();
  for (int64_t i = 0; i < g; ++i) {
    if (rc[i] != MANS_OK) {
      for (mans_corpus* s : c->shards)
        if (s) mans_corpus_destroy(s);
      delete c;
      return fail(rc[i], "shard " + std::to_string(i) + ": " + msg[i]);
    }
  }
  *out = c;
  return MANS_OK;
}

int32_t group_flat_search(mans_ctx* ctx, const mans_corpus* corpus, const float* queries,
                          int64_t nq, int64_t dim, int32_t k, int32_t metric, float* out_dist,
                          uint32_t* out_ids, int32_t* out_counts) {
  const int g = static_cast<int>(ctx->members.size());
  const int32_t kout = std::min<int32_t>(k, MANS_MAX_TOPK);
  const int64_t words = 2 * nq * kout + nq;
  const int64_t stride = (words + 3) / 4 * 4;  // 16-byte aligned slots
  std::vector<mans_workspace*> ws(g, nullptr);
  int32_t rc = MANS_OK;
  for (int i = 0; i < g && rc == MANS_OK; ++i) {
    DeviceGuard dg(ctx->members[i]->device);
    ws[i] = acquire_workspace(ctx->members[i]);
    if (!ws[i]) rc = fail(MANS_ERR_OOM, "cannot create a workspace stream");
  }
  int32_t* gather = nullptr;
  if (rc == MANS_OK) {
    DeviceGuard dg(ctx->members[0]->device);
    rc = ws[0]->gather.reserve(static_cast<size_t>(g) * stride * sizeof(int32_t));
    gather = static_cast<int32_t*>(ws[0]->gather.ptr);
    if (rc == MANS_OK)
      rc = ws[0]->out_dist.reserve(nq * kout * sizeof(float));
    if (rc == MANS_OK) rc = ws[0]->out_ids.reserve(nq * kout * sizeof(uint32_t));
    if (rc == MANS_OK) rc = ws[0]->out_counts.reserve(nq * sizeof(int32_t));
  }
  // 1. every shard on its own GPU, its block stored into slot i on GPU 0
  for (int i = 0; i < g && rc == MANS_OK; ++i) {
    mans_ctx* m = ctx->members[i];
    mans_workspace* w = ws[i];
    DeviceGuard dg(m->device);
    cudaStream_t st = w->stream;
    if ((rc = w->queries.reserve(nq * dim * sizeof(float))) != MANS_OK) break;
    if ((rc = w->out_dist.reserve(nq * kout * sizeof(float))) != MANS_OK) break;
    if ((rc = w->out_ids.reserve(nq * kout * sizeof(uint32_t))) != MANS_OK) break;
    if ((rc = w->out_counts.reserve(nq * sizeof(int32_t))) != MANS_OK) break;
    if (!w->done && cudaEventCreateWithFlags(&w->done, cudaEventDisableTiming) != cudaSuccess) {
      w->done = nullptr;
      rc = fail(MANS_ERR_EXEC, "cudaEventCreate");
      break;
    }
    cudaError_t e = cudaMemcpyAsync(w->queries.ptr, queries, nq * dim * sizeof(float),
                                    cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) {
      rc = fail_cuda(e, "query upload");
      break;
    }
    rc = run_flat_search(m, corpus->shards[i], w, static_cast<const float*>(w->queries.ptr), nq,
                         k, metric, static_cast<float*>(w->out_dist.ptr),
                         static_cast<uint32_t*>(w->out_ids.ptr),
                         static_cast<int32_t*>(w->out_counts.ptr), st);
    if (rc != MANS_OK) break;
    const int blocks = static_cast<int>(std::min<int64_t>((words + 255) / 256, 64));
    publish_block_kernel<<<blocks, 256, 0, st>>>(
        static_cast<const float*>(w->out_dist.ptr), static_cast<const uint32_t*>(w->out_ids.ptr),
        static_cast<const int32_t*>(w->out_counts.ptr), nq, kout,
        gather + static_cast<int64_t>(i) * stride);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaEventRecord(w->done, st);
    if (e != cudaSuccess) rc = fail_cuda(e, "shard block publish");
  }
  // 2. GPU 0 waits for every block, merges and downloads
  if (rc == MANS_OK) {
    DeviceGuard dg(ctx->members[0]->device);
    cudaStream_t st = ws[0]->stream;
    cudaError_t e = cudaSuccess;
    for (int i = 1; i < g && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(st, ws[i]->done, 0);
    if (e != cudaSuccess) rc = fail_cuda(e, "cross-GPU event wait");
    if (rc == MANS_OK && (rc = ws[0]->err.reserve(sizeof(int))) == MANS_OK) {
      MergeParams mp{};
      mp.in_dist = reinterpret_cast<const float*>(gather);
      mp.in_ids = reinterpret_cast<const uint32_t*>(gather + nq * kout);
      mp.in_counts = gather + 2 * nq * kout;
      mp.n_lists = g;
      mp.list_stride = stride;
      mp.kp_in = kout;
      mp.nq = nq;
      mp.k = kout;
      mp.kp = pow2_at_least(kout);
      mp.kout = kout;
      mp.out_dist = static_cast<float*>(ws[0]->out_dist.ptr);
      mp.out_ids = static_cast<uint32_t*>(ws[0]->out_ids.ptr);
      mp.out_counts = static_cast<int32_t*>(ws[0]->out_counts.ptr);
      mp.err = static_cast<int*>(ws[0]->err.ptr);
      e = launch_merge(mp, st);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(out_dist, ws[0]->out_dist.ptr, nq * kout * sizeof(float),
                            cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(out_ids, ws[0]->out_ids.ptr, nq * kout * sizeof(uint32_t),
                            cudaMemcpyDeviceToHost, st);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(out_counts, ws[0]->out_counts.ptr, nq * sizeof(int32_t),
                            cudaMemcpyDeviceToHost, st);
      if (e != cudaSuccess) rc = fail_cuda(e, "merge and download");
    }
  }
  // 3. every GPU's stream finished (also after a failure: nothing may still
  // write into the gather buffer when the workspaces return to their pools);
  // a device-side failure of any shard fails the call
  for (int i = 0; i < g; ++i) {
    if (!ws[i]) continue;
    DeviceGuard dg(ctx->members[i]->device);
    int32_t r = check_device_error(ws[i], ws[i]->stream);
    if (rc == MANS_OK) rc = r;
  }
  for (int i = 0; i < g; ++i)
    if (ws[i]) release_workspace(ctx->members[i], ws[i]);
  return rc;
}

}  // namespace mans

extern "C" {

int32_t mans_ctx_create_multi(const int32_t* devices, int32_t n_devices, mans_ctx** out_ctx) {
  using namespace mans;
  if (!out_ctx || !devices) return fail(MANS_ERR_INVALID, "null devices or output");
  *out_ctx = nullptr;
  if (n_devices < 1) return fail(MANS_ERR_INVALID, "a multi-GPU context needs at least one device");
  for (int32_t i = 0; i < n_devices; ++i)
    for (int32_t j = 0; j < i; ++j)
      if (devices[i] == devices[j]) return fail(MANS_ERR_INVALID, "a device is listed twice");
  std::vector<mans_ctx*> members;
  auto undo = [&] {
    for (mans_ctx* m : members) mans_ctx_destroy(m);
  };
  for (int32_t i = 0; i < n_devices; ++i) {
    mans_ctx* m = nullptr;
    int32_t rc = mans_ctx_create(devices[i], &m);
    if (rc != MANS_OK) {
      undo();
      return rc;
    }
    members.push_back(m);
  }
  // every GPU stores its block into the first GPU's memory
  for (int32_t i = 1; i < n_devices; ++i) {
    int can = 0;
    cudaError_t e = cudaDeviceCanAccessPeer(&can, devices[i], devices[0]);
    if (e != cudaSuccess || !can) {
      undo();
      return fail(MANS_ERR_DEVICE, "a device of the group cannot reach the first one (no peer access)");
    }
    DeviceGuard dg(devices[i]);
    e = cudaDeviceEnablePeerAccess(devices[0], 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
      cudaGetLastError();  // not sticky: take it out of the last-error slot
      e = cudaSuccess;
    }
    if (e != cudaSuccess) {
      undo();
      return fail_cuda(e, "cudaDeviceEnablePeerAccess");
    }
  }
  mans_ctx* ctx = new mans_ctx();
  ctx->device = members[0]->device;
  ctx->num_sms = members[0]->num_sms;
  ctx->max_smem = members[0]->max_smem;
  ctx->members = members;
  *out_ctx = ctx;
  return MANS_OK;
}

int32_t mans_ctx_device_count(const mans_ctx* ctx) {
  if (!ctx) return 0;
  return ctx->members.empty() ? 1 : static_cast<int32_t>(ctx->members.size());
}

}  // extern "C"
