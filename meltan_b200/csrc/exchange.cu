// exchange.cu -- all-gather of the per-shard top-k blocks over peer memory
// (NVLink), fused with the final (distance, id) merge.
//
// Each rank owns one device buffer, shared with the other ranks through CUDA
// IPC handles: for both parities b of the call counter,
//   slots[b][world][stride]  int32 words: rank r's packed block
//                            [distances | ids | counts] lands in slots[b][r]
//   flags[b][world]          uint32: rank r release-stores the call's epoch
//                            after its block
// A call publishes this rank's block into slot [rank] of every rank (P2P
// stores, then a system fence and a release store of the flag) and launches
// the merge kernel, which acquire-waits (bounded) for all flags of its
// parity and merges the world blocks.  A rank can run at most one call ahead
// of a peer (its next merge needs the peer's next block, which the peer
// publishes only after finishing the current merge), so two parities keep a
// block from being overwritten while it is read.  This replaces the NCCL
// all-gather of mergeSorted's inputs (ParallelFlatScan.swift:288-315 applied
// to row shards) with one small kernel and no library call.

#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "mans_cuda.h"

struct mans_exchange {
  mans_ctx* ctx = nullptr;
  int32_t world = 1;
  int32_t rank = 0;
  int64_t stride = 0;          // words per slot (multiple of 4)
  int32_t* local = nullptr;    // this rank's buffer
  size_t bytes = 0;
  std::vector<int32_t*> peer;  // mapped buffers (peer[rank] = local)
  int32_t** d_peer = nullptr;  // device copy of `peer`
  uint32_t epoch = 0;
};

namespace mans {
namespace {

__host__ __device__ inline size_t flags_offset_words(int32_t world, int64_t stride) {
  return static_cast<size_t>(2) * world * stride;
}

// grid = world blocks: block p writes this rank's block into peer p's slot
__global__ void publish_kernel(int32_t* const* peers, int32_t rank, int32_t world, int64_t stride,
                               const int32_t* __restrict__ block, int64_t words, int parity,
                               uint32_t epoch) {
  int32_t* dst_base = peers[blockIdx.x];
  int32_t* dst = dst_base + (static_cast<size_t>(parity) * world + rank) * stride;
  const bool vec = (reinterpret_cast<uintptr_t>(block) & 15) == 0 && (words & 3) == 0;
  if (vec) {
    const int4* s4 = reinterpret_cast<const int4*>(block);
    int4* d4 = reinterpret_cast<int4*>(dst);
    for (int64_t i = threadIdx.x; i < words / 4; i += blockDim.x) d4[i] = s4[i];
  } else {
    for (int64_t i = threadIdx.x; i < words; i += blockDim.x) dst[i] = block[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* flag = reinterpret_cast<uint32_t*>(dst_base + flags_offset_words(world, stride)) +
                     parity * world + rank;
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(epoch) : "memory");
  }
}

}  // namespace
}  // namespace mans

extern "C" {

int32_t mans_exchange_create(mans_ctx* ctx, int32_t world, int32_t rank, int64_t max_block_words,
                             mans_exchange** out) {
  using namespace mans;
  if (!ctx || !out) return fail(MANS_ERR_INVALID, "null context or output");
  *out = nullptr;
  if (int32_t r = reject_group(ctx, nullptr, "mans_exchange_create")) return r;
  if (world < 1 || rank < 0 || rank >= world || max_block_words <= 0)
    return fail(MANS_ERR_INVALID, "bad exchange shape");
  DeviceGuard g(ctx->device);
  mans_exchange* ex = new mans_exchange();
  ex->ctx = ctx;
  ex->world = world;
  ex->rank = rank;
  ex->stride = (max_block_words + 3) / 4 * 4;
  ex->bytes = (flags_offset_words(world, ex->stride) + 2 * static_cast<size_t>(world)) * 4;
  cudaError_t e = cudaMalloc(&ex->local, ex->bytes);
  if (e == cudaSuccess) e = cudaMemset(ex->local, 0, ex->bytes);
  if (e == cudaSuccess) e = cudaMalloc(&ex->d_peer, world * sizeof(int32_t*));
  if (e != cudaSuccess) {
    if (ex->local) cudaFree(ex->local);
    delete ex;
    return fail_cuda(e, "exchange buffer");
  }
  ex->peer.assign(world, nullptr);
  ex->peer[rank] = ex->local;
  *out = ex;
  return MANS_OK;
}

int32_t mans_exchange_handle(const mans_exchange* ex, void* out_handle) {
  using namespace mans;
  if (!ex || !out_handle) return fail(MANS_ERR_INVALID, "null exchange or output");
  DeviceGuard g(ex->ctx->device);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ex->local);
  if (e != cudaSuccess) return fail_cuda(e, "cudaIpcGetMemHandle");
  std::memcpy(out_handle, &h, sizeof h);
  return MANS_OK;
}

int32_t mans_exchange_open(mans_exchange* ex, const void* handles) {
  using namespace mans;
  if (!ex || !handles) return fail(MANS_ERR_INVALID, "null exchange or handles");
  DeviceGuard g(ex->ctx->device);
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int32_t r = 0; r < ex->world; ++r) {
    if (r == ex->rank || ex->peer[r]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hb + static_cast<size_t>(r) * MANS_IPC_HANDLE_BYTES, sizeof h);
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return fail_cuda(e, "cudaIpcOpenMemHandle");
    ex->peer[r] = static_cast<int32_t*>(p);
  }
  cudaError_t e = cudaMemcpy(ex->d_peer, ex->peer.data(), ex->world * sizeof(int32_t*),
                             cudaMemcpyHostToDevice);
  return e == cudaSuccess ? MANS_OK : fail_cuda(e, "exchange peers");
}

int32_t mans_exchange_allgather(mans_exchange* ex, mans_workspace* ws, const int32_t* d_block,
                                int64_t nq, int32_t kin, int32_t k, float* d_out_dist,
                                uint32_t* d_out_ids, int32_t* d_out_counts, void* cuda_stream) {
  using namespace mans;
  if (!ex || !ws || !d_block) return fail(MANS_ERR_INVALID, "null exchange, workspace or block");
  if (nq <= 0 || kin <= 0 || k <= 0) return fail(MANS_ERR_INVALID, "bad merge shape");
  const int64_t words = 2 * nq * kin + nq;
  if (words > ex->stride) return fail(MANS_ERR_INVALID, "block larger than the exchange slots");
  for (int32_t r = 0; r < ex->world; ++r)
    if (!ex->peer[r]) return fail(MANS_ERR_INVALID, "exchange not opened to every rank");
  DeviceGuard g(ex->ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  int32_t rc;
  if ((rc = ws->err.reserve(sizeof(int))) != MANS_OK) return rc;
  if (!ws->err_cleared) {
    cudaError_t e = cudaMemsetAsync(ws->err.ptr, 0, sizeof(int), st);
    if (e != cudaSuccess) return fail_cuda(e, "cudaMemsetAsync(err)");
    ws->err_cleared = true;
  }
  const uint32_t epoch = ++ex->epoch;
  const int parity = static_cast<int>(epoch & 1u);
  cudaEvent_t st_stop = stage_begin(ws, st, MANS_STAGE_MERGE);
  publish_kernel<<<ex->world, 256, 0, st>>>(ex->d_peer, ex->rank, ex->world, ex->stride, d_block,
                                           words, parity, epoch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "publish launch");
  const int32_t* base = ex->local + static_cast<size_t>(parity) * ex->world * ex->stride;
  const int32_t kout = std::min<int32_t>(k, MANS_MAX_TOPK);
  MergeParams m{};
  m.in_dist = reinterpret_cast<const float*>(base);
  m.in_ids = reinterpret_cast<const uint32_t*>(base + nq * kin);
  m.in_counts = base + 2 * nq * kin;
  m.n_lists = ex->world;
  m.list_stride = ex->stride;
  m.kp_in = kin;
  m.nq = nq;
  m.k = kout;
  m.kp = pow2_at_least(kout);
  m.kout = kout;
  m.out_dist = d_out_dist;
  m.out_ids = d_out_ids;
  m.out_counts = d_out_counts;
  m.err = static_cast<int*>(ws->err.ptr);
  m.wait_flags = reinterpret_cast<const uint32_t*>(ex->local + flags_offset_words(ex->world, ex->stride)) +
                 parity * ex->world;
  m.wait_count = ex->world;
  m.wait_epoch = epoch;
  m.empty_on_error = true;  // a peer that never published: empty results, not a partial merge
  e = launch_merge(m, st);
  if (e != cudaSuccess) return fail_cuda(e, "exchange merge launch");
  timing_end(st_stop, st);
  ws->launches += 2;
  return MANS_OK;
}

int32_t mans_exchange_destroy(mans_exchange* ex) {
  using namespace mans;
  if (!ex) return MANS_OK;
  DeviceGuard g(ex->ctx->device);
  cudaDeviceSynchronize();
  for (int32_t r = 0; r < ex->world; ++r)
    if (r != ex->rank && ex->peer[r]) cudaIpcCloseMemHandle(ex->peer[r]);
  if (ex->d_peer) cudaFree(ex->d_peer);
  if (ex->local) cudaFree(ex->local);
  delete ex;
  return MANS_OK;
}

}  // extern "C"
