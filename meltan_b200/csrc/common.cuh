// common.cuh -- device helpers shared by the search kernels (sm_100a).
//
// mbarrier / TMA wrappers are thin inline-PTX shims.  Every wait is bounded by
// the global nanosecond timer: a wait that runs past kWaitLimitNs records
// kErrTimeout in the launch's error word and returns false, so no kernel can
// spin forever.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace mans {

constexpr int kMaxTopK = 256;
constexpr uint32_t kEmptyId = 0xFFFFFFFFu;
constexpr uint64_t kKeyMax = ~0ull;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

enum Metric : int { kCosine = 0, kL2 = 1, kIP = 2, kHamming = 3 };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ---------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false (and
// records kErrTimeout) when kWaitLimitNs passes first.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u && global_ns() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, kErrTimeout);
      return false;
    }
  }
}

// ---- TMA ----------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Contiguous bulk copy global -> shared (no multicast) completing on `bar`.
// Both addresses 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- rows staged one per lane ---------------------------------------------------
//
// A warp stages up to 32 rows into shared memory with one bulk copy per lane
// (a row pitch of ld + 4 floats puts the rows of a quarter-warp 4 banks apart,
// so their 16-byte reads hit distinct banks), and each lane scores its row.

// dot(q_i, row) for i < nq (independent chains), each in index order with
// separately rounded multiply and add; the staged row and the queries are
// zero past dim, and adding +0 leaves a sum that started at +0 unchanged.
template <int NQ>
__device__ __forceinline__ void row_dots(const float* srow, const float* q, int qw, int nq, int ld,
                                         float (&acc)[NQ]) {
#pragma unroll
  for (int i = 0; i < NQ; ++i) acc[i] = 0.0f;
  const float4* r4 = reinterpret_cast<const float4*>(srow);
#pragma unroll 4
  for (int c = 0; c < ld / 4; ++c) {
    const float4 v = r4[c];
#pragma unroll
    for (int i = 0; i < NQ; ++i) {
      if (i >= nq) break;
      const float4 b = reinterpret_cast<const float4*>(q + i * qw)[c];
      float a = acc[i];
      a = __fadd_rn(a, __fmul_rn(v.x, b.x));
      a = __fadd_rn(a, __fmul_rn(v.y, b.y));
      a = __fadd_rn(a, __fmul_rn(v.z, b.z));
      a = __fadd_rn(a, __fmul_rn(v.w, b.w));
      acc[i] = a;
    }
  }
}

// Stages row src (ld floats, 16-byte aligned) into dst with one bulk copy
// that completes on `bar` (one barrier per staged row).  The proxy fence orders this thread's earlier
// reads of dst before the copy overwrites it.
__device__ __forceinline__ void stage_row(float* dst, const float* src, int ld, uint64_t* bar) {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  const uint32_t bytes = static_cast<uint32_t>(ld) * 4;
  mbar_arrive_expect_tx(bar, bytes);
  bulk_load(dst, src, bytes, bar);
}

// Waits for this lane's staged row (lanes without a row pass); false for the
// whole warp when a wait gave up, after one more bounded wait for the copy.
__device__ __forceinline__ bool wait_row(uint64_t* bar, uint32_t ph, bool has_row, int* err) {
  const bool ok = !has_row || mbar_wait_bounded(bar, ph, err);
  if (__any_sync(0xFFFFFFFFu, !ok)) {
    if (has_row && ok == false) mbar_wait_bounded(bar, ph, nullptr);
    return false;
  }
  return true;
}

// ---- programmatic dependent launch ----------------------------------------------
//
// A kernel launched with programmatic stream serialization may start while the
// previous kernel on the stream still runs; pdl_wait() blocks until that kernel
// has completed and its memory is visible (a no-op for a plain launch).
// pdl_trigger() lets the next such kernel start once every block of this one
// has issued it or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- named barriers -----------------------------------------------------------

__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- (distance, id) keys ---------------------------------------------------------
//
// A 64-bit key orders candidates by (distance, id): the high word is the
// distance mapped to an order-preserving unsigned integer, the low word the id.
// -0.0 is folded onto +0.0 first so that keys order exactly like float `<`
// (which treats the two zeros as equal, leaving the id to break the tie).

__device__ __forceinline__ uint32_t float_to_ordered(float f) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float ordered_to_float(uint32_t o) {
  uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
  return __uint_as_float(u);
}

__device__ __forceinline__ uint64_t make_key(float d, uint32_t id) {
  return (static_cast<uint64_t>(float_to_ordered(d)) << 32) | id;
}

__device__ __forceinline__ float key_distance(uint64_t key) {
  return ordered_to_float(static_cast<uint32_t>(key >> 32));
}

__device__ __forceinline__ uint32_t key_id(uint64_t key) { return static_cast<uint32_t>(key); }

// ---- metric finalize ---------------------------------------------------------------
//
// The reference CPU exact path (ParallelFlatScan.swift:237-258,
// IVFFlatSearch.swift:293-311) with every operation rounded on its own:
//   IP     : -dot
//   L2     : max(0, (qn - 2*dot) + vn)
//   cosine : denom = sqrt(qn*vn); denom < 1e-10 ? 1 : 1 - dot/denom

__device__ __forceinline__ float finalize_distance(int metric, float dot, float qn, float vn) {
  if (metric == kIP) return -dot;
  if (metric == kL2) {
    float t = __fadd_rn(__fsub_rn(qn, __fmul_rn(2.0f, dot)), vn);
    return t > 0.0f ? t : 0.0f;
  }
  float denom = __fsqrt_rn(__fmul_rn(qn, vn));
  if (denom < 1e-10f) return 1.0f;
  return __fsub_rn(1.0f, __fdiv_rn(dot, denom));
}

// SIMDDistance semantics (SIMDDistance.swift:17-80): `acc` is sum((q-v)^2)
// for L2 and dot(q, v) otherwise; cosine divides by sqrt(|q|^2)*sqrt(|v|^2).
__device__ __forceinline__ float finalize_simd(int metric, float acc, float qn, float vn) {
  if (metric == kL2) return acc;
  if (metric == kIP) return -acc;
  float denom = __fmul_rn(__fsqrt_rn(qn), __fsqrt_rn(vn));
  if (denom < 1e-10f) return 1.0f;
  return __fsub_rn(1.0f, __fdiv_rn(acc, denom));
}

// ---- block bitonic sort over shared-memory keys -------------------------------------
//
// Sorts n (a power of two) keys ascending with NT threads that share named
// barrier `bar_id`.  The caller synchronises before the call; the call ends
// with a barrier.
template <int NT>
__device__ __forceinline__ void bitonic_sort_keys(uint64_t* a, int n, int tid, int bar_id) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n; i += NT) {
        int ixj = i ^ j;
        if (ixj > i) {
          uint64_t x = a[i], y = a[ixj];
          bool up = (i & k) == 0;
          if ((x > y) == up) {
            a[i] = y;
            a[ixj] = x;
          }
        }
      }
      named_sync(bar_id, NT);
    }
  }
}

// ---- warp sort of one key per lane -------------------------------------------------

__device__ __forceinline__ uint64_t key_min(uint64_t a, uint64_t b) { return a < b ? a : b; }
__device__ __forceinline__ uint64_t key_max(uint64_t a, uint64_t b) { return a < b ? b : a; }

// Ascending bitonic sort of one key per lane.
__device__ __forceinline__ uint64_t warp_sort32(uint64_t x, int lane) {
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const uint64_t y = __shfl_xor_sync(0xFFFFFFFFu, x, j);
      x = (((lane & j) == 0) == ((lane & k) == 0)) ? key_min(x, y) : key_max(x, y);
    }
  return x;
}

// ---- warp-resident top-k of 64-bit keys (at most 32 kept) ----------------

// The 32 smallest of two ascending lane-sorted lists, ascending: the lane-wise
// minimum of t and x reversed is a bitonic sequence holding them, which a
// half-cleaner cascade sorts.
__device__ __forceinline__ uint64_t warp_merge32(uint64_t t, uint64_t x, int lane) {
  uint64_t y = key_min(t, __shfl_sync(0xFFFFFFFFu, x, 31 - lane));
#pragma unroll
  for (int j = 16; j > 0; j >>= 1) {
    const uint64_t z = __shfl_xor_sync(0xFFFFFFFFu, y, j);
    y = (lane & j) == 0 ? key_min(y, z) : key_max(y, z);
  }
  return y;
}

// Offers one key per lane to the warp's ascending list of its k smallest keys
// (lane i holds the (i+1)-th; `kth` is the warp-uniform k-th key, kept
// current): a batch where more than six keys beat the k-th is sorted by
// shuffles and merged in, fewer are inserted one by one at their rank (keys
// are distinct; a key that no longer beats the k-th after an earlier
// insertion lands at rank k or drops out, which is harmless).
__device__ __forceinline__ void warp_topk_offer(uint64_t& best, uint64_t& kth, uint64_t key,
                                                int k, int lane) {
  uint32_t pass = __ballot_sync(0xFFFFFFFFu, key < kth);
  if (!pass) return;
  if (__popc(pass) > 6) {
    best = warp_merge32(best, warp_sort32(key < kth ? key : kKeyMax, lane), lane);
  } else {
    while (pass) {
      const int src = __ffs(pass) - 1;
      pass &= pass - 1;
      const uint64_t x = __shfl_sync(0xFFFFFFFFu, key, src);
      const int at = __popc(__ballot_sync(0xFFFFFFFFu, best < x));
      const uint64_t up = __shfl_up_sync(0xFFFFFFFFu, best, 1);
      best = lane < at ? best : (lane == at ? x : up);
    }
  }
  kth = __shfl_sync(0xFFFFFFFFu, best, k - 1);
}

// Running top-k of one query inside a thread block:
//   buf[0, kp)      -- the current best keys (ascending, `nbest` of them valid)
//   buf[kp, sortn)  -- an append queue of candidates below the threshold
// merge() sorts both regions together and keeps the first k keys.
struct TopKState {
  uint64_t* buf;
  int* qcount;  // queue fill
  int* nbest;   // valid best keys (<= k)
  uint64_t* thr;  // k-th best key, or kKeyMax while fewer than k are known
};

template <int NT>
__device__ __forceinline__ void topk_merge(TopKState s, int k, int kp, int sortn, int tid,
                                           int bar_id) {
  int qc = *s.qcount;
  int nb = *s.nbest;
  // sort only the occupied prefix, rounded up to a power of two
  int n = kp;
  while (n < kp + qc) n <<= 1;
  if (n > sortn) n = sortn;
  for (int i = tid; i < n; i += NT) {
    bool keep = (i < nb) || (i >= kp && i < kp + qc);
    if (!keep) s.buf[i] = kKeyMax;
  }
  named_sync(bar_id, NT);
  bitonic_sort_keys<NT>(s.buf, n, tid, bar_id);
  if (tid == 0) {
    int total = nb + qc;
    int keep = total < k ? total : k;
    *s.nbest = keep;
    *s.qcount = 0;
    *s.thr = keep == k ? s.buf[k - 1] : kKeyMax;
  }
  named_sync(bar_id, NT);
}

// Appends `key` to the queue when it beats the threshold.  Warp-aggregated:
// one shared atomic per warp and query.
__device__ __forceinline__ void topk_offer(TopKState s, int kp, uint64_t key, bool valid) {
  bool pass = valid && key < *s.thr;
  unsigned mask = __ballot_sync(0xFFFFFFFFu, pass);
  if (mask == 0) return;
  int lane = threadIdx.x & 31;
  int leader = __ffs(mask) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(s.qcount, __popc(mask));
  base = __shfl_sync(0xFFFFFFFFu, base, leader);
  if (pass) {
    int pos = base + __popc(mask & ((1u << lane) - 1u));
    s.buf[kp + pos] = key;
  }
}

// Exclusive prefix sum of in[0, n) into out[0, n] by the whole block (at
// most 1024 threads; part: 64 ints of shared memory).
__device__ inline void block_exclusive_scan(const int32_t* in, int n, int32_t* out, int32_t* part) {
  const int t = threadIdx.x, nt = blockDim.x;
  const int per = (n + nt - 1) / nt;
  const int b = t * per;
  const int e = min(n, b + per);
  int32_t sum = 0;
  for (int i = b; i < e; ++i) sum += in[i];
  // warp-level inclusive scan of the per-thread sums, then across warps
  const int lane = t & 31, w = t >> 5;
  int32_t v = sum;
  for (int o = 1; o < 32; o <<= 1) {
    int32_t u = __shfl_up_sync(0xFFFFFFFFu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) part[w] = v;
  __syncthreads();
  if (w == 0) {
    int32_t x = lane < (nt >> 5) ? part[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      int32_t u = __shfl_up_sync(0xFFFFFFFFu, x, o);
      if (lane >= o) x += u;
    }
    part[32 + lane] = x;  // inclusive warp totals
  }
  __syncthreads();
  int32_t acc = v - sum + (w > 0 ? part[32 + w - 1] : 0);
  for (int i = b; i < e; ++i) {
    out[i] = acc;
    acc += in[i];
  }
  if (t == nt - 1) out[n] = acc;
  __syncthreads();
}

}  // namespace mans
