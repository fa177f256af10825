// tc.h -- parameters of the tensor-core (tcgen05) batched exact search.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mans {

// One pass of the bf16 candidate GEMM over rows [row0, row0 + rows).
struct TcParams {
  int64_t row0;
  int64_t rows;
  int64_t nq;
  int32_t dim;
  int32_t qblocks;          // ceil(nq / 128)
  int32_t groups;           // > 0: row groups walked in step by the query blocks
  int32_t stream_queries;   // 1: stream the query block with every stage instead of keeping it
  const float* row_beta;    // per-row additive term (L2: |r|^2), may be null
  const float* row_w;       // int8 pass: per-row factor of the integer dot
  const float* q_alpha;     // per-query additive term
  const float* q_gamma;     // per-query factor of the dot
  const float* q_c;         // filter constant in the score domain (filter mode)
  float* dense_out;         // dense mode: dense_out[q * dense_ld + (row - row0) / dense_group]
  int64_t dense_ld;
  int32_t dense_group;      // 1: every row's distance; 32: the minimum of each 32-row group
  uint64_t* cand;           // filter mode: (distance, row) keys, cand_cap per query
  int32_t* cand_count;
  int32_t cand_cap;
  int32_t cand_reserve;     // list slots a thread reserves per atomic (unused ones padded)
  int* err;
  // Fused sampling (sample_tiles > 0): each block first runs its first
  // sample_tiles tiles as a sample (32-row group minima into samp_out
  // [q][groups][sample_tiles][8]), meets the grid at a barrier, derives the
  // thresholds of a share of its block's queries, meets it again and then
  // runs its whole range filtered.  Needs a cooperative (co-resident) launch.
  int32_t sample_tiles;
  float* samp_out;
  int64_t samp_ld;              // groups * sample_tiles * 8
  unsigned long long* bar;      // grid barrier counter (monotonic across calls)
  unsigned long long bar_base;  // its value at launch
  int32_t k;
  const float* q_eps;
  const float* q_scale;
  float* thr_out;               // per query: sample k-th + 2 eps
  float* c_out;                 // per query: score-domain constant (also read as q_c)
  // Dynamic tail of a fused pass (pool != null): block c streams the static
  // tiles [c * static_tiles, (c + 1) * static_tiles), then claims tiles
  // pool_first + t, t = atomicAdd(pool, 1), while t < pool_tiles, so blocks
  // whose stream runs faster take more of the tail.  *pool is zeroed by the
  // query prep of the same search.
  unsigned long long* pool;
  int64_t static_tiles;
  int64_t pool_first;
  int64_t pool_tiles;
};

// Corpus-wide terms of the error bound (maxima over rows, rounded up).
struct TcCorpusStats {
  float max_norm;       // max |r|
  float max_resid;      // max |r - bf16(r)|
  float max_norm_bf16;  // max |bf16(r)|
  float min_norm;       // min |r|
  float max_sqnorm;     // max |r|^2 (L2)
};

}  // namespace mans
