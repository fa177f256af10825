/*
 * mans_cuda.h -- C ABI of the B200 search hot path for MetalANNS.
 *
 * This library replaces the Metal dispatch layer under MetalANNSCore's search
 * path: the exact flat scan with top-k, the IVF-flat probe-and-scan and the
 * IVF-PQ asymmetric-distance scoring.  Paths below are relative to the
 * MetalANNS source tree.
 *
 * Conventions (the style of Sources/MetalANNSC/include/MetalANNSC.h:13-38):
 *   - plain C, int64_t counts, caller-owned host inputs read only during the
 *     call, caller-owned outputs;
 *   - every function returns an int32_t status (MANS_OK == 0);
 *   - search results are sorted ascending by (distance, id): equal distances
 *     are ordered by ascending id (the GPU tier order pinned by
 *     Tests/MetalANNSTests/BoundedSelectionTests.swift:257-277), except IVF-PQ,
 *     which keeps the reference's newest-first rule (BoundedSelection.swift
 *     :158-214);
 *   - a result row holds kout = min(k, MANS_MAX_TOPK) entries; entries past
 *     out_counts[q] are (+inf, MANS_EMPTY_ID);
 *   - distances follow the reference's CPU exact path (ParallelFlatScan.swift
 *     :237-258): IP = -dot, L2 = max(0, |q|^2 - 2 dot + |v|^2), cosine =
 *     1 - dot / sqrt(|q|^2 |v|^2) (1 when the denominator is below 1e-10),
 *     with dot accumulated in the order of Sources/MetalANNSC/dots.c:40-47
 *     (one fp32 accumulator, index order, no fused multiply-add) and squared
 *     norms by the same sequential rule, so returned distances are bit-equal
 *     to the reference's x86-64 build of dots.c.
 *
 * Thread safety: every entry point may be called concurrently on one context
 * (each host-pointer call takes a private workspace and stream from a pool,
 * like FlatGPUSearch's FlatWorkspacePool, FlatGPUSearch.swift:1070-1139).
 * Objects must not be destroyed while calls that use them are running.
 */
#ifndef MANS_CUDA_H
#define MANS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__cplusplus)
extern "C" {
#endif

/* Metric codes, FlatGPUSearch.swift:134-140. */
#define MANS_METRIC_COSINE 0
#define MANS_METRIC_L2 1
#define MANS_METRIC_IP 2
#define MANS_METRIC_HAMMING 3

/* FlatGPUSearch.maxTopK (FlatGPUSearch.swift:13) and emptyID (:19). */
#define MANS_MAX_TOPK 256
#define MANS_EMPTY_ID 0xFFFFFFFFu

/* Status codes.  Each maps to one ANNSError case (Errors.swift:6-21); the
 * tier-degradeable ones (Errors.swift:23-30) are PIPELINE, OOM, EXEC, SEARCH. */
#define MANS_OK 0
#define MANS_ERR_DIM 1      /* dimensionMismatch(expected:got:) */
#define MANS_ERR_SEARCH 2   /* searchFailed(_:) */
#define MANS_ERR_PIPELINE 3 /* gpuPipelineUnavailable(_:) */
#define MANS_ERR_OOM 4      /* gpuResourceExhausted(_:) */
#define MANS_ERR_EXEC 5     /* gpuExecutionFailed(_:), includes device wait timeouts */
#define MANS_ERR_INVALID 6  /* constructionFailed(_:) (bad argument or handle) */
#define MANS_ERR_DEVICE 7   /* deviceNotSupported */
#define MANS_ERR_CORRUPT 8  /* corruptFile(_:) (index file loader) */

typedef struct mans_ctx mans_ctx;
typedef struct mans_corpus mans_corpus;
typedef struct mans_workspace mans_workspace;
typedef struct mans_ivf mans_ivf;
typedef struct mans_ivfpq mans_ivfpq;

/* ---- context ------------------------------------------------------------ */

/* Replaces `MetalContext()` creation (Sources/MetalANNSCore/MetalDevice.swift
 * :40-81, called at Sources/MetalANNS/ANNSIndex.swift:35 and IVFPQIndex.swift
 * :51).  Fails with MANS_ERR_DEVICE when `device` is not an sm_100 GPU, which
 * the caller treats like a nil MetalContext (host tiers only). */
int32_t mans_ctx_create(int32_t device, mans_ctx **out_ctx);
int32_t mans_ctx_destroy(mans_ctx *ctx);

/* One context over several GPUs of this process (the reference's one
 * MetalContext per index, ANNSIndex.swift:35, given all the GPUs of the
 * machine).  A corpus created or loaded on it (mans_corpus_create,
 * mans_corpus_load_mann) is split into contiguous row shards, one per device
 * in `devices` order (the first n % n_devices shards hold one extra row), and
 * mans_flat_search with host buffers searches every shard on its own GPU at
 * once: each GPU stores its shard's top-k over NVLink into the first GPU's
 * memory (peer access is enabled between the GPUs of the group), which merges
 * them by (distance, id) -- ParallelFlatScan.mergeSorted
 * (ParallelFlatScan.swift:288-315) over the shards.  Results equal the
 * single-GPU search of the whole corpus.  The corpus calls and
 * mans_flat_search accept such a context; the device-pointer calls, the
 * workspaces and the IVF / IVF-PQ objects need a single-device context
 * (MANS_ERR_INVALID).  Fails with MANS_ERR_DEVICE when a device is not an
 * sm_100 GPU or cannot reach the first device over peer access. */
int32_t mans_ctx_create_multi(const int32_t *devices, int32_t n_devices, mans_ctx **out_ctx);
/* Number of GPUs of a context (1 for mans_ctx_create). */
int32_t mans_ctx_device_count(const mans_ctx *ctx);

/* Message of the last failed call on the calling thread (NUL-terminated,
 * truncated to buf_len).  Replaces the String payloads of ANNSError. */
int32_t mans_last_error_message(char *buf, size_t buf_len);

/* Number of streaming multiprocessors of the context's device. */
int32_t mans_ctx_sm_count(const mans_ctx *ctx);

/* "sha256:<hex>" digest of the CUDA sources and headers this library was
 * built from (NUL-terminated, truncated to buf_len), so a deployment can tell
 * which sources a binary belongs to.  No reference counterpart. */
int32_t mans_build_info(char *buf, size_t buf_len);

/* Query batches of at least `min_batch` queries run on the tensor cores
 * (bf16 tcgen05 candidate GEMM with a certified error bound, then an exact
 * fp32 re-score, so results are identical to the exact scan); smaller batches
 * use the exact CUDA-core scan.  0 disables the tensor-core path.  Default 16.
 * No reference counterpart (the reference has one GPU tier,
 * FlatGPUSearch.swift:652-707). */
int32_t mans_ctx_set_tensor_core_batch(mans_ctx *ctx, int32_t min_batch);
/* (Batches smaller than min_batch also take that path when the corpus holds at
 * least 2^25 elements, where reading half the bytes outweighs its fixed cost.) */

/* Operand format of that path.  MANS_TC_BF16: bf16 rows; MANS_TC_INT8:
 * signed 8-bit codes quantised as the reference's int8 prefilter does
 * (Int8CodeBuffer.fill, Int8CodeCache.swift:64-99; query quantised as
 * BoundedExactScan.swift:52-64), half the bytes per row and a looser bound;
 * MANS_TC_AUTO (default): bf16 (on L2-normalised 384-d rows the int8 bound is
 * about 6x wider and its larger candidate sets cost more than the halved row
 * bytes save).  Results are identical to the exact scan in every format.  The
 * GPU counterpart of BoundedExactScan.search (BoundedExactScan.swift:30-122):
 * a bounded low-precision pass, then an exact fp32 re-score of the provable
 * candidates. */
#define MANS_TC_AUTO 0
#define MANS_TC_BF16 1
#define MANS_TC_INT8 2
int32_t mans_ctx_set_tensor_core_format(mans_ctx *ctx, int32_t format);

/* ---- corpus (VectorBuffer) --------------------------------------------- */

/* Uploads a row-major fp32 corpus (n x dim), the layout of VectorBuffer
 * (Sources/MetalANNSCore/VectorBuffer.swift:12-111) and of the zero-copy MANN
 * v3 vector section (MmapIndexLoader.swift:117-123), and computes the row
 * squared norms on the device (replaces the host norm cache of
 * FlatGPUSearch.withCorpusSquaredNorms, FlatGPUSearch.swift:465-521).
 * `id_offset` is added to every row index when results are reported (row
 * shards of one corpus use their first global row). */
int32_t mans_corpus_create(mans_ctx *ctx, const float *rows, int64_t n, int64_t dim,
                           uint32_t id_offset, mans_corpus **out_corpus);

/* Overwrites rows [start, start+count) and refreshes their norms; mirrors
 * VectorBuffer.insert + FlatGPUSearch.invalidateHostNormCache
 * (VectorBuffer.swift:44-51,77-91). */
int32_t mans_corpus_update_rows(mans_corpus *corpus, int64_t start, const float *rows,
                                int64_t count);
int32_t mans_corpus_destroy(mans_corpus *corpus);
int64_t mans_corpus_count(const mans_corpus *corpus);
int64_t mans_corpus_dim(const mans_corpus *corpus);

/* Host copy of the corpus's signed 8-bit codes (n x dim, row-major) and
 * per-row scales u, as Int8CodeBuffer.fill computes them
 * (Int8CodeCache.swift:64-99); either output may be null.  Builds the int8
 * copy on the device when it does not exist yet. */
int32_t mans_corpus_int8_codes(mans_corpus *corpus, int8_t *codes, float *scales);

/* ---- index files (loadReadOnly) ------------------------------------------ */

/* Header and section offsets of a reference index file (IndexSerializer
 * format versions 1-3, Sources/MetalANNSCore/IndexSerializer.swift:11-137;
 * version 3 is the page-aligned layout MmapIndexLoader maps,
 * MmapIndexLoader.swift:38-200). */
typedef struct {
  uint32_t version, count, degree, dim, metric, storage; /* storage 0 fp32, 1 fp16, 2 binary */
  uint32_t page_size;                                    /* version 3: the writer's page size */
  uint32_t idmap_bytes, entry_point;
  uint64_t vector_offset, vector_bytes, adjacency_offset, distance_offset, idmap_offset;
} mans_mann_info;

/* Parses and validates the file (the checks of IndexSerializer.load /
 * MmapIndexLoader.load); no GPU work.  MANS_ERR_CORRUPT on a bad file. */
int32_t mans_mann_read_info(const char *path, mans_mann_info *out);

/* ANNSIndex.loadReadOnly(.mmap)'s vector section into a device corpus: the
 * file is memory-mapped and rows [r0, r1) of shard `shard_index` of
 * `shard_count` (the first count % shard_count shards hold one extra row)
 * are uploaded with id_offset = r0; fp16 storage is widened to fp32 exactly;
 * binary storage fails with MANS_ERR_SEARCH.  The graph sections and the JSON
 * IDMap stay with the caller (mans_mann_read_info gives their offsets). */
int32_t mans_corpus_load_mann(mans_ctx *ctx, const char *path, int32_t shard_index,
                              int32_t shard_count, mans_corpus **out_corpus);

/* ---- workspaces (device-pointer calls) ---------------------------------- */

/* A workspace owns the scratch of one in-flight device-pointer search.  It
 * must not be used by two calls at once. */
int32_t mans_workspace_create(mans_ctx *ctx, mans_workspace **out_ws);
int32_t mans_workspace_destroy(mans_workspace *ws);
/* Waits for the stream of the last call made with `ws` and reports a device
 * side failure (MANS_ERR_EXEC) recorded by its kernels. */
int32_t mans_workspace_check(mans_workspace *ws, void *cuda_stream);
/* Number of queries of the last tensor-core search made with `ws` whose
 * certificate failed and that were re-scanned exactly (synchronises). */
int32_t mans_workspace_fallbacks(mans_workspace *ws, int32_t *out);
/* Path of the last flat search made with `ws`: 0 the exact CUDA-core scan,
 * 1 the bf16 tensor-core pass, 2 the int8 tensor-core pass (no reference
 * counterpart; for measurement). */
int32_t mans_workspace_last_path(mans_workspace *ws, int32_t *out);

/* Measurement hooks (no reference counterpart; the reference's benchmark CLI
 * times whole calls, Sources/MetalANNSBenchmarks/HotPathProfiler.swift:22-304).
 * `enable` bit 0: every later search made with `ws` brackets its dominant
 * kernel (the scan) with CUDA events on the launching stream;
 * mans_workspace_stats waits for them, returns the summed kernel time, the
 * number of timed launches and the number of library kernels enqueued, and
 * resets the counters.
 * `enable` bit 1: every stage of a flat search (MANS_STAGE_*: query prep,
 * sample pass, thresholds, the full pass or exact scan, the re-rank, and the
 * merges -- slot merge, shard merge, peer exchange) is bracketed the same
 * way; mans_workspace_stage_times waits for them and returns, per stage, the
 * summed time in ms and the number of timed launches, then resets.  Events
 * between the kernels keep the next kernel from launching early
 * (programmatic dependent launch), so the stages sum to a little more than
 * an untimed search. */
#define MANS_STAGE_QUERY_PREP 0
#define MANS_STAGE_SAMPLE 1
#define MANS_STAGE_THRESHOLD 2
#define MANS_STAGE_PASS 3
#define MANS_STAGE_RERANK 4
#define MANS_STAGE_MERGE 5
#define MANS_STAGES 6
int32_t mans_workspace_set_timing(mans_workspace *ws, int32_t enable);
int32_t mans_workspace_stats(mans_workspace *ws, double *kernel_ms, int64_t *kernel_launches,
                             int64_t *total_launches);
int32_t mans_workspace_stage_times(mans_workspace *ws, double *stage_ms, int64_t *stage_counts,
                                   int32_t n_stages);

/* ---- exact flat search -------------------------------------------------- */

/* Exact batched search, host buffers.  Replaces FlatGPUSearch.batchSearch's
 * GPU tier: runChunk's `flat_scan_distances` dispatch plus the host
 * selectTopK/boundedTopK (FlatGPUSearch.swift:103-181, 652-707, 786-933).
 * queries: nq x dim row-major; out_dist/out_ids: nq x kout; out_counts: nq.
 * Validation follows batchSearch: dim != corpus dim -> MANS_ERR_DIM; metric
 * hamming -> MANS_ERR_SEARCH; k <= 0 or an empty corpus -> all counts 0. */
int32_t mans_flat_search(mans_ctx *ctx, const mans_corpus *corpus, const float *queries,
                         int64_t nq, int64_t dim, int32_t k, int32_t metric, float *out_dist,
                         uint32_t *out_ids, int32_t *out_counts);

/* Same search with device pointers, enqueued on `cuda_stream` (a
 * cudaStream_t; NULL = legacy default stream) without synchronising.
 * Scratch comes from `ws`; call mans_workspace_check to surface device errors. */
int32_t mans_flat_search_device(mans_ctx *ctx, const mans_corpus *corpus, mans_workspace *ws,
                                const float *d_queries, int64_t nq, int32_t k, int32_t metric,
                                float *d_out_dist, uint32_t *d_out_ids, int32_t *d_out_counts,
                                void *cuda_stream);

/* Exact search with device pointers that allocates nothing.  No counterpart
 * in the reference: it exists for callers that may not allocate device
 * memory while searching -- a search recorded into a CUDA graph during stream
 * capture, a service whose device memory is owned by its own allocator, or a
 * latency-critical loop that cannot take cudaMalloc's implicit
 * synchronisation.  Results equal mans_flat_search_device.  Scratch is a
 * fixed 4 MiB __device__ array held by every GPU that loads the library until
 * exit.  One call needs 256 + round_up(4 S, 256) + 8 S kp bytes of it, with
 * S = G qb splits, qb = the smallest power of two >= nq capped at 8,
 * G = ceil(nq / qb), splits = min(max(1, SMs / G), ceil(n / 256)) and kp = the
 * smallest power of two >= min(k, 256, n) (so k = 129 costs as much as
 * k = 256); a request needing more fails with MANS_ERR_OOM and a message
 * naming the sizes.  The first call on a device resolves the array's
 * address (cudaGetSymbolAddress) and should come before any stream capture.
 * All calls on a device share the array: calls whose GPU work may overlap race
 * and must be serialised by the caller.  The call enqueues on `cuda_stream`
 * and returns argument and launch errors only; a device wait that timed out
 * (a stalled GPU) turns every query's result empty (count 0) instead of
 * leaving a partial top-k. */
int32_t mans_flat_search_noalloc(mans_ctx *ctx, const mans_corpus *corpus,
                                 const float *d_queries, int64_t nq, int32_t k, int32_t metric,
                                 float *d_out_dist, uint32_t *d_out_ids, int32_t *d_out_counts,
                                 void *cuda_stream);

/* Merges `n_lists` per-shard result blocks (each nq x kin, sorted ascending by
 * (distance, id)) into the global top-k per query, by (distance, id).  This is
 * the device form of ParallelFlatScan.mergeSorted (ParallelFlatScan.swift
 * :288-315) used after the all-gather of row-shard results.  Block l starts at
 * d_in_dist + l*list_stride, d_in_ids + l*list_stride and d_in_counts +
 * l*list_stride (elements of 4 bytes); list_stride 0 means the plain
 * list-major layout (dist/ids stride nq*kin, counts stride nq).  A packed
 * per-shard buffer [dist | ids | counts] lets one all-gather move all three.
 * Device pointers, async on the stream. */
int32_t mans_topk_merge_device(mans_ctx *ctx, mans_workspace *ws, const float *d_in_dist,
                               const uint32_t *d_in_ids, const int32_t *d_in_counts,
                               int32_t n_lists, int64_t list_stride, int64_t nq, int32_t kin,
                               int32_t k, float *d_out_dist, uint32_t *d_out_ids,
                               int32_t *d_out_counts, void *cuda_stream);

/* ---- peer-memory exchange (row shards on several GPUs) -------------------- */

/* All-gather of the per-shard packed top-k blocks [distances | ids | counts]
 * over NVLink peer memory, fused with the final (distance, id) merge -- the
 * exchange step of ParallelFlatScan.mergeSorted (ParallelFlatScan.swift:
 * 288-315) applied to row shards, without a collective library.  One
 * exchange per rank (one process per GPU): create it, share the 64-byte IPC
 * handle of every rank (any host channel), open, then every rank calls
 * allgather in the same order.  A rank whose peers do not publish within 2 s
 * gets MANS_ERR_EXEC from its next mans_workspace_check.  No reference
 * counterpart (the reference runs on one GPU). */
typedef struct mans_exchange mans_exchange;
#define MANS_IPC_HANDLE_BYTES 64
int32_t mans_exchange_create(mans_ctx *ctx, int32_t world, int32_t rank, int64_t max_block_words,
                             mans_exchange **out);
int32_t mans_exchange_handle(const mans_exchange *ex, void *out_handle);
/* handles: world x MANS_IPC_HANDLE_BYTES, rank order. */
int32_t mans_exchange_open(mans_exchange *ex, const void *handles);
/* d_block: this rank's packed block for nq queries of kin entries; outputs:
 * the merged top-min(k, 256) per query (device pointers, enqueued on the
 * stream). */
int32_t mans_exchange_allgather(mans_exchange *ex, mans_workspace *ws, const int32_t *d_block,
                                int64_t nq, int32_t kin, int32_t k, float *d_out_dist,
                                uint32_t *d_out_ids, int32_t *d_out_counts, void *cuda_stream);
int32_t mans_exchange_destroy(mans_exchange *ex);

/* ---- IVF-flat ------------------------------------------------------------ */

/* Uploads an IVF-flat partition in the layout of IVFFlatSearch.Partition
 * (Sources/MetalANNSCore/IVFFlatSearch.swift:39-95): `centroids` nlist x dim,
 * `packed_rows` n x dim with packed[p] = corpus[list_ids[p]], list p of
 * list_offsets[l]..list_offsets[l+1].  Centroid and packed-row squared norms
 * are computed on the device (the centroidNormSq / packedNormSq arrays). */
int32_t mans_ivf_create(mans_ctx *ctx, const float *centroids, int32_t nlist, int64_t dim,
                        const float *packed_rows, const uint32_t *list_ids,
                        const int64_t *list_offsets, int64_t n, mans_ivf **out_ivf);
int32_t mans_ivf_destroy(mans_ivf *ivf);
int64_t mans_ivf_list_count(const mans_ivf *ivf);

/* IVFFlatSearch.assignRows (IVFFlatSearch.swift:633-703) on the device: for
 * every row of `corpus` the list whose centroid (host, nlist x dim) has the
 * smallest host-tier key, ties to the lower list.  The row's dot with each
 * centroid uses the reference's sequential fp32 order (the reference calls
 * cblas_sgemm, whose order is closed).  out_assign: host, n entries. */
int32_t mans_ivf_assign(mans_ctx *ctx, mans_corpus *corpus, const float *centroids,
                        int32_t nlist, int32_t metric, int32_t *out_assign);
/* IVFFlatSearch.buildPartition after its k-means (IVFFlatSearch.swift:
 * 559-631): assignment as mans_ivf_assign, list sizes, offsets, list ids in
 * ascending row order per list, packed rows and norms -- all on the device,
 * from a corpus already uploaded; the result equals mans_ivf_create on the
 * host-built layout.  The list ids carry the corpus's id_offset, so a row
 * shard's partition reports global ids.  Centroid training (KMeans.cluster,
 * seeded by Swift's generator) stays with the caller. */
int32_t mans_ivf_build(mans_ctx *ctx, mans_corpus *corpus, const float *centroids,
                       int32_t nlist, int32_t metric, mans_ivf **out_ivf);
/* Host copy of the partition layout: offsets (nlist + 1) and list ids (n);
 * either may be null. */
int32_t mans_ivf_layout(const mans_ivf *ivf, int64_t *list_offsets, uint32_t *list_ids);

/* IVF-flat probe-and-scan, replacing IVFFlatSearch.search(query:partition:k:
 * nprobe:metric:) / scanProbedLists (IVFFlatSearch.swift:115-133, 214-291)
 * for a batch: nprobe is clamped to [1, nlist]; the nprobe lists with the
 * smallest centroid keys (ties to the lower list) are scanned exactly and the
 * top min(k, 256, candidates) are returned by (distance, id).  nprobe >= nlist
 * scans every list (exact).  256 < nprobe < nlist fails with MANS_ERR_SEARCH. */
int32_t mans_ivf_search(mans_ctx *ctx, mans_ivf *ivf, const float *queries, int64_t nq,
                        int64_t dim, int32_t k, int32_t nprobe, int32_t metric, float *out_dist,
                        uint32_t *out_ids, int32_t *out_counts);
int32_t mans_ivf_search_device(mans_ctx *ctx, mans_ivf *ivf, mans_workspace *ws,
                               const float *d_queries, int64_t nq, int32_t k, int32_t nprobe,
                               int32_t metric, float *d_out_dist, uint32_t *d_out_ids,
                               int32_t *d_out_counts, void *cuda_stream);

/* ---- IVF-PQ ---------------------------------------------------------------- */

/* Uploads a trained IVF-PQ index in the layout of _IVFPQIndex
 * (Sources/MetalANNS/IVFPQIndex.swift:6-35): coarse centroids nlist x dim,
 * codebooks m x ks x (dim/m) (GPUADCSearch.flattenCodebooks order,
 * GPUADCSearch.swift:194-205), codes n x m stored per internal id
 * (PQVectorBuffer, PQVectorBuffer.swift:26,34-51), and the inverted lists as
 * CSR (list l = lists[list_offsets[l] .. list_offsets[l+1]), in insertion
 * order).  ks must be 256 (IVFPQIndex.swift:45-47); metric 0/1/2.
 * list_positions (may be NULL) gives each entry's position in its full list
 * when this index holds one row shard of a larger one, so that insertion
 * order survives the cross-shard merge.  Candidates are ordered by a 32-bit
 * insertion sequence (probe rank, then list position), so a search with
 * nprobe p needs every list position below 2^(32 - ceil(log2 p)) (capped at
 * 2^31): lists of up to 2^27 entries at nprobe 32; beyond that the search
 * fails with MANS_ERR_SEARCH. */
int32_t mans_ivfpq_create(mans_ctx *ctx, const float *coarse, int32_t nlist, int64_t dim,
                          const float *codebooks, int32_t m, int32_t ks, const uint8_t *codes,
                          int64_t n, const int64_t *list_offsets, const uint32_t *lists,
                          const uint32_t *list_positions, int32_t metric, mans_ivfpq **out);
int32_t mans_ivfpq_destroy(mans_ivfpq *ix);

/* IVFPQIndex.add's encoding on the device: per vector the nearest coarse
 * centroid (nearestCoarseCentroid, IVFPQIndex.swift:514-550: SIMDDistance,
 * strict '<', first index wins) and the codes of the residual
 * (ProductQuantizer.encode(vector:subtracting:), ProductQuantizer.swift:
 * 120-169: sequential fp32 sum of ((v - c) - cb)^2 over the subspace, strict
 * '<').  vectors: host n x dim; coarse: nlist x dim; codebooks: m x ks x
 * (dim/m); out_codes: host n x m; out_assign (may be null): host n. */
int32_t mans_pq_encode(mans_ctx *ctx, const float *vectors, int64_t n, int64_t dim,
                       const float *coarse, int32_t nlist, const float *codebooks, int32_t m,
                       int32_t ks, int32_t metric, uint8_t *out_codes, int32_t *out_assign);

/* _IVFPQIndex.search(query:k:nprobe:) (IVFPQIndex.swift:177-226) for a batch:
 * coarse SIMDDistance ranking with newest-first ties, residual LUT
 * (ProductQuantizer.distanceTableFlattened) and sequential ADC sums per
 * probed list, merged with the BoundedSortedList rule.  out_ids are internal
 * ids; results are k wide (the reference's list has no cap beyond k): up to
 * k = 256 the candidates stay in on-chip top-k lists, above it every probed
 * entry's key is sorted per query in device memory (workspace scratch of
 * 16 bytes per probed entry).  A query of the wrong width yields an empty
 * result, as the reference returns []. */
int32_t mans_ivfpq_search(mans_ctx *ctx, mans_ivfpq *ix, const float *queries, int64_t nq,
                          int64_t dim, int32_t k, int32_t nprobe, float *out_dist,
                          uint32_t *out_ids, int32_t *out_counts);
int32_t mans_ivfpq_search_device(mans_ctx *ctx, mans_ivfpq *ix, mans_workspace *ws,
                                 const float *d_queries, int64_t nq, int32_t k, int32_t nprobe,
                                 float *d_out_dist, uint32_t *d_out_ids, int32_t *d_out_counts,
                                 void *cuda_stream);

/* Shards of one IVF-PQ index (one process per GPU; every shard holds the
 * same coarse centroids and codebooks, its entries' codes, and for each list
 * entry its position in the global list, `list_positions` of
 * mans_ivfpq_create).  A shard may hold row ranges (entries of every list)
 * or whole lists (the other lists empty: their distance tables are never
 * built, so the table work divides over the shards).  Each shard writes a packed block of nq*(3*kin + 1)
 * int32 words, kin = 2*min(k, 256): [scores | sequences | internal ids |
 * counts], its (score, insertion sequence) 2k-smallest candidates; after an
 * all-gather, mans_ivfpq_resolve_device merges the blocks (block r at
 * d_blocks + r*block_stride words) and applies the BoundedSortedList outcome
 * (BoundedSelection.swift:158-214) -- the same result as the unsharded
 * search, newest-first ties included.  No reference counterpart (one GPU). */
int32_t mans_ivfpq_search_partial_device(mans_ctx *ctx, mans_ivfpq *ix, mans_workspace *ws,
                                         const float *d_queries, int64_t nq, int32_t k,
                                         int32_t nprobe, int32_t *d_block, void *cuda_stream);
int32_t mans_ivfpq_resolve_device(mans_ctx *ctx, mans_workspace *ws, const int32_t *d_blocks,
                                  int32_t n_blocks, int64_t block_stride, int64_t nq, int32_t k,
                                  float *d_out_dist, uint32_t *d_out_ids, int32_t *d_out_counts,
                                  void *cuda_stream);

/* ---- index training (k-means) -------------------------------------------- */

/* KMeans.cluster's Lloyd iterations (Sources/MetalANNSCore/KMeans.swift:
 * 95-254) on the device, from the initial centroids the caller passes (the
 * reference seeds them by k-means++ with Swift's random number API,
 * KMeans.swift:256-328, which stays with the caller).  Row i's vector is
 * vectors[i*row_stride + offset .. + dim) (host; offset/dim select a subspace,
 * as KMeans.clusterSubspace does).  Each iteration assigns every row to the
 * centroid of smallest SIMDDistance (`metric`, strict '<', first minimum
 * wins), stops when no assignment changed, else sets every non-empty cluster
 * to sum * (1 / count) in fp32.  `workers` is the reference's
 * activeProcessorCount: with workers > 1, n >= 512 and k >= 8 the rows are
 * summed in `workers` chunks of ceil(n / workers) rows, added in chunk order
 * (useParallelLloyd), otherwise in one running sum -- the same fp32 order, so
 * centroids and assignments are bit-equal to the reference's Lloyd loop run
 * with that many cores.  centroids: host k x dim, read and overwritten;
 * out_assignments (may be null): host n, the last assignment;
 * out_iterations (may be null): centroid updates performed.  Validation
 * follows KMeans.cluster: n = 0 or k outside [1, n] -> MANS_ERR_INVALID. */
int32_t mans_kmeans_lloyd(mans_ctx *ctx, const float *vectors, int64_t n, int64_t row_stride,
                          int64_t offset, int64_t dim, int32_t k, int32_t max_iterations,
                          int32_t metric, int32_t workers, float *centroids,
                          int32_t *out_assignments, int32_t *out_iterations);

/* ProductQuantizer.train (Sources/MetalANNSCore/ProductQuantizer.swift:10-86)
 * from initial codebooks: for each of the m subspaces of `vectors` (host,
 * n x dim), mans_kmeans_lloyd with L2, k = ks = 256 and `max_iterations`.
 * codebooks: host m x ks x (dim/m), read and overwritten (the
 * GPUADCSearch.flattenCodebooks order, GPUADCSearch.swift:194-205).  Checks of
 * the reference: ks must be 256, n >= 256, dim divisible by m. */
int32_t mans_pq_train(mans_ctx *ctx, const float *vectors, int64_t n, int64_t dim, int32_t m,
                      int32_t ks, int32_t max_iterations, int32_t workers, float *codebooks);

/* GPUADCSearch.computeDistances(context:query:pq:packedCodes:vectorCount:
 * flatCodebooks:) (GPUADCSearch.swift:35-173): squared-L2 LUT of `query`
 * against the codebooks (pq_compute_distance_table) and the sequential sum
 * per code (pq_adc_scan).  Codes >= ks -> MANS_ERR_SEARCH, as the reference's
 * validation; count == 0 -> nothing written. */
int32_t mans_pq_adc_list(mans_ctx *ctx, const float *query, int64_t dim, const float *codebooks,
                         int32_t m, int32_t ks, const uint8_t *codes, int64_t count,
                         float *out_dist);

#if defined(__cplusplus)
}
#endif

#endif /* MANS_CUDA_H */
