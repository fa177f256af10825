/*
 * mans_oracle.c -- CPU restatement of the MetalANNS search hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library in meltan_b200/: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  Nothing in
 * the product path calls into it.
 *
 * Every function restates the reference algorithm it cites (paths are
 * relative to the MetalANNS source tree).  Floating-point rules:
 *   - built with -ffp-contract=off, so `a + b * c` rounds the product and the
 *     sum separately, exactly like Swift (which never contracts) and like the
 *     scalar branch of Sources/MetalANNSC/dots.c:40-47 on x86-64;
 *   - Apple Accelerate calls in the reference (vDSP_dotpr, vDSP_vsq +
 *     cblas_sgemv, vDSP_distancesq, cblas_sgemm) have a closed summation
 *     order; they are restated as sequential fp32 sums (index 0 first).
 *
 * Parity pins: orc_dot_rows_seq is checked bit-for-bit against the
 * reference's own mans_f32_dot_rows compiled from dots.c (oracle/build.py
 * -> oracle/_ref/), and the generators / tie rules against the reference
 * tests' own restated brute force (tests/golden/).
 */
#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_COSINE 0
#define ORC_L2 1
#define ORC_IP 2
#define ORC_HAMMING 3
#define ORC_MAX_TOPK 256 /* FlatGPUSearch.maxTopK, FlatGPUSearch.swift:13 */

typedef void (*orc_dot_rows_fn)(const float *corpus, const float *query, int64_t rows,
                                int64_t dim, float *out);

/* ------------------------------------------------------------------------ */
/* Generators                                                                */
/* ------------------------------------------------------------------------ */

/* Portable LCG of Tests/MetalANNSTests/FlatSearchTests.swift:15-22 (and
 * ExactSearchIntegrationTests.swift:23-30): 24 bits of state>>33 mapped to
 * [-1, 1] with fp32 divide, multiply by 2, subtract 1. */
void orc_lcg_vectors(uint64_t seed, int64_t count, int64_t dim, float *out) {
    uint64_t state = seed;
    for (int64_t i = 0; i < count * dim; ++i) {
        state = state * 6364136223846793005ULL + 1442695040888963407ULL;
        float u = (float)((state >> 33) & 0xFFFFFFULL) / (float)0xFFFFFF;
        out[i] = u * 2.0f - 1.0f;
    }
}

/* Variant of Tests/MetalANNSTests/BoundedExactScanTests.swift:23-34: seed is
 * scrambled first and 32 bits of state>>33 are used (the Float conversions
 * round, as Swift's Float(UInt64) does). */
void orc_lcg32_vectors(uint64_t seed, int64_t count, int64_t dim, float *out) {
    uint64_t state = seed * 0x9E3779B97F4A7C15ULL + 0xD1B54A32D192ED03ULL;
    for (int64_t i = 0; i < count * dim; ++i) {
        state = state * 6364136223846793005ULL + 1442695040888963407ULL;
        float u = (float)((state >> 33) & 0xFFFFFFFFULL) / (float)0xFFFFFFFFULL;
        out[i] = u * 2.0f - 1.0f;
    }
}

/* ------------------------------------------------------------------------ */
/* Int8 codes (Sources/MetalANNSCore/Int8CodeCache.swift:64-99)              */
/* ------------------------------------------------------------------------ */

/* Int8CodeBuffer.fill: per row, maxAbs (exact), scale = maxAbs / 127 (1 for a
 * zero row), inverse = 1 / scale, code = Int32(v * inverse +- 0.5) (the
 * conversion truncates toward zero, so this rounds half away from zero),
 * clamped to +-127; every step in fp32. */
void orc_int8_fill(const float *rows, int64_t n, int64_t dim, int8_t *codes, float *scales) {
    for (int64_t r = 0; r < n; ++r) {
        const float *v = rows + r * dim;
        float max_abs = 0.0f;
        for (int64_t d = 0; d < dim; ++d) {
            float a = fabsf(v[d]);
            if (a > max_abs) max_abs = a;
        }
        float scale = max_abs > 0.0f ? max_abs / 127.0f : 1.0f;
        float inverse = 1.0f / scale;
        for (int64_t d = 0; d < dim; ++d) {
            float scaled = v[d] * inverse;
            float shifted = scaled >= 0.0f ? scaled + 0.5f : scaled - 0.5f;
            int32_t rounded = (int32_t)shifted;
            if (rounded > 127) rounded = 127;
            else if (rounded < -127) rounded = -127;
            codes[r * dim + d] = (int8_t)rounded;
        }
        scales[r] = scale;
    }
}

/* ------------------------------------------------------------------------ */
/* Dot products (Sources/MetalANNSC/dots.c)                                   */
/* ------------------------------------------------------------------------ */

/* Scalar branch of mans_f32_dot_rows (dots.c:40-47): one fp32 accumulator,
 * index order, product rounded before the add. */
void orc_dot_rows_seq(const float *corpus, const float *query, int64_t rows, int64_t dim,
                      float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *row = corpus + r * dim;
        float acc = 0.0f;
        for (int64_t d = 0; d < dim; ++d) {
            float p = row[d] * query[d];
            acc = acc + p;
        }
        out[r] = acc;
    }
}

/* arm64 branch of mans_f32_dot_rows (dots.c:14-37) for dim >= 16, dim % 4 == 0:
 * sixteen fused-multiply-add lanes (lane s takes columns = s mod 16), the
 * 4-wide tail folds into lanes 0..3, then acc0+(acc1+(acc2+acc3)) per lane,
 * (l0+l2, l1+l3) and the final pair add.  Other shapes take the scalar order.
 * Restated with fmaf so it runs on any host; it cannot be executed against
 * the NEON original on this machine (x86-64). */
void orc_dot_rows_neon(const float *corpus, const float *query, int64_t rows, int64_t dim,
                       float *out) {
    if (!(dim >= 16 && (dim & 3) == 0)) {
        orc_dot_rows_seq(corpus, query, rows, dim, out);
        return;
    }
    for (int64_t r = 0; r < rows; ++r) {
        const float *row = corpus + r * dim;
        float acc[16];
        for (int s = 0; s < 16; ++s) acc[s] = 0.0f;
        int64_t d = 0;
        for (; d + 16 <= dim; d += 16)
            for (int s = 0; s < 16; ++s) acc[s] = fmaf(row[d + s], query[d + s], acc[s]);
        for (; d < dim; d += 4)
            for (int s = 0; s < 4; ++s) acc[s] = fmaf(row[d + s], query[d + s], acc[s]);
        float v[4];
        for (int s = 0; s < 4; ++s) v[s] = acc[s] + (acc[4 + s] + (acc[8 + s] + acc[12 + s]));
        float lo0 = v[0] + v[2];
        float lo1 = v[1] + v[3];
        out[r] = lo0 + lo1;
    }
}

/* Squared norm of one vector, sequential fp32 (FlatGPUSearch.swift:532-535,
 * hostScan's query norm; also stands in for the closed vDSP order of
 * vDSP_vsq+cblas_sgemv at :484-501 and vDSP_dotpr at IVFFlatSearch.swift:226). */
float orc_norm_sq(const float *v, int64_t dim) {
    float s = 0.0f;
    for (int64_t d = 0; d < dim; ++d) {
        float p = v[d] * v[d];
        s = s + p;
    }
    return s;
}

void orc_row_norms(const float *corpus, int64_t n, int64_t dim, float *out) {
    for (int64_t r = 0; r < n; ++r) out[r] = orc_norm_sq(corpus + r * dim, dim);
}

/* Host-tier metric finalize, ParallelFlatScan.swift:237-258 and
 * IVFFlatSearch.swift:293-311: IP = -dot; L2 = max(0, qn - 2dot + vn);
 * cosine = 1 - dot / sqrt(qn*vn), 1 when the denominator is below 1e-10. */
float orc_distance(int metric, float dot, float qn, float vn) {
    switch (metric) {
    case ORC_IP:
        return -dot;
    case ORC_L2: {
        float t = qn - 2.0f * dot;
        t = t + vn;
        return t > 0.0f ? t : 0.0f;
    }
    case ORC_COSINE: {
        float denom = sqrtf(qn * vn);
        if (denom < 1e-10f) return 1.0f;
        return 1.0f - dot / denom;
    }
    default:
        return FLT_MAX;
    }
}

/* ------------------------------------------------------------------------ */
/* (distance, id) ordering helpers                                            */
/* ------------------------------------------------------------------------ */

typedef struct {
    float d;
    uint32_t id;
} orc_pair;

static int pair_less(orc_pair a, orc_pair b) {
    return a.d < b.d || (a.d == b.d && a.id < b.id);
}

/* Bounded max-heap under the strict (distance, id) total order: the same
 * admission rule as IVFFlatSearch.TopKHeap (IVFFlatSearch.swift:384-444). */
typedef struct {
    orc_pair *e;
    int size, cap;
} orc_lexheap;

static void lexheap_push(orc_lexheap *h, orc_pair p) {
    if (h->cap <= 0) return;
    if (h->size < h->cap) {
        int pos = h->size++;
        h->e[pos] = p;
        while (pos > 0) {
            int parent = (pos - 1) / 2;
            if (pair_less(h->e[parent], h->e[pos])) {
                orc_pair t = h->e[parent];
                h->e[parent] = h->e[pos];
                h->e[pos] = t;
                pos = parent;
            } else {
                break;
            }
        }
    } else if (pair_less(p, h->e[0])) {
        h->e[0] = p;
        int pos = 0;
        for (;;) {
            int l = 2 * pos + 1, r = l + 1, big = pos;
            if (l < h->size && pair_less(h->e[big], h->e[l])) big = l;
            if (r < h->size && pair_less(h->e[big], h->e[r])) big = r;
            if (big == pos) break;
            orc_pair t = h->e[big];
            h->e[big] = h->e[pos];
            h->e[pos] = t;
            pos = big;
        }
    }
}

static int cmp_pair(const void *a, const void *b) {
    orc_pair x = *(const orc_pair *)a, y = *(const orc_pair *)b;
    if (pair_less(x, y)) return -1;
    if (pair_less(y, x)) return 1;
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Exact flat search (the product's result contract)                           */
/* ------------------------------------------------------------------------ */

/* Exact top-k under the strict (distance, id) order, the ordering the GPU tier
 * reports (FlatGPUSearch.swift:917-932 sorts ties by id; BoundedSelectionTests
 * .swift:257-277 pins it).  k is capped at min(k, 256, n) as batchSearch does
 * (FlatGPUSearch.swift:130).  `dot_rows` selects the summation order (NULL =
 * orc_dot_rows_seq); norms may be NULL for IP.  Output rows are kout = min(k,
 * 256) wide; unused tail slots hold (+inf, 0xFFFFFFFF). */
void orc_flat_search(const float *corpus, const float *norms, int64_t n, int64_t dim,
                     const float *queries, int64_t nq, int32_t k, int32_t metric,
                     orc_dot_rows_fn dot_rows, float *out_d, uint32_t *out_i,
                     int32_t *out_count) {
    int kout = k < ORC_MAX_TOPK ? k : ORC_MAX_TOPK;
    int keff = (int64_t)kout < n ? kout : (int)n;
    if (!dot_rows) dot_rows = orc_dot_rows_seq;
    float *dots = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    orc_pair *heap = (orc_pair *)malloc(sizeof(orc_pair) * (size_t)(keff > 0 ? keff : 1));
    for (int64_t q = 0; q < nq; ++q) {
        const float *qv = queries + q * dim;
        float qn = (metric == ORC_COSINE || metric == ORC_L2) ? orc_norm_sq(qv, dim) : 0.0f;
        orc_lexheap h = {heap, 0, keff};
        if (n > 0) dot_rows(corpus, qv, n, dim, dots);
        for (int64_t r = 0; r < n; ++r) {
            float vn = norms ? norms[r] : 0.0f;
            orc_pair p = {orc_distance(metric, dots[r], qn, vn), (uint32_t)r};
            lexheap_push(&h, p);
        }
        qsort(heap, (size_t)h.size, sizeof(orc_pair), cmp_pair);
        for (int i = 0; i < kout; ++i) {
            out_d[q * kout + i] = i < h.size ? heap[i].d : INFINITY;
            out_i[q * kout + i] = i < h.size ? heap[i].id : 0xFFFFFFFFu;
        }
        out_count[q] = h.size;
    }
    free(dots);
    free(heap);
}

/* ------------------------------------------------------------------------ */
/* ParallelFlatScan (the reference CPU exact path; CPU baseline)              */
/* ------------------------------------------------------------------------ */

typedef struct {
    float d;
    uint32_t id;
} orc_entry;

/* Distance-only max-heap of ParallelFlatScan.selectTopK (ParallelFlatScan.
 * swift:188-263): strict `<` admission against the root, sift on distance
 * alone, so ties keep heap-dependent order. */
static void pfs_append(orc_entry *e, int *count, int topk, float d, uint32_t id) {
    if (*count < topk) {
        int pos = (*count)++;
        e[pos].d = d;
        e[pos].id = id;
        while (pos > 0) {
            int parent = (pos - 1) / 2;
            if (e[pos].d > e[parent].d) {
                orc_entry t = e[pos];
                e[pos] = e[parent];
                e[parent] = t;
                pos = parent;
            } else {
                break;
            }
        }
    } else if (d < e[0].d) {
        e[0].d = d;
        e[0].id = id;
        int pos = 0;
        for (;;) {
            int l = 2 * pos + 1, r = l + 1, big = pos;
            if (l < *count && e[l].d > e[big].d) big = l;
            if (r < *count && e[r].d > e[big].d) big = r;
            if (big == pos) break;
            orc_entry t = e[pos];
            e[pos] = e[big];
            e[big] = t;
            pos = big;
        }
    }
}

/* heapSortedAscending, ParallelFlatScan.swift:266-285. */
static void pfs_heap_sorted_ascending(orc_entry *e, int count) {
    while (count > 1) {
        orc_entry t = e[0];
        e[0] = e[count - 1];
        e[count - 1] = t;
        count -= 1;
        int pos = 0;
        for (;;) {
            int l = 2 * pos + 1, r = l + 1, big = pos;
            if (l < count && e[l].d > e[big].d) big = l;
            if (r < count && e[r].d > e[big].d) big = r;
            if (big == pos) break;
            orc_entry u = e[pos];
            e[pos] = e[big];
            e[big] = u;
            pos = big;
        }
    }
}

typedef struct {
    const float *query, *corpus, *norms;
    float qn;
    int64_t dim, n, chunk;
    int topk, metric;
    orc_dot_rows_fn dot_rows;
    float *dots;
    orc_entry *results; /* slices x topk */
    int *counts;
    int slice;
} pfs_work;

static void pfs_run_slice(pfs_work *w) {
    int64_t start = (int64_t)w->slice * w->chunk;
    int64_t end = start + w->chunk < w->n ? start + w->chunk : w->n;
    w->counts[w->slice] = 0;
    if (start >= end) return;
    int64_t rows = end - start;
    float *dots = w->dots + start;
    w->dot_rows(w->corpus + start * w->dim, w->query, rows, w->dim, dots);
    orc_entry *e = w->results + (size_t)w->slice * w->topk;
    int count = 0;
    for (int64_t r = 0; r < rows; ++r) {
        float vn = w->norms ? w->norms[start + r] : 0.0f;
        pfs_append(e, &count, w->topk, orc_distance(w->metric, dots[r], w->qn, vn),
                   (uint32_t)(start + r));
    }
    pfs_heap_sorted_ascending(e, count);
    w->counts[w->slice] = count;
}

static void *pfs_thread(void *arg) {
    pfs_run_slice((pfs_work *)arg);
    return NULL;
}

/* ParallelFlatScan.search (ParallelFlatScan.swift:96-155) for one query:
 * slices = max(1, min(cores, 32, n / 2048)) (:84-88), one heap per slice, then
 * the k-way mergeSorted (:288-315) that takes the lowest slice on ties.
 * Returns the number of entries written (min(topk, n)). */
int orc_parallel_flat_scan(const float *query, const float *corpus, const float *norms,
                           float qn, int64_t n, int64_t dim, int32_t topk, int32_t metric,
                           int32_t cores, orc_dot_rows_fn dot_rows, float *out_d,
                           uint32_t *out_i) {
    if (n <= 0 || topk <= 0) return 0;
    if (!dot_rows) dot_rows = orc_dot_rows_seq;
    int k = (int64_t)topk < n ? topk : (int)n;
    int64_t by_work = n / 2048 > 1 ? n / 2048 : 1;
    int64_t slices = cores;
    if (slices > 32) slices = 32;
    if (slices > by_work) slices = by_work;
    if (slices < 1) slices = 1;
    int64_t chunk = (n + slices - 1) / slices;
    float *dots = (float *)malloc(sizeof(float) * (size_t)(slices * chunk));
    orc_entry *res = (orc_entry *)malloc(sizeof(orc_entry) * (size_t)(slices * k));
    int *counts = (int *)calloc((size_t)slices, sizeof(int));
    pfs_work *work = (pfs_work *)malloc(sizeof(pfs_work) * (size_t)slices);
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)slices);
    for (int64_t s = 0; s < slices; ++s) {
        pfs_work w = {query, corpus, norms, qn, dim, n, chunk, k, metric, dot_rows,
                      dots, res, counts, (int)s};
        work[s] = w;
    }
    if (slices == 1) {
        pfs_run_slice(&work[0]);
    } else {
        for (int64_t s = 0; s < slices; ++s) pthread_create(&th[s], NULL, pfs_thread, &work[s]);
        for (int64_t s = 0; s < slices; ++s) pthread_join(th[s], NULL);
    }
    /* mergeSorted: repeatedly take the strictly smallest head, lowest slice
     * first on ties; +inf heads are never taken (bestDistance starts at inf).
     * With a single non-empty list the list prefix is returned as is. */
    int *cursor = (int *)calloc((size_t)slices, sizeof(int));
    int written = 0;
    int live = 0, live_slice = 0;
    for (int64_t s = 0; s < slices; ++s)
        if (counts[s] > 0) {
            live += 1;
            live_slice = (int)s;
        }
    if (live == 1 && slices > 1) {
        written = counts[live_slice] < k ? counts[live_slice] : k;
        for (int i = 0; i < written; ++i) {
            out_d[i] = res[(size_t)live_slice * k + i].d;
            out_i[i] = res[(size_t)live_slice * k + i].id;
        }
        written = -written - 1; /* marks "done" for the loop below */
    }
    while (written >= 0 && written < k) {
        int best = -1;
        float best_d = INFINITY;
        for (int64_t s = 0; s < slices; ++s) {
            if (cursor[s] < counts[s]) {
                float c = res[(size_t)s * k + cursor[s]].d;
                if (c < best_d) {
                    best_d = c;
                    best = (int)s;
                }
            }
        }
        if (best < 0) break;
        orc_entry e = res[(size_t)best * k + cursor[best]];
        out_d[written] = e.d;
        out_i[written] = e.id;
        cursor[best] += 1;
        written += 1;
    }
    if (written < 0) written = -written - 1;
    if (slices == 1) {
        /* single-slice path returns the slice list itself (mergeSorted is not
         * called, ParallelFlatScan.swift:110-115) */
        written = counts[0] < k ? counts[0] : k;
        for (int i = 0; i < written; ++i) {
            out_d[i] = res[i].d;
            out_i[i] = res[i].id;
        }
    }
    free(cursor);
    free(th);
    free(work);
    free(counts);
    free(res);
    free(dots);
    return written;
}

/* GPU-tier host selection over one distance row, FlatGPUSearch.boundedTopK
 * (FlatGPUSearch.swift:849-933): distance-only max-heap with strict `<`
 * admission, root-first extraction reversed, then a (distance, id) sort when
 * any tie exists.  Returns the count written. */
int orc_gpu_tier_topk(const float *row, int64_t count, int32_t topk, float *out_d,
                      uint32_t *out_i) {
    if (count <= 0 || topk <= 0) return 0;
    orc_entry *h = (orc_entry *)malloc(sizeof(orc_entry) * (size_t)topk);
    int size = 0;
    for (int64_t i = 0; i < count; ++i) pfs_append(h, &size, topk, row[i], (uint32_t)i);
    /* root-first extraction gives descending order; reversing yields the same
     * sequence as heapSortedAscending on this heap. */
    pfs_heap_sorted_ascending(h, size);
    int ties = 0;
    for (int i = 1; i < size; ++i)
        if (h[i].d == h[i - 1].d) ties = 1;
    orc_pair *p = (orc_pair *)malloc(sizeof(orc_pair) * (size_t)(size > 0 ? size : 1));
    for (int i = 0; i < size; ++i) {
        p[i].d = h[i].d;
        p[i].id = h[i].id;
    }
    if (ties) qsort(p, (size_t)size, sizeof(orc_pair), cmp_pair);
    for (int i = 0; i < size; ++i) {
        out_d[i] = p[i].d;
        out_i[i] = p[i].id;
    }
    free(p);
    free(h);
    return size;
}

/* ------------------------------------------------------------------------ */
/* IVF-flat (Sources/MetalANNSCore/IVFFlatSearch.swift)                       */
/* ------------------------------------------------------------------------ */

/* assignRows (IVFFlatSearch.swift:633-703): per row the metric key against
 * every centroid (row norm as the "query" norm, centroid norm as the row
 * norm), smallest key wins, ties to the lower cluster.  cblas_sgemm's dot
 * order is closed; dots here are sequential. */
void orc_ivf_assign(const float *corpus, const float *row_norms, int64_t n, int64_t dim,
                    const float *centroids, const float *centroid_norms, int32_t nlist,
                    int32_t metric, int32_t *out_assign) {
    float *dots = (float *)malloc(sizeof(float) * (size_t)nlist);
    for (int64_t r = 0; r < n; ++r) {
        orc_dot_rows_seq(centroids, corpus + r * dim, nlist, dim, dots);
        int best = 0;
        float best_key = FLT_MAX;
        for (int c = 0; c < nlist; ++c) {
            float key = orc_distance(metric, dots[c], row_norms[r], centroid_norms[c]);
            if (key < best_key || (key == best_key && c < best)) {
                best_key = key;
                best = c;
            }
        }
        out_assign[r] = best;
    }
    free(dots);
}

/* Counting-sort layout of buildPartition (IVFFlatSearch.swift:583-614):
 * list sizes -> offsets (nlist+1), list ids in ascending row order, packed
 * rows and packed norms gathered through the ids. */
void orc_ivf_layout(const float *corpus, const float *row_norms, int64_t n, int64_t dim,
                    const int32_t *assign, int32_t nlist, int64_t *offsets, uint32_t *list_ids,
                    float *packed, float *packed_norms) {
    for (int c = 0; c <= nlist; ++c) offsets[c] = 0;
    for (int64_t r = 0; r < n; ++r) offsets[assign[r] + 1] += 1;
    for (int c = 0; c < nlist; ++c) offsets[c + 1] += offsets[c];
    int64_t *write_at = (int64_t *)malloc(sizeof(int64_t) * (size_t)(nlist > 0 ? nlist : 1));
    for (int c = 0; c < nlist; ++c) write_at[c] = offsets[c];
    for (int64_t r = 0; r < n; ++r) list_ids[write_at[assign[r]]++] = (uint32_t)r;
    for (int64_t p = 0; p < n; ++p) {
        memcpy(packed + p * dim, corpus + (int64_t)list_ids[p] * dim, sizeof(float) * (size_t)dim);
        packed_norms[p] = row_norms[list_ids[p]];
    }
    free(write_at);
}

/* smallestIndices (IVFFlatSearch.swift:314-382): the `count` smallest keys
 * with ties to the lower index, returned sorted by (key, index). */
static int ivf_smallest(const float *keys, int nkeys, int count, int *out) {
    int limit = count < nkeys ? count : nkeys;
    if (limit <= 0) return 0;
    orc_pair *h = (orc_pair *)malloc(sizeof(orc_pair) * (size_t)limit);
    orc_lexheap heap = {h, 0, limit};
    for (int i = 0; i < nkeys; ++i) {
        orc_pair p = {keys[i], (uint32_t)i};
        lexheap_push(&heap, p);
    }
    qsort(h, (size_t)heap.size, sizeof(orc_pair), cmp_pair);
    for (int i = 0; i < heap.size; ++i) out[i] = (int)h[i].id;
    int sz = heap.size;
    free(h);
    return sz;
}

static int cmp_int(const void *a, const void *b) {
    int x = *(const int *)a, y = *(const int *)b;
    return (x > y) - (x < y);
}

/* scanProbedLists (IVFFlatSearch.swift:214-291) with the search() clamps of
 * :115-133 (k <- min(k, n), nprobe <- clamp to [1, nlist]): centroid keys,
 * nprobe smallest (ties to lower list), probed lists visited in ascending
 * list id, TopKHeap over (distance, id), output sorted by (distance, id).
 * Output rows are min(k, 256) wide; out_count = min(k, candidates). */
void orc_ivf_search(const float *centroids, const float *centroid_norms, int32_t nlist,
                    const float *packed, const float *packed_norms, const uint32_t *list_ids,
                    const int64_t *offsets, int64_t n, int64_t dim, const float *queries,
                    int64_t nq, int32_t k, int32_t nprobe, int32_t metric, float *out_d,
                    uint32_t *out_i, int32_t *out_count) {
    int kout = k < ORC_MAX_TOPK ? k : ORC_MAX_TOPK;
    int probe = nprobe < 1 ? 1 : (nprobe > nlist ? nlist : nprobe);
    float *cdots = (float *)malloc(sizeof(float) * (size_t)nlist);
    float *ckeys = (float *)malloc(sizeof(float) * (size_t)nlist);
    int *probed = (int *)malloc(sizeof(int) * (size_t)nlist);
    float *dots = (float *)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    orc_pair *heap = (orc_pair *)malloc(sizeof(orc_pair) * (size_t)(kout > 0 ? kout : 1));
    for (int64_t q = 0; q < nq; ++q) {
        const float *qv = queries + q * dim;
        for (int i = 0; i < kout; ++i) {
            out_d[q * kout + i] = INFINITY;
            out_i[q * kout + i] = 0xFFFFFFFFu;
        }
        out_count[q] = 0;
        if (k <= 0 || n <= 0) continue;
        float qn = (metric == ORC_COSINE || metric == ORC_L2) ? orc_norm_sq(qv, dim) : 0.0f;
        orc_dot_rows_seq(centroids, qv, nlist, dim, cdots);
        for (int c = 0; c < nlist; ++c) ckeys[c] = orc_distance(metric, cdots[c], qn, centroid_norms[c]);
        int np = ivf_smallest(ckeys, nlist, probe, probed);
        qsort(probed, (size_t)np, sizeof(int), cmp_int);
        int64_t cand = 0;
        for (int i = 0; i < np; ++i) cand += offsets[probed[i] + 1] - offsets[probed[i]];
        if (cand == 0) continue;
        int kk = kout < (int64_t)n ? kout : (int)n;
        int topk = (int64_t)kk < cand ? kk : (int)cand;
        orc_lexheap h = {heap, 0, topk};
        for (int i = 0; i < np; ++i) {
            int64_t start = offsets[probed[i]];
            int64_t rows = offsets[probed[i] + 1] - start;
            if (rows <= 0) continue;
            orc_dot_rows_seq(packed + start * dim, qv, rows, dim, dots);
            for (int64_t l = 0; l < rows; ++l) {
                orc_pair p = {orc_distance(metric, dots[l], qn, packed_norms[start + l]),
                              list_ids[start + l]};
                lexheap_push(&h, p);
            }
        }
        qsort(heap, (size_t)h.size, sizeof(orc_pair), cmp_pair);
        for (int i = 0; i < h.size; ++i) {
            out_d[q * kout + i] = heap[i].d;
            out_i[q * kout + i] = heap[i].id;
        }
        out_count[q] = h.size;
    }
    free(heap);
    free(dots);
    free(probed);
    free(ckeys);
    free(cdots);
}

/* ------------------------------------------------------------------------ */
/* IVF-PQ (Sources/MetalANNS/IVFPQIndex.swift, ProductQuantizer.swift)        */
/* ------------------------------------------------------------------------ */

/* SIMDDistance.distance for one pair (SIMDDistance.swift:17-80,131-160) with
 * sequential sums in place of vDSP: cosine via sqrt(na)*sqrt(nb), squared L2,
 * IP = -dot. */
float orc_simd_distance(const float *a, const float *b, int64_t dim, int32_t metric) {
    if (metric == ORC_L2) {
        if (dim <= 0) return 0.0f;
        float s = 0.0f;
        for (int64_t d = 0; d < dim; ++d) {
            float t = a[d] - b[d];
            float p = t * t;
            s = s + p;
        }
        return s;
    }
    if (metric == ORC_IP) {
        if (dim <= 0) return 0.0f;
        float s = 0.0f;
        for (int64_t d = 0; d < dim; ++d) {
            float p = a[d] * b[d];
            s = s + p;
        }
        return -s;
    }
    if (metric == ORC_COSINE) {
        if (dim <= 0) return 1.0f;
        float dot = 0.0f, na = 0.0f, nb = 0.0f;
        for (int64_t d = 0; d < dim; ++d) {
            float p = a[d] * b[d];
            dot = dot + p;
        }
        na = orc_norm_sq(a, dim);
        nb = orc_norm_sq(b, dim);
        float denom = sqrtf(na) * sqrtf(nb);
        return denom < 1e-10f ? 1.0f : 1.0f - dot / denom;
    }
    return FLT_MAX;
}

/* distanceTableFlattened (ProductQuantizer.swift:223-253): LUT[m*ks + c] =
 * SIMDDistance.distance(query sub-vector m, codebook[m][c]). */
void orc_pq_lut(const float *query, const float *codebooks, int32_t m, int32_t ks,
                int32_t sub, int32_t metric, float *out) {
    for (int32_t s = 0; s < m; ++s)
        for (int32_t c = 0; c < ks; ++c)
            out[s * ks + c] = orc_simd_distance(query + (int64_t)s * sub,
                                                codebooks + ((int64_t)s * ks + c) * sub, sub, metric);
}

/* encode(vector:subtracting:) (ProductQuantizer.swift:120-169): per subspace
 * argmin over centroids of the sequential sum of ((v - c) - cb)^2, strict `<`
 * (first index wins on ties). */
void orc_pq_encode_subtracting(const float *v, const float *centroid, const float *codebooks,
                               int32_t m, int32_t ks, int32_t sub, uint8_t *out) {
    for (int32_t s = 0; s < m; ++s) {
        int best = 0;
        float best_d = FLT_MAX;
        for (int32_t c = 0; c < ks; ++c) {
            const float *cb = codebooks + ((int64_t)s * ks + c) * sub;
            float sum = 0.0f;
            for (int32_t d = 0; d < sub; ++d) {
                float delta = v[s * sub + d] - centroid[s * sub + d];
                delta = delta - cb[d];
                float p = delta * delta;
                sum = sum + p;
            }
            if (sum < best_d) {
                best_d = sum;
                best = c;
            }
        }
        out[s] = (uint8_t)best;
    }
}

/* nearestCoarseCentroid (IVFPQIndex.swift:514-550): strict `<`, first wins. */
int32_t orc_nearest_coarse(const float *v, const float *coarse, int32_t nlist, int64_t dim,
                           int32_t metric) {
    int best = 0;
    float best_d = FLT_MAX;
    for (int32_t c = 0; c < nlist; ++c) {
        float d = orc_simd_distance(v, coarse + (int64_t)c * dim, dim, metric);
        if (d < best_d) {
            best_d = d;
            best = c;
        }
    }
    return best;
}

/* KMeans.cluster's Lloyd iterations (Sources/MetalANNSCore/KMeans.swift:
 * 95-254) from given initial centroids (the k-means++ seeding, :256-328,
 * stays with the caller).  Row i's sub-vector is vectors[i*stride + offset ..
 * + dim).  Per iteration: every row goes to the centroid of smallest
 * SIMDDistance (strict `<` from FLT_MAX: the first minimum wins); the loop
 * stops before the update when no assignment changed; otherwise each
 * non-empty cluster becomes sum * (1 / count).  With workers > 1, n >= 512
 * and k >= 8 the reference splits the rows into `workers` chunks of
 * ceil(n / workers) (useParallelLloyd, :89-90,103-190): each chunk sums its
 * rows per cluster in row order from 0, and the chunk sums are added to the
 * cluster total in chunk order; otherwise one running sum per cluster in row
 * order (:191-233) -- the same as a single chunk.  All sums are fp32.
 * Returns the number of centroid updates; assign[i] is the last assignment. */
int32_t orc_kmeans_lloyd(const float *vectors, int64_t n, int64_t stride, int64_t offset,
                         int64_t dim, int32_t k, int32_t max_iter, int32_t metric,
                         int32_t workers, float *centroids, int32_t *assign) {
    int64_t W = workers < 1 ? 1 : workers;
    if (W > n) W = n;
    if (!(W > 1 && n >= 512 && k >= 8)) W = 1;
    const int64_t chunk = (n + W - 1) / W;
    float *sums = (float *)calloc((size_t)(W * k * dim), sizeof(float));
    int64_t *counts = (int64_t *)calloc((size_t)(W * k), sizeof(int64_t));
    int32_t updates = 0;
    for (int64_t i = 0; i < n; ++i) assign[i] = -1;
    for (int32_t it = 0; it < max_iter; ++it) {
        memset(sums, 0, sizeof(float) * (size_t)(W * k * dim));
        memset(counts, 0, sizeof(int64_t) * (size_t)(W * k));
        int changed = 0;
        for (int64_t i = 0; i < n; ++i) {
            const float *v = vectors + i * stride + offset;
            int32_t best = 0;
            float best_d = FLT_MAX;
            for (int32_t c = 0; c < k; ++c) {
                float d = orc_simd_distance(v, centroids + (int64_t)c * dim, dim, metric);
                if (d < best_d) {
                    best_d = d;
                    best = c;
                }
            }
            if (assign[i] != best) changed = 1;
            assign[i] = best;
            const int64_t w = i / chunk;
            counts[w * k + best] += 1;
            float *acc = sums + (w * k + best) * dim;
            for (int64_t d = 0; d < dim; ++d) acc[d] = acc[d] + v[d];
        }
        if (!changed) break;
        for (int32_t c = 0; c < k; ++c) {
            int64_t cnt = 0;
            for (int64_t w = 0; w < W; ++w) cnt += counts[w * k + c];
            if (cnt == 0) continue;
            const float scale = 1.0f / (float)cnt;
            for (int64_t d = 0; d < dim; ++d) {
                float total = 0.0f;
                for (int64_t w = 0; w < W; ++w) total = total + sums[(w * k + c) * dim + d];
                centroids[(int64_t)c * dim + d] = total * scale;
            }
        }
        ++updates;
    }
    free(sums);
    free(counts);
    return updates;
}

/* BoundedSortedList (BoundedSelection.swift:158-214) over (score, payload):
 * best-first by score; an equal-score newcomer is rejected when the list is
 * full and otherwise placed ahead of earlier equal scores (lowerBound). */
typedef struct {
    float s;
    uint32_t a; /* payload: cluster index or internal id */
} orc_scored;

static void bsl_insert(orc_scored *list, int *count, int cap, orc_scored x) {
    if (cap <= 0) return;
    if (*count >= cap && !(x.s < list[*count - 1].s)) return;
    int lo = 0, hi = *count;
    while (lo < hi) {
        int mid = (lo + hi) / 2;
        if (list[mid].s < x.s)
            lo = mid + 1;
        else
            hi = mid;
    }
    int last = *count < cap ? *count : cap - 1;
    for (int i = last; i > lo; --i) list[i] = list[i - 1];
    list[lo] = x;
    if (*count < cap) *count += 1;
}

/* _IVFPQIndex.search (IVFPQIndex.swift:177-226): probe = clamp(nprobe, 1,
 * nlist); coarse centroids ranked by SIMDDistance in a BoundedSortedList
 * (:484-512); for each probed cluster in that order the residual q - c
 * (:366-368), the LUT over the residual and the sequential ADC sum
 * (cpuADCDistances, :418-452), each candidate inserted in list order into a
 * BoundedSortedList of capacity k.  `lists`/`list_offsets` are the inverted
 * lists in insertion order (internal ids); `codes` is row-major [id][m].
 * Output rows are k wide: the list has no cap beyond k (IVFPQIndex.swift:197). */
void orc_ivfpq_search(const float *coarse, int32_t nlist, int64_t dim, const float *codebooks,
                      int32_t m, int32_t ks, const uint8_t *codes, const int64_t *list_offsets,
                      const uint32_t *lists, const float *queries, int64_t nq, int32_t k,
                      int32_t nprobe, int32_t metric, float *out_d, uint32_t *out_i,
                      int32_t *out_count) {
    int kout = k > 0 ? k : 0;
    int32_t sub = (int32_t)(dim / m);
    int probe = nprobe < 1 ? 1 : (nprobe > nlist ? nlist : nprobe);
    orc_scored *closest = (orc_scored *)malloc(sizeof(orc_scored) * (size_t)probe);
    orc_scored *merged = (orc_scored *)malloc(sizeof(orc_scored) * (size_t)(kout > 0 ? kout : 1));
    float *resid = (float *)malloc(sizeof(float) * (size_t)dim);
    float *lut = (float *)malloc(sizeof(float) * (size_t)m * ks);
    for (int64_t q = 0; q < nq; ++q) {
        const float *qv = queries + q * dim;
        for (int i = 0; i < kout; ++i) {
            out_d[q * kout + i] = INFINITY;
            out_i[q * kout + i] = 0xFFFFFFFFu;
        }
        out_count[q] = 0;
        if (k <= 0 || nlist <= 0) continue;
        int nc = 0;
        for (int32_t c = 0; c < nlist; ++c) {
            orc_scored x = {orc_simd_distance(qv, coarse + (int64_t)c * dim, dim, metric), (uint32_t)c};
            bsl_insert(closest, &nc, probe, x);
        }
        int nm = 0;
        for (int p = 0; p < nc; ++p) {
            int32_t c = (int32_t)closest[p].a;
            for (int64_t d = 0; d < dim; ++d) resid[d] = qv[d] - coarse[(int64_t)c * dim + d];
            orc_pq_lut(resid, codebooks, m, ks, sub, metric, lut);
            for (int64_t j = list_offsets[c]; j < list_offsets[c + 1]; ++j) {
                uint32_t id = lists[j];
                const uint8_t *code = codes + (int64_t)id * m;
                float total = 0.0f;
                for (int32_t s = 0; s < m; ++s) total = total + lut[s * ks + code[s]];
                orc_scored x = {total, id};
                bsl_insert(merged, &nm, kout, x);
            }
        }
        for (int i = 0; i < nm; ++i) {
            out_d[q * kout + i] = merged[i].s;
            out_i[q * kout + i] = merged[i].a;
        }
        out_count[q] = nm;
    }
    free(lut);
    free(resid);
    free(merged);
    free(closest);
}

/* pq_adc_scan / cpuADCDistances for one list (PQDistance.metal:32-66,
 * IVFPQIndex.swift:418-452): sequential sum of LUT entries over m; a code
 * >= ks yields FLT_MAX. */
void orc_pq_adc(const float *lut, int32_t m, int32_t ks, const uint8_t *codes, int64_t count,
                float *out) {
    for (int64_t i = 0; i < count; ++i) {
        float total = 0.0f;
        for (int32_t s = 0; s < m; ++s) {
            int c = codes[i * m + s];
            if (c >= ks) {
                total = FLT_MAX;
                break;
            }
            total = total + lut[s * ks + c];
        }
        out[i] = total;
    }
}

/* ------------------------------------------------------------------------ */
/* BoundedExactScan: the int8-prefiltered exact scan of the CPU batch route   */
/* (Sources/MetalANNSCore/BoundedExactScan.swift, Int8CodeCache.swift,        */
/* FlatGPUSearch.swift:754-779,1024-1035)                                     */
/* ------------------------------------------------------------------------ */

typedef void (*orc_i8_dot_rows_fn)(const int8_t *codes, const int8_t *query_codes, int64_t rows,
                                   int64_t dim, float *out);
typedef void (*orc_dot_gather_fn)(const float *corpus, const float *query, const uint32_t *ids,
                                  int64_t count, int64_t dim, float *out);

/* Portable branch of mans_i8_dot_rows_f32 (dots.c:50-88): exact int32 sum,
 * one conversion to fp32. */
void orc_i8_dot_rows(const int8_t *codes, const int8_t *query_codes, int64_t rows, int64_t dim,
                     float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const int8_t *row = codes + r * dim;
        int32_t total = 0;
        for (int64_t d = 0; d < dim; ++d) total += (int32_t)row[d] * (int32_t)query_codes[d];
        out[r] = (float)total;
    }
}

/* Scalar branch of mans_f32_dot_rows_gather (dots.c:90-125). */
void orc_dot_rows_gather(const float *corpus, const float *query, const uint32_t *ids,
                         int64_t count, int64_t dim, float *out) {
    for (int64_t i = 0; i < count; ++i) {
        const float *row = corpus + (int64_t)ids[i] * dim;
        float acc = 0.0f;
        for (int64_t d = 0; d < dim; ++d) {
            float p = row[d] * query[d];
            acc = acc + p;
        }
        out[i] = acc;
    }
}

/* Int8CodeBuffer.fill (Int8CodeCache.swift:64-99): the codes of orc_int8_fill
 * plus the planes u = scale, w = scale * eBase with eBase = (|c|_1 / 2 +
 * dim / 4) * (1 + 1e-6) + 16, the sequential fp32 |v|^2 and 1 / sqrt(|v|^2)
 * (0 below 1e-20); every step in fp32. */
void orc_int8_planes(const float *rows, int64_t n, int64_t dim, int8_t *codes, float *u,
                     float *w, float *norm_sq, float *inv_sqrt) {
    for (int64_t r = 0; r < n; ++r) {
        const float *v = rows + r * dim;
        float max_abs = 0.0f;
        for (int64_t d = 0; d < dim; ++d) {
            float a = fabsf(v[d]);
            if (a > max_abs) max_abs = a;
        }
        float scale = max_abs > 0.0f ? max_abs / 127.0f : 1.0f;
        float inverse = 1.0f / scale;
        int32_t abs_sum = 0;
        float nsq = 0.0f;
        for (int64_t d = 0; d < dim; ++d) {
            float value = v[d];
            float p = value * value;
            nsq = nsq + p;
            float scaled = value * inverse;
            float shifted = scaled >= 0.0f ? scaled + 0.5f : scaled - 0.5f;
            int32_t rounded = (int32_t)shifted;
            if (rounded > 127) rounded = 127;
            else if (rounded < -127) rounded = -127;
            codes[r * dim + d] = (int8_t)rounded;
            abs_sum += rounded < 0 ? -rounded : rounded;
        }
        float ebase = ((float)abs_sum / 2.0f + (float)dim / 4.0f) * (1.0f + 1e-6f) + 16.0f;
        u[r] = scale;
        w[r] = scale * ebase;
        norm_sq[r] = nsq;
        inv_sqrt[r] = nsq > 1e-20f ? 1.0f / sqrtf(nsq) : 0.0f;
    }
}

typedef struct {
    float key;
    uint32_t id;
} bes_entry;

/* admit / siftUpHeap / siftDownHeap (BoundedExactScan.swift:238-276): a
 * key-only max-heap, a newcomer replaces the root only when strictly lower. */
static void bes_sift_down(bes_entry *h, int pos, int size) {
    for (;;) {
        int l = 2 * pos + 1, r = l + 1, big = pos;
        if (l < size && h[l].key > h[big].key) big = l;
        if (r < size && h[r].key > h[big].key) big = r;
        if (big == pos) return;
        bes_entry t = h[pos];
        h[pos] = h[big];
        h[big] = t;
        pos = big;
    }
}

static void bes_admit(bes_entry *h, int *count, int cap, float key, uint32_t id) {
    if (*count < cap) {
        int pos = (*count)++;
        h[pos].key = key;
        h[pos].id = id;
        while (pos > 0) {
            int parent = (pos - 1) / 2;
            if (h[pos].key > h[parent].key) {
                bes_entry t = h[pos];
                h[pos] = h[parent];
                h[parent] = t;
                pos = parent;
            } else {
                break;
            }
        }
    } else if (key < h[0].key) {
        h[0].key = key;
        h[0].id = id;
        bes_sift_down(h, 0, *count);
    }
}

/* heapSortedAscending (:279-288). */
static void bes_sorted_ascending(bes_entry *h, int count) {
    while (count > 1) {
        bes_entry t = h[0];
        h[0] = h[count - 1];
        h[count - 1] = t;
        count -= 1;
        bes_sift_down(h, 0, count);
    }
}

static int cmp_entry(const void *a, const void *b) {
    const orc_entry *x = (const orc_entry *)a, *y = (const orc_entry *)b;
    if (x->d < y->d) return -1;
    if (y->d < x->d) return 1;
    return x->id < y->id ? -1 : (x->id > y->id ? 1 : 0);
}

/* BoundedExactScan.search (:30-122) for one query, its slices run in turn
 * (the caller parallelises over queries, as parallelHostBatchSearch does).
 * The query is quantised in double (:52-64); each slice ranks its rows by the
 * metric's lower-bound key (:178-228, same operation order and types) in a
 * heap of min(budget, chunk); the slices' ascending lists are merged
 * (:290-316, lowest slice first on equal keys) into `budget` candidates whose
 * last key is the cutoff; the candidates are rescored in fp32 with the
 * ParallelFlatScan formulas (:320-369) and sorted; the result is proven when
 * cutoff >= tau + max(1e-7, |tau| 1e-6) (tau = k-th rescored distance) or
 * every row is a candidate, else the budget grows x4.  Swift's sort of the
 * rescored entries is unstable; here equal distances order by id.
 * Returns the count written, or -1 where the reference returns nil (fewer
 * than 16384 rows, hamming, or missing norms for cosine / L2). */
int orc_bounded_exact_scan(const float *query, const float *corpus, const float *norms, float qn,
                           int64_t n, int64_t dim, int32_t topk, int32_t metric, int32_t slices_in,
                           const int8_t *codes, const float *u, const float *w,
                           const float *norm_sq, const float *inv_sqrt, orc_i8_dot_rows_fn i8dot,
                           orc_dot_gather_fn gather, float *out_d, uint32_t *out_i) {
    if (n < 16384 || dim <= 0 || topk <= 0 || metric == ORC_HAMMING) return -1;
    if ((metric == ORC_COSINE || metric == ORC_L2) && !norms) return -1;
    if (!i8dot) i8dot = orc_i8_dot_rows;
    if (!gather) gather = orc_dot_rows_gather;
    int k = (int64_t)topk < n ? topk : (int)n;
    float qmax = 0.0f;
    for (int64_t d = 0; d < dim; ++d) {
        float a = fabsf(query[d]);
        if (a > qmax) qmax = a;
    }
    double qscale = qmax > 0.0f ? (double)qmax / 127.0 : 1.0;
    int8_t *qc = (int8_t *)malloc((size_t)dim);
    int64_t qabs = 0;
    for (int64_t d = 0; d < dim; ++d) {
        double scaled = (double)query[d] / qscale;
        int32_t r = (int32_t)(scaled >= 0 ? scaled + 0.5 : scaled - 0.5);
        if (r > 127) r = 127;
        else if (r < -127) r = -127;
        qc[d] = (int8_t)r;
        qabs += r < 0 ? -r : r;
    }
    const float qs = (float)qscale;
    const float qabs_half = (float)qabs / 2.0f;
    const float qs_dot = qs, qs_w = qs, qs_qh = qs * qabs_half;
    const float inv_q = qn > 1e-20f ? 1.0f / sqrtf(qn) : 0.0f;
    const float cos_dot = qs * inv_q, cos_h = qs * qabs_half * inv_q, cos_w = qs * inv_q;
    const double qn_d = (double)qn;
    const float two_dot = 2.0f * qs_dot, two_qh = 2.0f * qs_qh, two_w = 2.0f * qs_w;

    int64_t slices = slices_in > 0 ? slices_in : 1;
    int64_t chunk = (n + slices - 1) / slices;
    float *dots = (float *)malloc(sizeof(float) * (size_t)(slices * chunk));
    int64_t budget = k * 16 > 256 ? (int64_t)k * 16 : 256;
    int result = -1;
    for (;;) {
        /* selectCandidates recomputes the slice dots every round (:154-172) */
        for (int64_t s = 0; s < slices; ++s) {
            int64_t start = s * chunk, end = start + chunk < n ? start + chunk : n;
            if (start < end) i8dot(codes + start * dim, qc, end - start, dim, dots + start);
        }
        int64_t per = budget < chunk ? budget : chunk;
        bes_entry *heaps = (bes_entry *)malloc(sizeof(bes_entry) * (size_t)(slices * per));
        int *cnt = (int *)calloc((size_t)slices, sizeof(int));
        for (int64_t s = 0; s < slices; ++s) {
            int64_t start = s * chunk, end = start + chunk < n ? start + chunk : n;
            bes_entry *h = heaps + s * per;
            for (int64_t r = start; r < end; ++r) {
                float key;
                if (metric == ORC_IP) {
                    float a = qs_dot * u[r] * dots[r];
                    float b = qs_qh * u[r];
                    float c = qs_w * w[r];
                    key = -(a + b + c);
                } else if (metric == ORC_L2) {
                    double t = qn_d + (double)norm_sq[r];
                    t = t - (double)(two_dot * u[r] * dots[r]);
                    t = t - (double)(two_qh * u[r]);
                    t = t - (double)(two_w * w[r]);
                    key = (float)t;
                } else {
                    float a = cos_dot * u[r] * dots[r];
                    float b = cos_h * u[r];
                    float c = cos_w * w[r];
                    float inner = a + b + c;
                    key = 1.0f - inner * inv_sqrt[r];
                }
                bes_admit(h, &cnt[s], (int)per, key, (uint32_t)r);
            }
            bes_sorted_ascending(h, cnt[s]);
        }
        /* mergeAscending */
        uint32_t *ids = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)budget);
        int *cur = (int *)calloc((size_t)slices, sizeof(int));
        int64_t taken = 0;
        double cutoff = INFINITY;
        while (taken < budget) {
            int best = -1;
            float best_key = INFINITY;
            for (int64_t s = 0; s < slices; ++s)
                if (cur[s] < cnt[s] && heaps[s * per + cur[s]].key < best_key) {
                    best_key = heaps[s * per + cur[s]].key;
                    best = (int)s;
                }
            if (best < 0) break;
            ids[taken++] = heaps[(int64_t)best * per + cur[best]].id;
            cutoff = (double)best_key;
            cur[best] += 1;
        }
        /* rescore */
        float *rd = (float *)malloc(sizeof(float) * (size_t)(taken > 0 ? taken : 1));
        orc_entry *ent = (orc_entry *)malloc(sizeof(orc_entry) * (size_t)(taken > 0 ? taken : 1));
        if (taken > 0) gather(corpus, query, ids, taken, dim, rd);
        for (int64_t i = 0; i < taken; ++i) {
            float vn = norms ? norms[ids[i]] : 0.0f;
            ent[i].d = orc_distance(metric, rd[i], qn, vn);
            ent[i].id = ids[i];
        }
        qsort(ent, (size_t)taken, sizeof(orc_entry), cmp_entry);
        int done = 0;
        if (taken < k) {
            for (int64_t i = 0; i < taken; ++i) {
                out_d[i] = ent[i].d;
                out_i[i] = ent[i].id;
            }
            result = (int)taken;
            done = 1;
        } else {
            double tau = (double)ent[k - 1].d;
            double margin = fabs(tau) * 1e-6 > 1e-7 ? fabs(tau) * 1e-6 : 1e-7;
            if (cutoff >= tau + margin || taken >= n) {
                for (int i = 0; i < k; ++i) {
                    out_d[i] = ent[i].d;
                    out_i[i] = ent[i].id;
                }
                result = k;
                done = 1;
            }
        }
        free(ent);
        free(rd);
        free(cur);
        free(ids);
        free(cnt);
        free(heaps);
        if (done || budget >= n) break;
        budget = budget * 4 < n ? budget * 4 : n;
    }
    free(dots);
    free(qc);
    return result;
}

typedef struct {
    const float *queries, *corpus, *norms, *qnorms;
    int64_t n, dim, nq;
    int32_t topk, metric, slices, kout, stride;
    const int8_t *codes;
    const float *u, *w, *norm_sq, *inv_sqrt;
    orc_i8_dot_rows_fn i8dot;
    orc_dot_gather_fn gather;
    float *out_d;
    uint32_t *out_i;
    int32_t *out_c;
    int t;
} bes_work;

static void *bes_thread(void *arg) {
    bes_work *b = (bes_work *)arg;
    for (int64_t q = b->t; q < b->nq; q += b->stride) {
        int c = orc_bounded_exact_scan(b->queries + q * b->dim, b->corpus, b->norms,
                                       b->qnorms ? b->qnorms[q] : 0.0f, b->n, b->dim, b->topk,
                                       b->metric, b->slices, b->codes, b->u, b->w, b->norm_sq,
                                       b->inv_sqrt, b->i8dot, b->gather, b->out_d + q * b->kout,
                                       b->out_i + q * b->kout);
        b->out_c[q] = c;
    }
    return NULL;
}

/* parallelHostBatchSearch (FlatGPUSearch.swift:754-779) over the bounded
 * scan: queries spread over `threads` workers, each query's slices run by
 * its worker.  out_* are nq x kout (kout >= min(topk, n)); counts of -1 mark
 * queries the bounded scan declines. */
void orc_bounded_exact_batch(const float *queries, int64_t nq, const float *qnorms,
                             const float *corpus, const float *norms, int64_t n, int64_t dim,
                             int32_t topk, int32_t metric, int32_t slices, int32_t threads,
                             const int8_t *codes, const float *u, const float *w,
                             const float *norm_sq, const float *inv_sqrt, orc_i8_dot_rows_fn i8dot,
                             orc_dot_gather_fn gather, int32_t kout, float *out_d, uint32_t *out_i,
                             int32_t *out_c) {
    if (threads < 1) threads = 1;
    if (threads > nq) threads = (int32_t)(nq > 0 ? nq : 1);
    bes_work *work = (bes_work *)malloc(sizeof(bes_work) * (size_t)threads);
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    for (int t = 0; t < threads; ++t) {
        bes_work b = {queries, corpus, norms, qnorms, n, dim, nq, topk, metric, slices, kout,
                      threads, codes, u, w, norm_sq, inv_sqrt, i8dot, gather, out_d, out_i,
                      out_c, t};
        work[t] = b;
    }
    if (threads == 1) {
        bes_thread(&work[0]);
    } else {
        for (int t = 0; t < threads; ++t) pthread_create(&th[t], NULL, bes_thread, &work[t]);
        for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
    }
    free(th);
    free(work);
}
