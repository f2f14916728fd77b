/*
 * CPU ORACLE for the exact learned-sparse scoring path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file is the checker, never the product: only the tests, the smoke check and
 * bench.py's CPU-baseline / reference arm may load it.  The product path
 * (gpu-sparse_b200/) never calls into it and fails loudly when its CUDA library is
 * missing.
 *
 * Contents
 *   1. orc_synth_*   - the deterministic synthetic SPLADE-shaped corpus/query generator.
 *                      It is an independent twin of the GPU generator in
 *                      gpu-sparse_b200/csrc/synth.cu; the GPU tests assert the two
 *                      produce byte-identical CSR matrices.
 *   2. orc_build_*   - term-major inverted-index build from a document-term CSR,
 *                      restating src/run_correctness_verification.py:32-84 (stable sort
 *                      by term so postings ascend by doc id, pad every list to a
 *                      multiple of 32 with doc id -1 / weight 0, exclusive prefix sum of
 *                      padded lengths -> offsets, per-term max weight) as a stable
 *                      counting sort.
 *   3. orc_score_topk - exhaustive scatter-add scoring + top-k, restating
 *                      src/triton_kernel.py:93-156 (_fast_scatter_add_kernel: for every
 *                      query term id in [0, V), add q_w * d_w into the document's fp32
 *                      accumulator; ids < 0 or >= V are skipped, :126-128) and :199
 *                      (torch.topk over the dense [B, N] matrix).  The reference's
 *                      summation order is unspecified (global atomics), so the oracle
 *                      fixes the canonical order the CUDA path also uses: a query's
 *                      (term id, slot) pairs in ascending order, the terms of an
 *                      optional "head" set (the index's densest terms) before all
 *                      others, each contribution added as acc = fma(q_w, d_w, acc):
 *                      one fused multiply-add, a single IEEE fp32 rounding (C99 fmaf;
 *                      nothing else may be contracted: build with -ffp-contract=off).
 *                      Ties in top-k are broken by ascending doc id.
 *   4. orc_score_dense_f64 - the exhaustive dense reference (src/remeasure_2026_09.py:
 *                      238-258, Q @ D^T) evaluated in fp64 for tolerance checks.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

/* ------------------------------------------------------------------ 1. generator */

/* SplitMix64 finaliser (Steele, Lea, Flood: "Fast splittable pseudorandom number
 * generators", OOPSLA 2014). */
static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* Key of one (seed, stream, item): every draw for that item is mix64(key + ctr*golden). */
static inline uint64_t item_key(uint64_t seed, uint32_t stream, uint64_t item) {
    uint64_t z = mix64(seed ^ (0x9E3779B97F4A7C15ULL * (uint64_t)(stream + 1)));
    return mix64(z ^ (item * 0xD1B54A32D192ED03ULL));
}
static inline uint64_t draw64(uint64_t key, uint64_t ctr) {
    return mix64(key + (ctr + 1) * 0x9E3779B97F4A7C15ULL);
}
static inline double u53(uint64_t x) { return (double)(x >> 11) * (1.0 / 9007199254740992.0); }

/* first index i in [0, n) with cdf[i] > u (cdf[n-1] == 1.0 > u always) */
static inline int64_t upper_idx(const double* cdf, int64_t n, double u) {
    int64_t lo = 0, hi = n - 1;
    while (lo < hi) {
        int64_t mid = lo + ((hi - lo) >> 1);
        if (cdf[mid] > u) hi = mid; else lo = mid + 1;
    }
    return lo;
}

/* The same answer as upper_idx(cdf, n, u), searched only inside the guide interval:
 * guide[j] = upper_idx(cdf, n, j / GUIDE) for j <= GUIDE (guide[GUIDE] = n - 1), and the
 * answer is monotone in u, so it lies in [guide[j], guide[j+1]] for u in [j, j+1) / GUIDE. */
#define GUIDE 65536
static inline int64_t upper_idx_guided(const double* cdf, const int32_t* guide, double u) {
    int32_t j = (int32_t)(u * (double)GUIDE);
    int64_t lo = guide[j], hi = guide[j + 1];
    while (lo < hi) {
        int64_t mid = lo + ((hi - lo) >> 1);
        if (cdf[mid] > u) hi = mid; else lo = mid + 1;
    }
    return lo;
}

/* stream ids: items of kind `kind` (0 = documents, 1 = queries) use 3 streams */
#define STREAM_NNZ(kind)  (3u * (kind) + 0u)
#define STREAM_TERM(kind) (3u * (kind) + 1u)
#define STREAM_W(kind)    (3u * (kind) + 2u)
#define WTAB_SEGS 65536

static int32_t item_nnz(uint64_t seed, uint32_t kind, uint64_t item, const double* nnz_cdf,
                        int32_t n_nnz, int32_t nnz_lo, int32_t V, int32_t min_nnz_item0) {
    double u = u53(draw64(item_key(seed, STREAM_NNZ(kind), item), 0));
    int32_t n = nnz_lo + (int32_t)upper_idx(nnz_cdf, n_nnz, u);
    if (item == 0 && n < min_nnz_item0) n = min_nnz_item0;
    if (n > V) n = V;
    return n;
}

/* piecewise-linear quantile of the weight law; every step is one IEEE double op */
static inline float weight_of(uint64_t x, const double* wtab) {
    double u = u53(x);
    double s = u * (double)WTAB_SEGS;           /* exact: power-of-two scaling */
    int32_t i = (int32_t)s;                      /* floor, u < 1 so i < WTAB_SEGS */
    double f = s - (double)i;                    /* exact */
    double a = wtab[i], b = wtab[i + 1];
    double d = b - a;
    double m = f * d;
    double w = a + m;
    return (float)w;
}

int orc_synth_nnz(uint64_t seed, uint32_t kind, uint64_t first, int64_t n, int32_t V,
                  const double* nnz_cdf, int32_t n_nnz, int32_t nnz_lo, int32_t min_nnz_item0,
                  int32_t* out) {
    for (int64_t i = 0; i < n; ++i)
        out[i] = item_nnz(seed, kind, first + (uint64_t)i, nnz_cdf, n_nnz, nnz_lo, V, min_nnz_item0);
    return 0;
}

typedef struct {
    uint64_t seed; uint32_t kind; uint64_t first; int64_t n0, n1; int32_t V;
    const double* term_cdf; const int32_t* guide; const double* wtab; const int64_t* indptr;
    int32_t* indices; float* data;
} fill_job;

static void* fill_worker(void* arg) {
    fill_job* j = (fill_job*)arg;
    int32_t V = j->V;
    uint8_t* seen = (uint8_t*)calloc((size_t)V, 1);
    if (!seen) return (void*)1;
    for (int64_t i = j->n0; i < j->n1; ++i) {
        uint64_t item = j->first + (uint64_t)i;
        int64_t p0 = j->indptr[i], p1 = j->indptr[i + 1];
        int32_t need = (int32_t)(p1 - p0), got = 0;
        uint64_t tkey = item_key(j->seed, STREAM_TERM(j->kind), item);
        uint64_t wkey = item_key(j->seed, STREAM_W(j->kind), item);
        /* successive sampling: i.i.d. draws from the Zipf law, keep first occurrences */
        int64_t cap = 64 * (int64_t)need + 4096;
        for (int64_t c = 0; c < cap && got < need; ++c) {
            int32_t t = (int32_t)upper_idx_guided(j->term_cdf, j->guide, u53(draw64(tkey, (uint64_t)c)));
            if (!seen[t]) { seen[t] = 1; j->indices[p0 + got] = t; ++got; }
        }
        /* deterministic completion if the draw cap was hit: smallest unused ids */
        for (int32_t t = 0; got < need && t < V; ++t)
            if (!seen[t]) { seen[t] = 1; j->indices[p0 + got] = t; ++got; }
        for (int32_t s = 0; s < need; ++s) {
            j->data[p0 + s] = weight_of(draw64(wkey, (uint64_t)s), j->wtab);
            seen[j->indices[p0 + s]] = 0;
        }
    }
    free(seen);
    return NULL;
}

int orc_synth_fill(uint64_t seed, uint32_t kind, uint64_t first, int64_t n, int32_t V,
                   const double* term_cdf, const int32_t* guide, const double* wtab,
                   const int64_t* indptr, int32_t* indices, float* data, int32_t nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256]; fill_job jobs[256];
    for (int32_t t = 0; t < nthreads; ++t) {
        jobs[t] = (fill_job){seed, kind, first, n * t / nthreads, n * (t + 1) / nthreads, V,
                             term_cdf, guide, wtab, indptr, indices, data};
        pthread_create(&th[t], NULL, fill_worker, &jobs[t]);
    }
    int rc = 0;
    for (int32_t t = 0; t < nthreads; ++t) { void* r; pthread_join(th[t], &r); if (r) rc = 1; }
    return rc;
}

/* ------------------------------------------------------------------ 2. index build */

/* lengths[t] = number of CSR entries with column t (run_correctness_verification.py:52-54) */
int orc_build_lengths(int64_t nnz, int32_t V, const int32_t* indices, int32_t* lengths) {
    memset(lengths, 0, sizeof(int32_t) * (size_t)V);
    for (int64_t e = 0; e < nnz; ++e) {
        int32_t t = indices[e];
        if (t < 0 || t >= V) return 1;
        lengths[t]++;
    }
    return 0;
}

/* Stable counting sort of the CSR by column into the padded term-major arrays.
 * offsets[] are the exclusive prefix sums of the 32-padded lengths (:55-58); the
 * arrays must be pre-filled with -1 / 0 (:61-62).  Rows are visited in order and
 * entries within a row in order, which is exactly what np.argsort(kind='stable') on
 * the COO column array gives (:47). */
int orc_build_fill(int64_t N, int32_t V, const int64_t* indptr, const int32_t* indices,
                   const float* data, const int64_t* offsets, int32_t* doc_ids, float* scores,
                   float* max_scores) {
    int64_t* cur = (int64_t*)malloc(sizeof(int64_t) * (size_t)V);
    if (!cur) return 2;
    memcpy(cur, offsets, sizeof(int64_t) * (size_t)V);
    for (int32_t t = 0; t < V; ++t) max_scores[t] = 0.0f;
    uint8_t* has = (uint8_t*)calloc((size_t)V, 1);
    for (int64_t d = 0; d < N; ++d) {
        for (int64_t e = indptr[d]; e < indptr[d + 1]; ++e) {
            int32_t t = indices[e];
            int64_t p = cur[t]++;
            doc_ids[p] = (int32_t)d;
            scores[p] = data[e];
            /* max over the list (:71); numpy's max of an all-negative list is negative */
            if (!has[t] || data[e] > max_scores[t]) { max_scores[t] = data[e]; has[t] = 1; }
        }
    }
    free(has);
    free(cur);
    return 0;
}

/* ------------------------------------------------------------------ 3. scoring */

typedef struct { int32_t tail; int32_t t; int32_t slot; float w; } qent;

static int qent_cmp(const void* a, const void* b) {
    const qent* x = (const qent*)a; const qent* y = (const qent*)b;
    if (x->tail != y->tail) return x->tail < y->tail ? -1 : 1;
    if (x->t != y->t) return x->t < y->t ? -1 : 1;
    return x->slot < y->slot ? -1 : (x->slot > y->slot);
}

/* order-preserving map of a float to uint32 (-0 folded onto +0) */
static inline uint32_t fkey(float f) {
    f = f + 0.0f;
    uint32_t b; memcpy(&b, &f, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
/* better(a,b): score desc, doc id asc */
static inline int better(float sa, int64_t da, float sb, int64_t db) {
    uint32_t ka = fkey(sa), kb = fkey(sb);
    if (ka != kb) return ka > kb;
    return da < db;
}

typedef struct { float s; int64_t d; } cand;

/* min-heap of the k best by `better` (root = worst kept) */
static void heap_sift_down(cand* h, int64_t n, int64_t i) {
    for (;;) {
        int64_t l = 2 * i + 1, r = l + 1, m = i;
        if (l < n && better(h[m].s, h[m].d, h[l].s, h[l].d)) m = l;
        if (r < n && better(h[m].s, h[m].d, h[r].s, h[r].d)) m = r;
        if (m == i) return;
        cand tmp = h[i]; h[i] = h[m]; h[m] = tmp; i = m;
    }
}
static void heap_sift_up(cand* h, int64_t i) {
    while (i > 0) {
        int64_t p = (i - 1) / 2;
        if (better(h[p].s, h[p].d, h[i].s, h[i].d)) { cand tmp = h[i]; h[i] = h[p]; h[p] = tmp; i = p; }
        else return;
    }
}
static int cand_cmp_desc(const void* a, const void* b) {
    const cand* x = (const cand*)a; const cand* y = (const cand*)b;
    if (better(x->s, x->d, y->s, y->d)) return -1;
    if (better(y->s, y->d, x->s, x->d)) return 1;
    return 0;
}

/* top-k of acc[0..N) (score desc, doc asc); ids are offset by id_base */
static void topk_row(const float* acc, int64_t N, int64_t k, int64_t id_base, cand* heap,
                     float* out_s, int64_t* out_i) {
    int64_t n = 0;
    for (int64_t d = 0; d < N; ++d) {
        float s = acc[d];
        if (n < k) { heap[n].s = s; heap[n].d = d; heap_sift_up(heap, n); ++n; }
        else if (better(s, d, heap[0].s, heap[0].d)) { heap[0].s = s; heap[0].d = d; heap_sift_down(heap, n, 0); }
    }
    qsort(heap, (size_t)n, sizeof(cand), cand_cmp_desc);
    for (int64_t j = 0; j < n; ++j) { out_s[j] = heap[j].s; out_i[j] = heap[j].d + id_base; }
}

typedef struct {
    int64_t N; int32_t V; const int32_t* doc_ids; const float* w; const int64_t* offsets;
    const int32_t* lengths; int64_t W; const int32_t* qi; const float* qs; int64_t k;
    int64_t b0, b1; float* out_s; int64_t* out_i; float* out_acc; int64_t id_base;
    const uint8_t* head;   /* [V] 1 for head terms, or NULL */
} score_job;

/* acc = fma(qw, w, acc) over the query's postings in canonical (term, slot) order.  The
 * FMA-capable clone is picked at load time where the CPU has the instruction; both clones
 * compute the same correctly rounded fmaf. */
__attribute__((target_clones("fma", "default")))
static void score_one(const score_job* j, int64_t b, float* acc, qent* ents) {
    memset(acc, 0, sizeof(float) * (size_t)j->N);
    int64_t ne = 0;
    for (int64_t s = 0; s < j->W; ++s) {
        int32_t t = j->qi[b * j->W + s];
        if (t < 0 || t >= j->V) continue;           /* triton_kernel.py:126-128 */
        ents[ne].tail = (j->head && j->head[t]) ? 0 : 1;
        ents[ne].t = t; ents[ne].slot = (int32_t)s; ents[ne].w = j->qs[b * j->W + s]; ++ne;
    }
    qsort(ents, (size_t)ne, sizeof(qent), qent_cmp);
    for (int64_t e = 0; e < ne; ++e) {
        const float qw = ents[e].w;
        const int64_t o = j->offsets[ents[e].t];
        const int32_t L = j->lengths[ents[e].t];
        for (int32_t p = 0; p < L; ++p) {
            const int32_t d = j->doc_ids[o + p];
            if (d < 0) continue;                     /* padding (:156 mask) */
            acc[d] = fmaf(qw, j->w[o + p], acc[d]);  /* one rounding (fused) */
        }
    }
}

static void* score_worker(void* arg) {
    score_job* j = (score_job*)arg;
    float* acc = j->out_acc ? NULL : (float*)malloc(sizeof(float) * (size_t)(j->N > 0 ? j->N : 1));
    qent* ents = (qent*)malloc(sizeof(qent) * (size_t)(j->W > 0 ? j->W : 1));
    cand* heap = (cand*)malloc(sizeof(cand) * (size_t)(j->k > 0 ? j->k : 1));
    if ((!acc && !j->out_acc) || !ents || !heap) return (void*)1;
    for (int64_t b = j->b0; b < j->b1; ++b) {
        float* a = j->out_acc ? j->out_acc + b * j->N : acc;
        score_one(j, b, a, ents);
        if (j->k > 0 && j->out_s)
            topk_row(a, j->N, j->k, j->id_base, heap, j->out_s + b * j->k, j->out_i + b * j->k);
    }
    free(acc); free(ents); free(heap);
    return NULL;
}

static int run_score(score_job base, int64_t B, int32_t nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (nthreads > B) nthreads = (int32_t)(B > 0 ? B : 1);
    pthread_t th[256]; score_job jobs[256];
    for (int32_t t = 0; t < nthreads; ++t) {
        jobs[t] = base; jobs[t].b0 = B * t / nthreads; jobs[t].b1 = B * (t + 1) / nthreads;
        pthread_create(&th[t], NULL, score_worker, &jobs[t]);
    }
    int rc = 0;
    for (int32_t t = 0; t < nthreads; ++t) { void* r; pthread_join(th[t], &r); if (r) rc = 1; }
    return rc;
}

/* Exhaustive scoring of B queries over all N documents + exact top-k.
 * weights are fp32 (quantised indexes pass their dequantised weights). */
int orc_score_topk(int64_t N, int32_t V, const int32_t* doc_ids, const float* weights,
                   const int64_t* offsets, const int32_t* lengths, int64_t B, int64_t W,
                   const int32_t* qi, const float* qs, int64_t k, int64_t id_base,
                   int32_t nthreads, float* out_scores, int64_t* out_ids, const uint8_t* head) {
    if (k > N) k = N;
    score_job j = {N, V, doc_ids, weights, offsets, lengths, W, qi, qs, k, 0, 0,
                   out_scores, out_ids, NULL, id_base, head};
    return run_score(j, B, nthreads);
}

/* The full [B, N] fp32 score matrix in the canonical order (small cases only). */
int orc_score_full(int64_t N, int32_t V, const int32_t* doc_ids, const float* weights,
                   const int64_t* offsets, const int32_t* lengths, int64_t B, int64_t W,
                   const int32_t* qi, const float* qs, int32_t nthreads, float* out_acc,
                   const uint8_t* head) {
    score_job j = {N, V, doc_ids, weights, offsets, lengths, W, qi, qs, 0, 0, 0,
                   NULL, NULL, out_acc, 0, head};
    return run_score(j, B, nthreads);
}

/* ------------------------------------------------------------------ 4. fp64 dense */

/* S[b, d] = sum over query slots with 0 <= t < V of qs * D[d, t], accumulated in fp64
 * straight from the document CSR (duplicates summed, as Q_dense @ D_dense^T does).
 * Queries are split over nthreads threads. */
typedef struct {
    int64_t N; int32_t V; const int64_t* indptr; const int32_t* indices; const float* data;
    int64_t W; const int32_t* qi; const float* qs; double* out; int64_t b0, b1;
} dense_job;

static void* dense_worker(void* arg) {
    dense_job* j = (dense_job*)arg;
    double* qd = (double*)calloc((size_t)j->V, sizeof(double));
    if (!qd) return (void*)1;
    for (int64_t b = j->b0; b < j->b1; ++b) {
        for (int64_t s = 0; s < j->W; ++s) {
            int32_t t = j->qi[b * j->W + s];
            if (t >= 0 && t < j->V) qd[t] += (double)j->qs[b * j->W + s];
        }
        for (int64_t d = 0; d < j->N; ++d) {
            double acc = 0.0;
            for (int64_t e = j->indptr[d]; e < j->indptr[d + 1]; ++e)
                acc += qd[j->indices[e]] * (double)j->data[e];
            j->out[b * j->N + d] = acc;
        }
        for (int64_t s = 0; s < j->W; ++s) {
            int32_t t = j->qi[b * j->W + s];
            if (t >= 0 && t < j->V) qd[t] = 0.0;
        }
    }
    free(qd);
    return NULL;
}

int orc_score_dense_f64(int64_t N, int32_t V, const int64_t* indptr, const int32_t* indices,
                        const float* data, int64_t B, int64_t W, const int32_t* qi,
                        const float* qs, double* out, int32_t nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (nthreads > B) nthreads = (int32_t)(B > 0 ? B : 1);
    pthread_t th[256]; dense_job jobs[256];
    for (int32_t t = 0; t < nthreads; ++t) {
        dense_job j = {N, V, indptr, indices, data, W, qi, qs, out, B * t / nthreads,
                       B * (t + 1) / nthreads};
        jobs[t] = j;
        pthread_create(&th[t], NULL, dense_worker, &jobs[t]);
    }
    int rc = 0;
    for (int32_t t = 0; t < nthreads; ++t) { void* r; pthread_join(th[t], &r); if (r) rc = 2; }
    return rc;
}
