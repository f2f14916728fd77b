/*
 * gpusparse.h -- C ABI of the B200 (sm_100a) exact learned-sparse scoring library
 * (libgpusparse.so).  Plain pointers, sizes and a cudaStream_t passed as void*; no torch
 * types.  Every entry point returns an int status (GSP_OK = 0); gsp_last_error() returns
 * a human-readable message for the calling thread's last failure.
 *
 * Reference interfaces replaced (paths inside the GPUSparse checkout):
 *   gsp_index_*           src/run_correctness_verification.py:32-84  build_gpu_index_from_csr
 *                         lsr_benchmark_engine/gpusparse_retrieval.py:81-115  build_index
 *                         src/gpu_inverted_index.py:21-35  GPUInvertedIndex layout
 *   gsp_chunk_bounds      src/triton_kernel_chunked.py:83-122  build_chunk_boundaries
 *   gsp_score_topk        src/triton_kernel.py:159-200  triton_fused_score
 *                         src/triton_kernel_chunked.py:125-170  triton_chunked_score
 *                         src/fused_topk.py:106-160  triton_chunked_score_fused
 *   gsp_compacted_topk    src/fused_topk.py:71-103  compacted_topk
 *   gsp_merge_topk        src/comprehensive_benchmark.py:472-480 (host-side shard merge),
 *                         src/triton_kernel_chunked.py:162-168 (running top-k merge)
 *   gsp_synth_*           src/gpu_inverted_index.py:137-174  generate_synthetic_splade_data
 *                         (the seeded SPLADE-shaped law of the benchmark configs)
 *
 * Layout of an index on the device (one shard of `n_docs` documents, ids local to it):
 *   doc_ids      int32 [P_pad]  term-major postings, ascending doc id within a term,
 *                               each list padded to a multiple of 32 with -1
 *   weights      fp32 / bf16 / uint8 [P_pad]  (padding weight 0)
 *   term_scale   fp32 [V]       uint8 mode only: weight = q * term_scale[t]
 *   offsets      int64 [V]      first posting of term t (a multiple of 32)
 *   lengths      int32 [V]      real postings of term t
 *   padded       int32 [V]      lengths rounded up to 32
 *   max_scores   fp32 [V]       max weight of term t (0 for an empty list)
 *   block_starts uint32 [n_blocks+1, V]  postings of term t with doc id < b*block_docs
 */
#ifndef GPUSPARSE_H
#define GPUSPARSE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes; the Python wrapper maps them to the reference's exception types */
#define GSP_OK 0
#define GSP_ERR_ARG 1          /* ValueError: bad size, pointer, dtype or range        */
#define GSP_ERR_UNSORTED 2     /* ValueError: a posting list is not ascending          */
#define GSP_ERR_OVERFLOW 3     /* RuntimeError: a fixed-capacity structure overflowed  */
#define GSP_ERR_CUDA 4         /* RuntimeError: a CUDA runtime call failed             */
#define GSP_ERR_TIMEOUT 5      /* RuntimeError: a bounded device wait ran out          */
#define GSP_ERR_UNSUPPORTED 6  /* RuntimeError: input outside the supported envelope   */
#define GSP_ERR_BLOCK_PL 7     /* AssertionError: block_pl is not a positive power of 2 */

/* weight dtypes */
#define GSP_W_F32 0
#define GSP_W_BF16 1
#define GSP_W_U8 2

const char* gsp_last_error(void);
int gsp_version(void);

/* Exclusive prefix sum of n int32 values into int64 out[0..n] (out[n] = total). */
int gsp_scan_i32(const int32_t* in, int64_t n, int64_t* out, void* ws, int64_t ws_bytes,
                 void* stream);
int64_t gsp_scan_ws_bytes(int64_t n);

/* ---------------------------------------------------------------- synthetic data */
/* Items [first, first+n) of the seeded SPLADE-shaped law (kind 0 = documents,
 * 1 = queries).  Tables (device, fp64): nnz_cdf[n_nnz] over nnz = nnz_lo.., term_cdf[V],
 * wtab[65537].  Step 1 writes nnz[n]; the caller scans it into indptr; step 2 fills. */
int gsp_synth_nnz(uint64_t seed, uint32_t kind, uint64_t first, int64_t n, int32_t V,
                  const double* nnz_cdf, int32_t n_nnz, int32_t nnz_lo, int32_t min_nnz_item0,
                  int32_t* nnz, void* stream);
int gsp_synth_fill(uint64_t seed, uint32_t kind, uint64_t first, int64_t n, int32_t V,
                   const double* term_cdf, const int32_t* term_guide, const double* wtab,
                   const int64_t* indptr, int32_t* indices, float* data, void* stream);

/* ---------------------------------------------------------------- index build */
/* Workspace bytes for the index build calls below on a CSR of n_docs rows. */
int64_t gsp_index_ws_bytes(int64_t n_docs, int32_t V, int32_t block_docs);
/* Pass 1 (replaces the argsort/bincount/cumsum of build_gpu_index_from_csr :47-58):
 * lengths, padded, offsets and block_starts on the device; *total_padded on the host
 * (this call synchronises the stream).  Column ids outside [0, V) -> GSP_ERR_ARG. */
int gsp_index_count(int64_t n_docs, int32_t V, int32_t block_docs, const int64_t* indptr,
                    const int32_t* indices, int32_t* lengths, int32_t* padded,
                    int64_t* offsets, uint32_t* block_starts, int64_t* total_padded,
                    void* ws, int64_t ws_bytes, void* stream);
/* Pass 2 (replaces the fill loop :60-72): stable scatter of every CSR entry to its
 * term's list (doc ids ascend), -1/0 padding, max_scores. */
int gsp_index_fill(int64_t n_docs, int32_t V, int32_t block_docs, const int64_t* indptr,
                   const int32_t* indices, const float* data, const int64_t* offsets,
                   const int32_t* lengths, const uint32_t* block_starts, int64_t total_padded,
                   int32_t* doc_ids, float* weights, float* max_scores, void* ws,
                   int64_t ws_bytes, void* stream);
/* Streamed build (no counterpart in the reference, whose builder needs the whole CSR on
 * the device): the two passes above, split so that only one chunk of CSR rows is on the
 * device at a time.  Order on one stream:
 *   gsp_index_count_chunk for every chunk (the chunk at first_doc 0 first),
 *   gsp_index_count_finish (synchronises; *total_padded sizes doc_ids/weights),
 *   gsp_index_fill_chunk for every chunk with the same rows,
 *   gsp_index_fill_finish (padding, max_scores, checks; synchronises).
 * A chunk is documents [first_doc, first_doc + chunk_docs) of n_docs: first_doc a
 * multiple of block_docs, chunk_docs too unless the chunk ends the corpus.  Its indptr
 * has chunk_docs + 1 entries indexing its own indices/data (indptr[0] need not be 0).
 * block_starts [n_blocks + 1, V] accumulates the counts of each block in place.  Writes
 * stay inside each block's counted slice of a list: a chunk filled with more postings of
 * a term than were counted is reported by gsp_index_fill_finish as GSP_ERR_ARG, and so
 * are lists left out of order or with doc ids outside [0, n_docs) (e.g. a chunk never
 * filled); a chunk filled with other rows of the same shape is not detectable. */
int gsp_index_count_chunk(int64_t n_docs, int32_t V, int32_t block_docs, int64_t first_doc,
                          int64_t chunk_docs, const int64_t* indptr, const int32_t* indices,
                          uint32_t* block_starts, void* ws, int64_t ws_bytes, void* stream);
int gsp_index_count_finish(int64_t n_docs, int32_t V, int32_t block_docs, int32_t* lengths,
                           int32_t* padded, int64_t* offsets, uint32_t* block_starts,
                           int64_t* total_padded, void* ws, int64_t ws_bytes, void* stream);
int gsp_index_fill_chunk(int64_t n_docs, int32_t V, int32_t block_docs, int64_t first_doc,
                         int64_t chunk_docs, const int64_t* indptr, const int32_t* indices,
                         const float* data, const int64_t* offsets, const uint32_t* block_starts,
                         int32_t* doc_ids, float* weights, void* ws, int64_t ws_bytes,
                         void* stream);
int gsp_index_fill_finish(int64_t n_docs, int32_t V, const int64_t* offsets,
                          const int32_t* lengths, int32_t* doc_ids, float* weights,
                          float* max_scores, void* ws, int64_t ws_bytes, void* stream);
/* Duplicate (document, term) entries.  The reference keeps a term that one CSR row lists
 * twice as two postings and its scatter-add sums both (lsr_benchmark_engine/
 * gpusparse_retrieval.py:84-105, src/triton_kernel.py:93-156); the scorer here needs each
 * document once per list, so the builders merge them first: the first occurrence keeps
 * its place and its weight becomes the fp32 sum of all occurrences' weights in row order.
 * count: nnz[r] = distinct terms of row r (rows [0, n_rows) of indptr, whose first entry
 * need not be 0), *n_dropped (host; the call synchronises) = entries merged away;
 * ws >= 8 bytes of device scratch; V (the vocabulary size, or 0 if unknown) lets the count
 * use a bitmap of the vocabulary (terms outside [0, V) count as distinct there).  fill: the merged rows at new_indptr (n_rows + 1
 * entries, e.g. the scan of nnz) relative to new_indptr[0]; data and out_data may both be
 * NULL to merge the indices only. */
int gsp_csr_dedup_count(int64_t n_rows, int32_t V, const int64_t* indptr,
                        const int32_t* indices, int32_t* nnz, int64_t* n_dropped, void* ws,
                        int64_t ws_bytes, void* stream);
int gsp_csr_dedup_fill(int64_t n_rows, const int64_t* indptr, const int32_t* indices,
                       const float* data, const int64_t* new_indptr, int32_t* out_indices,
                       float* out_data, void* stream);
/* fp32 weights -> bf16 (round to nearest even) or uint8 impacts with per-term scale
 * max_scores[t] / 255 (q = clamp(rint(w / scale), 0, 255)). */
int gsp_index_quantize(int32_t V, int64_t total_padded, const int64_t* offsets,
                       const int32_t* padded, const float* max_scores, const float* weights,
                       int32_t wdtype, void* out_weights, float* term_scale, void* stream);
/* Dense rows of H "head" terms (no reference counterpart: a scorer-side copy of the
 * densest posting lists).  rows [H, ld] (caller zero-filled, dtype = wdtype): row h holds
 * the weight of term head_ids[h] in every document, 0 where the term is absent; ld is a
 * multiple of block_docs >= n_docs. */
int gsp_index_head_rows(int32_t H, const int32_t* head_ids, const int64_t* offsets,
                        const int32_t* lengths, const int32_t* doc_ids, const void* weights,
                        int32_t wdtype, int64_t ld, void* rows, void* stream);
/* lo[i] = rows[i] - trunc_tf32(rows[i]) for n fp32 values (no reference counterpart): the
 * low parts of the dense head rows for the tensor-core head phase (gsp_index_view.head_lo).
 * The tensor core reads an fp32 operand as tf32 by ignoring its low 13 mantissa bits, so
 * rows + lo carry the full fp32 value through a 3xTF32 product. */
int gsp_index_head_lo(int64_t n, const float* rows, float* lo, void* stream);
/* Counts posting lists that are not ascending in doc id (*n_bad) and, when n_dup is not
 * NULL, lists that repeat a doc id (*n_dup); both written on the host (this call
 * synchronises the stream).  ws: at least GSP_CHECK_WS_BYTES of device scratch.  The
 * scorer needs strictly ascending lists (the CSR builders merge a term listed twice in one
 * row first); a caller that assembles an index itself checks n_dup == 0.
 * Replaces the check in src/triton_kernel_chunked.py:99-108. */
#define GSP_CHECK_WS_BYTES 16
int gsp_check_sorted(int32_t V, const int32_t* doc_ids, const int64_t* offsets,
                     const int32_t* lengths, int64_t* n_bad, int64_t* n_dup, void* ws,
                     int64_t ws_bytes, void* stream);

/* ---------------------------------------------------------------- chunk bounds */
/* build_chunk_boundaries: out int64 [n_chunks+1, V], out[c][t] = offsets[t] + number of
 * postings of t with doc id < min(c*doc_chunk, n_docs).  GSP_ERR_UNSORTED if any list
 * is not ascending (the reference raises ValueError).  ws: GSP_CHECK_WS_BYTES of device
 * scratch for the order check (which synchronises the stream). */
int gsp_chunk_bounds(int64_t n_docs, int32_t V, int64_t doc_chunk, const int32_t* doc_ids,
                     const int64_t* offsets, const int32_t* lengths, int64_t* out, void* ws,
                     int64_t ws_bytes, void* stream);

/* ---------------------------------------------------------------- scoring */
typedef struct gsp_index_view {
    int64_t n_docs;            /* documents in this shard (local ids 0..n_docs-1) */
    int64_t doc_base;          /* global id of local document 0 */
    int32_t V;
    int32_t block_docs;        /* documents per block_starts row */
    int32_t wdtype;            /* GSP_W_* */
    int32_t pad_;
    const int32_t* doc_ids;
    const void* weights;
    const float* term_scale;   /* uint8 mode only */
    const int64_t* offsets;
    const int32_t* lengths;
    const uint32_t* block_starts;
    /* head terms scored from dense rows instead of their posting lists (n_head may be 0) */
    int32_t n_head;
    int32_t head_wdtype;       /* GSP_W_* of head_rows: wdtype, or GSP_W_F32 with wdtype
                                  GSP_W_U8 (rows hold the dequantised q * scale_t values) */
    const int32_t* head_slot;  /* [V]: row of term t in head_rows, or -1 */
    const void* head_rows;     /* [n_head, head_ld], head_wdtype */
    int64_t head_ld;
    /* fp32 head rows only, optional: head_rows[i] - (head_rows[i] with its low 13 mantissa
       bits cleared), the second tf32 term of each element for the tensor-core head phase
       (gsp_index_head_lo); NULL keeps the head terms on the CUDA cores */
    const float* head_lo;
} gsp_index_view;

/* How the head terms (those with dense rows) are summed (no reference counterpart):
 *   GSP_HEAD_AUTO          the library's choice, currently GSP_HEAD_CUDA_CORES for every
 *                          index (the default): on B200 the tensor-core path measured slower
 *                          for fp32 head rows (48.9 against 35.1 ms per batch at 8.8M
 *                          documents, 1000 queries, k = 1000), its operand stream being
 *                          limited by TMA throughput
 *   GSP_HEAD_CUDA_CORES    acc = fma(q_w, d_w, acc) in the canonical order: results bitwise
 *                          equal to the CPU oracle's
 *   GSP_HEAD_TENSOR_CORES  tcgen05 MMAs (tf32, operands split 3xTF32: fp32 accuracy to about
 *                          1e-6 relative) for indexes with fp32 head rows and head_lo, any
 *                          batch size; other indexes keep the CUDA cores.  A query's weights
 *                          for a repeated head term are added before the product; the tail
 *                          terms then follow in the canonical order, and results are bitwise
 *                          reproducible run to run.
 * Applies to calls issued after it; process-wide. */
#define GSP_HEAD_AUTO 0
#define GSP_HEAD_CUDA_CORES 1
#define GSP_HEAD_TENSOR_CORES 2
int gsp_set_head_mode(int32_t mode);
int32_t gsp_get_head_mode(void);

/* Workspace bytes for gsp_score_topk with this batch shape (a negative status on error). */
int64_t gsp_score_ws_bytes(const gsp_index_view* ix, int64_t B, int64_t W, int64_t k);
/* Exact scores of B queries (qi int32 [B, W], -1 padded; ids outside [0, V) skipped;
 * qs fp32 [B, W]) against every document, then the exact top-k per query:
 * out_scores fp32 [B, k'] descending, out_ids int64 [B, k'] global doc ids, with
 * k' = min(k, n_docs) and ties broken by ascending doc id.  Each document's score is
 * accumulated as acc = fma(q_w, d_w, acc) over the query's terms, head terms (those with
 * dense rows) first, each group in ascending (term id, slot) order, so results are
 * bitwise reproducible.  Optionally also writes the packed (score key << 32 | ~doc id)
 * top-k to out_keys [B, k'] for a later gsp_merge_topk.  If an internal bounded wait
 * ever ran out (it should not), the scores of that call are NaN and the ids -1.
 * Replaces src/triton_kernel.py:159-200 (triton_fused_score). */
int gsp_score_topk(const gsp_index_view* ix, const int32_t* qi, const float* qs, int64_t B,
                   int64_t W, int64_t k, float* out_scores, int64_t* out_ids,
                   uint64_t* out_keys, void* ws, int64_t ws_bytes, void* stream);

/* gsp_score_topk without any device allocation, for callers that cannot allocate device
 * memory on the call path (a serving loop where cudaMalloc would synchronise the device,
 * or a host that gives the library only its input and output buffers).  No counterpart in
 * the reference.  Scratch is a fixed 32 MiB array compiled into the library, placed on
 * every GPU that loads it and held until exit.  When a batch does not fit with the default
 * per-query candidate capacity, the capacity shrinks toward its minimum of k' + 1024 keys
 * (more frequent compactions, same result; the default equals that minimum up to
 * k' = 2048, so only larger k' shrink); a batch that still does not fit (about
 * B * 3 * (2k + 2048) * 8 bytes plus the plan: some 330 queries at k = 1000), or with
 * k' > 8192, is rejected with GSP_ERR_UNSUPPORTED.
 * Results equal gsp_score_topk's.  Every call whose stream is not being captured looks up
 * the array's device address (cudaGetSymbolAddress) in the current context; a call during
 * a stream capture reuses the address of the device's last call outside one, so make the
 * first call on each device (and the first after a device reset) before any capture.
 * All calls on a device share the one array: calls that overlap on the GPU (different
 * streams, or threads) race and must be serialised. */
int gsp_score_topk_noalloc(const gsp_index_view* ix, const int32_t* qi, const float* qs,
                           int64_t B, int64_t W, int64_t k, float* out_scores, int64_t* out_ids,
                           uint64_t* out_keys, void* stream);

/* gsp_score_topk for shard `shard` of n_shards doc-range shards of one corpus that score
 * the same batch at the same time, one per GPU (no counterpart in the reference, whose
 * shards exchange nothing before the merge).  Every shard has a board [n_shards, B]
 * (device, uint64 keys, row s = shard s) and peer_boards holds the other n_shards - 1
 * shards' boards (usually IPC mappings of other GPUs' memory; host array of device
 * pointers).  After each compaction a shard writes into its row of every board (atomic
 * max) a key that at least ceil(k / n_shards) of its candidates reach; the minimum over
 * the rows is then a lower bound of the corpus-wide k-th best key (the shards hold at
 * least k candidates at or above it), and every shard drops candidates below it.  The
 * call never clears a board (a row of 0 means "no bound yet"), nothing waits on a peer,
 * and the merge of all shards' keys (gsp_merge_topk) is exactly the corpus top-k; a
 * shard may return fewer than k' real entries (the rest are -inf / -1 / key 0).  A
 * board must not hold rows from another batch.  n_shards <= 9; n_shards == 1 is
 * gsp_score_topk. */
int gsp_score_topk_shared(const gsp_index_view* ix, const int32_t* qi, const float* qs,
                          int64_t B, int64_t W, int64_t k, float* out_scores, int64_t* out_ids,
                          uint64_t* out_keys, void* ws, int64_t ws_bytes, uint64_t* board,
                          int32_t shard, int32_t n_shards, uint64_t* const* peer_boards,
                          void* stream);

/* Threshold boards for gsp_score_topk_shared (no reference counterpart).  alloc: n zeroed
 * uint64 on the current device (cudaMalloc) and, if ipc_handle is not NULL, its
 * GSP_IPC_HANDLE_BYTES-byte CUDA IPC handle for the other processes; open / close map and
 * unmap another process's board; clear zeroes n entries on a stream. */
#define GSP_IPC_HANDLE_BYTES 64
int gsp_board_alloc(int64_t n, uint64_t** board, void* ipc_handle);
int gsp_board_free(uint64_t* board);
int gsp_board_open(const void* ipc_handle, uint64_t** board);
int gsp_board_close(uint64_t* board);
int gsp_board_clear(uint64_t* board, int64_t n, void* stream);

/* Timing of the scoring kernel itself (no reference counterpart; used by the benchmark
 * for its roofline figure): while enabled, every gsp_score_topk brackets its main kernel
 * launch with CUDA events on the caller's stream; collect synchronises on them and returns
 * the summed duration and the number of launches, then resets.  One device per process. */
int gsp_profile_enable(int on);

/* Polls a scoring call's bounded waits make before giving up (no reference counterpart;
 * a diagnostic control, default 2^21, about a second).  A wait that gives up records a
 * fault and that call returns NaN scores and ids -1 instead of a result; the context stays
 * usable.  0 makes every wait give up at once (tests use it to exercise that path).
 * Applies to calls issued after it; process-wide. */
int gsp_set_wait_limit(int32_t polls);
int32_t gsp_get_wait_limit(void);

/* Scheduling jitter of the CUDA-core scorer (no reference counterpart; a test control,
 * default 0 = off): lane 0 of every scoring warp sleeps about `ns` nanoseconds at the start
 * of half of its work items (a fixed hash of the item picks them), which reshuffles how the
 * lanes of a warp and the warps of an SM interleave.  Results must not change: the tests
 * score under it to show that the canonical summation order does not depend on scheduling.
 * No work is skipped.  Applies to calls issued after it; process-wide; 0 <= ns <= 1000000. */
int gsp_set_schedule_jitter(int32_t ns);
int32_t gsp_get_schedule_jitter(void);

/* Small-batch mode (no reference counterpart).  A batch with 256 <= k' <= 1024, at most
 * 24576 (query, 1024-document tile) pairs and per-tile lists of at most `bytes`
 * (B x ceil(n_docs / 1024) x k' x 8; default 256 MiB) skips the shared candidate
 * buffers: every tile writes its own exact top-k' and a tree of merges (8 lists per
 * node) reduces them, with no atomics and no waits.  That is faster when few queries
 * spread over many tiles (their shared buffers would serialise on compactions).  Results
 * are identical either way; 0 turns the mode off.  Applies to calls issued after it;
 * process-wide.  gsp_score_ws_bytes accounts for it. */
int gsp_set_tree_limit(int64_t bytes);
int64_t gsp_get_tree_limit(void);
int gsp_profile_collect(double* total_ms, int64_t* launches);

/* ---------------------------------------------------------------- selection */
/* Merge R candidate lists per query into the exact top-k.  keys: packed uint64
 * (fkey(score) << 32 | (0xFFFFFFFF - doc id)), list r of query b at
 * keys + b*stride_b + r*stride_r, holding counts[r] valid entries.  Writes k' =
 * min(k, sum(counts)) results per query (scores fp32, ids int64 and, if non-null,
 * keys).  ws: gsp_merge_ws_bytes(B, k) bytes of device scratch (0, and ws may be NULL,
 * for k <= 8192; above that the keys are sorted in global memory).
 * Replaces the host-side shard merge and the running torch.topk merge. */
int64_t gsp_merge_ws_bytes(int64_t B, int64_t k);
int gsp_merge_topk(const uint64_t* keys, int64_t B, int64_t R, int64_t stride_b,
                   int64_t stride_r, const int32_t* counts_host, int64_t k,
                   float* out_scores, int64_t* out_ids, uint64_t* out_keys, void* ws,
                   int64_t ws_bytes, void* stream);
/* compacted_topk: top-min(k, L) of row entries >= tau[b] of scores [B, L] (row stride
 * `stride` floats), (score desc, column asc), padded with (-inf, 0) when fewer. */
int64_t gsp_compacted_ws_bytes(int64_t B, int64_t L, int64_t k, int64_t max_cand);
int gsp_compacted_topk(const float* scores, int64_t B, int64_t L, int64_t stride,
                       const float* tau, int64_t k, int64_t max_cand, float* out_v,
                       int64_t* out_i, void* ws, int64_t ws_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GPUSPARSE_H */
