// Exact batched scoring with fused threshold selection (sm_100a).
//
// Replaces src/triton_kernel.py:93-200 (_fast_scatter_add_kernel + torch.zeros +
// torch.topk), src/triton_kernel_chunked.py:34-170 and src/fused_topk.py:33-160.
//
// Work decomposition.  A work item is one (document tile, query) pair.  Warps take items
// from one global counter in tile-major order, so the whole GPU works on a window of a few
// tiles at any moment (their postings and dense head rows stay in L2) and no warp idles
// while items are left.  A tile is a whole number of index blocks (one, 1024 documents,
// by default), so the window of every term's postings inside a tile is
// [block_starts[first block][t], block_starts[last block + 1][t]) with no search.  The
// warp owns the tile's fp32 accumulators, so every (query, document) cell has exactly one
// writer, and the result does not depend on which warp scored which item.
//
// Candidates.  Each query has two candidate buffers used in turn and a keep list of the k
// best keys found so far, shared by all warps; a 64-bit word (generation << 32 | reserved
// slots) says which buffer is open (the generation's low bit) and how far it is reserved.
// A buffer is all zeros when its generation opens, and a key is never zero, so a slot
// that holds a key has been written.  A warp reserves room for its keys with one
// atomicAdd on the word, which also tells it the generation, and below the capacity
// writes the keys; nothing else (no fence, no counter).  The warp whose reservation
// crosses the capacity writes its keys into the buffer's spare tail, waits for the
// previous compaction to finish (it read the other buffer, wrote the keep list and zeroed
// that buffer), opens the next generation on the other buffer so that the other warps go
// on appending there, waits until every slot below its own reservation holds a key, and
// then keeps the k largest of that buffer and the keep list as the new keep list,
// publishes the k-th as the query's threshold and zeroes every slot its generation used.
// The zeroing is ordered before any key of the buffer's next generation, two generations
// on: the compactor fences before it marks the compaction finished, the next crossing
// warp waits for that mark and fences before it opens the next generation, and a key's
// slot is known only from the reservation that reads the opened word.  Warps that reserved
// past the capacity wait only until the next generation is open.
// Every wait is bounded; one that runs out records a fault, and the merge then reports
// NaN scores instead of a result.
//
// Doc-range shards of one corpus scored at the same time (one per GPU) also share a
// bound: after each compaction a shard writes into its row of every shard's board
// (remote atomics over NVLink) a key that ceil(k / n_shards) of its kept keys reach, and
// a tile's selection uses the minimum over the rows when it is higher than the query's
// own threshold.  The shards together hold k keys at or above that minimum, so it is a
// lower bound of the corpus-wide k-th key and dropping keys below it loses nothing.
//
// Per tile:
//  1. head terms (the index's densest terms, stored as dense rows): the warp keeps the
//     accumulators of one part of the tile in registers (512 documents, 16 per lane, with
//     four CTAs per SM) and streams the matching slice of each of the query's head rows
//     with coalesced 16-byte loads: acc = fma(q_w, w, acc) for every document;
//  2. the accumulators go to shared memory and the tail terms (all others), in ascending
//     term id, are scattered into them: a run whose window is long (or that a query
//     repeats) is streamed on its own, four 32-posting chunks in flight (two consecutive
//     long runs of at most 64 postings share one such window); consecutive short runs are
//     flattened into full 32-lane chunks, and lanes that hit the same document (different
//     terms) are applied in term order, one rank at a time (match_any);
//  3. every score becomes a packed key (order-preserving score bits << 32 | ~doc id:
//     larger is better, ties go to the lower doc id) and the keys whose score reaches the
//     query's threshold go to its candidate buffer.  A discarded key is beaten by k kept
//     keys, so the final top-k (merge_kernel in select.cu) is exact.  In the small-batch
//     mode (kModeTree) the tile instead writes its own exact top-k' to a list of its own, and
//     a merge tree reduces the lists (no shared buffers, atomics or waits).
// Each cell therefore accumulates acc = fma(q_w, d_w, acc) in a fixed order -- head terms
// by term id, then tail terms by term id, a repeated term in query-slot order -- with one
// fp32 rounding per fused multiply-add: bitwise reproducible, and equal to the CPU
// oracle's canonical order.
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <stdio.h>
#include <stdlib.h>
#include <utility>
#include <vector>

namespace gsp {

#ifndef GSP_SCORE_WARPS
#define GSP_SCORE_WARPS 8          // warps per scoring CTA
#endif
constexpr int kWarps = GSP_SCORE_WARPS;
#ifndef GSP_SCORE_CTAS_PER_SM
#define GSP_SCORE_CTAS_PER_SM 4   // resident scoring CTAs per SM (register budget 65536 / (256 * this))
#endif
constexpr int kCtasPerSm = GSP_SCORE_CTAS_PER_SM;
constexpr int kPlanThreads = 256;
constexpr int kMaxWidth = 16384;  // query slots (W) supported: the plan sorts them in shared memory
constexpr int kBlock = 1024;      // documents per index block (block_starts row)
#ifndef GSP_TILE_BLOCKS
#define GSP_TILE_BLOCKS 1         // index blocks per scoring tile
#endif
constexpr int kTile = kBlock * GSP_TILE_BLOCKS;   // documents per scoring tile
constexpr int kSel = 1024;        // documents one selection pass marks (32 per lane)
constexpr int kTileBlocksI = GSP_TILE_BLOCKS;
// the head rows are summed over parts of the tile, 1024 documents each with 80 registers
// per thread (768 threads per SM), 512 with 64 (1024 threads), 256 with fewer, so that the
// accumulators and row values of one part fit in registers
constexpr int kRegsPerThread = 65536 / (kWarps * 32 * kCtasPerSm);
constexpr int kHeadPart = kRegsPerThread >= 80 ? 1024 : (kRegsPerThread >= 64 ? 512 : 256);
constexpr int kHeadParts = kTile / kHeadPart;
constexpr int kHeadVec = kHeadPart / 128;   // float4 accumulators per lane per part
constexpr int kLongRun = 24;      // tail windows at least this long are streamed on their own
constexpr int kSpinLimit = 1 << 21;   // default polls of a bounded wait (about a second)
constexpr int kCompactUnroll = 8;     // keys per lane loaded together by a compaction pass
constexpr int kMaxPeers = 8;          // other shards' threshold boards one launch raises
constexpr int kTreeMinK = 256;        // small-batch mode: smallest k' and most query-tiles
constexpr int64_t kTreeMaxTiles = 24576;
constexpr int64_t kDenseBytes = int64_t(2) << 30;   // dense mode: keys of one query window

struct ScoreParams {
  const int32_t* doc_ids;
  const void* weights;
  const float* term_scale;
  const uint32_t* block_starts;
  const void* head_rows;
  int64_t head_ld;
  int64_t n_docs;
  int64_t doc_base;
  int32_t V;
  int32_t n_blocks;     // scoring tiles
  int32_t n_iblocks;    // index blocks (block_starts has n_iblocks + 1 rows)
  int32_t B;
  int32_t k;
  int32_t ecap;      // plan capacity per query (= W)
  int32_t cap;       // candidate buffer capacity per query (keys), > k
  int64_t cand_stride;   // keys per buffer: cap + kSel (the crossing warp's spare tail) + k (the keep list, for a compaction)
  // plan, per query: head entries and tail runs
  const int32_t* n_head_e;
  const uint16_t* head_h;
  const float* head_w;
  const float* head_scale;
  const int32_t* n_runs;
  const int32_t* run_term;
  const uint32_t* run_base32;
  const uint16_t* run_end;
  const float* run_w0;
  const float* ent_w;
  uint64_t* cand;              // [B, 3, cand_stride]: keep list, buffer 0, buffer 1
  unsigned long long* gthr;    // [B] published lower bound of each query's k-th key (zeroed)
  unsigned long long* rg;      // [B] generation << 32 | reserved slots (zeroed)
  int32_t* cdone;              // [B] finished compactions (zeroed)
  int32_t* counts;             // [B, 3] final candidates: keep list, buffer 0, buffer 1
  unsigned long long* item_next;   // next work item (zeroed)
  int32_t* fault;              // a bounded wait ran out (zeroed)
  int32_t wait_limit;          // polls before a wait gives up
  int32_t jitter_ns;           // > 0: lane 0 sleeps this long at the start of half the items
  // Doc-range shards of one batch scored at the same time (n_shards > 1) share a bound:
  // row s of every shard's board [n_shards, B] holds, per query, a key that shard s has at
  // least kg = ceil(k / n_shards) candidates at or above.  The minimum over the rows is a
  // lower bound of the k-th best key of the whole corpus (the shards hold n_shards * kg
  // >= k keys at or above it), so every shard may drop candidates below it.
  unsigned long long* board;                  // this shard's board (local memory)
  unsigned long long* peer_thr[kMaxPeers];    // the other shards' boards (peer memory)
  int32_t n_peers;                            // n_shards - 1
  int32_t n_shards, shard, kg;
  // Small batches: instead of the shared candidate buffers, every tile writes its exact
  // top tile_k keys to tile_out [B, n_blocks, tile_k] (0 in unused slots) and a tree of
  // merges reduces them (no atomics, no waits).
  uint64_t* tile_out;
  int32_t tile_k;
  // Queries [q_lo, q_lo + q_n) are this launch's (all B except in the dense mode, which
  // scores the batch a window of queries at a time).
  int32_t q_lo, q_n;
  // Dense mode (k above what the candidate buffers hold): every tile writes the keys of
  // all its documents to dense [q_n, dense_ld] (0 past the last document).
  uint64_t* dense;
  int64_t dense_ld;
};

// How a launch selects: shared candidate buffers, per-tile lists and a merge tree (small
// batches), or every key written out (k above kMaxSmemK).
constexpr int kModeBuffers = 0;
constexpr int kModeTree = 1;
constexpr int kModeDense = 2;

namespace {

// ---------------------------------------------------------------------------- plan
// One CTA per query: sort the query's (term, slot) pairs (bitonic in shared memory), then
// split them into head entries (terms with a dense row) and tail runs (distinct other
// terms, each with its entries in slot order).
__global__ void __launch_bounds__(kPlanThreads)
plan_kernel(const int32_t* __restrict__ qi, const float* __restrict__ qs, int32_t B, int32_t W,
            int32_t V, int32_t npow2, const int64_t* __restrict__ offsets,
            const int32_t* __restrict__ head_slot, int32_t n_head, const float* __restrict__ term_scale,
            ScoreParams p) {
  extern __shared__ uint64_t keys[];
  __shared__ int32_t s_head, s_tail, s_runs;
  __shared__ int32_t w_head[kPlanThreads / 32], w_tail[kPlanThreads / 32], w_runs[kPlanThreads / 32];
  const int32_t q = blockIdx.x;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int32_t i = threadIdx.x; i < npow2; i += blockDim.x) {
    uint64_t key = ~0ull;
    if (i < W) {
      const int32_t t = qi[int64_t(q) * W + i];
      if (t >= 0 && t < V) key = (uint64_t(uint32_t(t)) << 32) | uint64_t(i);
    }
    keys[i] = key;
  }
  __syncthreads();
  for (int32_t size = 2; size <= npow2; size <<= 1) {
    for (int32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (int32_t i = threadIdx.x; i < npow2; i += blockDim.x) {
        const int32_t j = i ^ stride;
        if (j > i) {
          const uint64_t a = keys[i], b = keys[j];
          const bool up = (i & size) == 0;
          if ((a > b) == up) {
            keys[i] = b;
            keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  if (threadIdx.x == 0) s_head = s_tail = s_runs = 0;
  __syncthreads();
  const int64_t ob = int64_t(q) * p.ecap;
  uint16_t* head_h = const_cast<uint16_t*>(p.head_h) + ob;
  float* head_w = const_cast<float*>(p.head_w) + ob;
  float* head_sc = const_cast<float*>(p.head_scale) + ob;
  int32_t* run_term = const_cast<int32_t*>(p.run_term) + ob;
  uint32_t* run_b32 = const_cast<uint32_t*>(p.run_base32) + ob;
  uint16_t* run_end = const_cast<uint16_t*>(p.run_end) + ob;
  float* run_w0 = const_cast<float*>(p.run_w0) + ob;
  float* ent_w = const_cast<float*>(p.ent_w) + ob;
  for (int32_t i0 = 0; i0 < npow2; i0 += blockDim.x) {
    const int32_t i = i0 + threadIdx.x;
    const uint64_t key = keys[i];
    const bool valid = key != ~0ull;
    const int32_t t = int32_t(key >> 32);
    const int32_t s = int32_t(key & 0xFFFFFFFFu);
    const int32_t h = (valid && n_head > 0) ? head_slot[t] : -1;
    const bool is_head = valid && h >= 0;
    const bool is_tail = valid && h < 0;
    const bool start = is_tail && (i == 0 || int32_t(keys[i - 1] >> 32) != t);
    const bool last = is_tail && (i + 1 >= npow2 || int32_t(keys[i + 1] >> 32) != t);
    const uint32_t bh = __ballot_sync(FULL, is_head), bt = __ballot_sync(FULL, is_tail),
                   bs = __ballot_sync(FULL, start);
    if (lane == 0) {
      w_head[wid] = __popc(bh);
      w_tail[wid] = __popc(bt);
      w_runs[wid] = __popc(bs);
    }
    __syncthreads();
    int32_t oh = s_head, ot = s_tail, orr = s_runs;
    for (int w = 0; w < wid; ++w) {
      oh += w_head[w];
      ot += w_tail[w];
      orr += w_runs[w];
    }
    const uint32_t lt = lanemask_lt();
    const float qw = valid ? qs[int64_t(q) * W + s] : 0.f;
    if (is_head) {
      const int32_t e = oh + __popc(bh & lt);
      head_h[e] = uint16_t(h);
      head_w[e] = qw;
      head_sc[e] = term_scale ? term_scale[t] : 1.0f;
    }
    if (is_tail) {
      const int32_t e = ot + __popc(bt & lt);
      const int32_t r = orr + __popc(bs & lt) - (start ? 0 : 1);
      ent_w[e] = qw;
      if (start) {
        run_term[r] = t;
        run_b32[r] = uint32_t(offsets[t] >> 5);
        run_w0[r] = qw;
      }
      if (last) run_end[r] = uint16_t(e + 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 0; w < kPlanThreads / 32; ++w) {
        s_head += w_head[w];
        s_tail += w_tail[w];
        s_runs += w_runs[w];
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const_cast<int32_t*>(p.n_head_e)[q] = s_head;
    const_cast<int32_t*>(p.n_runs)[q] = s_runs;
  }
}

// ---------------------------------------------------------------------------- scoring

// Shared memory of one warp: its accumulator tile and a radix histogram.
struct WarpLayout {
  static constexpr int acc = 0;
  static constexpr int hist = kTile * 4;
  static constexpr int total = hist + 256 * 4;
};

// Radix select over the distinct keys buf[0..n) (n >= k >= 1): returns a key value P such
// that exactly k keys are >= P (P is the k-th largest key with its low bits cleared below
// the digit that decided it).  The buffer is written by warps of other SMs, so it is read
// through L2 (ld.global.cg).
__device__ uint64_t warp_select(const uint64_t* __restrict__ buf, int32_t n, int32_t k,
                                uint32_t* __restrict__ hist) {
  const int lane = lane_id();
  // All keys share the bytes above the highest bit where the smallest and largest differ;
  // the digit passes start below them.  Every pass issues kCompactUnroll loads per lane
  // before it uses any.
  uint64_t mn = ~0ull, mx = 0ull;
  for (int32_t i0 = 0; i0 < n; i0 += 32 * kCompactUnroll) {
    uint64_t kk[kCompactUnroll];
#pragma unroll
    for (int u = 0; u < kCompactUnroll; ++u) {
      const int32_t i = i0 + 32 * u + lane;
      kk[u] = i < n ? __ldcg(buf + i) : 0ull;
    }
#pragma unroll
    for (int u = 0; u < kCompactUnroll; ++u) {
      if (i0 + 32 * u + lane < n) {
        mn = min(mn, kk[u]);
        mx = max(mx, kk[u]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    mn = min(mn, (uint64_t)__shfl_xor_sync(FULL, (unsigned long long)mn, o));
    mx = max(mx, (uint64_t)__shfl_xor_sync(FULL, (unsigned long long)mx, o));
  }
  const uint64_t diff = mn ^ mx;
  const int top = diff ? 63 - __clzll((long long)diff) : 0;
  const int start = (top / 8) * 8;
  uint64_t prefix = start == 56 ? 0ull : (mn & (~0ull << (start + 8)));
  int32_t need = k;
  for (int shift = start; shift >= 0; shift -= 8) {
    for (int j = lane; j < 256; j += 32) hist[j] = 0u;
    __syncwarp();
    const uint64_t pmask = shift == 56 ? 0ull : (~0ull << (shift + 8));
    for (int32_t i0 = 0; i0 < n; i0 += 32 * kCompactUnroll) {
      uint64_t kk[kCompactUnroll];
#pragma unroll
      for (int u = 0; u < kCompactUnroll; ++u) {
        const int32_t i = i0 + 32 * u + lane;
        kk[u] = i < n ? __ldcg(buf + i) : 0ull;
      }
#pragma unroll
      for (int u = 0; u < kCompactUnroll; ++u) {
        const bool live = i0 + 32 * u + lane < n && (kk[u] & pmask) == prefix;
        const uint32_t dig = live ? uint32_t((kk[u] >> shift) & 255u) : 0x100u;
        const uint32_t peers = __match_any_sync(FULL, dig);
        if (live && (peers & lanemask_lt()) == 0u) hist[dig] += __popc(peers);
        __syncwarp();
      }
    }
    // digit D with (count above D) < need <= (count above D) + hist[D]
    int32_t s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += int32_t(hist[255 - 8 * lane - j]);
    int32_t incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t hit = __ballot_sync(FULL, incl >= need);
    const int L = __ffs(hit) - 1;
    int32_t above = incl - s, D = 0, cD = 0;
    if (lane == L) {
      for (int j = 0; j < 8; ++j) {
        const int bin = 255 - 8 * lane - j;
        const int32_t c = int32_t(hist[bin]);
        if (above + c >= need) {
          D = bin;
          cD = c;
          break;
        }
        above += c;
      }
    }
    D = __shfl_sync(FULL, D, L);
    cD = __shfl_sync(FULL, cD, L);
    above = __shfl_sync(FULL, above, L);
    need -= above;
    prefix |= uint64_t(D) << shift;
    __syncwarp();
    if (cD == need) break;
  }
  return prefix;
}

// Write exactly the k largest keys of buf[0..n) (n > k, keys distinct) to dst[0..k) in
// buffer order and return the smallest key value that is kept-or-better.  dst may be buf
// itself (in place: the writes never pass the loaded chunks) or an array that does not
// overlap it.
__device__ uint64_t warp_compact(const uint64_t* buf, int32_t n, int32_t k, uint32_t* __restrict__ hist,
                                 uint64_t* dst) {
  const int lane = lane_id();
  const uint64_t prefix = warp_select(buf, n, k, hist);
  // stable compaction of keys >= prefix
  int32_t out = 0;
  for (int32_t i0 = 0; i0 < n; i0 += 32 * kCompactUnroll) {
    uint64_t kk[kCompactUnroll];
#pragma unroll
    for (int u = 0; u < kCompactUnroll; ++u) {
      const int32_t i = i0 + 32 * u + lane;
      kk[u] = i < n ? __ldcg(buf + i) : 0ull;
    }
    __syncwarp();
#pragma unroll
    for (int u = 0; u < kCompactUnroll; ++u) {
      const bool keep = i0 + 32 * u + lane < n && kk[u] >= prefix;
      const uint32_t bal = __ballot_sync(FULL, keep);
      if (keep) dst[out + __popc(bal & lanemask_lt())] = kk[u];
      out += __popc(bal);
    }
  }
  __syncwarp();
  return prefix;
}

// acc[col] = fma(qw, w, acc[col]); the column test keeps a list that breaks the
// ascending-doc-id invariant from ever addressing outside the tile.
__device__ __forceinline__ void acc_add(float* __restrict__ acc, int32_t col, uint32_t span, float qw,
                                        float w) {
  if (uint32_t(col) < span) {
    float* a = acc + col;
    *a = __fmaf_rn(qw, w, *a);
  }
}

constexpr int kUnroll = 4;   // posting chunks of one run in flight together

// Postings [0, n) of one run (pd/pw point at its window) applied to its NE entries (NE = 1
// or 2 in registers; NE = 0: ne entries read from ew).  Every pass issues the loads of
// kUnroll chunks (predicated past n) before it applies any, so a run costs one memory
// round trip per 32 * kUnroll postings.  A list holds each document at most once (the
// index build merges repeats), so the pass reads all its accumulators, updates them in
// registers and writes them back without ordering the shared-memory accesses within it;
// the warp barrier at the end orders it before the next run, whose lanes may hold the
// same documents.
template <typename WT, int NE>
__device__ __forceinline__ void run_window(const int32_t* __restrict__ pd, const WT* __restrict__ pw,
                                           float scale, int32_t n, int32_t d0i, uint32_t span,
                                           float* __restrict__ acc, float w_a, float w_b,
                                           const float* __restrict__ ew, int32_t ne) {
  const int lane = lane_id();
  for (int32_t base = 0; base < n; base += 32 * kUnroll) {
    int32_t col[kUnroll];
    float w[kUnroll], v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int32_t i = base + 32 * u + lane;
      col[u] = -1;
      w[u] = 0.f;
      if (i < n) {
        col[u] = __ldg(pd + i) - d0i;
        w[u] = WDecode<WT>::get(pw, i, scale);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = uint32_t(col[u]) < span ? acc[col[u]] : 0.f;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if constexpr (NE >= 1) v[u] = __fmaf_rn(w_a, w[u], v[u]);
      if constexpr (NE >= 2) v[u] = __fmaf_rn(w_b, w[u], v[u]);
      if constexpr (NE == 0) {
        for (int32_t e = 0; e < ne; ++e) v[u] = __fmaf_rn(ew[e], w[u], v[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (uint32_t(col[u]) < span) acc[col[u]] = v[u];
    }
  }
  // the next run may add to the same documents from other lanes: this run's stores first
  __syncwarp();
}

// Two consecutive runs of one entry each and at most 64 postings each (A then B, in term
// order): the loads of both (two chunks each) in flight together, then A's chunks applied,
// a warp barrier, then B's (A and B may share documents, held by different lanes).
template <typename WT>
__device__ __forceinline__ void run_pair(const int32_t* __restrict__ pa, const WT* __restrict__ wa, float sa,
                                         int32_t na, float qa, const int32_t* __restrict__ pb,
                                         const WT* __restrict__ wb, float sb, int32_t nb, float qb,
                                         int32_t d0i, uint32_t span, float* __restrict__ acc) {
  const int lane = lane_id();
  int32_t col[4];
  float w[4], v[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int32_t i = 32 * (u & 1) + lane;
    const bool a = u < 2;
    col[u] = -1;
    w[u] = 0.f;
    if (i < (a ? na : nb)) {
      col[u] = __ldg((a ? pa : pb) + i) - d0i;
      w[u] = WDecode<WT>::get(a ? wa : wb, i, a ? sa : sb);
    }
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const float q = hh == 0 ? qa : qb;
#pragma unroll
    for (int u = 2 * hh; u < 2 * hh + 2; ++u) v[u] = uint32_t(col[u]) < span ? acc[col[u]] : 0.f;
#pragma unroll
    for (int u = 2 * hh; u < 2 * hh + 2; ++u) v[u] = __fmaf_rn(q, w[u], v[u]);
#pragma unroll
    for (int u = 2 * hh; u < 2 * hh + 2; ++u) {
      if (uint32_t(col[u]) < span) acc[col[u]] = v[u];
    }
    // B's lanes read a document only after A's lanes have stored it (the lanes of a warp
    // need not run in step between the phases)
    __syncwarp();
  }
}

// four consecutive weights of a dense head row, decoded to fp32
template <typename WT>
struct Vec4;
template <>
struct Vec4<float> {
  __device__ __forceinline__ static float4 get(const float* p, float) {
    return __ldg(reinterpret_cast<const float4*>(p));
  }
};
template <>
struct Vec4<__nv_bfloat16> {
  __device__ __forceinline__ static float4 get(const __nv_bfloat16* p, float) {
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
  }
};
template <>
struct Vec4<uint8_t> {
  __device__ __forceinline__ static float4 get(const uint8_t* p, float s) {
    const uint32_t u = __ldg(reinterpret_cast<const unsigned int*>(p));
    return make_float4(__fmul_rn(float(u & 255u), s), __fmul_rn(float((u >> 8) & 255u), s),
                       __fmul_rn(float((u >> 16) & 255u), s), __fmul_rn(float(u >> 24), s));
  }
};

__device__ __forceinline__ void fma4(float4& a, float qw, const float4 v) {
  a.x = __fmaf_rn(qw, v.x, a.x);
  a.y = __fmaf_rn(qw, v.y, a.y);
  a.z = __fmaf_rn(qw, v.z, a.z);
  a.w = __fmaf_rn(qw, v.w, a.w);
}

// Bit 4 * i + j of the result: document 128 * i + 4 * lane + j of the tile (below span)
// has a score at or above the score of threshold key thr.
__device__ __forceinline__ uint32_t mark_tile(const float* __restrict__ acc, int lane, uint32_t span,
                                              uint64_t thr) {
  const uint32_t thi = uint32_t(thr >> 32);
  const float ts = thi < 0x00800000u ? -INFINITY : fkey_inv(thi);
  uint32_t m = 0;
  if (span >= uint32_t(kSel)) {
    // a whole tile: set.ge gives an all-ones word per passing score, masked into its bit
#pragma unroll
    for (int i = 0; i < kSel / 128; ++i) {
      const float4 v = *reinterpret_cast<const float4*>(acc + 128 * i + 4 * lane);
      uint32_t r0, r1, r2, r3;
      asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(r0) : "f"(v.x), "f"(ts));
      asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(r1) : "f"(v.y), "f"(ts));
      asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(r2) : "f"(v.z), "f"(ts));
      asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(r3) : "f"(v.w), "f"(ts));
      m |= r0 & (1u << (4 * i));
      m |= r1 & (2u << (4 * i));
      m |= r2 & (4u << (4 * i));
      m |= r3 & (8u << (4 * i));
    }
    return m;
  }
#pragma unroll
  for (int i = 0; i < kSel / 128; ++i) {
    const float4 v = *reinterpret_cast<const float4*>(acc + 128 * i + 4 * lane);
    const uint32_t c = uint32_t(128 * i + 4 * lane);
    m |= uint32_t(c < span && v.x >= ts) << (4 * i);
    m |= uint32_t(c + 1 < span && v.y >= ts) << (4 * i + 1);
    m |= uint32_t(c + 2 < span && v.z >= ts) << (4 * i + 2);
    m |= uint32_t(c + 3 < span && v.w >= ts) << (4 * i + 3);
  }
  return m;
}

// Inclusive warp prefix sum.
__device__ __forceinline__ int32_t lane_scan(int32_t x) {
  const int lane = lane_id();
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  return x;
}

// Bounded polls of a word that other warps of this launch update (read through L2).
__device__ __forceinline__ bool wait_equal(const int32_t* a, int32_t v, int32_t limit) {
  for (int i = 0; i < limit; ++i) {
    if (*reinterpret_cast<const volatile int32_t*>(a) == v) return true;
    __nanosleep(64);
  }
  return false;
}
__device__ __forceinline__ bool wait_generation(const unsigned long long* a, uint32_t g, int32_t limit) {
  for (int i = 0; i < limit; ++i) {
    if (uint32_t(*reinterpret_cast<const volatile unsigned long long*>(a) >> 32) != g) return true;
    __nanosleep(64);
  }
  return false;
}

// Bounded wait until every slot of buf[0, n) holds a key (is not zero); read through L2,
// kCompactUnroll slots per lane at a time.  Warp-uniform result.
__device__ __noinline__ bool wait_keys(const uint64_t* buf, int32_t n, int32_t limit) {
  const int lane = lane_id();
  bool ok = true;
  for (int32_t i0 = 0; i0 < n; i0 += 32 * kCompactUnroll) {
    uint64_t kk[kCompactUnroll];
#pragma unroll
    for (int u = 0; u < kCompactUnroll; ++u) {
      const int32_t i = i0 + 32 * u + lane;
      kk[u] = i < n ? __ldcg(buf + i) : 1ull;
    }
#pragma unroll
    for (int u = 0; u < kCompactUnroll; ++u) {
      const volatile unsigned long long* slot =
          reinterpret_cast<const volatile unsigned long long*>(buf + i0 + 32 * u + lane);
      for (int32_t w = 0; kk[u] == 0ull && ok; ++w) {
        if (w >= limit) {
          ok = false;
          break;
        }
        __nanosleep(64);
        kk[u] = *slot;
      }
    }
  }
  return __all_sync(FULL, ok);
}

// Per-query state of the shared candidate buffers.
struct QueryBuf {
  uint64_t* region;            // keep list, buffer 0, buffer 1, stride keys apart
  int64_t stride;
  unsigned long long* gthr;
  unsigned long long* rg;
  int32_t* cdone;
  int32_t* fault;
  int32_t cap, k;
  int32_t wait_limit;
  int32_t kg;                  // > 0: also return the kg-th best key after a compaction
};

// Appends the tile's documents whose score reaches threshold key thr (marked in m) to a
// query's candidate buffers, following the protocol described at the top of the file.
// Called only for tiles with a candidate.  Returns 0, or, when this warp compacted and
// qb.kg > 0, a key that at least qb.kg keys of the new keep list reach.
__device__ __noinline__ uint64_t append_candidates(QueryBuf qb, const float* __restrict__ acc, uint32_t span,
                                               uint32_t dbase, uint32_t* __restrict__ hist, uint64_t thr,
                                               uint32_t m) {
  const int lane = lane_id();
  for (bool first = true;; first = false) {
    if (!first) m = mark_tile(acc, lane, span, thr);
    const int32_t cnt = __popc(m);
    const int32_t incl = lane_scan(cnt);
    const int32_t total = __shfl_sync(FULL, incl, 31);
    if (total == 0) return 0;
    // one atomic gives the reservation and the generation it belongs to
    unsigned long long word = 0;
    if (lane == 0) word = atomicAdd(qb.rg, (unsigned long long)total);
    word = __shfl_sync(FULL, word, 0);
    const int32_t pos = int32_t(uint32_t(word));
    const uint32_t g0 = uint32_t(word >> 32);
    const int bsel = int(g0 & 1u);
    uint64_t* __restrict__ buf = qb.region + (1 + bsel) * qb.stride;
    if (pos <= qb.cap) {
      // below the capacity: write the keys (a crossing reservation runs into the spare tail)
      int32_t o = pos + incl - cnt;
      while (m) {
        const int bit = __ffs(m) - 1;
        m &= m - 1;
        const int32_t col = 128 * (bit >> 2) + 4 * lane + (bit & 3);
        buf[o++] = pack_key(acc[col], dbase + uint32_t(col));
      }
      __syncwarp();
      // below the capacity the keys themselves mark their slots written
      if (pos + total <= qb.cap) return 0;
      // this warp crossed the capacity of generation g0
      bool ok = true;
      if (lane == 0) {
        // the previous compaction read the other buffer, wrote the keep list and zeroed
        // that buffer
        ok = wait_equal(qb.cdone, int32_t(g0), qb.wait_limit);
        // open generation g0 + 1 on the other buffer: the other warps go on there
        __threadfence();
        atomicExch(qb.rg, static_cast<unsigned long long>(g0 + 1u) << 32);
      }
      // every earlier reservation of generation g0 is written: its slots hold keys
      ok = wait_keys(buf, pos, qb.wait_limit) && __shfl_sync(FULL, int(ok), 0) != 0;
      if (!ok && lane == 0) atomicOr(qb.fault, 1);
      __syncwarp();
      __threadfence();
      // the k largest of this buffer and the keep list become the keep list
      int32_t n = pos + total;
      uint64_t* __restrict__ keep = qb.region;
      if (g0 > 0) {
        // the keep list appended behind the buffer's keys, kCompactUnroll loads per lane in
        // flight
        for (int32_t j0 = 0; j0 < qb.k; j0 += 32 * kCompactUnroll) {
          uint64_t kk[kCompactUnroll];
#pragma unroll
          for (int u = 0; u < kCompactUnroll; ++u) {
            const int32_t j = j0 + 32 * u + lane;
            kk[u] = j < qb.k ? __ldcg(keep + j) : 0ull;
          }
#pragma unroll
          for (int u = 0; u < kCompactUnroll; ++u) {
            const int32_t j = j0 + 32 * u + lane;
            if (j < qb.k) buf[n + j] = kk[u];
          }
        }
        n += qb.k;
        __syncwarp();
        __threadfence();
      }
      // the k largest straight into the keep list (its old keys are in buf now)
      const uint64_t t = warp_compact(buf, n, qb.k, hist, keep);
      __syncwarp();
      __threadfence();
      // the shared-bound key, read while this warp still owns the keep list: the next
      // compaction of this query, which rewrites it, waits for the cdone below
      const uint64_t pc = qb.kg > 0 ? warp_select(keep, qb.k, qb.kg, hist) : 0ull;
      // this generation's slots back to zero for the buffer's next generation
      for (int32_t j = lane; j < n; j += 32) buf[j] = 0ull;
      __syncwarp();
      __threadfence();
      if (lane == 0) {
        atomicMax(qb.gthr, (unsigned long long)t);
        __threadfence();
        atomicExch(qb.cdone, int32_t(g0 + 1u));
      }
      __syncwarp();
      return pc;
    }
    // generation g0 is full: wait until its crossing warp opens the next one, then retry
    // against the raised threshold
    bool ok = true;
    if (lane == 0) ok = wait_generation(qb.rg, g0, qb.wait_limit);
    ok = __shfl_sync(FULL, int(ok), 0) != 0;
    if (!ok) {
      if (lane == 0) atomicOr(qb.fault, 1);
      return 0;
    }
    thr = max(thr, uint64_t(__ldcg(qb.gthr)));
  }
}

// The kk (<= span) largest keys of one tile's scores (acc[col] for col < span, document
// dbase + col), written to out[0..kk) in column order, and zeros in out[kk..slots).  A
// radix select over the order-preserving score bits finds the kk-th largest score; every
// score above it is kept, and of the scores equal to it the lowest columns (the larger
// keys) until kk are kept, so the kept keys are exactly the kk largest.
__device__ __noinline__ void tile_topk(const float* __restrict__ acc, uint32_t span, uint32_t dbase,
                                       int32_t kk, int32_t slots, uint32_t* __restrict__ hist,
                                       uint64_t* __restrict__ out) {
  const int lane = lane_id();
  uint32_t u[kSel / 32];   // element 4 * i + j: column 128 * i + 4 * lane + j
#pragma unroll
  for (int i = 0; i < kSel / 128; ++i) {
    const float4 v = *reinterpret_cast<const float4*>(acc + 128 * i + 4 * lane);
    const uint32_t c = uint32_t(128 * i + 4 * lane);
    u[4 * i + 0] = c + 0 < span ? fkey(v.x) : 0u;
    u[4 * i + 1] = c + 1 < span ? fkey(v.y) : 0u;
    u[4 * i + 2] = c + 2 < span ? fkey(v.z) : 0u;
    u[4 * i + 3] = c + 3 < span ? fkey(v.w) : 0u;
  }
  uint32_t prefix = 0;
  int32_t need = kk;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int j = lane; j < 256; j += 32) hist[j] = 0u;
    __syncwarp();
    const uint32_t pmask = shift == 24 ? 0u : (~0u << (shift + 8));
#pragma unroll
    for (int e = 0; e < kSel / 32; ++e) {
      const bool live = (u[e] & pmask) == prefix;
      const uint32_t dig = live ? ((u[e] >> shift) & 255u) : 0x100u;
      const uint32_t peers = __match_any_sync(FULL, dig);
      if (live && (peers & lanemask_lt()) == 0u) hist[dig] += __popc(peers);
      __syncwarp();
    }
    // digit D with (count above D) < need <= (count above D) + hist[D]
    int32_t sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += int32_t(hist[255 - 8 * lane - j]);
    const int32_t incl = lane_scan(sum);
    const int L = __ffs(__ballot_sync(FULL, incl >= need)) - 1;
    int32_t above = incl - sum, D = 0;
    if (lane == L) {
      for (int j = 0; j < 8; ++j) {
        const int bin = 255 - 8 * lane - j;
        const int32_t c = int32_t(hist[bin]);
        if (above + c >= need) {
          D = bin;
          break;
        }
        above += c;
      }
    }
    D = __shfl_sync(FULL, D, L);
    above = __shfl_sync(FULL, above, L);
    need -= above;
    prefix |= uint32_t(D) << shift;
    __syncwarp();
  }
  // prefix is the kk-th largest score key; take every key above it and the first `need`
  // equal to it in column order
  int32_t base = 0, eq_seen = 0;
#pragma unroll
  for (int i = 0; i < kSel / 128; ++i) {
    uint32_t gtm = 0, eqm = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      gtm |= uint32_t(u[4 * i + j] > prefix) << j;
      eqm |= uint32_t(u[4 * i + j] == prefix && u[4 * i + j] != 0u) << j;
    }
    const int32_t neq = __popc(eqm);
    const int32_t eq_incl = lane_scan(neq);
    int32_t r = eq_seen + eq_incl - neq;
    uint32_t take = gtm;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if ((eqm >> j) & 1u) {
        if (r < need) take |= 1u << j;
        ++r;
      }
    }
    const int32_t nt = __popc(take);
    const int32_t t_incl = lane_scan(nt);
    int32_t o = base + t_incl - nt;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if ((take >> j) & 1u) {
        const int32_t col = 128 * i + 4 * lane + j;
        if (o < kk) out[o] = pack_key(acc[col], dbase + uint32_t(col));   // o < kk by construction
        ++o;
      }
    }
    base += __shfl_sync(FULL, t_incl, 31);
    eq_seen += __shfl_sync(FULL, eq_incl, 31);
  }
  for (int32_t j = kk + lane; j < slots; j += 32) out[j] = 0ull;
}

// Final candidate counts of every query: the keep list (k once a compaction happened) and
// the open buffer (its reserved slots, all written once the scorer has ended; a generation
// reserved past the capacity was compacted and closed by its crossing warp); the other
// buffer was compacted into the keep list.
__global__ void final_counts_kernel(int32_t B, int32_t k, int32_t cap, const unsigned long long* __restrict__ rg,
                                    const int32_t* __restrict__ cdone, int32_t* __restrict__ counts) {
  const int32_t q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= B) return;
  const unsigned long long w = rg[q];
  const int b = int((w >> 32) & 1ull);
  const int32_t n = int32_t(min(uint32_t(w), uint32_t(cap)));
  counts[3 * q + 0] = cdone[q] > 0 ? k : 0;
  counts[3 * q + 1] = b == 0 ? n : 0;
  counts[3 * q + 2] = b == 1 ? n : 0;
}

// Steps 2 and 3 of one work item (query q, tile b), after the head terms are in acc: the
// tail runs scattered into the shared-memory accumulators in ascending term id, then the
// selection of the launch's mode.  Shared by the CUDA-core scorer and the tensor-core one.
template <typename WT, int kMode>
__device__ __forceinline__ void item_tail_select(const ScoreParams& p, const int32_t q, const int32_t b,
                                                 float* __restrict__ acc, uint32_t* __restrict__ hist) {
  const int lane = lane_id();
  const WT* __restrict__ wts = static_cast<const WT*>(p.weights);
  const int32_t* __restrict__ doc_ids = p.doc_ids;
  const int64_t pbase = int64_t(q) * p.ecap;
  const int32_t nr = p.n_runs[q];
  const int32_t* __restrict__ run_term = p.run_term + pbase;
  const uint32_t* __restrict__ run_b32 = p.run_base32 + pbase;
  const uint16_t* __restrict__ run_end = p.run_end + pbase;
  const float* __restrict__ run_w0 = p.run_w0 + pbase;
  const float* __restrict__ ent_w = p.ent_w + pbase;
  const int32_t d0i = b * kTile;
  const int32_t d1 = int32_t(min64(int64_t(b + 1) * kTile, p.n_docs));
  const uint32_t span = uint32_t(d1 - d0i);
  const unsigned long long g_pub = __ldcg(p.gthr + q);   // consumed by the selection
  unsigned long long bnd = ~0ull;                        // lane s: shard s's row
  if (p.n_shards > 1 && lane < p.n_shards) bnd = __ldcg(p.board + int64_t(lane) * p.B + q);

  // 2. tail runs in ascending term id
  const uint32_t* __restrict__ brow = p.block_starts + int64_t(b) * kTileBlocksI * p.V;
  const uint32_t* __restrict__ brow_end =
      p.block_starts + int64_t(min((b + 1) * kTileBlocksI, p.n_iblocks)) * p.V;
  for (int32_t rb = 0; rb < nr; rb += 32) {
    const int32_t ri = rb + lane;
    uint32_t lo = 0, hi = 0, b32 = 0;
    int32_t e0 = 0, ne = 0;
    float w0 = 0.f, scale = 1.0f;
    if (ri < nr) {
      const int32_t t = run_term[ri];
      lo = __ldg(brow + t);
      hi = __ldg(brow_end + t);
      e0 = ri ? int32_t(run_end[ri - 1]) : 0;
      ne = int32_t(run_end[ri]) - e0;
      b32 = run_b32[ri];
      w0 = run_w0[ri];
      if constexpr (std::is_same<WT, uint8_t>::value) scale = __ldg(p.term_scale + t);
    }
    const int32_t n = int32_t(hi - lo);
    const uint32_t act = __ballot_sync(FULL, n > 0);
    const uint32_t lng = __ballot_sync(FULL, n > 0 && (n >= kLongRun || ne > 1));
    int c = 0;  // next run (lane) to process
    while (c < 32) {
      const uint32_t from = c ? ~((1u << c) - 1u) : FULL;
      if (!(act & from)) break;
      const uint32_t nl = lng & from;
      const int next_long = nl ? __ffs(nl) - 1 : 32;
      const uint32_t upto = next_long < 32 ? ((1u << next_long) - 1u) : FULL;
      const uint32_t seg = act & ~lng & from & upto;
      if (seg) {
        // consecutive short runs flattened into full 32-lane chunks
        const int m = __popc(seg);
        const int src = lane < m ? int(__fns(seg, 0, lane + 1)) : 0;
        const int32_t n_c = __shfl_sync(FULL, n, src);
        const uint32_t lo_c = __shfl_sync(FULL, lo, src), b32_c = __shfl_sync(FULL, b32, src);
        const float w_c = __shfl_sync(FULL, w0, src), s_c = __shfl_sync(FULL, scale, src);
        const int32_t sz = lane < m ? n_c : 0;
        int32_t incl = sz;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int32_t y = __shfl_up_sync(FULL, incl, o);
          if (lane >= o) incl += y;
        }
        const int32_t P = incl - sz;
        const int32_t total = __shfl_sync(FULL, incl, 31);
        for (int32_t F = 0; F < total; F += 32) {
          const int32_t f = F + lane;
          const bool valid = f < total;
          const uint32_t bit = (lane < m && P >= F && P < F + 32) ? (1u << (P - F)) : 0u;
          const uint32_t S = __reduce_or_sync(FULL, bit);
          const int jF = __popc(__ballot_sync(FULL, lane < m && P <= F)) - 1;
          int j = jF + __popc(S & (lanemask_lt() | (1u << lane)) & ~1u);
          j = valid ? j : 0;
          const int32_t Pj = __shfl_sync(FULL, P, j);
          const uint32_t loj = __shfl_sync(FULL, lo_c, j), bj = __shfl_sync(FULL, b32_c, j);
          const float wj = __shfl_sync(FULL, w_c, j), sj = __shfl_sync(FULL, s_c, j);
          int32_t col = -1;
          float wv = 0.f;
          if (valid) {
            const int64_t pos = (int64_t(bj) << 5) + loj + (f - Pj);
            col = __ldg(doc_ids + pos) - d0i;
            wv = WDecode<WT>::get(wts, pos, sj);
          }
          // lanes on the same document (different terms) apply in term (= lane) order
          const int32_t dkey = (valid && uint32_t(col) < span) ? col : -1 - lane;
          const uint32_t peers = __match_any_sync(FULL, dkey);
          const int rank = __popc(peers & lanemask_lt());
          const int top = int(__reduce_max_sync(FULL, uint32_t(rank)));
          for (int rr = 0; rr <= top; ++rr) {
            if (rank == rr) acc_add(acc, col, span, wj, wv);
            __syncwarp();
          }
        }
      }
      if (next_long >= 32) break;
      // one long (or multi-entry) run
      const int jl = next_long;
      const int32_t nl_n = __shfl_sync(FULL, n, jl);
      const uint32_t lo_l = __shfl_sync(FULL, lo, jl), b32_l = __shfl_sync(FULL, b32, jl);
      const int32_t e0_l = __shfl_sync(FULL, e0, jl), ne_l = __shfl_sync(FULL, ne, jl);
      const float w0_l = __shfl_sync(FULL, w0, jl), sc_l = __shfl_sync(FULL, scale, jl);
      const int64_t base = (int64_t(b32_l) << 5) + lo_l;
      if (ne_l == 1 && nl_n <= 64) {
        // the next run, if it is long with one entry and nothing lies between: as a pair
        const uint32_t after = act & ~((2u << jl) - 1u);
        const int j2 = after ? __ffs(after) - 1 : 32;
        if (j2 < 32 && ((lng >> j2) & 1u)) {
          const int32_t n2 = __shfl_sync(FULL, n, j2), ne2 = __shfl_sync(FULL, ne, j2);
          const uint32_t lo2 = __shfl_sync(FULL, lo, j2), b322 = __shfl_sync(FULL, b32, j2);
          const float w02 = __shfl_sync(FULL, w0, j2), sc2 = __shfl_sync(FULL, scale, j2);
          if (ne2 == 1 && n2 <= 64) {
            const int64_t base2 = (int64_t(b322) << 5) + lo2;
            run_pair<WT>(doc_ids + base, wts + base, sc_l, nl_n, w0_l, doc_ids + base2, wts + base2, sc2, n2,
                         w02, d0i, span, acc);
            c = j2 + 1;
            continue;
          }
        }
      }
      if (ne_l == 1) {
        run_window<WT, 1>(doc_ids + base, wts + base, sc_l, nl_n, d0i, span, acc, w0_l, 0.f, nullptr, 0);
      } else if (ne_l == 2) {
        run_window<WT, 2>(doc_ids + base, wts + base, sc_l, nl_n, d0i, span, acc, w0_l, ent_w[e0_l + 1],
                          nullptr, 0);
      } else {
        run_window<WT, 0>(doc_ids + base, wts + base, sc_l, nl_n, d0i, span, acc, 0.f, 0.f, ent_w + e0_l,
                          ne_l);
      }
      c = jl + 1;
    }
  }
  __syncwarp();

  // 3. fused selection: the documents whose score reaches the query's threshold go to
  // its candidate buffer (a superset of the keys >= threshold is harmless: only the k
  // largest survive the compactions and the merge)
  uint64_t thr = uint64_t(g_pub);
  if (p.n_shards > 1) {
#pragma unroll
    for (int o = 16; o; o >>= 1) bnd = min(bnd, __shfl_xor_sync(FULL, bnd, o));
    thr = max(thr, uint64_t(bnd));
  }
  if constexpr (kMode == kModeTree) {
    // small-batch mode (one selection pass per tile): the tile's own exact top-k
    tile_topk(acc, span, uint32_t(p.doc_base + d0i), min(p.tile_k, int32_t(span)), p.tile_k, hist,
              p.tile_out + (int64_t(q) * p.n_blocks + b) * p.tile_k);
  } else if constexpr (kMode == kModeDense) {
    // every document's key (lane writes columns 128 i + 4 lane .. + 3, two 16-byte stores)
    uint64_t* __restrict__ row = p.dense + int64_t(q - p.q_lo) * p.dense_ld + d0i;
    const uint32_t dbase = uint32_t(p.doc_base + d0i);
#pragma unroll
    for (int i = 0; i < kTile / 128; ++i) {
      const uint32_t c = uint32_t(128 * i + 4 * lane);
      const float4 v = *reinterpret_cast<const float4*>(acc + c);
      ulonglong2 k0, k1;
      k0.x = c + 0 < span ? pack_key(v.x, dbase + c + 0) : 0ull;
      k0.y = c + 1 < span ? pack_key(v.y, dbase + c + 1) : 0ull;
      k1.x = c + 2 < span ? pack_key(v.z, dbase + c + 2) : 0ull;
      k1.y = c + 3 < span ? pack_key(v.w, dbase + c + 3) : 0ull;
      *reinterpret_cast<ulonglong2*>(row + c) = k0;
      *reinterpret_cast<ulonglong2*>(row + c + 2) = k1;
    }
  } else {
#pragma unroll
  for (int h = 0; h < kTile / kSel; ++h) {
    if (uint32_t(h * kSel) >= span) break;
    const uint32_t sp = min(span - uint32_t(h * kSel), uint32_t(kSel));
    const uint32_t m = mark_tile(acc + h * kSel, lane, sp, thr);
    if (__any_sync(FULL, m != 0u)) {
      QueryBuf qb{p.cand + int64_t(q) * 3 * p.cand_stride, p.cand_stride, p.gthr + q, p.rg + q,
                  p.cdone + q, p.fault, p.cap, p.k, p.wait_limit, p.kg};
      const uint64_t pub =
          append_candidates(qb, acc + h * kSel, sp, uint32_t(p.doc_base + d0i + h * kSel), hist, thr, m);
      // this shard's row of every board: local, then the peers' (remote reductions over
      // NVLink; nothing waits on them)
      if (pub != 0ull) {
        const int64_t slot = int64_t(p.shard) * p.B + q;
        if (lane == 0) atomicMax(p.board + slot, (unsigned long long)pub);
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r) {
          if (r < p.n_peers && lane == r + 1) atomicMax(p.peer_thr[r] + slot, (unsigned long long)pub);
        }
      }
    }
  }
  }
}

// WT: posting weight type; HT: head row type (WT, or float rows for uint8 postings);
// kMode: kModeBuffers, kModeTree (per-tile top-k lists instead of the shared candidate
// buffers) or kModeDense (every key written out).
template <typename WT, typename HT, int kMode>
__global__ void __launch_bounds__(kWarps * 32, kCtasPerSm)
score_kernel(const ScoreParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = lane_id(), wid = threadIdx.x >> 5;
  unsigned char* wsm = smem + size_t(wid) * WarpLayout::total;
  float* acc = reinterpret_cast<float*>(wsm + WarpLayout::acc);
  uint32_t* hist = reinterpret_cast<uint32_t*>(wsm + WarpLayout::hist);
  const HT* __restrict__ hrows = static_cast<const HT*>(p.head_rows);
  const unsigned long long n_items = (unsigned long long)p.q_n * unsigned(p.n_blocks);
  unsigned long long nit = 0;   // the claimed item (lane 0)
  if (lane == 0) nit = atomicAdd(p.item_next, 1ull);
  for (;;) {
    const unsigned long long it = __shfl_sync(FULL, nit, 0);
    if (it >= n_items) break;
    // claim the next item now, so the atomic's round trip overlaps this item's work
    if (lane == 0) nit = atomicAdd(p.item_next, 1ull);
    // items stay below 2^31 (make_cfg), so 32-bit division suffices
    const uint32_t it32 = uint32_t(it);
    if (p.jitter_ns > 0 && lane == 0 && ((it32 * 2654435761u) >> 31) != 0u) __nanosleep(uint32_t(p.jitter_ns));
    const int32_t b = int32_t(it32 / uint32_t(p.q_n));
    const int32_t q = p.q_lo + int32_t(it32 - uint32_t(b) * uint32_t(p.q_n));
    const int64_t pbase = int64_t(q) * p.ecap;
    const int32_t nhe = p.n_head_e[q];
    const uint16_t* __restrict__ head_h = p.head_h + pbase;
    const float* __restrict__ head_w = p.head_w + pbase;
    const float* __restrict__ head_sc = p.head_scale + pbase;
    {
      const int32_t d0i = b * kTile;

      // 1. head rows, accumulators in registers: in each of the kHeadParts parts of the
      // tile, lane owns documents part * kTile / kHeadParts + 128 * i + 4 * lane + j
#pragma unroll 1
      for (int part = 0; part < kHeadParts; ++part) {
        const int32_t pofs = part * (kTile / kHeadParts);
        float4 a[kHeadVec];
#pragma unroll
        for (int i = 0; i < kHeadVec; ++i) a[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int32_t e = 0; e < nhe; ++e) {
          const int32_t h = head_h[e];
          const float qw = head_w[e];
          float sc = 1.0f;
          if constexpr (std::is_same<HT, uint8_t>::value) sc = head_sc[e];
          const HT* row = hrows + int64_t(h) * p.head_ld + d0i + pofs + 4 * lane;
          float4 v[kHeadVec];
#pragma unroll
          for (int i = 0; i < kHeadVec; ++i) v[i] = Vec4<HT>::get(row + 128 * i, sc);
#pragma unroll
          for (int i = 0; i < kHeadVec; ++i) fma4(a[i], qw, v[i]);
        }
#pragma unroll
        for (int i = 0; i < kHeadVec; ++i) *reinterpret_cast<float4*>(acc + pofs + 128 * i + 4 * lane) = a[i];
      }
      __syncwarp();
      item_tail_select<WT, kMode>(p, q, b, acc, hist);
    }
  }
}

#include "score_tc.cuh"

struct Cfg {
  bool tree = false;   // small-batch mode: per-tile top-k lists and a merge tree
  bool dense = false;  // k above kMaxSmemK: all keys written, a window of queries at a time
  bool tc = false;     // head terms on the tensor cores (score_tc_kernel)
  int64_t qh_rows = 0, off_qh = 0, off_qhlo = 0;
  int64_t dense_q = 0, dense_ld = 0, off_dense = 0, off_large = 0;
  int64_t off_tiles = 0, off_lv0 = 0, off_lv1 = 0;
  int npow2 = 0, cap = 0, smem = 0, ctas_per_sm = 0, grid = 0;
  int64_t ecap = 0, n_blocks = 0, n_iblocks = 0, kk = 0, stride = 0;
  int64_t off_nhe = 0, off_hh = 0, off_hw = 0, off_hs = 0, off_nruns = 0, off_rterm = 0, off_rb32 = 0,
          off_rend = 0, off_rw0 = 0, off_entw = 0, off_cand = 0, off_counts = 0, off_zero = 0, zero_bytes = 0,
          total = 0;
};

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }
std::atomic<int32_t> g_wait_limit{kSpinLimit};
std::atomic<int32_t> g_jitter_ns{0};
// How head terms are summed.  The automatic mode uses the CUDA cores: for the fp32 head rows
// of fp32 and uint8 indexes the tensor-core path measured slower on B200 (see score_tc.cuh),
// and bf16 rows have no tensor-core path.
std::atomic<int32_t> g_head_mode{GSP_HEAD_AUTO};

PFN_cuTensorMapEncodeTiled_v12000 tma_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      f = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}
// largest per-tile list buffer (B x tiles x k keys) for which a batch takes the merge tree
std::atomic<int64_t> g_tree_limit{int64_t(256) << 20};
int64_t align8(int64_t x) { return (x + 7) / 8 * 8; }

// Workspace layout of one call for the configured buffer capacity.
void set_layout(Cfg& c, int64_t B) {
  int64_t o = 0;
  const int64_t E = B * c.ecap;
  c.stride = c.cap + kSel + c.kk;
  c.off_nhe = o; o = align256(o + B * 4);
  c.off_hh = o; o = align256(o + E * 2);
  c.off_hw = o; o = align256(o + E * 4);
  c.off_hs = o; o = align256(o + E * 4);
  c.off_nruns = o; o = align256(o + B * 4);
  c.off_rterm = o; o = align256(o + E * 4);
  c.off_rb32 = o; o = align256(o + E * 4);
  c.off_rend = o; o = align256(o + E * 2);
  c.off_rw0 = o; o = align256(o + E * 4);
  c.off_entw = o; o = align256(o + E * 4);
  c.off_cand = o; o = align256(o + (c.dense ? 0 : B * 3 * c.stride * 8));
  c.off_counts = o; o = align256(o + B * 3 * 4);
  // cleared by every call: thresholds [B] u64, reservation words [B] u64, finished
  // compactions [B], item counter u64, fault flag
  c.off_zero = o; c.zero_bytes = align8(2 * B * 8 + B * 4) + 24; o = align256(o + c.zero_bytes);
  if (c.tc) {
    c.qh_rows = (B + tc::kUnitQ - 1) / tc::kUnitQ * tc::kUnitQ;
    c.off_qh = o; o = align256(o + c.qh_rows * 128 * 4);
    c.off_qhlo = o; o = align256(o + c.qh_rows * 128 * 4);
  }
  if (c.tree) {
    const int64_t g1 = (c.n_blocks + kTreeFanIn - 1) / kTreeFanIn;
    c.off_tiles = o; o = align256(o + B * c.n_blocks * c.kk * 8);
    c.off_lv0 = o; o = align256(o + B * g1 * c.kk * 8);
    c.off_lv1 = o; o = align256(o + B * ((g1 + kTreeFanIn - 1) / kTreeFanIn) * c.kk * 8);
  }
  if (c.dense) {
    c.off_dense = o; o = align256(o + c.dense_q * c.dense_ld * 8);
    c.off_large = o; o = align256(o + large_k_ws_bytes(c.dense_q, c.kk));
  }
  c.total = o;
}

int make_cfg(const gsp_index_view* ix, int64_t B, int64_t W, int64_t k, Cfg& c) {
  GSP_REQUIRE(ix && ix->V > 0 && ix->n_docs >= 0 && ix->block_docs > 0, GSP_ERR_ARG,
              "score: bad index view");
  GSP_REQUIRE(ix->block_docs == kBlock, GSP_ERR_UNSUPPORTED,
              "score: the scorer needs index blocks of %d documents (this index has %d)", kBlock,
              ix->block_docs);
  GSP_REQUIRE(B >= 0 && W >= 1 && k >= 1, GSP_ERR_ARG, "score: bad batch shape (B=%lld W=%lld k=%lld)",
              (long long)B, (long long)W, (long long)k);
  GSP_REQUIRE(W <= kMaxWidth, GSP_ERR_UNSUPPORTED,
              "score: query width %lld exceeds the supported maximum %d", (long long)W, kMaxWidth);
  GSP_REQUIRE(ix->n_head >= 0 && ix->n_head <= 65535 && (ix->n_head == 0 || (ix->head_slot && ix->head_rows)),
              GSP_ERR_ARG, "score: bad head rows");
  c.kk = std::min<int64_t>(k, ix->n_docs);
  GSP_REQUIRE(c.kk < 0x7FFFFFFFll, GSP_ERR_UNSUPPORTED, "score: top_k %lld too large", (long long)c.kk);
  const int sms = num_sms();
  c.ecap = W;
  c.smem = WarpLayout::total * kWarps;
  c.ctas_per_sm = kCtasPerSm;
  c.npow2 = kPlanThreads;
  while (c.npow2 < W) c.npow2 <<= 1;
  c.n_blocks = (ix->n_docs + kTile - 1) / kTile;
  c.n_iblocks = (ix->n_docs + kBlock - 1) / kBlock;
  // one persistent CTA per resident slot; fewer when the batch has fewer items
  const int64_t items = B * c.n_blocks;
  c.grid = int(std::max<int64_t>(1, std::min<int64_t>(int64_t(sms) * c.ctas_per_sm, (items + kWarps - 1) / kWarps)));
  // a compaction keeps k keys; the rest of the capacity takes at least one selection
  // pass's candidates.  Small buffers compact more often and so raise the threshold
  // sooner, which measured slightly faster than larger ones.
  c.cap = int(((c.kk + std::max<int64_t>(kSel, c.kk / 2) + 31) / 32) * 32);
  // Small batches spread every query over thousands of warps that would all append to one
  // candidate buffer, so the shared buffers serialise on its compactions; there each tile
  // keeps its own top-k instead and a merge tree reduces the lists.
  // Measured on B200: the tree wins for k' of a few hundred and more while B x tiles stays
  // within a few times the number of warps (~24K); for small k' the shared buffers'
  // compactions are short anyway.
  c.tree = kTile == kSel && c.kk <= kSel && c.kk >= kTreeMinK && c.n_blocks > 0 && B > 0 &&
           B * c.n_blocks <= kTreeMaxTiles && B * c.n_blocks * c.kk * 8 <= g_tree_limit.load();
  // Above kMaxSmemK keys per query the candidate buffers and the shared-memory sort do not
  // apply: every key is written out for a window of queries whose keys (and the global
  // sort's two buffers) fit about kDenseBytes, and the windows are selected one by one.
  c.dense = c.kk > kMaxSmemK;
  // head terms on the tensor cores: fp32 head rows (fp32 and uint8 indexes) with their 3xTF32
  // low parts, unless the caller asked for the canonical CUDA-core order
  const int32_t mode = g_head_mode.load();
  c.tc = mode == GSP_HEAD_TENSOR_CORES && B > 0 && c.n_blocks > 0 && ix->n_head >= tc::kKC &&
         ix->n_head <= 128 && ix->head_lo != nullptr && ix->head_wdtype == GSP_W_F32 &&
         tma_encoder() != nullptr;
  if (c.dense) {
    c.dense_ld = c.n_blocks * kTile;
    const int64_t per_q = c.dense_ld * 8 + large_k_ws_bytes(1, c.kk);
    c.dense_q = std::max<int64_t>(1, std::min<int64_t>(B, kDenseBytes / per_q));
    GSP_REQUIRE(c.dense_q * c.n_blocks < (int64_t(1) << 31), GSP_ERR_UNSUPPORTED,
                "score: too many documents for the dense selection");
  }
  set_layout(c, B);
  return GSP_OK;
}

// Optional timing of the scoring kernel's launches with CUDA events on the launching
// stream (one device per process); read back by gsp_profile_collect.
struct Profile {
  std::mutex mu;
  bool on = false;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;
  size_t used = 0;
};
Profile& profile() {
  static Profile p;
  return p;
}

// The profiling event pair of the next scoring launch, or null when profiling is off.
int profile_slot(std::pair<cudaEvent_t, cudaEvent_t>** evp) {
  Profile& pr = profile();
  *evp = nullptr;
  std::lock_guard<std::mutex> g(pr.mu);
  if (pr.on) {
    if (pr.used == pr.ev.size()) {
      cudaEvent_t a, b;
      GSP_CUDA(cudaEventCreate(&a));
      GSP_CUDA(cudaEventCreate(&b));
      pr.ev.emplace_back(a, b);
    }
    *evp = &pr.ev[pr.used++];
  }
  return GSP_OK;
}

template <typename WT, typename HT>
int launch_score(const ScoreParams& p, const Cfg& c, cudaStream_t st) {
  auto kern = c.dense ? score_kernel<WT, HT, kModeDense>
                      : (c.tree ? score_kernel<WT, HT, kModeTree> : score_kernel<WT, HT, kModeBuffers>);
  if (int rc = ensure_smem(reinterpret_cast<const void*>(kern), c.smem)) return rc;
  std::pair<cudaEvent_t, cudaEvent_t>* evp = nullptr;
  if (int rc = profile_slot(&evp)) return rc;
  if (evp) GSP_CUDA(cudaEventRecord(evp->first, st));
  kern<<<unsigned(c.grid), kWarps * 32, c.smem, st>>>(p);
  GSP_CHECK_LAUNCH();
  if (evp) GSP_CUDA(cudaEventRecord(evp->second, st));
  return GSP_OK;
}

// The tensor-core scorer over queries [p.q_lo, p.q_lo + p.q_n): one persistent CTA per SM.
template <typename WT>
int launch_score_tc(const ScoreParams& p, TcParams& tp, const Cfg& c, cudaStream_t st) {
  auto kern = c.dense ? score_tc_kernel<WT, kModeDense>
                      : (c.tree ? score_tc_kernel<WT, kModeTree> : score_tc_kernel<WT, kModeBuffers>);
  const int smem = tc::kSmem + 1024;
  if (int rc = ensure_smem(reinterpret_cast<const void*>(kern), smem)) return rc;
  tp.n_groups = (p.q_n + tc::kUnitQ - 1) / tc::kUnitQ;
  tp.n_units = int32_t(c.n_blocks) * tp.n_groups;
  GSP_CUDA(cudaMemsetAsync(tp.unit_next, 0, sizeof(unsigned long long), st));
  std::pair<cudaEvent_t, cudaEvent_t>* evp = nullptr;
  if (int rc = profile_slot(&evp)) return rc;
  if (evp) GSP_CUDA(cudaEventRecord(evp->first, st));
  const int grid = std::max(1, std::min(num_sms(), tp.n_units));
  kern<<<unsigned(grid), tc::kThreads, smem, st>>>(p, tp);
  GSP_CHECK_LAUNCH();
  if (evp) GSP_CUDA(cudaEventRecord(evp->second, st));
  return GSP_OK;
}

// Tensor maps of the head rows (hi = the rows, lo = their 3xTF32 low parts) and of the
// batch's dense query head weights.
int make_tc_params(const gsp_index_view* ix, const Cfg& c, float* qh, float* qh_lo, TcParams& tp) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tma_encoder();
  GSP_REQUIRE(enc, GSP_ERR_CUDA, "score: cuTensorMapEncodeTiled is not available");
  GSP_REQUIRE(ix->head_ld % 32 == 0 && (reinterpret_cast<uintptr_t>(ix->head_rows) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(ix->head_lo) & 15) == 0,
              GSP_ERR_ARG, "score: head rows must be 16-byte aligned with a multiple of 32 columns");
  {
    const cuuint64_t dims[3] = {32, cuuint64_t(ix->n_head), cuuint64_t(ix->head_ld / 32)};
    const cuuint64_t strides[2] = {cuuint64_t(ix->head_ld) * 4, 128};
    const cuuint32_t box[3] = {32, tc::kKC, 4};
    const cuuint32_t es[3] = {1, 1, 1};
    const void* src[2] = {ix->head_rows, ix->head_lo};
    CUtensorMap* dst[2] = {&tp.a_hi, &tp.a_lo};
    for (int i = 0; i < 2; ++i) {
      const CUresult r = enc(dst[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(src[i]), dims, strides, box,
                             es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      GSP_REQUIRE(r == CUDA_SUCCESS, GSP_ERR_CUDA, "score: head-row tensor map failed (%d)", int(r));
    }
  }
  {
    const cuuint64_t dims[2] = {128, cuuint64_t(c.qh_rows)};
    const cuuint64_t strides[1] = {128 * 4};
    const cuuint32_t box[2] = {tc::kKC, tc::kUnitQ};
    const cuuint32_t es[2] = {1, 1};
    float* src[2] = {qh, qh_lo};
    CUtensorMap* dst[2] = {&tp.b_hi, &tp.b_lo};
    for (int i = 0; i < 2; ++i) {
      const CUresult r = enc(dst[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, src[i], dims, strides, box, es,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      GSP_REQUIRE(r == CUDA_SUCCESS, GSP_ERR_CUDA, "score: query-weight tensor map failed (%d)", int(r));
    }
  }
  tp.n_kc = (ix->n_head + tc::kKC - 1) / tc::kKC;
  return GSP_OK;
}

}  // namespace
}  // namespace gsp

using namespace gsp;

extern "C" int64_t gsp_score_ws_bytes(const gsp_index_view* ix, int64_t B, int64_t W, int64_t k) {
  Cfg c;
  const int rc = make_cfg(ix, B, W, k, c);
  if (rc != GSP_OK) return -int64_t(rc);  // negative status; gsp_last_error() has the reason
  return c.total;
}

// Everything after the configuration: plan, scoring kernel, merge, with the workspace at ws.
static int score_with_cfg(const gsp_index_view* ix, const int32_t* qi, const float* qs, int64_t B,
                          int64_t W, const Cfg& c, float* out_scores, int64_t* out_ids,
                          uint64_t* out_keys, void* ws, cudaStream_t st, uint64_t* board = nullptr,
                          int32_t shard = 0, int32_t n_shards = 1, uint64_t* const* peers = nullptr) {
  int rc = GSP_OK;
  GSP_REQUIRE(ix->doc_ids && ix->weights && ix->offsets && ix->lengths && ix->block_starts &&
                  (ix->wdtype != GSP_W_U8 || ix->term_scale),
              GSP_ERR_ARG, "gsp_score_topk: null index array");
  GSP_REQUIRE(ix->doc_base >= 0 && ix->doc_base + ix->n_docs <= 0xFFFFFFFEll, GSP_ERR_UNSUPPORTED,
              "gsp_score_topk: global doc ids must stay below 2^32 - 1");
  if (B == 0 || c.kk == 0) return GSP_OK;
  GSP_REQUIRE(qi && qs && out_scores && out_ids, GSP_ERR_ARG, "gsp_score_topk: null argument");
  GSP_REQUIRE(ix->n_head == 0 || ix->head_ld >= c.n_blocks * kTile, GSP_ERR_ARG,
              "gsp_score_topk: head rows shorter than the block-padded document count");
  char* w = static_cast<char*>(ws);
  ScoreParams p;
  p.doc_ids = ix->doc_ids;
  p.weights = ix->weights;
  p.term_scale = ix->term_scale;
  p.block_starts = ix->block_starts;
  p.head_rows = ix->head_rows;
  p.head_ld = ix->head_ld;
  p.n_docs = ix->n_docs;
  p.doc_base = ix->doc_base;
  p.V = ix->V;
  p.n_blocks = int32_t(c.n_blocks);
  p.n_iblocks = int32_t(c.n_iblocks);
  p.B = int32_t(B);
  p.k = int32_t(c.kk);
  p.ecap = int32_t(c.ecap);
  p.cap = c.cap;
  p.wait_limit = g_wait_limit.load();
  p.jitter_ns = g_jitter_ns.load();
  p.cand_stride = c.stride;
  p.n_head_e = reinterpret_cast<int32_t*>(w + c.off_nhe);
  p.head_h = reinterpret_cast<uint16_t*>(w + c.off_hh);
  p.head_w = reinterpret_cast<float*>(w + c.off_hw);
  p.head_scale = reinterpret_cast<float*>(w + c.off_hs);
  p.n_runs = reinterpret_cast<int32_t*>(w + c.off_nruns);
  p.run_term = reinterpret_cast<int32_t*>(w + c.off_rterm);
  p.run_base32 = reinterpret_cast<uint32_t*>(w + c.off_rb32);
  p.run_end = reinterpret_cast<uint16_t*>(w + c.off_rend);
  p.run_w0 = reinterpret_cast<float*>(w + c.off_rw0);
  p.ent_w = reinterpret_cast<float*>(w + c.off_entw);
  p.cand = reinterpret_cast<uint64_t*>(w + c.off_cand);
  char* z = w + c.off_zero;
  p.gthr = reinterpret_cast<unsigned long long*>(z);
  p.rg = reinterpret_cast<unsigned long long*>(z + B * 8);
  p.cdone = reinterpret_cast<int32_t*>(z + 2 * B * 8);
  p.counts = reinterpret_cast<int32_t*>(w + c.off_counts);
  p.item_next = reinterpret_cast<unsigned long long*>(z + align8(2 * B * 8 + B * 4));
  p.fault = reinterpret_cast<int32_t*>(p.item_next + 1);
  unsigned long long* unit_next = p.item_next + 2;
  GSP_REQUIRE(n_shards >= 1 && n_shards <= kMaxPeers + 1 && shard >= 0 && shard < n_shards &&
                  (n_shards == 1 || (board && peers)),
              GSP_ERR_ARG, "gsp_score_topk_shared: bad shard arguments (shard %d of %d, at most %d)", shard,
              n_shards, kMaxPeers + 1);
  p.board = reinterpret_cast<unsigned long long*>(board);
  p.n_shards = n_shards;
  p.shard = shard;
  p.n_peers = n_shards - 1;
  p.kg = n_shards > 1 ? int32_t((c.kk + n_shards - 1) / n_shards) : 0;
  p.tile_out = c.tree ? reinterpret_cast<uint64_t*>(w + c.off_tiles) : nullptr;
  p.tile_k = int32_t(c.kk);
  p.q_lo = 0;
  p.q_n = int32_t(B);
  p.dense = c.dense ? reinterpret_cast<uint64_t*>(w + c.off_dense) : nullptr;
  p.dense_ld = c.dense_ld;
  for (int r = 0; r < kMaxPeers; ++r) {
    p.peer_thr[r] = r < p.n_peers ? reinterpret_cast<unsigned long long*>(peers[r]) : nullptr;
    GSP_REQUIRE(r >= p.n_peers || p.peer_thr[r], GSP_ERR_ARG, "gsp_score_topk_shared: null peer board %d", r);
  }
  GSP_CUDA(cudaMemsetAsync(z, 0, size_t(c.zero_bytes), st));
  if (!c.tree && !c.dense && B > 0) {
    // both candidate buffers of every query start empty (all zeros); the keep lists are
    // written before they are read
    GSP_CUDA(cudaMemset2DAsync(p.cand + c.stride, size_t(3 * c.stride * 8), 0, size_t(2 * c.stride * 8), size_t(B),
                               st));
  }

  const size_t plan_smem = size_t(c.npow2) * 8;
  rc = ensure_smem(reinterpret_cast<const void*>(plan_kernel), int(plan_smem));
  if (rc) return rc;
  plan_kernel<<<unsigned(B), kPlanThreads, plan_smem, st>>>(
      qi, qs, int32_t(B), int32_t(W), ix->V, c.npow2, ix->offsets, ix->head_slot, ix->n_head,
      ix->wdtype == GSP_W_U8 ? ix->term_scale : nullptr, p);
  GSP_CHECK_LAUNCH();

  // head rows share the postings' type, except that uint8 postings may have fp32 rows
  const int32_t hdt = ix->n_head > 0 ? ix->head_wdtype : ix->wdtype;
  GSP_REQUIRE(hdt == ix->wdtype || (ix->wdtype == GSP_W_U8 && hdt == GSP_W_F32), GSP_ERR_ARG,
              "gsp_score_topk: head rows of type %d do not go with weights of type %d", hdt, ix->wdtype);
  TcParams tp;
  if (c.tc) {
    float* qh = reinterpret_cast<float*>(w + c.off_qh);
    float* qh_lo = reinterpret_cast<float*>(w + c.off_qhlo);
    qhead_kernel<<<unsigned(c.qh_rows), 128, 0, st>>>(p, int32_t(B), ix->n_head, qh, qh_lo);
    GSP_CHECK_LAUNCH();
    rc = make_tc_params(ix, c, qh, qh_lo, tp);
    if (rc) return rc;
    tp.unit_next = unit_next;
  }
  auto launch = [&](const ScoreParams& pp) -> int {
    if (c.tc) {
      // fp32 head rows: fp32 postings, or uint8 postings with dequantised rows
      return ix->wdtype == GSP_W_U8 ? launch_score_tc<uint8_t>(pp, tp, c, st) : launch_score_tc<float>(pp, tp, c, st);
    }
    switch (ix->wdtype) {
      case GSP_W_F32: return launch_score<float, float>(pp, c, st);
      case GSP_W_BF16: return launch_score<__nv_bfloat16, __nv_bfloat16>(pp, c, st);
      case GSP_W_U8:
        return hdt == GSP_W_F32 ? launch_score<uint8_t, float>(pp, c, st) : launch_score<uint8_t, uint8_t>(pp, c, st);
      default: set_error("gsp_score_topk: unknown weight dtype %d", ix->wdtype); return GSP_ERR_ARG;
    }
  };
  if (c.dense) {
    // a window of dense_q queries at a time: all their keys, then the exact top-k' of each
    // row (radix select over the row, global sort of the k' keys)
    for (int64_t q0 = 0; q0 < B; q0 += c.dense_q) {
      const int64_t qn = std::min<int64_t>(c.dense_q, B - q0);
      ScoreParams pw = p;
      pw.q_lo = int32_t(q0);
      pw.q_n = int32_t(qn);
      GSP_CUDA(cudaMemsetAsync(p.item_next, 0, sizeof(unsigned long long), st));
      rc = launch(pw);
      if (rc) return rc;
      const int32_t row_len = int32_t(c.dense_ld);
      rc = merge_topk_device(pw.dense, qn, 1, c.dense_ld, c.dense_ld, nullptr, 0, &row_len, c.kk,
                             out_scores + q0 * c.kk, out_ids + q0 * c.kk, out_keys ? out_keys + q0 * c.kk : nullptr,
                             st, -1, p.fault, w + c.off_large);
      if (rc) return rc;
    }
    return GSP_OK;
  }
  if (c.n_blocks > 0) {
    rc = launch(p);
    if (rc) return rc;
  }
  if (c.tree) {
    // merge tree over the per-tile lists: kTreeFanIn lists per node, the last level into
    // the output
    const uint64_t* in = p.tile_out;
    int32_t n_in = int32_t(c.n_blocks);
    uint64_t* lv[2] = {reinterpret_cast<uint64_t*>(w + c.off_lv0), reinterpret_cast<uint64_t*>(w + c.off_lv1)};
    for (int level = 0;; ++level) {
      const int32_t groups = (n_in + kTreeFanIn - 1) / kTreeFanIn;
      const bool last = groups == 1;
      uint64_t* out = last ? out_keys : lv[level & 1];
      rc = merge_tree_level(in, B, n_in, int32_t(c.kk), c.kk, last ? out_scores : nullptr,
                            last ? out_ids : nullptr, out, st, -1);
      if (rc || last) return rc;
      in = out;
      n_in = groups;
    }
  }
  final_counts_kernel<<<unsigned((B + 255) / 256), 256, 0, st>>>(int32_t(B), int32_t(c.kk), int32_t(c.cap), p.rg,
                                                                 p.cdone, p.counts);
  GSP_CHECK_LAUNCH();
  return merge_topk_device(p.cand, B, 3, 3 * c.stride, c.stride, p.counts, 3, nullptr, c.kk, out_scores,
                           out_ids, out_keys, st, -1, p.fault);
}

extern "C" int gsp_set_wait_limit(int32_t polls) {
  GSP_REQUIRE(polls >= 0, GSP_ERR_ARG, "gsp_set_wait_limit: negative limit");
  g_wait_limit.store(polls);
  return GSP_OK;
}

extern "C" int32_t gsp_get_wait_limit(void) { return g_wait_limit.load(); }

extern "C" int gsp_set_schedule_jitter(int32_t ns) {
  GSP_REQUIRE(ns >= 0 && ns <= 1000000, GSP_ERR_ARG, "gsp_set_schedule_jitter: %d ns outside [0, 1000000]", ns);
  g_jitter_ns.store(ns);
  return GSP_OK;
}
extern "C" int32_t gsp_get_schedule_jitter(void) { return g_jitter_ns.load(); }

extern "C" int gsp_set_head_mode(int32_t mode) {
  GSP_REQUIRE(mode == GSP_HEAD_AUTO || mode == GSP_HEAD_CUDA_CORES || mode == GSP_HEAD_TENSOR_CORES, GSP_ERR_ARG,
              "gsp_set_head_mode: unknown mode %d", mode);
  g_head_mode.store(mode);
  return GSP_OK;
}

extern "C" int32_t gsp_get_head_mode(void) { return g_head_mode.load(); }

extern "C" int gsp_set_tree_limit(int64_t bytes) {
  GSP_REQUIRE(bytes >= 0, GSP_ERR_ARG, "gsp_set_tree_limit: negative limit");
  g_tree_limit.store(bytes);
  return GSP_OK;
}

extern "C" int64_t gsp_get_tree_limit(void) { return g_tree_limit.load(); }

extern "C" int gsp_profile_enable(int on) {
  Profile& pr = profile();
  std::lock_guard<std::mutex> g(pr.mu);
  pr.on = on != 0;
  pr.used = 0;
  return GSP_OK;
}

extern "C" int gsp_profile_collect(double* total_ms, int64_t* launches) {
  GSP_REQUIRE(total_ms && launches, GSP_ERR_ARG, "gsp_profile_collect: null argument");
  Profile& pr = profile();
  std::lock_guard<std::mutex> g(pr.mu);
  double tot = 0.0;
  for (size_t i = 0; i < pr.used; ++i) {
    GSP_CUDA(cudaEventSynchronize(pr.ev[i].second));
    float ms = 0.f;
    GSP_CUDA(cudaEventElapsedTime(&ms, pr.ev[i].first, pr.ev[i].second));
    tot += ms;
  }
  *total_ms = tot;
  *launches = int64_t(pr.used);
  pr.used = 0;
  return GSP_OK;
}

extern "C" int gsp_score_topk(const gsp_index_view* ix, const int32_t* qi, const float* qs, int64_t B,
                              int64_t W, int64_t k, float* out_scores, int64_t* out_ids,
                              uint64_t* out_keys, void* ws, int64_t ws_bytes, void* stream) {
  Cfg c;
  int rc = make_cfg(ix, B, W, k, c);
  if (rc) return rc;
  GSP_REQUIRE(ws && ws_bytes >= c.total, GSP_ERR_ARG, "gsp_score_topk: workspace too small (%lld < %lld)",
              (long long)ws_bytes, (long long)c.total);
  return score_with_cfg(ix, qi, qs, B, W, c, out_scores, out_ids, out_keys, ws, as_stream(stream));
}

extern "C" int gsp_score_topk_shared(const gsp_index_view* ix, const int32_t* qi, const float* qs,
                                     int64_t B, int64_t W, int64_t k, float* out_scores,
                                     int64_t* out_ids, uint64_t* out_keys, void* ws, int64_t ws_bytes,
                                     uint64_t* board, int32_t shard, int32_t n_shards,
                                     uint64_t* const* peer_boards, void* stream) {
  Cfg c;
  int rc = make_cfg(ix, B, W, k, c);
  if (rc) return rc;
  GSP_REQUIRE(ws && ws_bytes >= c.total, GSP_ERR_ARG,
              "gsp_score_topk_shared: workspace too small (%lld < %lld)", (long long)ws_bytes,
              (long long)c.total);
  return score_with_cfg(ix, qi, qs, B, W, c, out_scores, out_ids, out_keys, ws, as_stream(stream), board,
                        shard, n_shards, peer_boards);
}

// ---------------------------------------------------------------------------------------
// Scoring without any device allocation.
//
// Some callers cannot allocate device memory while they serve a batch: a serving loop
// where a cudaMalloc would synchronise the device and stall every other stream, or a host
// application (for example a search engine that loads this library as a native plug-in
// through a C FFI) that hands the library only its input and output buffers and owns no
// device allocator to lend it a workspace.  gsp_score_topk_noalloc serves them: its
// scratch (query plan, candidate buffers, work counter, thresholds) lives in the
// file-scope array below, which the CUDA runtime places on every GPU that loads this
// library and keeps until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;   // 32 MiB per GPU
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[256] = {nullptr};   // device address of the array, per device ordinal
}  // namespace

// Host code may not use g_noalloc_scratch as an address (it is a host-side stand-in), so
// the device address is looked up with the device current.  It is looked up again on every
// call whose stream is not being captured (the address belongs to the current context, so
// a device reset or another driver-API context gets its own), and remembered per device for
// calls made during a stream capture, which reuse the address of the last call outside one.
static int noalloc_scratch(void** out, cudaStream_t st) {
  int dev = 0;
  GSP_CUDA(cudaGetDevice(&dev));
  GSP_REQUIRE(dev >= 0 && dev < 256, GSP_ERR_UNSUPPORTED, "noalloc: device ordinal %d out of range", dev);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
    (void)cudaGetLastError();
    cs = cudaStreamCaptureStatusActive;   // cannot tell: treat it as a capture
  }
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (cs == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error("gsp_score_topk_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return GSP_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  GSP_REQUIRE(g_noalloc_ptr[dev], GSP_ERR_UNSUPPORTED,
              "gsp_score_topk_noalloc: the first call on a device must come before any stream capture");
  *out = g_noalloc_ptr[dev];
  return GSP_OK;
}

extern "C" int gsp_score_topk_noalloc(const gsp_index_view* ix, const int32_t* qi, const float* qs,
                                      int64_t B, int64_t W, int64_t k, float* out_scores,
                                      int64_t* out_ids, uint64_t* out_keys, void* stream) {
  Cfg c;
  int rc = make_cfg(ix, B, W, k, c);
  if (rc) return rc;
  // a smaller candidate capacity means more frequent compactions, never another result;
  // the smallest one keeps k keys plus a whole tile.  The default capacity is already that
  // minimum up to k' = 2048, so only larger k' can shrink.
  const int min_cap = int(((c.kk + kSel + 31) / 32) * 32);
  GSP_REQUIRE(!c.dense, GSP_ERR_UNSUPPORTED,
              "gsp_score_topk_noalloc: top_k %lld is above %d; use gsp_score_topk with a workspace",
              (long long)c.kk, kMaxSmemK);
  if (c.tree) {   // the per-tile lists would not fit the fixed scratch: shared buffers only
    c.tree = false;
    set_layout(c, B);
  }
  while (c.total > int64_t(kNoAllocScratchBytes) && c.cap > min_cap) {
    c.cap = std::max(min_cap, c.cap / 2 / 32 * 32);
    set_layout(c, B);
  }
  GSP_REQUIRE(c.total <= int64_t(kNoAllocScratchBytes), GSP_ERR_UNSUPPORTED,
              "gsp_score_topk_noalloc: this batch needs %lld bytes of scratch, more than the "
              "fixed %lld (lower the batch size or top_k, or use gsp_score_topk with a workspace)",
              (long long)c.total, (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch, as_stream(stream));
  if (rc) return rc;
  // Every buffer in the scratch is written before it is read within a call except the
  // per-query thresholds and buffer counters, the item counter and the fault flag, which
  // score_with_cfg clears on the stream; the array keeps the previous call's contents
  // otherwise.
  return score_with_cfg(ix, qi, qs, B, W, c, out_scores, out_ids, out_keys, scratch, as_stream(stream));
}
