// Term-major inverted index built on the GPU from a document-term CSR.
//
// Same layout as the reference builder (src/run_correctness_verification.py:32-84):
// postings grouped by term, ascending doc id inside a term (the stable-sort invariant the
// chunked path depends on), every list padded to a multiple of 32 entries with doc id -1
// and weight 0, offsets = exclusive prefix sum of the padded lengths.  The reference does
// a host argsort; here it is a two-pass counting sort over fixed document blocks:
//
//   count : per block b, per term t, how many postings (shared-memory histogram)
//   scan  : per term, exclusive prefix over blocks -> block_starts[b][t] (kept in the
//           index: the posting of t at which block b begins), lengths, padded lengths;
//           then offsets = exclusive scan of the padded lengths
//   fill  : one warp per block walks its documents in order and appends each posting at
//           offsets[t] + block_starts[b][t] + (running count of t in b); documents are
//           visited in ascending order, so every list comes out sorted by doc id.
//
// Both passes work on any run of whole blocks, so a corpus can also be built in chunks of
// documents (count every chunk, finish the counts, fill every chunk, finish the fill):
// only one chunk of the CSR needs to be on the device at a time.
#include "common.cuh"

#include <algorithm>

namespace gsp {
namespace {

constexpr int kCountThreads = 512;

__global__ void __launch_bounds__(kCountThreads)
count_kernel(int64_t n_docs, int32_t V, int32_t block_docs, const int64_t* __restrict__ indptr,
             const int32_t* __restrict__ indices, uint32_t* __restrict__ counts, int32_t use_smem,
             int32_t* __restrict__ err) {
  extern __shared__ uint32_t hist[];
  const int64_t b = blockIdx.x;               // block of this chunk (documents local to it)
  const int64_t d0 = b * block_docs;
  const int64_t d1 = min(d0 + block_docs, n_docs);
  uint32_t* row = counts + b * int64_t(V);    // counts: the chunk's first block row
  if (use_smem) {
    for (int32_t t = threadIdx.x; t < V; t += blockDim.x) hist[t] = 0u;
    __syncthreads();
  }
  const int64_t e0 = indptr[d0], e1 = indptr[d1];
  for (int64_t e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
    const int32_t t = indices[e];
    if (t < 0 || t >= V) {
      atomicExch(err, 1);
      continue;
    }
    if (use_smem) atomicAdd(&hist[t], 1u);
    else atomicAdd(&row[t], 1u);
  }
  if (use_smem) {
    __syncthreads();
    for (int32_t t = threadIdx.x; t < V; t += blockDim.x) row[t] = hist[t];
  }
}

// per term: exclusive prefix over blocks, in place (rows 0..n_blocks-1 hold the counts on
// entry; row n_blocks receives the totals), lengths, padded lengths
__global__ void scan_blocks_kernel(int32_t V, int64_t n_blocks, uint32_t* __restrict__ block_starts,
                                   int32_t* __restrict__ lengths, int32_t* __restrict__ padded,
                                   int32_t* __restrict__ err) {
  const int32_t t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= V) return;
  uint64_t run = 0;
  uint32_t max_c = 0;
  for (int64_t b = 0; b < n_blocks; ++b) {
    const uint32_t c = block_starts[b * V + t];
    max_c = max(max_c, c);
    block_starts[b * V + t] = uint32_t(run);
    run += c;
  }
  block_starts[n_blocks * V + t] = uint32_t(run);
  if (run > 0x7FFFFFE0ull || max_c > 0xFFFFu) atomicExch(err, 2);
  lengths[t] = int32_t(run);
  padded[t] = int32_t((run + kPostingPad - 1) / kPostingPad * kPostingPad);
}

// One warp per document block; u16 running counts per term in shared memory.  A posting
// is written only inside its block's slice of the term's list, [block_starts[b][t],
// block_starts[b+1][t]); rows that hold more postings of a term than the count pass saw
// (a chunk filled with other rows than it was counted with) set err = 3 and are dropped.
__global__ void __launch_bounds__(32)
fill_kernel(int64_t n_docs, int32_t V, int32_t block_docs, int64_t first_doc,
            const int64_t* __restrict__ indptr, const int32_t* __restrict__ indices,
            const float* __restrict__ data, const int64_t* __restrict__ offsets,
            const uint32_t* __restrict__ block_starts, int32_t* __restrict__ doc_ids,
            float* __restrict__ weights, int32_t* __restrict__ err) {
  extern __shared__ uint16_t run16[];
  const int lane = lane_id();
  const int64_t b = blockIdx.x;               // block of this chunk (documents local to it)
  const int64_t d0 = b * block_docs;
  const int64_t d1 = min(d0 + block_docs, n_docs);
  const uint32_t* bstart = block_starts + (first_doc / block_docs + b) * int64_t(V);
  for (int32_t t = lane; t < V; t += 32) run16[t] = 0;
  __syncwarp();
  for (int64_t d = d0; d < d1; ++d) {
    const int64_t e0 = indptr[d], e1 = indptr[d + 1];
    for (int64_t e = e0; e < e1; e += 32) {
      const int32_t tr = e + lane < e1 ? indices[e + lane] : -1;
      const bool live = tr >= 0 && tr < V;   // ids outside [0, V) were rejected by the count pass
      const int32_t t = live ? tr : -1;
      const float w = live ? data[e + lane] : 0.0f;
      // duplicated term ids inside one document keep their CSR order
      const uint32_t live_mask = __ballot_sync(FULL, live);
      const uint32_t peers = __match_any_sync(FULL, t) & live_mask;
      const int rank = __popc(peers & lanemask_lt());
      const int leader = live ? (__ffs(peers) - 1) : 0;
      uint32_t old = 0;
      if (live && rank == 0) {
        old = run16[t];
        run16[t] = uint16_t(old + __popc(peers));
      }
      old = __shfl_sync(FULL, old, leader);
      if (live) {
        const uint32_t s0 = __ldg(bstart + t), s1 = __ldg(bstart + V + t);
        if (old + rank < s1 - s0) {
          const int64_t pos = offsets[t] + int64_t(s0) + old + rank;
          doc_ids[pos] = int32_t(first_doc + d);
          weights[pos] = w;
        } else {
          atomicExch(err, 3);
        }
      }
      __syncwarp();
    }
  }
}

// One block per term, after every posting is in place: writes the list's padding (doc id
// -1, weight 0), its max weight (0 for an empty list), and counts lists that are out of
// order or hold a doc id outside [0, n_docs) (n_bad[0]) and lists that repeat a doc id
// (n_bad[1]).  A block, not a warp, per term: the longest lists hold every document.
constexpr int kFinishThreads = 256;
__global__ void __launch_bounds__(kFinishThreads)
finish_kernel(int64_t n_docs, int32_t V, const int64_t* __restrict__ offsets,
              const int32_t* __restrict__ lengths, int32_t* __restrict__ doc_ids,
              float* __restrict__ weights, float* __restrict__ max_scores,
              unsigned long long* __restrict__ n_bad) {
  __shared__ float s_max[kFinishThreads / 32];
  __shared__ int s_bad[kFinishThreads / 32], s_dup[kFinishThreads / 32];
  const int32_t t = blockIdx.x;
  const int lane = lane_id(), wid = threadIdx.x >> 5;
  const int64_t o = offsets[t];
  const int32_t L = lengths[t];
  const int32_t P = (L + kPostingPad - 1) / kPostingPad * kPostingPad;
  float m = -INFINITY;
  bool bad = false, dup = false;
  for (int32_t p = threadIdx.x; p < L; p += kFinishThreads) {
    m = fmaxf(m, weights[o + p]);
    const int32_t b = doc_ids[o + p];
    bad |= b < 0 || int64_t(b) >= n_docs;
    if (p > 0) {
      const int32_t a = doc_ids[o + p - 1];
      bad |= b < a;
      dup |= b == a;
    }
  }
  for (int32_t p = L + threadIdx.x; p < P; p += kFinishThreads) {
    doc_ids[o + p] = -1;
    weights[o + p] = 0.0f;
  }
#pragma unroll
  for (int sh = 16; sh; sh >>= 1) m = fmaxf(m, __shfl_xor_sync(FULL, m, sh));
  const bool wbad = __any_sync(FULL, bad), wdup = __any_sync(FULL, dup);
  if (lane == 0) {
    s_max[wid] = m;
    s_bad[wid] = wbad;
    s_dup[wid] = wdup;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = -INFINITY;
    int bb = 0, dd = 0;
    for (int w = 0; w < kFinishThreads / 32; ++w) {
      mm = fmaxf(mm, s_max[w]);
      bb |= s_bad[w];
      dd |= s_dup[w];
    }
    max_scores[t] = L > 0 ? mm : 0.0f;
    if (bb) atomicAdd(n_bad, 1ull);
    if (dd) atomicAdd(n_bad + 1, 1ull);
  }
}

__global__ void quant_kernel(int32_t V, const int64_t* __restrict__ offsets,
                             const int32_t* __restrict__ padded, const float* __restrict__ max_scores,
                             const float* __restrict__ weights, int32_t wdtype, void* out,
                             float* __restrict__ term_scale) {
  const int32_t t = (int32_t)((int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = lane_id();
  if (t >= V) return;
  const int64_t o = offsets[t];
  const int32_t P = padded[t];
  if (wdtype == GSP_W_BF16) {
    __nv_bfloat16* q = static_cast<__nv_bfloat16*>(out);
    for (int32_t p = lane; p < P; p += 32) q[o + p] = __float2bfloat16_rn(weights[o + p]);
    return;
  }
  uint8_t* q = static_cast<uint8_t*>(out);
  const float mx = fmaxf(max_scores[t], 0.0f);
  const float scale = __fdiv_rn(mx, 255.0f);
  if (lane == 0 && term_scale) term_scale[t] = scale;
  for (int32_t p = lane; p < P; p += 32) {
    int v = 0;
    if (scale > 0.0f) {
      v = __float2int_rn(__fdiv_rn(weights[o + p], scale));
      v = min(max(v, 0), 255);
    }
    q[o + p] = uint8_t(v);
  }
}

// n_bad[0]: lists with a descending step; n_bad[1]: lists that repeat a doc id.
__global__ void check_sorted_kernel(int32_t V, const int32_t* __restrict__ doc_ids,
                                    const int64_t* __restrict__ offsets,
                                    const int32_t* __restrict__ lengths,
                                    unsigned long long* __restrict__ n_bad) {
  const int32_t t = (int32_t)((int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = lane_id();
  if (t >= V) return;
  const int64_t o = offsets[t];
  const int32_t L = lengths[t];
  bool bad = false, dup = false;
  for (int32_t p = lane + 1; p < L; p += 32) {
    const int32_t a = doc_ids[o + p - 1], b = doc_ids[o + p];
    bad |= b < a;
    dup |= b == a;
  }
  if (__any_sync(FULL, bad) && lane == 0) atomicAdd(n_bad, 1ull);
  if (__any_sync(FULL, dup) && lane == 0) atomicAdd(n_bad + 1, 1ull);
}

// out[c][t] = offsets[t] + #postings of t with doc id < min(c*chunk, n_docs); one warp per
// term, binary search per boundary (lists are ascending, the caller checked).
__global__ void chunk_bounds_kernel(int64_t n_docs, int32_t V, int64_t chunk, int64_t n_chunks,
                                    const int32_t* __restrict__ doc_ids,
                                    const int64_t* __restrict__ offsets,
                                    const int32_t* __restrict__ lengths, int64_t* __restrict__ out) {
  const int32_t t = (int32_t)((int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = lane_id();
  if (t >= V) return;
  const int64_t o = offsets[t];
  const int32_t L = lengths[t];
  for (int64_t c = lane; c <= n_chunks; c += 32) {
    const int64_t edge = c < n_chunks ? c * chunk : n_docs;
    int32_t lo = 0, hi = L;  // first p with doc_ids[o+p] >= edge
    while (lo < hi) {
      const int32_t mid = (lo + hi) >> 1;
      if (int64_t(doc_ids[o + mid]) < edge) lo = mid + 1; else hi = mid;
    }
    out[c * V + t] = o + lo;
  }
}

// Dense rows of the head terms: row h holds term head_ids[h]'s weight for every document
// (0 where the term is absent).  One warp per head term scatters its postings.
template <typename WT>
__global__ void head_rows_kernel(int32_t H, const int32_t* __restrict__ head_ids,
                                 const int64_t* __restrict__ offsets, const int32_t* __restrict__ lengths,
                                 const int32_t* __restrict__ doc_ids, const WT* __restrict__ weights,
                                 int64_t ld, WT* __restrict__ rows) {
  const int32_t h = blockIdx.x;
  if (h >= H) return;
  const int32_t t = head_ids[h];
  const int64_t o = offsets[t];
  const int32_t L = lengths[t];
  WT* __restrict__ row = rows + int64_t(h) * ld;
  for (int32_t i = threadIdx.x; i < L; i += blockDim.x) {
    const int32_t d = doc_ids[o + i];
    if (d >= 0 && d < ld) row[d] = weights[o + i];
  }
}

// ---- duplicate (document, term) entries of a CSR ------------------------------------
// The reference keeps a term that one CSR row lists twice as two postings, and its
// scatter-add sums both into the document's score.  The scorer here updates a list's
// documents in parallel and needs each document once per list, so the builders merge such
// entries first: the first occurrence keeps its place in the row, and its weight becomes
// the fp32 sum of every occurrence's weight, left to right in CSR order.  One warp per row;
// an entry is compared with every earlier entry of its row (32 at a time), which costs
// O(nnz^2 / 32) per row: a few milliseconds for millions of SPLADE-sized rows.

// rows [0, n_rows) of indptr (indptr[0] need not be 0): nnz[r] = distinct terms of row r;
// dropped += entries that repeat an earlier term of their row
__global__ void dedup_count_kernel(int64_t n_rows, const int64_t* __restrict__ indptr,
                                   const int32_t* __restrict__ indices, int32_t* __restrict__ nnz,
                                   unsigned long long* __restrict__ dropped) {
  const int lane = lane_id();
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  unsigned long long drop = 0;
  for (int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n_rows; r += warps) {
    const int64_t e0 = indptr[r], e1 = indptr[r + 1];
    int32_t kept = 0;
    for (int64_t j0 = e0; j0 < e1; j0 += 32) {
      const bool valid = j0 + lane < e1;
      const int32_t t = valid ? indices[j0 + lane] : 0;
      bool dup = false;
      for (int64_t i0 = e0; i0 < j0; i0 += 32) {   // earlier chunks are whole
        const int32_t u = indices[i0 + lane];
#pragma unroll 8
        for (int sl = 0; sl < 32; ++sl) dup |= __shfl_sync(FULL, u, sl) == t;
      }
      const uint32_t vmask = __ballot_sync(FULL, valid);
      const uint32_t peers = __match_any_sync(FULL, valid ? t : int32_t(0x80000000u) + lane) & vmask;
      dup |= (peers & lanemask_lt()) != 0u;
      kept += __popc(__ballot_sync(FULL, valid && !dup));
    }
    if (lane == 0) {
      nnz[r] = kept;
      drop += uint64_t(e1 - e0 - kept);
    }
  }
  if (lane == 0 && drop) atomicAdd(dropped, drop);
}

// The same count with a bitmap of the vocabulary per warp in shared memory (V bits): an
// entry repeats an earlier chunk's term if its bit is set, and an earlier lane of its own
// chunk (match_any); then the chunk's bits are set, and the row's bits cleared at its end.
// O(nnz) per row; used when 8 warps' bitmaps fit the shared memory.
__global__ void __launch_bounds__(256)
dedup_count_bitmap_kernel(int64_t n_rows, int32_t V, const int64_t* __restrict__ indptr,
                          const int32_t* __restrict__ indices, int32_t* __restrict__ nnz,
                          unsigned long long* __restrict__ dropped) {
  extern __shared__ uint32_t bm_all[];
  const int lane = lane_id(), wid = threadIdx.x >> 5;
  const int32_t words = (V + 31) >> 5;
  uint32_t* bm = bm_all + int64_t(wid) * words;
  for (int32_t i = lane; i < words; i += 32) bm[i] = 0u;
  __syncwarp();
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  unsigned long long drop = 0;
  for (int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + wid; r < n_rows; r += warps) {
    const int64_t e0 = indptr[r], e1 = indptr[r + 1];
    int32_t kept = 0;
    for (int64_t j0 = e0; j0 < e1; j0 += 32) {
      const bool valid = j0 + lane < e1;
      const int32_t t = valid ? indices[j0 + lane] : 0;
      const bool inv = valid && (t < 0 || t >= V);   // out of range: counted as distinct here,
                                                     // refused by the index build's count pass
      const uint32_t bit = 1u << (t & 31);
      bool dup = valid && !inv && (bm[t >> 5] & bit) != 0u;
      const uint32_t vmask = __ballot_sync(FULL, valid);
      const uint32_t peers = __match_any_sync(FULL, valid ? t : int32_t(0x80000000u) + lane) & vmask;
      dup |= (peers & lanemask_lt()) != 0u;
      kept += __popc(__ballot_sync(FULL, valid && !dup));
      __syncwarp();
      if (valid && !inv) atomicOr(&bm[t >> 5], bit);
      __syncwarp();
    }
    for (int64_t j0 = e0; j0 < e1; j0 += 32) {
      if (j0 + lane < e1) {
        const int32_t t = indices[j0 + lane];
        if (t >= 0 && t < V) bm[t >> 5] = 0u;
      }
    }
    __syncwarp();
    if (lane == 0) {
      nnz[r] = kept;
      drop += uint64_t(e1 - e0 - kept);
    }
  }
  if (lane == 0 && drop) atomicAdd(dropped, drop);
}

// out row r (at new_indptr[r] - new_indptr[0]) = the first occurrence of every term of in
// row r, in row order, each with the fp32 sum of its occurrences' weights in row order
// (data and out_data may be null: indices only)
__global__ void dedup_fill_kernel(int64_t n_rows, const int64_t* __restrict__ indptr,
                                  const int32_t* __restrict__ indices, const float* __restrict__ data,
                                  const int64_t* __restrict__ new_indptr, int32_t* __restrict__ out_indices,
                                  float* __restrict__ out_data) {
  const int lane = lane_id();
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n_rows; r += warps) {
    const int64_t e0 = indptr[r], e1 = indptr[r + 1];
    int64_t o = new_indptr[r] - new_indptr[0];
    for (int64_t j0 = e0; j0 < e1; j0 += 32) {
      const bool valid = j0 + lane < e1;
      const int32_t t = valid ? indices[j0 + lane] : 0;
      float w = (valid && data) ? data[j0 + lane] : 0.0f;
      bool dup = false;
      for (int64_t i0 = e0; i0 < j0; i0 += 32) {
        const int32_t u = indices[i0 + lane];
#pragma unroll 8
        for (int sl = 0; sl < 32; ++sl) dup |= __shfl_sync(FULL, u, sl) == t;
      }
      const uint32_t vmask = __ballot_sync(FULL, valid);
      const int32_t tk = valid ? t : int32_t(0x80000000u) + lane;
      const uint32_t peers = __match_any_sync(FULL, tk) & vmask;
      dup |= (peers & lanemask_lt()) != 0u;
      const bool first = valid && !dup;
      if (data) {
        // later occurrences in this chunk, then in the chunks after it, in row order
        const float dv = valid ? data[j0 + lane] : 0.0f;
        for (int sl = 0; sl < 32; ++sl) {
          const float x = __shfl_sync(FULL, dv, sl);
          if (first && sl > lane && ((peers >> sl) & 1u)) w = __fadd_rn(w, x);
        }
        for (int64_t i0 = j0 + 32; i0 < e1; i0 += 32) {
          const bool iv = i0 + lane < e1;
          const int32_t u = iv ? indices[i0 + lane] : 0;
          const float x = iv ? data[i0 + lane] : 0.0f;
          const uint32_t um = __ballot_sync(FULL, iv);
          for (int sl = 0; sl < 32; ++sl) {
            const int32_t us = __shfl_sync(FULL, u, sl);
            const float xs = __shfl_sync(FULL, x, sl);
            if (first && ((um >> sl) & 1u) && us == t) w = __fadd_rn(w, xs);
          }
        }
      }
      const uint32_t fm = __ballot_sync(FULL, first);
      if (first) {
        const int64_t pos = o + __popc(fm & lanemask_lt());
        out_indices[pos] = t;
        if (out_data) out_data[pos] = w;
      }
      o += __popc(fm);
    }
  }
}

// lo = x - (x with its low 13 mantissa bits cleared): exact in fp32
__global__ void head_lo_kernel(int64_t n, const float4* __restrict__ rows, float4* __restrict__ lo) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float4 v = rows[i];
    float4 r;
    r.x = __fsub_rn(v.x, __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u));
    r.y = __fsub_rn(v.y, __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u));
    r.z = __fsub_rn(v.z, __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u));
    r.w = __fsub_rn(v.w, __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u));
    lo[i] = r;
  }
}

int64_t n_blocks_of(int64_t n_docs, int32_t block_docs) {
  return (n_docs + block_docs - 1) / block_docs;
}

}  // namespace
}  // namespace gsp

using namespace gsp;

// workspace: err int32 at 0 | finish counters (2 x u64) at 64 | scan ws at 256.  The block
// counts are accumulated in block_starts itself and scanned in place.
constexpr int64_t kWsCounters = 64;
constexpr int64_t kWsScan = 256;
// gsp_check_sorted / gsp_chunk_bounds: two uint64 counters
constexpr int64_t kCheckWsBytes = 16;

extern "C" int64_t gsp_index_ws_bytes(int64_t n_docs, int32_t V, int32_t block_docs) {
  if (n_docs < 0 || V <= 0 || block_docs <= 0) return -1;
  return kWsScan + gsp_scan_ws_bytes(V);
}

static int check_csr_args(int64_t n_docs, int32_t V, int32_t block_docs, const int64_t* indptr) {
  GSP_REQUIRE(n_docs >= 0 && V > 0 && block_docs > 0 && block_docs <= 65536 && indptr, GSP_ERR_ARG,
              "index build: bad arguments (n_docs=%lld V=%d block_docs=%d)", (long long)n_docs, V,
              block_docs);
  GSP_REQUIRE(n_docs < 0x7FFFFFFFll, GSP_ERR_UNSUPPORTED, "index build: n_docs must be < 2^31");
  return GSP_OK;
}

static int check_chunk_args(int64_t n_docs, int32_t V, int32_t block_docs, int64_t first_doc,
                            int64_t chunk_docs, const int64_t* indptr, void* ws, int64_t ws_bytes) {
  int rc = check_csr_args(n_docs, V, block_docs, indptr);
  if (rc) return rc;
  GSP_REQUIRE(ws && ws_bytes >= gsp_index_ws_bytes(n_docs, V, block_docs), GSP_ERR_ARG,
              "index build: workspace too small");
  GSP_REQUIRE(first_doc >= 0 && chunk_docs >= 0 && first_doc + chunk_docs <= n_docs &&
                  first_doc % block_docs == 0 &&
                  (chunk_docs % block_docs == 0 || first_doc + chunk_docs == n_docs),
              GSP_ERR_ARG,
              "index build: chunk [%lld, %lld) of %lld documents is not a run of whole %d-document "
              "blocks",
              (long long)first_doc, (long long)(first_doc + chunk_docs), (long long)n_docs, block_docs);
  return GSP_OK;
}

extern "C" int gsp_index_count_chunk(int64_t n_docs, int32_t V, int32_t block_docs, int64_t first_doc,
                                     int64_t chunk_docs, const int64_t* indptr, const int32_t* indices,
                                     uint32_t* block_starts, void* ws, int64_t ws_bytes, void* stream) {
  int rc = check_chunk_args(n_docs, V, block_docs, first_doc, chunk_docs, indptr, ws, ws_bytes);
  if (rc) return rc;
  GSP_REQUIRE(block_starts, GSP_ERR_ARG, "gsp_index_count_chunk: block_starts is null");
  cudaStream_t st = as_stream(stream);
  int32_t* err = static_cast<int32_t*>(ws);
  if (first_doc == 0) GSP_CUDA(cudaMemsetAsync(err, 0, sizeof(int32_t), st));
  const int64_t nb = n_blocks_of(chunk_docs, block_docs);
  if (nb == 0) return GSP_OK;
  uint32_t* rows = block_starts + (first_doc / block_docs) * int64_t(V);
  const size_t smem = size_t(V) * 4;
  const int use_smem = smem <= size_t(max_smem_optin()) ? 1 : 0;
  if (use_smem) {
    rc = ensure_smem(reinterpret_cast<const void*>(count_kernel), int(smem));
    if (rc) return rc;
  } else {
    GSP_CUDA(cudaMemsetAsync(rows, 0, size_t(nb) * V * 4, st));
  }
  count_kernel<<<unsigned(nb), kCountThreads, use_smem ? smem : 0, st>>>(
      chunk_docs, V, block_docs, indptr, indices, rows, use_smem, err);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

extern "C" int gsp_index_count_finish(int64_t n_docs, int32_t V, int32_t block_docs, int32_t* lengths,
                                      int32_t* padded, int64_t* offsets, uint32_t* block_starts,
                                      int64_t* total_padded, void* ws, int64_t ws_bytes, void* stream) {
  int64_t dummy_indptr = 0;
  int rc = check_chunk_args(n_docs, V, block_docs, 0, 0, &dummy_indptr, ws, ws_bytes);
  if (rc) return rc;
  GSP_REQUIRE(lengths && padded && offsets && block_starts && total_padded, GSP_ERR_ARG,
              "gsp_index_count_finish: bad arguments");
  cudaStream_t st = as_stream(stream);
  const int64_t nb = n_blocks_of(n_docs, block_docs);
  char* w = static_cast<char*>(ws);
  int32_t* err = reinterpret_cast<int32_t*>(w);
  if (n_docs == 0) GSP_CUDA(cudaMemsetAsync(err, 0, sizeof(int32_t), st));
  scan_blocks_kernel<<<unsigned((V + 255) / 256), 256, 0, st>>>(V, nb, block_starts, lengths, padded,
                                                                err);
  GSP_CHECK_LAUNCH();
  rc = gsp_scan_i32(padded, V, offsets, w + kWsScan, gsp_scan_ws_bytes(V), stream);
  if (rc) return rc;
  // offsets holds V entries; the total is the last offset plus the last padded length
  int64_t last_off = 0;
  int32_t last_pad = 0, herr = 0;
  GSP_CUDA(cudaMemcpyAsync(&last_off, offsets + (V - 1), sizeof(int64_t), cudaMemcpyDeviceToHost, st));
  GSP_CUDA(cudaMemcpyAsync(&last_pad, padded + (V - 1), sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  GSP_CUDA(cudaMemcpyAsync(&herr, err, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  GSP_CUDA(cudaStreamSynchronize(st));
  GSP_REQUIRE(herr != 1, GSP_ERR_ARG, "index build: a column id is outside [0, %d)", V);
  GSP_REQUIRE(herr != 2, GSP_ERR_UNSUPPORTED,
              "index build: a posting list exceeds 2^31 entries or a term repeats more than "
              "65535 times inside one document block");
  *total_padded = last_off + last_pad;
  return GSP_OK;
}

extern "C" int gsp_index_fill_chunk(int64_t n_docs, int32_t V, int32_t block_docs, int64_t first_doc,
                                    int64_t chunk_docs, const int64_t* indptr, const int32_t* indices,
                                    const float* data, const int64_t* offsets,
                                    const uint32_t* block_starts, int32_t* doc_ids, float* weights,
                                    void* ws, int64_t ws_bytes, void* stream) {
  int rc = check_chunk_args(n_docs, V, block_docs, first_doc, chunk_docs, indptr, ws, ws_bytes);
  if (rc) return rc;
  GSP_REQUIRE(offsets && block_starts && (chunk_docs == 0 || (indices && data && doc_ids && weights)),
              GSP_ERR_ARG, "gsp_index_fill_chunk: bad arguments");
  const int64_t nb = n_blocks_of(chunk_docs, block_docs);
  if (nb == 0) return GSP_OK;
  const size_t smem = size_t(V) * 2;
  GSP_REQUIRE(smem <= size_t(max_smem_optin()), GSP_ERR_UNSUPPORTED,
              "index build: vocabulary %d too large", V);
  rc = ensure_smem(reinterpret_cast<const void*>(fill_kernel), int(smem));
  if (rc) return rc;
  fill_kernel<<<unsigned(nb), 32, smem, as_stream(stream)>>>(chunk_docs, V, block_docs, first_doc,
                                                             indptr, indices, data, offsets,
                                                             block_starts, doc_ids, weights,
                                                             static_cast<int32_t*>(ws));
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

extern "C" int gsp_index_fill_finish(int64_t n_docs, int32_t V, const int64_t* offsets,
                                     const int32_t* lengths, int32_t* doc_ids, float* weights,
                                     float* max_scores, void* ws, int64_t ws_bytes, void* stream) {
  GSP_REQUIRE(n_docs >= 0 && V > 0 && offsets && lengths && max_scores && ws &&
                  ws_bytes >= kWsCounters + 16,
              GSP_ERR_ARG, "gsp_index_fill_finish: bad arguments");
  cudaStream_t st = as_stream(stream);
  unsigned long long* d_cnt =
      reinterpret_cast<unsigned long long*>(static_cast<char*>(ws) + kWsCounters);
  GSP_CUDA(cudaMemsetAsync(d_cnt, 0, 16, st));
  int32_t herr = 0;
  GSP_CUDA(cudaMemcpyAsync(&herr, ws, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  finish_kernel<<<unsigned(V), kFinishThreads, 0, st>>>(n_docs, V, offsets, lengths, doc_ids, weights,
                                                        max_scores, d_cnt);
  GSP_CHECK_LAUNCH();
  unsigned long long h[2] = {0, 0};
  GSP_CUDA(cudaMemcpyAsync(h, d_cnt, 16, cudaMemcpyDeviceToHost, st));
  GSP_CUDA(cudaStreamSynchronize(st));
  GSP_REQUIRE(herr != 3, GSP_ERR_ARG,
              "index build: a chunk was filled with other rows than it was counted with");
  GSP_REQUIRE(h[0] == 0, GSP_ERR_ARG,
              "index build: %llu posting lists are out of place; every chunk must be counted and "
              "filled exactly once with the same CSR rows",
              h[0]);
  // a term listed twice in one document row would give one list a repeated doc id; the
  // scorer applies a list's postings to distinct documents in parallel, so the builders
  // merge such entries first (gsp_csr_dedup_*) and a repeat here means they were skipped
  GSP_REQUIRE(h[1] == 0, GSP_ERR_UNSORTED,
              "index build: %llu terms occur twice in one document row (duplicate (doc, term) "
              "entries); merge them first (gsp_csr_dedup_count / gsp_csr_dedup_fill)", h[1]);
  return GSP_OK;
}

extern "C" int gsp_index_count(int64_t n_docs, int32_t V, int32_t block_docs, const int64_t* indptr,
                               const int32_t* indices, int32_t* lengths, int32_t* padded,
                               int64_t* offsets, uint32_t* block_starts, int64_t* total_padded,
                               void* ws, int64_t ws_bytes, void* stream) {
  int rc = gsp_index_count_chunk(n_docs, V, block_docs, 0, n_docs, indptr, indices, block_starts, ws,
                                 ws_bytes, stream);
  if (rc) return rc;
  return gsp_index_count_finish(n_docs, V, block_docs, lengths, padded, offsets, block_starts,
                                total_padded, ws, ws_bytes, stream);
}

extern "C" int gsp_index_fill(int64_t n_docs, int32_t V, int32_t block_docs, const int64_t* indptr,
                              const int32_t* indices, const float* data, const int64_t* offsets,
                              const int32_t* lengths, const uint32_t* block_starts,
                              int64_t total_padded, int32_t* doc_ids, float* weights,
                              float* max_scores, void* ws, int64_t ws_bytes, void* stream) {
  GSP_REQUIRE(total_padded >= 0, GSP_ERR_ARG, "gsp_index_fill: total_padded < 0");
  int rc = gsp_index_fill_chunk(n_docs, V, block_docs, 0, n_docs, indptr, indices, data, offsets,
                                block_starts, doc_ids, weights, ws, ws_bytes, stream);
  if (rc) return rc;
  return gsp_index_fill_finish(n_docs, V, offsets, lengths, doc_ids, weights, max_scores, ws,
                               ws_bytes, stream);
}

extern "C" int gsp_csr_dedup_count(int64_t n_rows, int32_t V, const int64_t* indptr,
                                   const int32_t* indices, int32_t* nnz, int64_t* n_dropped, void* ws,
                                   int64_t ws_bytes, void* stream) {
  GSP_REQUIRE(n_rows >= 0 && indptr && nnz && n_dropped && ws && ws_bytes >= 8, GSP_ERR_ARG,
              "gsp_csr_dedup_count: bad arguments");
  cudaStream_t st = as_stream(stream);
  unsigned long long* d = static_cast<unsigned long long*>(ws);
  GSP_CUDA(cudaMemsetAsync(d, 0, 8, st));
  if (n_rows > 0) {
    const int64_t blocks = std::min<int64_t>((n_rows + 7) / 8, int64_t(num_sms()) * 32);
    const int64_t bm_bytes = 8 * int64_t((std::max(V, 1) + 31) / 32) * 4;
    if (V > 0 && bm_bytes <= 96 * 1024) {
      if (int rc = ensure_smem(reinterpret_cast<const void*>(dedup_count_bitmap_kernel), int(bm_bytes))) return rc;
      const int64_t bblocks = std::min<int64_t>((n_rows + 7) / 8, int64_t(num_sms()) * 2);
      dedup_count_bitmap_kernel<<<unsigned(bblocks), 256, size_t(bm_bytes), st>>>(n_rows, V, indptr, indices, nnz, d);
    } else {
      dedup_count_kernel<<<unsigned(blocks), 256, 0, st>>>(n_rows, indptr, indices, nnz, d);
    }
    GSP_CHECK_LAUNCH();
  }
  unsigned long long h = 0;
  GSP_CUDA(cudaMemcpyAsync(&h, d, 8, cudaMemcpyDeviceToHost, st));
  GSP_CUDA(cudaStreamSynchronize(st));
  *n_dropped = int64_t(h);
  return GSP_OK;
}

extern "C" int gsp_csr_dedup_fill(int64_t n_rows, const int64_t* indptr, const int32_t* indices,
                                  const float* data, const int64_t* new_indptr, int32_t* out_indices,
                                  float* out_data, void* stream) {
  GSP_REQUIRE(n_rows >= 0 && indptr && new_indptr && (n_rows == 0 || (indices && out_indices)) &&
                  ((data == nullptr) == (out_data == nullptr)),
              GSP_ERR_ARG, "gsp_csr_dedup_fill: bad arguments");
  if (n_rows == 0) return GSP_OK;
  const int64_t blocks = std::min<int64_t>((n_rows + 7) / 8, int64_t(num_sms()) * 32);
  dedup_fill_kernel<<<unsigned(blocks), 256, 0, as_stream(stream)>>>(n_rows, indptr, indices, data, new_indptr,
                                                                     out_indices, out_data);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

extern "C" int gsp_index_quantize(int32_t V, int64_t total_padded, const int64_t* offsets,
                                  const int32_t* padded, const float* max_scores,
                                  const float* weights, int32_t wdtype, void* out_weights,
                                  float* term_scale, void* stream) {
  GSP_REQUIRE(V > 0 && total_padded >= 0 && (wdtype == GSP_W_BF16 || wdtype == GSP_W_U8) &&
                  out_weights && (wdtype != GSP_W_U8 || term_scale),
              GSP_ERR_ARG, "gsp_index_quantize: bad arguments");
  quant_kernel<<<unsigned((int64_t(V) * 32 + 255) / 256), 256, 0, as_stream(stream)>>>(
      V, offsets, padded, max_scores, weights, wdtype, out_weights, term_scale);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

extern "C" int gsp_index_head_lo(int64_t n, const float* rows, float* lo, void* stream) {
  GSP_REQUIRE(n >= 0 && n % 4 == 0 && (n == 0 || (rows && lo)) && (reinterpret_cast<uintptr_t>(rows) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(lo) & 15) == 0,
              GSP_ERR_ARG, "gsp_index_head_lo: bad arguments (n a multiple of 4, 16-byte aligned arrays)");
  if (n == 0) return GSP_OK;
  const int64_t n4 = n / 4;
  const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, int64_t(num_sms()) * 16);
  head_lo_kernel<<<unsigned(blocks), 256, 0, as_stream(stream)>>>(n4, reinterpret_cast<const float4*>(rows),
                                                                 reinterpret_cast<float4*>(lo));
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

extern "C" int gsp_check_sorted(int32_t V, const int32_t* doc_ids, const int64_t* offsets,
                                const int32_t* lengths, int64_t* n_bad, int64_t* n_dup, void* ws,
                                int64_t ws_bytes, void* stream) {
  GSP_REQUIRE(V > 0 && doc_ids && offsets && lengths && n_bad && ws && ws_bytes >= kCheckWsBytes,
              GSP_ERR_ARG, "gsp_check_sorted: bad arguments (workspace needs %lld bytes)",
              (long long)kCheckWsBytes);
  cudaStream_t st = as_stream(stream);
  unsigned long long* d_bad = static_cast<unsigned long long*>(ws);
  GSP_CUDA(cudaMemsetAsync(d_bad, 0, 2 * sizeof(unsigned long long), st));
  check_sorted_kernel<<<unsigned((int64_t(V) * 32 + 255) / 256), 256, 0, st>>>(V, doc_ids, offsets,
                                                                                 lengths, d_bad);
  GSP_CHECK_LAUNCH();
  unsigned long long h[2] = {0, 0};
  GSP_CUDA(cudaMemcpyAsync(h, d_bad, sizeof(h), cudaMemcpyDeviceToHost, st));
  GSP_CUDA(cudaStreamSynchronize(st));
  *n_bad = int64_t(h[0]);
  if (n_dup) *n_dup = int64_t(h[1]);
  return GSP_OK;
}

extern "C" int gsp_chunk_bounds(int64_t n_docs, int32_t V, int64_t doc_chunk, const int32_t* doc_ids,
                                const int64_t* offsets, const int32_t* lengths, int64_t* out, void* ws,
                                int64_t ws_bytes, void* stream) {
  GSP_REQUIRE(n_docs >= 0 && V > 0 && doc_chunk > 0 && out, GSP_ERR_ARG,
              "gsp_chunk_bounds: bad arguments");
  int64_t n_bad = 0;
  int rc = gsp_check_sorted(V, doc_ids, offsets, lengths, &n_bad, nullptr, ws, ws_bytes, stream);
  if (rc) return rc;
  GSP_REQUIRE(n_bad == 0, GSP_ERR_UNSORTED,
              "%lld posting lists are not ascending in doc_id. Chunked scoring requires "
              "ascending lists; otherwise results are silently wrong.",
              (long long)n_bad);
  const int64_t n_chunks = (n_docs + doc_chunk - 1) / doc_chunk;
  chunk_bounds_kernel<<<unsigned((int64_t(V) * 32 + 255) / 256), 256, 0, as_stream(stream)>>>(
      n_docs, V, doc_chunk, n_chunks, doc_ids, offsets, lengths, out);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

extern "C" int gsp_index_head_rows(int32_t H, const int32_t* head_ids, const int64_t* offsets,
                                   const int32_t* lengths, const int32_t* doc_ids, const void* weights,
                                   int32_t wdtype, int64_t ld, void* rows, void* stream) {
  GSP_REQUIRE(H >= 0 && ld >= 0 && (H == 0 || (head_ids && offsets && lengths && doc_ids && weights && rows)),
              GSP_ERR_ARG, "gsp_index_head_rows: bad arguments");
  if (H == 0) return GSP_OK;
  cudaStream_t st = as_stream(stream);
  switch (wdtype) {
    case GSP_W_F32:
      head_rows_kernel<float><<<unsigned(H), 256, 0, st>>>(H, head_ids, offsets, lengths, doc_ids,
                                                           static_cast<const float*>(weights), ld,
                                                           static_cast<float*>(rows));
      break;
    case GSP_W_BF16:
      head_rows_kernel<__nv_bfloat16><<<unsigned(H), 256, 0, st>>>(
          H, head_ids, offsets, lengths, doc_ids, static_cast<const __nv_bfloat16*>(weights), ld,
          static_cast<__nv_bfloat16*>(rows));
      break;
    case GSP_W_U8:
      head_rows_kernel<uint8_t><<<unsigned(H), 256, 0, st>>>(H, head_ids, offsets, lengths, doc_ids,
                                                             static_cast<const uint8_t*>(weights), ld,
                                                             static_cast<uint8_t*>(rows));
      break;
    default:
      set_error("gsp_index_head_rows: unknown weight dtype %d", wdtype);
      return GSP_ERR_ARG;
  }
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}
