// Exact batched scoring with fused threshold selection (sm_100a).
//
// Replaces src/triton_kernel.py:93-200 (_fast_scatter_add_kernel + torch.zeros +
// torch.topk), src/triton_kernel_chunked.py:34-170 and src/fused_topk.py:33-160.
//
// Work decomposition.  Queries are cut into warp slots of QPW queries; a CTA holds
// kWarps slots (one query group) and one document range (a run of whole index blocks).
// Every warp owns fp32 accumulators acc[QPW][TILE] in shared memory for the current
// document tile, so each accumulator cell has exactly one writer and no atomics are
// needed.  Per tile the warp walks its "runs": the distinct terms of its queries in
// ascending term id, each with the (query, weight) entries that use it.  A run streams
// the term's postings that fall inside the tile (coalesced 32-wide loads from the cursor
// kept per run; postings ascend by doc id so the tile boundary is a ballot) and applies
// each posting to every entry of the run, so one posting load feeds all of the warp's
// queries that contain the term.  Each cell therefore receives its contributions in
// ascending (term id, slot) order with one fp32 rounding for the product and one for the
// sum: results are bitwise reproducible and equal to the CPU oracle's canonical order.
//
// Selection.  After a tile every (query, tile) score is turned into a packed 64-bit key
// (order-preserving score bits << 32 | ~doc id: larger is better, ties -> lower doc id)
// and appended to the query's candidate buffer for this range if it is >= the query's
// running threshold.  When the buffer would overflow, the owning warp radix-selects the
// k-th largest key (8-bit digits, most significant first, early exit once the boundary
// bucket is taken whole), compacts the buffer in place to exactly k keys and raises the
// threshold to that boundary.  Every discarded key is below k kept keys of the same
// query, so the final top-k is exact.  A merge kernel (select.cu) then reduces the
// ranges' k-lists of each query to the answer.
#include "common.cuh"

#include <algorithm>
#include <mutex>
#include <stdio.h>
#include <stdlib.h>
#include <utility>
#include <vector>

namespace gsp {

constexpr int kWarps = 8;
constexpr int kPlanThreads = 256;
constexpr int kMaxEntriesPerSlot = 2048;

struct ScoreParams {
  const int32_t* doc_ids;
  const void* weights;
  const float* term_scale;
  const int64_t* offsets;
  const int32_t* lengths;
  const uint32_t* block_starts;
  int64_t n_docs;
  int64_t doc_base;
  int32_t V;
  int32_t block_docs;
  int32_t n_blocks;
  int32_t B;
  int32_t W;
  int32_t k;
  const int32_t* run_term;
  const uint32_t* run_base32;
  const uint16_t* run_end;
  const uint8_t* ent_q;
  const float* ent_w;
  const int32_t* n_runs;
  int32_t ecap;
  int32_t C;
  int32_t n_ranges;
  int32_t n_slots;
  uint64_t* cand;
  int32_t* cand_cnt;
  uint32_t* work_counter;
};

namespace {

// ---------------------------------------------------------------------------- plan
// One CTA per warp slot: gather the slot's (term, query, slot) triples, sort them by
// that key (bitonic in shared memory) and emit runs of equal term ids.
__global__ void __launch_bounds__(kPlanThreads)
plan_kernel(const int32_t* __restrict__ qi, const float* __restrict__ qs, int32_t B, int32_t W,
            int32_t V, int32_t qpw, int32_t ecap, int32_t npow2, const int64_t* __restrict__ offsets,
            int32_t* __restrict__ run_term, uint32_t* __restrict__ run_base32,
            uint16_t* __restrict__ run_end, uint8_t* __restrict__ ent_q, float* __restrict__ ent_w,
            int32_t* __restrict__ n_runs) {
  extern __shared__ uint64_t keys[];
  __shared__ int32_t s_base;
  __shared__ int32_t warp_cnt[kPlanThreads / 32];
  const int32_t slot = blockIdx.x;
  const int64_t q0 = int64_t(slot) * qpw;
  const int32_t ne = qpw * W;
  for (int32_t i = threadIdx.x; i < npow2; i += blockDim.x) {
    uint64_t key = ~0ull;
    if (i < ne) {
      const int32_t qq = i / W, s = i - qq * W;
      const int64_t q = q0 + qq;
      if (q < B) {
        const int32_t t = qi[q * W + s];
        if (t >= 0 && t < V)
          key = (uint64_t(uint32_t(t)) << 32) | (uint64_t(qq) << 16) | uint64_t(s);
      }
    }
    keys[i] = key;
  }
  __syncthreads();
  // bitonic sort, ascending
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
  // runs: a new run starts where the term id changes; ordinal by a running ballot scan
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  const int64_t obase = int64_t(slot) * ecap;
  for (int32_t i0 = 0; i0 < npow2; i0 += blockDim.x) {
    const int32_t i = i0 + threadIdx.x;
    const uint64_t key = keys[i];
    const bool valid = key != ~0ull;
    const uint32_t t = uint32_t(key >> 32);
    const bool start = valid && (i == 0 || uint32_t(keys[i - 1] >> 32) != t);
    // block-wide exclusive count of starts before i
    const uint32_t bal = __ballot_sync(FULL, start);
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) warp_cnt[wid] = __popc(bal);
    __syncthreads();
    int32_t before = s_base;
    for (int w = 0; w < wid; ++w) before += warp_cnt[w];
    const int32_t rank = before + __popc(bal & lanemask_lt());
    if (valid) {
      const int32_t qq = int32_t((key >> 16) & 0xFFFF), s = int32_t(key & 0xFFFF);
      ent_q[obase + i] = uint8_t(qq);
      ent_w[obase + i] = qs[(q0 + qq) * W + s];
      if (start) {
        run_term[obase + rank] = int32_t(t);
        run_base32[obase + rank] = uint32_t(offsets[t] >> 5);
      }
      // end of the run containing i is written by its last entry
      const bool last = (i + 1 >= npow2) || keys[i + 1] == ~0ull || uint32_t(keys[i + 1] >> 32) != t;
      if (last) run_end[obase + rank - (start ? 0 : 1)] = uint16_t(i + 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int32_t tot = 0;
      for (int w = 0; w < kPlanThreads / 32; ++w) tot += warp_cnt[w];
      s_base += tot;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) n_runs[slot] = s_base;
}

// ---------------------------------------------------------------------------- scoring

__host__ __device__ constexpr int align16(int x) { return (x + 15) / 16 * 16; }

// Shared memory of one warp: its accumulator tile, a radix histogram and per-query
// selection state.  Run and entry lists stay in global memory (L1-resident).
struct WarpLayout {
  int acc, hist, thr, cnt, total;
  __host__ __device__ WarpLayout(int qpw, int tile) {
    acc = 0;
    hist = acc + qpw * tile * 4;
    thr = hist + 256 * 4;
    cnt = thr + align16(qpw * 8);
    total = cnt + align16(qpw * 4);
  }
};

// Radix-select the k-th largest key of buf[0..n) (n > k, keys distinct), keep exactly the
// k largest in place (stable) and return the smallest key value that is kept-or-better.
__device__ uint64_t warp_compact(uint64_t* __restrict__ buf, int32_t n, int32_t k,
                                 uint32_t* __restrict__ hist) {
  const int lane = lane_id();
  uint64_t prefix = 0;
  int32_t need = k;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int j = lane; j < 256; j += 32) hist[j] = 0u;
    __syncwarp();
    const uint64_t pmask = shift == 56 ? 0ull : (~0ull << (shift + 8));
    for (int32_t i0 = 0; i0 < n; i0 += 32) {
      const int32_t i = i0 + lane;
      const uint64_t key = i < n ? buf[i] : 0ull;
      const bool live = i < n && (key & pmask) == prefix;
      const uint32_t dig = live ? uint32_t((key >> shift) & 255u) : 0x100u;
      const uint32_t peers = __match_any_sync(FULL, dig);
      if (live && (peers & lanemask_lt()) == 0u) hist[dig] += __popc(peers);
      __syncwarp();
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
  // stable in-place compaction of keys >= prefix
  int32_t out = 0;
  for (int32_t i0 = 0; i0 < n; i0 += 32) {
    const int32_t i = i0 + lane;
    const uint64_t key = i < n ? buf[i] : 0ull;
    const bool keep = i < n && key >= prefix;
    const uint32_t bal = __ballot_sync(FULL, keep);
    if (keep) buf[out + __popc(bal & lanemask_lt())] = key;
    out += __popc(bal);
  }
  __syncwarp();
  return prefix;
}

// acc[d - d0] += fl(qw * w) for one posting; the column test keeps a list that breaks the
// ascending-doc-id invariant from ever addressing outside the tile.
__device__ __forceinline__ void acc_add(float* __restrict__ row, int32_t col, uint32_t span, float qw,
                                        float w) {
  if (uint32_t(col) < span) {
    float* a = row + col;
    *a = __fadd_rn(*a, __fmul_rn(qw, w));
  }
}

constexpr int kUnroll = 4;   // posting chunks of one run in flight together

// Apply the postings [wlo, whi) of one run to NE (1 or 2) entries held in registers, or to
// every entry of the run from global memory when NE == 0.
template <typename WT, int NE, int TILE>
__device__ __forceinline__ void run_window(const int32_t* __restrict__ pd, const WT* __restrict__ pw,
                                           float scale, int32_t n, int32_t d0i, uint32_t span,
                                           float* __restrict__ acc, int32_t q_a, float w_a, int32_t q_b,
                                           float w_b, const uint8_t* __restrict__ eq,
                                           const float* __restrict__ ew, int32_t ne) {
  const int lane = lane_id();
  float* row_a = acc + q_a * TILE;
  float* row_b = acc + q_b * TILE;
  for (int32_t base = 0; base < n; base += 32 * kUnroll) {
    int32_t col[kUnroll];
    float w[kUnroll];
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
    for (int u = 0; u < kUnroll; ++u) {
      if constexpr (NE >= 1) acc_add(row_a, col[u], span, w_a, w[u]);
      if constexpr (NE >= 2) acc_add(row_b, col[u], span, w_b, w[u]);
      if constexpr (NE == 0) {
        for (int32_t e = 0; e < ne; ++e) acc_add(acc + int32_t(eq[e]) * TILE, col[u], span, ew[e], w[u]);
      }
    }
  }
}

// Work items: (warp slot, document range).  Each warp takes items from a global counter
// in order item = range * n_slots + slot, so warps running concurrently share a range and
// its postings stay hot in L2.  Tiles are the index's document blocks, so every run's
// window of postings in a tile is [block_starts[b][t], block_starts[b+1][t]).
template <typename WT, int QPW, int TILE>
__global__ void __launch_bounds__(kWarps * 32, 3)
score_kernel(const ScoreParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = lane_id(), wid = threadIdx.x >> 5;
  const WarpLayout lay(QPW, TILE);
  unsigned char* wsm = smem + size_t(wid) * lay.total;
  float* acc = reinterpret_cast<float*>(wsm + lay.acc);
  uint32_t* hist = reinterpret_cast<uint32_t*>(wsm + lay.hist);
  uint64_t* kthr = reinterpret_cast<uint64_t*>(wsm + lay.thr);
  int32_t* cnt = reinterpret_cast<int32_t*>(wsm + lay.cnt);
  const WT* __restrict__ wts = static_cast<const WT*>(p.weights);
  const int32_t* __restrict__ doc_ids = p.doc_ids;
  const uint32_t* __restrict__ bstarts = p.block_starts;
  const int64_t n_items = int64_t(p.n_slots) * p.n_ranges;

  for (;;) {
    int64_t item = 0;
    if (lane == 0) item = int64_t(atomicAdd(p.work_counter, 1u));
    item = __shfl_sync(FULL, item, 0);
    if (item >= n_items) break;
    const int32_t slot = int32_t(item % p.n_slots);
    const int32_t r = int32_t(item / p.n_slots);
    const int64_t q0 = int64_t(slot) * QPW;
    if (q0 >= p.B) continue;
    const int64_t blk0 = int64_t(p.n_blocks) * r / p.n_ranges;
    const int64_t blk1 = int64_t(p.n_blocks) * (r + 1) / p.n_ranges;
    const int32_t nq = int32_t(min64(QPW, p.B - q0));
    const int64_t pbase = int64_t(slot) * p.ecap;
    const int32_t nr = p.n_runs[slot];
    const int32_t* __restrict__ run_term = p.run_term + pbase;
    const uint32_t* __restrict__ run_b32 = p.run_base32 + pbase;
    const uint16_t* __restrict__ run_end = p.run_end + pbase;
    const uint8_t* __restrict__ ent_q = p.ent_q + pbase;
    const float* __restrict__ ent_w = p.ent_w + pbase;
    if (lane < QPW) {
      kthr[lane] = 0ull;
      cnt[lane] = 0;
    }
    __syncwarp();

    for (int64_t b = blk0; b < blk1; ++b) {
      const int32_t d0i = int32_t(b * TILE);
      const int32_t d1 = int32_t(min64((b + 1) * TILE, p.n_docs));
      const uint32_t span = uint32_t(d1 - d0i);
      const uint32_t* __restrict__ brow = bstarts + b * int64_t(p.V);
      float4* a4 = reinterpret_cast<float4*>(acc);
#pragma unroll 4
      for (int i = lane; i < QPW * TILE / 4; i += 32) a4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      __syncwarp();

      for (int32_t rb = 0; rb < nr; rb += 32) {
        // this tile's window of up to 32 runs, one lane per run
        const int32_t ri = rb + lane;
        uint32_t lo = 0, hi = 0;
        int32_t e_lo = 0, e_hi = 0;
        uint32_t b32 = 0;
        if (ri < nr) {
          const int32_t t = run_term[ri];
          lo = __ldg(brow + t);
          hi = __ldg(brow + p.V + t);
          e_lo = ri ? int32_t(run_end[ri - 1]) : 0;
          e_hi = int32_t(run_end[ri]);
          b32 = run_b32[ri];
        }
        uint32_t am = __ballot_sync(FULL, hi > lo);
        while (am) {
          const int j = __ffs(am) - 1;
          am &= am - 1;
          const uint32_t wlo = __shfl_sync(FULL, lo, j), whi = __shfl_sync(FULL, hi, j);
          const int32_t e0 = __shfl_sync(FULL, e_lo, j), e1 = __shfl_sync(FULL, e_hi, j);
          const int64_t base = (int64_t(__shfl_sync(FULL, b32, j)) << 5) + wlo;
          float scale = 1.0f;
          if constexpr (std::is_same<WT, uint8_t>::value) scale = __ldg(p.term_scale + run_term[rb + j]);
          const int32_t n = int32_t(whi - wlo), ne = e1 - e0;
          const int32_t q_a = ent_q[e0];
          const float w_a = ent_w[e0];
          if (ne == 1) {
            run_window<WT, 1, TILE>(doc_ids + base, wts + base, scale, n, d0i, span, acc, q_a, w_a, 0,
                                    0.f, nullptr, nullptr, 0);
          } else if (ne == 2) {
            run_window<WT, 2, TILE>(doc_ids + base, wts + base, scale, n, d0i, span, acc, q_a, w_a,
                                    ent_q[e0 + 1], ent_w[e0 + 1], nullptr, nullptr, 0);
          } else {
            run_window<WT, 0, TILE>(doc_ids + base, wts + base, scale, n, d0i, span, acc, 0, 0.f, 0,
                                    0.f, ent_q + e0, ent_w + e0, ne);
          }
        }
      }
      __syncwarp();

      // fused selection of this tile
      for (int32_t qq = 0; qq < nq; ++qq) {
        uint64_t* __restrict__ buf = p.cand + ((q0 + qq) * p.n_ranges + r) * int64_t(p.C);
        uint64_t thr = kthr[qq];
        int32_t n = cnt[qq];
        for (int32_t c0 = 0; c0 < d1 - d0i; c0 += 32) {
          const int32_t col = c0 + lane;
          const bool valid = d0i + col < d1;
          const float s = acc[qq * TILE + (valid ? col : 0)];
          const uint64_t key = pack_key(s, uint32_t(p.doc_base + d0i + col));
          bool pass = valid && key >= thr;
          uint32_t bal = __ballot_sync(FULL, pass);
          if (!bal) continue;
          if (n + __popc(bal) > p.C) {
            thr = warp_compact(buf, n, p.k, hist);
            n = p.k;
            pass = pass && key >= thr;
            bal = __ballot_sync(FULL, pass);
          }
          if (pass) buf[n + __popc(bal & lanemask_lt())] = key;
          n += __popc(bal);
        }
        __syncwarp();
        if (lane == 0) {
          kthr[qq] = thr;
          cnt[qq] = n;
        }
        __syncwarp();
      }
    }

    for (int32_t qq = 0; qq < nq; ++qq) {
      uint64_t* __restrict__ buf = p.cand + ((q0 + qq) * p.n_ranges + r) * int64_t(p.C);
      int32_t n = cnt[qq];
      if (n > p.k) {
        warp_compact(buf, n, p.k, hist);
        n = p.k;
      }
      if (lane == 0) p.cand_cnt[(q0 + qq) * p.n_ranges + r] = n;
    }
    __syncwarp();
  }
}

struct Cfg {
  int qpw = 0, tile = 0, ecap = 0, npow2 = 0, n_groups = 0, n_slots = 0, R = 0, C = 0;
  int wbytes = 0, smem = 0, ctas_per_sm = 0, grid = 0;
  int64_t n_blocks = 0, kk = 0;
  int64_t off_run_term = 0, off_run_b32 = 0, off_run_end = 0, off_ent_q = 0, off_ent_w = 0, off_nruns = 0,
          off_cand = 0, off_cnt = 0, off_counter = 0, total = 0;
};

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

int warp_bytes(int qpw, int tile) { return WarpLayout(qpw, tile).total; }

// (queries per warp, tile) shapes that are compiled, preferred first for each tile
static const int kShapes[][2] = {{2, 1024}, {4, 1024}, {1, 1024}, {2, 2048}, {1, 2048}, {1, 4096},
                                 {4, 512},  {2, 512},  {4, 256}};

// Workspace layout of one call for the configured shape and range count.
void set_layout(Cfg& c, int64_t B) {
  int64_t o = 0;
  c.off_run_term = o; o = align256(o + int64_t(c.n_slots) * c.ecap * 4);
  c.off_run_b32 = o; o = align256(o + int64_t(c.n_slots) * c.ecap * 4);
  c.off_run_end = o; o = align256(o + int64_t(c.n_slots) * c.ecap * 2);
  c.off_ent_q = o; o = align256(o + int64_t(c.n_slots) * c.ecap * 1);
  c.off_ent_w = o; o = align256(o + int64_t(c.n_slots) * c.ecap * 4);
  c.off_nruns = o; o = align256(o + int64_t(c.n_slots) * 4);
  c.off_cand = o; o = align256(o + B * int64_t(c.R) * c.C * 8);
  c.off_cnt = o; o = align256(o + B * int64_t(c.R) * 4);
  c.off_counter = o; o = align256(o + 4);
  c.total = o;
}

int make_cfg(const gsp_index_view* ix, int64_t B, int64_t W, int64_t k, Cfg& c) {
  GSP_REQUIRE(ix && ix->V > 0 && ix->n_docs >= 0 && ix->block_docs > 0, GSP_ERR_ARG,
              "score: bad index view");
  GSP_REQUIRE(B >= 0 && W >= 1 && W <= 65535 && k >= 1, GSP_ERR_ARG,
              "score: bad batch shape (B=%lld W=%lld k=%lld)", (long long)B, (long long)W, (long long)k);
  GSP_REQUIRE(W <= kMaxEntriesPerSlot, GSP_ERR_UNSUPPORTED,
              "score: query width %lld exceeds the supported maximum %d", (long long)W,
              kMaxEntriesPerSlot);
  c.kk = std::min<int64_t>(k, ix->n_docs);
  GSP_REQUIRE(c.kk <= 8192, GSP_ERR_UNSUPPORTED, "score: top_k %lld exceeds the supported maximum 8192",
              (long long)c.kk);
  const int smem_max = max_smem_optin();
  const int sms = num_sms();
  // GSP_SCORE_QPW overrides the choice (tuning)
  int want_q = 0;
  if (const char* e = getenv("GSP_SCORE_QPW")) want_q = atoi(e);
  c.qpw = 0;
  c.tile = ix->block_docs;
  for (const auto& sh : kShapes) {
    const int qpw = sh[0], tile = sh[1];
    if (tile != c.tile || (want_q && qpw != want_q)) continue;
    if (qpw * W > kMaxEntriesPerSlot) continue;
    const int ecap = int(qpw * W);
    const int wb = warp_bytes(qpw, tile);
    if (wb * kWarps <= smem_max) {
      c.qpw = qpw;
      c.ecap = ecap;
      c.wbytes = wb;
      break;
    }
  }
  GSP_REQUIRE(c.qpw > 0, GSP_ERR_UNSUPPORTED,
              "score: no scoring kernel for index block size %d with query width %lld",
              ix->block_docs, (long long)W);
  c.smem = c.wbytes * kWarps;
  c.ctas_per_sm = std::max(1, std::min(8, (228 * 1024) / (c.smem + 1024)));
  c.npow2 = kPlanThreads;
  while (c.npow2 < c.qpw * W) c.npow2 <<= 1;
  const int64_t slots_needed = (B + c.qpw - 1) / c.qpw;
  c.n_groups = int((slots_needed + kWarps - 1) / kWarps);
  c.n_slots = c.n_groups * kWarps;
  c.n_blocks = (ix->n_docs + c.tile - 1) / c.tile;
  // about four work items per resident warp, ranges of whole blocks
  const int64_t warps = int64_t(sms) * c.ctas_per_sm * kWarps;
  int64_t R = std::max<int64_t>(1, (4 * warps + slots_needed - 1) / std::max<int64_t>(1, slots_needed));
  R = std::min<int64_t>(R, std::max<int64_t>(1, c.n_blocks));
  R = std::min<int64_t>(R, 4096);
  c.R = int(R);
  c.grid = int(std::min<int64_t>(int64_t(sms) * c.ctas_per_sm,
                                 (int64_t(c.n_slots) * c.R + kWarps - 1) / kWarps));
  c.C = int(((std::max<int64_t>(2 * c.kk, c.kk + 256) + 31) / 32) * 32);
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

template <typename WT, int QPW, int TILE>
int launch_score(const ScoreParams& p, const Cfg& c, cudaStream_t st) {
  auto kern = score_kernel<WT, QPW, TILE>;
  GSP_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, c.smem));
  Profile& pr = profile();
  std::pair<cudaEvent_t, cudaEvent_t>* evp = nullptr;
  {
    std::lock_guard<std::mutex> g(pr.mu);
    if (pr.on) {
      if (pr.used == pr.ev.size()) {
        cudaEvent_t a, b;
        GSP_CUDA(cudaEventCreate(&a));
        GSP_CUDA(cudaEventCreate(&b));
        pr.ev.emplace_back(a, b);
      }
      evp = &pr.ev[pr.used++];
    }
  }
  if (evp) GSP_CUDA(cudaEventRecord(evp->first, st));
  kern<<<unsigned(c.grid), kWarps * 32, c.smem, st>>>(p);
  GSP_CHECK_LAUNCH();
  if (evp) GSP_CUDA(cudaEventRecord(evp->second, st));
  return GSP_OK;
}

template <typename WT>
int dispatch_tile(const ScoreParams& p, const Cfg& c, cudaStream_t st) {
#define GSP_CASE(Q, T) \
  if (c.qpw == Q && c.tile == T) return launch_score<WT, Q, T>(p, c, st);
  GSP_CASE(2, 1024) GSP_CASE(4, 1024) GSP_CASE(1, 1024) GSP_CASE(2, 2048) GSP_CASE(1, 2048)
  GSP_CASE(1, 4096) GSP_CASE(4, 512) GSP_CASE(2, 512) GSP_CASE(4, 256)
#undef GSP_CASE
  set_error("score: no kernel instantiated for qpw=%d tile=%d", c.qpw, c.tile);
  return GSP_ERR_UNSUPPORTED;
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
                          uint64_t* out_keys, void* ws, cudaStream_t st) {
  int rc = GSP_OK;
  GSP_REQUIRE(ix->doc_ids && ix->weights && ix->offsets && ix->lengths && ix->block_starts &&
                  (ix->wdtype != GSP_W_U8 || ix->term_scale),
              GSP_ERR_ARG, "gsp_score_topk: null index array");
  GSP_REQUIRE(ix->doc_base >= 0 && ix->doc_base + ix->n_docs <= 0xFFFFFFFEll, GSP_ERR_UNSUPPORTED,
              "gsp_score_topk: global doc ids must stay below 2^32 - 1");
  if (B == 0 || c.kk == 0) return GSP_OK;
  GSP_REQUIRE(qi && qs && out_scores && out_ids, GSP_ERR_ARG, "gsp_score_topk: null argument");
  char* w = static_cast<char*>(ws);
  ScoreParams p;
  p.doc_ids = ix->doc_ids;
  p.weights = ix->weights;
  p.term_scale = ix->term_scale;
  p.offsets = ix->offsets;
  p.lengths = ix->lengths;
  p.block_starts = ix->block_starts;
  p.n_docs = ix->n_docs;
  p.doc_base = ix->doc_base;
  p.V = ix->V;
  p.block_docs = ix->block_docs;
  p.n_blocks = int32_t(c.n_blocks);
  p.B = int32_t(B);
  p.W = int32_t(W);
  p.k = int32_t(c.kk);
  p.run_term = reinterpret_cast<int32_t*>(w + c.off_run_term);
  p.run_base32 = reinterpret_cast<uint32_t*>(w + c.off_run_b32);
  p.run_end = reinterpret_cast<uint16_t*>(w + c.off_run_end);
  p.ent_q = reinterpret_cast<uint8_t*>(w + c.off_ent_q);
  p.ent_w = reinterpret_cast<float*>(w + c.off_ent_w);
  p.n_runs = reinterpret_cast<int32_t*>(w + c.off_nruns);
  p.ecap = c.ecap;
  p.C = c.C;
  p.n_ranges = c.R;
  p.n_slots = c.n_slots;
  p.cand = reinterpret_cast<uint64_t*>(w + c.off_cand);
  p.cand_cnt = reinterpret_cast<int32_t*>(w + c.off_cnt);
  p.work_counter = reinterpret_cast<uint32_t*>(w + c.off_counter);
  GSP_CUDA(cudaMemsetAsync(p.work_counter, 0, sizeof(uint32_t), st));

  const size_t plan_smem = size_t(c.npow2) * 8;
  GSP_CUDA(cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(plan_smem)));
  plan_kernel<<<unsigned(c.n_slots), kPlanThreads, plan_smem, st>>>(
      qi, qs, int32_t(B), int32_t(W), ix->V, c.qpw, c.ecap, c.npow2, ix->offsets,
      const_cast<int32_t*>(p.run_term), const_cast<uint32_t*>(p.run_base32), const_cast<uint16_t*>(p.run_end), const_cast<uint8_t*>(p.ent_q), const_cast<float*>(p.ent_w),
      const_cast<int32_t*>(p.n_runs));
  GSP_CHECK_LAUNCH();

  if (c.n_blocks > 0) {
    switch (ix->wdtype) {
      case GSP_W_F32: rc = dispatch_tile<float>(p, c, st); break;
      case GSP_W_BF16: rc = dispatch_tile<__nv_bfloat16>(p, c, st); break;
      case GSP_W_U8: rc = dispatch_tile<uint8_t>(p, c, st); break;
      default: set_error("gsp_score_topk: unknown weight dtype %d", ix->wdtype); return GSP_ERR_ARG;
    }
    if (rc) return rc;
  }
  return merge_topk_device(p.cand, B, c.R, int64_t(c.R) * c.C, c.C, p.cand_cnt, c.R, nullptr, c.kk,
                           out_scores, out_ids, out_keys, st);
}

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

// ---------------------------------------------------------------------------------------
// Scoring without any device allocation.
//
// Some callers cannot allocate device memory while they serve a batch: a serving loop
// where a cudaMalloc would synchronise the device and stall every other stream, or a host
// application (for example a search engine that loads this library as a native plug-in
// through a C FFI) that hands the library only its input and output buffers and owns no
// device allocator to lend it a workspace.  gsp_score_topk_noalloc serves them: its
// scratch (query plan, candidate buffers, work counter) lives in the file-scope array
// below, which the CUDA runtime places on every GPU that loads this library and keeps
// until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;   // 32 MiB per GPU
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[256] = {nullptr};   // device address of the array, per device ordinal
}  // namespace

// Host code may not use g_noalloc_scratch as an address (it is a host-side stand-in), so
// the device address is looked up once per device, with that device current.
static int noalloc_scratch(void** out) {
  int dev = 0;
  GSP_CUDA(cudaGetDevice(&dev));
  GSP_REQUIRE(dev >= 0 && dev < 256, GSP_ERR_UNSUPPORTED, "noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error("gsp_score_topk_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return GSP_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return GSP_OK;
}

extern "C" int gsp_score_topk_noalloc(const gsp_index_view* ix, const int32_t* qi, const float* qs,
                                      int64_t B, int64_t W, int64_t k, float* out_scores,
                                      int64_t* out_ids, uint64_t* out_keys, void* stream) {
  Cfg c;
  int rc = make_cfg(ix, B, W, k, c);
  if (rc) return rc;
  // fewer document ranges shrink the candidate buffers; the result does not depend on
  // the range count, only the parallelism does
  while (c.total > int64_t(kNoAllocScratchBytes) && c.R > 1) {
    c.R = std::max(1, c.R / 2);
    set_layout(c, B);
  }
  GSP_REQUIRE(c.total <= int64_t(kNoAllocScratchBytes), GSP_ERR_UNSUPPORTED,
              "gsp_score_topk_noalloc: this batch needs %lld bytes of scratch, more than the "
              "fixed %lld (lower the batch size or top_k, or use gsp_score_topk with a workspace)",
              (long long)c.total, (long long)kNoAllocScratchBytes);
  c.grid = int(std::min<int64_t>(int64_t(num_sms()) * c.ctas_per_sm,
                                 (int64_t(c.n_slots) * c.R + kWarps - 1) / kWarps));
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  // Every buffer in the scratch is written before it is read within a call except the
  // work counter, which score_with_cfg clears on the stream; the array keeps the previous
  // call's contents otherwise.
  return score_with_cfg(ix, qi, qs, B, W, c, out_scores, out_ids, out_keys, scratch, as_stream(stream));
}
