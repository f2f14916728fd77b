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
  const uint16_t* run_end;
  const uint8_t* ent_q;
  const float* ent_w;
  const int32_t* n_runs;
  int32_t ecap;
  int32_t C;
  int32_t n_ranges;
  uint64_t* cand;
  int32_t* cand_cnt;
};

namespace {

// ---------------------------------------------------------------------------- plan
// One CTA per warp slot: gather the slot's (term, query, slot) triples, sort them by
// that key (bitonic in shared memory) and emit runs of equal term ids.
__global__ void __launch_bounds__(kPlanThreads)
plan_kernel(const int32_t* __restrict__ qi, const float* __restrict__ qs, int32_t B, int32_t W,
            int32_t V, int32_t qpw, int32_t ecap, int32_t npow2, int32_t* __restrict__ run_term,
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
      if (start) run_term[obase + rank] = int32_t(t);
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

template <int QPW, int TILE>
struct WarpSmem {
  static constexpr int acc_bytes = QPW * TILE * 4;
  static constexpr int hist_bytes = 256 * 4;
  static constexpr int thr_bytes = ((QPW * 8 + 15) / 16) * 16;
  static constexpr int cnt_bytes = ((QPW * 4 + 15) / 16) * 16;
  __host__ __device__ static int bytes(int ecap) {
    const int run_bytes = ((ecap * 4 + 15) / 16) * 16;
    return acc_bytes + 2 * run_bytes + hist_bytes + thr_bytes + cnt_bytes;
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

template <typename WT, int QPW, int TILE>
__global__ void __launch_bounds__(kWarps * 32)
score_kernel(const ScoreParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  using SM = WarpSmem<QPW, TILE>;
  const int lane = lane_id(), wid = threadIdx.x >> 5;
  const int32_t slot = blockIdx.x * kWarps + wid;
  const int64_t q0 = int64_t(slot) * QPW;
  if (q0 >= p.B) return;  // no CTA-wide barriers below: warps are independent
  const int wbytes = SM::bytes(p.ecap);
  unsigned char* wsm = smem + size_t(wid) * wbytes;
  float* acc = reinterpret_cast<float*>(wsm);
  const int run_bytes = ((p.ecap * 4 + 15) / 16) * 16;
  uint32_t* cur = reinterpret_cast<uint32_t*>(wsm + SM::acc_bytes);
  int32_t* nd = reinterpret_cast<int32_t*>(wsm + SM::acc_bytes + run_bytes);
  uint32_t* hist = reinterpret_cast<uint32_t*>(wsm + SM::acc_bytes + 2 * run_bytes);
  uint64_t* kthr = reinterpret_cast<uint64_t*>(wsm + SM::acc_bytes + 2 * run_bytes + SM::hist_bytes);
  int32_t* cnt =
      reinterpret_cast<int32_t*>(wsm + SM::acc_bytes + 2 * run_bytes + SM::hist_bytes + SM::thr_bytes);

  const int32_t r = blockIdx.y;
  const int64_t blk0 = int64_t(p.n_blocks) * r / p.n_ranges;
  const int64_t blk1 = int64_t(p.n_blocks) * (r + 1) / p.n_ranges;
  const int64_t dbeg = blk0 * p.block_docs;
  const int64_t dend = min(blk1 * int64_t(p.block_docs), p.n_docs);
  const int32_t nq = int32_t(min64(QPW, p.B - q0));

  const int64_t pbase = int64_t(slot) * p.ecap;
  const int32_t* __restrict__ run_term = p.run_term + pbase;
  const uint16_t* __restrict__ run_end = p.run_end + pbase;
  const uint8_t* __restrict__ ent_q = p.ent_q + pbase;
  const float* __restrict__ ent_w = p.ent_w + pbase;
  const int32_t nr = p.n_runs[slot];
  const WT* __restrict__ wts = static_cast<const WT*>(p.weights);
  const int32_t* __restrict__ doc_ids = p.doc_ids;

  for (int32_t i = lane; i < nr; i += 32) {
    const int32_t t = run_term[i];
    const int64_t base = p.offsets[t];
    const int32_t len = p.lengths[t];
    const uint32_t c = p.block_starts[blk0 * p.V + t];
    cur[i] = c;
    nd[i] = int32_t(c) < len ? doc_ids[base + c] : INT_MAX;
  }
  if (lane < QPW) {
    kthr[lane] = 0ull;
    cnt[lane] = 0;
  }
  __syncwarp();

  for (int64_t d0 = dbeg; d0 < dend; d0 += TILE) {
    const int32_t d1 = int32_t(min64(d0 + TILE, dend));
    const int32_t d0i = int32_t(d0);
    float4* a4 = reinterpret_cast<float4*>(acc);
#pragma unroll 4
    for (int i = lane; i < QPW * TILE / 4; i += 32) a4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    __syncwarp();

    for (int32_t rb = 0; rb < nr; rb += 32) {
      const int32_t ri = rb + lane;
      uint32_t am = __ballot_sync(FULL, ri < nr && nd[ri] < d1);
      while (am) {
        const int32_t run = rb + __ffs(am) - 1;
        am &= am - 1;
        const int32_t t = run_term[run];
        const int32_t e0 = run ? int32_t(run_end[run - 1]) : 0;
        const int32_t e1 = int32_t(run_end[run]);
        const int64_t base = p.offsets[t];
        const int32_t len = p.lengths[t];
        float scale = 1.0f;
        if constexpr (std::is_same<WT, uint8_t>::value) scale = __ldg(p.term_scale + t);
        const int32_t ne = e1 - e0;
        int32_t my_q = 0;
        float my_w = 0.f;
        if (lane < ne) {
          my_q = ent_q[e0 + lane];
          my_w = ent_w[e0 + lane];
        }
        int32_t c = int32_t(cur[run]);
        int32_t next_doc;
        for (;;) {
          const int32_t pi = c + lane;
          const bool in = pi < len;
          const int32_t dj = in ? __ldg(doc_ids + base + pi) : INT_MAX;
          // in-tile test; the unsigned compare also rejects doc ids below the tile, so a
          // list that violates the ascending invariant can never index outside acc
          const int32_t col = dj - d0i;
          const bool m = in && uint32_t(col) < uint32_t(d1 - d0i);
          const uint32_t bal = __ballot_sync(FULL, m);
          const int32_t n = __popc(bal);
          if (n) {
            const float w = m ? WDecode<WT>::get(wts, base + pi, scale) : 0.0f;
            if (ne <= 32) {
              for (int32_t e = 0; e < ne; ++e) {
                const int32_t qq = __shfl_sync(FULL, my_q, e);
                const float qw = __shfl_sync(FULL, my_w, e);
                if (m) {
                  float* a = acc + qq * TILE + col;
                  *a = __fadd_rn(*a, __fmul_rn(qw, w));
                }
              }
            } else {
              for (int32_t e = e0; e < e1; ++e) {
                const int32_t qq = ent_q[e];
                const float qw = ent_w[e];
                if (m) {
                  float* a = acc + qq * TILE + col;
                  *a = __fadd_rn(*a, __fmul_rn(qw, w));
                }
              }
            }
          }
          c += n;
          if (n < 32) {
            next_doc = __shfl_sync(FULL, dj, n);
            break;
          }
        }
        if (lane == 0) {
          cur[run] = uint32_t(c);
          nd[run] = next_doc;
        }
        __syncwarp();
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
}

struct Cfg {
  int qpw = 0, tile = 0, ecap = 0, npow2 = 0, n_groups = 0, n_slots = 0, R = 0, C = 0;
  int wbytes = 0, smem = 0, ctas_per_sm = 0;
  int64_t n_blocks = 0, kk = 0;
  int64_t off_run_term = 0, off_run_end = 0, off_ent_q = 0, off_ent_w = 0, off_nruns = 0,
          off_cand = 0, off_cnt = 0, total = 0;
};

int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

int warp_bytes(int qpw, int tile, int ecap) {
  const int run_bytes = ((ecap * 4 + 15) / 16) * 16;
  return qpw * tile * 4 + 2 * run_bytes + 1024 + ((qpw * 8 + 15) / 16) * 16 + ((qpw * 4 + 15) / 16) * 16;
}

int make_cfg(const gsp_index_view* ix, int64_t B, int64_t W, int64_t k, Cfg& c) {
  GSP_REQUIRE(ix && ix->V > 0 && ix->n_docs >= 0 && ix->block_docs > 0 && ix->block_docs % 32 == 0,
              GSP_ERR_ARG, "score: bad index view");
  GSP_REQUIRE(B >= 0 && W >= 1 && W <= 65535 && k >= 1, GSP_ERR_ARG, "score: bad batch shape (B=%lld W=%lld k=%lld)",
              (long long)B, (long long)W, (long long)k);
  GSP_REQUIRE(W <= kMaxEntriesPerSlot, GSP_ERR_UNSUPPORTED,
              "score: query width %lld exceeds the supported maximum %d", (long long)W,
              kMaxEntriesPerSlot);
  c.kk = std::min<int64_t>(k, ix->n_docs);
  GSP_REQUIRE(c.kk <= 8192, GSP_ERR_UNSUPPORTED, "score: top_k %lld exceeds the supported maximum 8192",
              (long long)c.kk);
  const int smem_max = max_smem_optin();
  const int sms = num_sms();
  c.qpw = 0;
  for (int qpw : {4, 2, 1}) {
    if (qpw * W > kMaxEntriesPerSlot) continue;
    for (int tile : {512, 256, 128}) {
      const int ecap = int(qpw * W);
      const int wb = warp_bytes(qpw, tile, ecap);
      if (wb * kWarps <= smem_max) {
        c.qpw = qpw;
        c.tile = tile;
        c.ecap = ecap;
        c.wbytes = wb;
        break;
      }
    }
    if (c.qpw) break;
  }
  GSP_REQUIRE(c.qpw > 0, GSP_ERR_UNSUPPORTED, "score: no kernel configuration fits shared memory");
  c.smem = c.wbytes * kWarps;
  c.ctas_per_sm = std::max(1, std::min(8, (228 * 1024) / (c.smem + 1024)));
  c.npow2 = kPlanThreads;
  while (c.npow2 < c.qpw * W) c.npow2 <<= 1;
  const int64_t slots_needed = (B + c.qpw - 1) / c.qpw;
  c.n_groups = int((slots_needed + kWarps - 1) / kWarps);
  c.n_slots = c.n_groups * kWarps;
  c.n_blocks = (ix->n_docs + ix->block_docs - 1) / ix->block_docs;
  const int64_t target = int64_t(sms) * c.ctas_per_sm;
  int64_t R = c.n_groups > 0 ? std::max<int64_t>(1, target / std::max(1, c.n_groups)) : 1;
  R = std::min<int64_t>(R, std::max<int64_t>(1, c.n_blocks));
  R = std::min<int64_t>(R, 65535);
  c.R = int(R);
  c.C = int(((std::max<int64_t>(2 * c.kk, c.kk + 256) + 31) / 32) * 32);
  int64_t o = 0;
  c.off_run_term = o; o = align256(o + int64_t(c.n_slots) * c.ecap * 4);
  c.off_run_end = o; o = align256(o + int64_t(c.n_slots) * c.ecap * 2);
  c.off_ent_q = o; o = align256(o + int64_t(c.n_slots) * c.ecap * 1);
  c.off_ent_w = o; o = align256(o + int64_t(c.n_slots) * c.ecap * 4);
  c.off_nruns = o; o = align256(o + int64_t(c.n_slots) * 4);
  c.off_cand = o; o = align256(o + B * int64_t(c.R) * c.C * 8);
  c.off_cnt = o; o = align256(o + B * int64_t(c.R) * 4);
  c.total = o;
  return GSP_OK;
}

template <typename WT, int QPW, int TILE>
int launch_score(const ScoreParams& p, const Cfg& c, cudaStream_t st) {
  auto kern = score_kernel<WT, QPW, TILE>;
  GSP_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, c.smem));
  dim3 grid(unsigned(c.n_groups), unsigned(c.R));
  kern<<<grid, kWarps * 32, c.smem, st>>>(p);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

template <typename WT>
int dispatch_tile(const ScoreParams& p, const Cfg& c, cudaStream_t st) {
#define GSP_CASE(Q, T) \
  if (c.qpw == Q && c.tile == T) return launch_score<WT, Q, T>(p, c, st);
  GSP_CASE(4, 512) GSP_CASE(4, 256) GSP_CASE(4, 128)
  GSP_CASE(2, 512) GSP_CASE(2, 256) GSP_CASE(2, 128)
  GSP_CASE(1, 512) GSP_CASE(1, 256) GSP_CASE(1, 128)
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

extern "C" int gsp_score_topk(const gsp_index_view* ix, const int32_t* qi, const float* qs, int64_t B,
                              int64_t W, int64_t k, float* out_scores, int64_t* out_ids,
                              uint64_t* out_keys, void* ws, int64_t ws_bytes, void* stream) {
  Cfg c;
  int rc = make_cfg(ix, B, W, k, c);
  if (rc) return rc;
  GSP_REQUIRE(ws && ws_bytes >= c.total, GSP_ERR_ARG, "gsp_score_topk: workspace too small (%lld < %lld)",
              (long long)ws_bytes, (long long)c.total);
  GSP_REQUIRE(ix->doc_ids && ix->weights && ix->offsets && ix->lengths && ix->block_starts &&
                  (ix->wdtype != GSP_W_U8 || ix->term_scale),
              GSP_ERR_ARG, "gsp_score_topk: null index array");
  GSP_REQUIRE(ix->doc_base >= 0 && ix->doc_base + ix->n_docs <= 0xFFFFFFFEll, GSP_ERR_UNSUPPORTED,
              "gsp_score_topk: global doc ids must stay below 2^32 - 1");
  if (B == 0 || c.kk == 0) return GSP_OK;
  GSP_REQUIRE(qi && qs && out_scores && out_ids, GSP_ERR_ARG, "gsp_score_topk: null argument");
  cudaStream_t st = as_stream(stream);
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
  p.run_end = reinterpret_cast<uint16_t*>(w + c.off_run_end);
  p.ent_q = reinterpret_cast<uint8_t*>(w + c.off_ent_q);
  p.ent_w = reinterpret_cast<float*>(w + c.off_ent_w);
  p.n_runs = reinterpret_cast<int32_t*>(w + c.off_nruns);
  p.ecap = c.ecap;
  p.C = c.C;
  p.n_ranges = c.R;
  p.cand = reinterpret_cast<uint64_t*>(w + c.off_cand);
  p.cand_cnt = reinterpret_cast<int32_t*>(w + c.off_cnt);

  const size_t plan_smem = size_t(c.npow2) * 8;
  GSP_CUDA(cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(plan_smem)));
  plan_kernel<<<unsigned(c.n_slots), kPlanThreads, plan_smem, st>>>(
      qi, qs, int32_t(B), int32_t(W), ix->V, c.qpw, c.ecap, c.npow2, const_cast<int32_t*>(p.run_term),
      const_cast<uint16_t*>(p.run_end), const_cast<uint8_t*>(p.ent_q), const_cast<float*>(p.ent_w),
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
