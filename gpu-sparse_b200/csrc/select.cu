// Exact top-k selection over packed candidate keys (sm_100a).
//
// A candidate is one uint64: fkey(score) << 32 | (0xFFFFFFFF - doc id).  Larger keys are
// better (higher score, then lower doc id), and keys of one query are distinct, so "the k
// largest keys" is exactly the reference's top-k with deterministic tie-breaking.
//
// merge_kernel: one CTA per query.  Radix-select the k-th largest key over the query's R
// candidate lists (8-bit digits, most significant first, shared-memory histogram with
// warp-aggregated increments, early exit once the boundary bucket is taken whole), gather
// the k keys at or above the boundary into shared memory, bitonic-sort them descending
// and decode (score, doc id).  If the producer of the candidates reported a fault, the
// query's output is NaN scores and ids -1 instead.
//
// Above kMaxK keys per query (the reference's torch.topk takes any k) the k keys do not fit
// one CTA's shared memory: merge_kernel gathers them, unsorted, into a global buffer, every
// run of kRun keys is sorted in shared memory (sort_runs_kernel), and merge passes over
// global memory (merge_pass_kernel, one merge-path split per thread) double the sorted
// runs until each query's k keys are one descending list.  This replaces torch.topk over the dense matrix
// (src/triton_kernel.py:199), the running cat/topk/gather merge
// (src/triton_kernel_chunked.py:162-168) and the host-side shard merge
// (src/comprehensive_benchmark.py:472-480).
#include "common.cuh"

#include <algorithm>

namespace gsp {

constexpr int kMergeThreads = 512;
constexpr int kMaxParamCounts = 64;
constexpr int kMaxK = kMaxSmemK;   // largest k sorted in one CTA's shared memory
constexpr int kRun = 4096;         // keys per run sorted in shared memory (large k)
constexpr int kRunThreads = 1024;
constexpr int kMergeOut = 8;       // outputs per thread of a merge pass
constexpr int kMergePassThreads = 256;

struct CountsParam {
  int32_t c[kMaxParamCounts];
};

namespace {

// The R candidate lists of one query at kb + r * stride_r, with counts from the kernel
// parameter or from counts_dev[b * cstride_b + r].
struct Lists {
  const uint64_t* base;
  int64_t stride_r;
  const int32_t* counts_dev;
  int64_t cstride_b;
  int32_t b, n;
  bool use_param;
  __device__ __forceinline__ int32_t count(int32_t r, const CountsParam& cp) const {
    return use_param ? cp.c[r] : counts_dev[int64_t(b) * cstride_b + r];
  }
  __device__ __forceinline__ const uint64_t* list(int32_t r) const { return base + int64_t(r) * stride_r; }
};

__global__ void __launch_bounds__(kMergeThreads)
merge_kernel(const uint64_t* __restrict__ keys, int64_t stride_b, int64_t stride_r, int32_t R,
             const int32_t* __restrict__ fault, const int32_t* __restrict__ counts_dev, int64_t cstride_b,
             const CountsParam cp, int32_t use_param, int32_t k, int32_t k_out, int32_t kpow2,
             int64_t pad_id, float* __restrict__ out_s, int64_t* __restrict__ out_i,
             uint64_t* __restrict__ out_k, int32_t tree_groups, int32_t tree_n_in,
             uint64_t* __restrict__ gather_g) {
  extern __shared__ uint64_t sk[];
  __shared__ uint32_t hist[256];
  __shared__ int32_t s_total, s_n, s_D, s_above, s_cD;
  __shared__ int32_t s_part[kMergeThreads / 32];
  const int32_t b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int64_t ob = int64_t(b) * k_out;
  if (fault && *fault) {
    // the producer of the candidates reported a fault: no result (with a global gather
    // buffer the decode pass reports it)
    if (gather_g) return;
    for (int32_t j = tid; j < k_out; j += blockDim.x) {
      if (out_s) out_s[ob + j] = __int_as_float(0x7fc00000);
      if (out_i) out_i[ob + j] = -1;
      if (out_k) out_k[ob + j] = 0ull;
    }
    return;
  }
  Lists L;
  L.use_param = use_param != 0;
  L.counts_dev = counts_dev;
  L.cstride_b = cstride_b;
  L.stride_r = stride_r;
  L.b = b;
  L.base = keys + int64_t(b) * stride_b;
  L.n = R;
  if (tree_groups > 0) {
    // one level of a merge tree: row b merges lists g*R .. g*R+R-1 (those that exist) of
    // the tree_n_in lists of its query, stored one after another
    const int32_t g = b % tree_groups;
    L.base = keys + (int64_t(b / tree_groups) * tree_n_in + int64_t(g) * R) * stride_r;
    L.n = min(R, tree_n_in - g * R);
  }

  int32_t part = 0;
  for (int32_t r = tid; r < L.n; r += blockDim.x) part += L.count(r, cp);
  for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(FULL, part, o);
  if (lane == 0) s_part[wid] = part;
  __syncthreads();
  if (tid == 0) {
    int32_t tot = 0;
    for (int w = 0; w < kMergeThreads / 32; ++w) tot += s_part[w];
    s_total = tot;
    s_n = 0;
  }
  __syncthreads();
  const int32_t total = s_total;
  const int32_t kk = min(k, total);

  uint64_t prefix = 0;
  if (kk > 0 && kk < total) {
    int32_t need = kk;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int j = tid; j < 256; j += blockDim.x) hist[j] = 0u;
      __syncthreads();
      const uint64_t pmask = shift == 56 ? 0ull : (~0ull << (shift + 8));
      for (int32_t r = 0; r < L.n; ++r) {
        const int32_t cnt = L.count(r, cp);
        const uint64_t* __restrict__ kr = L.list(r);
        for (int32_t i0 = 0; i0 < cnt; i0 += blockDim.x) {
          const int32_t i = i0 + tid;
          const uint64_t key = i < cnt ? kr[i] : 0ull;
          const bool live = i < cnt && (key & pmask) == prefix;
          const uint32_t dig = live ? uint32_t((key >> shift) & 255u) : 0x100u;
          const uint32_t peers = __match_any_sync(FULL, dig);
          if (live && (peers & lanemask_lt()) == 0u) atomicAdd(&hist[dig], uint32_t(__popc(peers)));
        }
      }
      __syncthreads();
      if (wid == 0) {
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
        if (lane == L) {
          int32_t above = incl - s;
          for (int j = 0; j < 8; ++j) {
            const int bin = 255 - 8 * lane - j;
            const int32_t c = int32_t(hist[bin]);
            if (above + c >= need) {
              s_D = bin;
              s_cD = c;
              s_above = above;
              break;
            }
            above += c;
          }
        }
      }
      __syncthreads();
      need -= s_above;
      prefix |= uint64_t(s_D) << shift;
      const bool done = s_cD == need;
      __syncthreads();
      if (done) break;
    }
  }

  // gather the kk keys >= prefix (all keys when kk == total)
  for (int32_t r = 0; r < L.n && kk > 0; ++r) {
    const int32_t cnt = L.count(r, cp);
    const uint64_t* __restrict__ kr = L.list(r);
    for (int32_t i0 = 0; i0 < cnt; i0 += blockDim.x) {
      const int32_t i = i0 + tid;
      const uint64_t key = i < cnt ? kr[i] : 0ull;
      const bool keep = i < cnt && key >= prefix;
      const uint32_t bal = __ballot_sync(FULL, keep);
      int32_t base = 0;
      if (lane == 0 && bal) base = atomicAdd(&s_n, __popc(bal));
      base = __shfl_sync(FULL, base, 0);
      if (keep) {
        const int32_t slot = base + __popc(bal & lanemask_lt());
        if (gather_g) {
          if (slot < k) gather_g[int64_t(b) * k + slot] = key;
        } else if (slot < kpow2) {
          sk[slot] = key;
        }
      }
    }
  }
  __syncthreads();
  if (gather_g) {
    // large k: the kk keys stay unsorted in the global buffer, zeros after them
    for (int32_t j = min(s_n, k) + tid; j < k; j += blockDim.x) gather_g[int64_t(b) * k + j] = 0ull;
    return;
  }
  const int32_t n = min(s_n, kpow2);
  for (int32_t i = n + tid; i < kpow2; i += blockDim.x) sk[i] = 0ull;
  __syncthreads();
  // bitonic sort, descending (an inner level of a merge tree passes its keys on unsorted)
  const bool sort = out_s != nullptr || out_i != nullptr || tree_groups == 0;
  for (int32_t size = 2; sort && size <= kpow2; size <<= 1) {
    for (int32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (int32_t i = tid; i < kpow2; i += blockDim.x) {
        const int32_t j = i ^ stride;
        if (j > i) {
          const uint64_t a = sk[i], c = sk[j];
          const bool desc = (i & size) == 0;
          if ((a < c) == desc) {
            sk[i] = c;
            sk[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int32_t j = tid; j < k_out; j += blockDim.x) {
    // key 0 is no document (an unused slot of a candidate list): a pad like a missing one
    const uint64_t key = (j < kk && j < n) ? sk[j] : 0ull;
    if (key != 0ull) {
      if (out_s) out_s[ob + j] = key_score(key);
      if (out_i) out_i[ob + j] = int64_t(key_doc(key));
    } else {
      if (out_s) out_s[ob + j] = -INFINITY;
      if (out_i) out_i[ob + j] = pad_id;
    }
    if (out_k) out_k[ob + j] = key;
  }
}

// keys of the entries >= tau[b] of a dense score row, compacted per row (order within a
// row is irrelevant: the merge sorts them)
__global__ void compact_rows_kernel(const float* __restrict__ scores, int64_t L, int64_t stride,
                                    const float* __restrict__ tau, uint64_t* __restrict__ out,
                                    int32_t* __restrict__ counts) {
  const int64_t b = blockIdx.y;
  const float t = tau[b];
  const float* __restrict__ row = scores + b * stride;
  uint64_t* __restrict__ o = out + b * L;
  const int lane = lane_id();
  for (int64_t i0 = int64_t(blockIdx.x) * blockDim.x; i0 < L; i0 += int64_t(gridDim.x) * blockDim.x) {
    const int64_t i = i0 + threadIdx.x;
    const float s = i < L ? row[i] : 0.0f;
    const bool keep = i < L && s >= t;
    const uint32_t bal = __ballot_sync(FULL, keep);
    int32_t base = 0;
    if (lane == 0 && bal) base = atomicAdd(counts + b, __popc(bal));
    base = __shfl_sync(FULL, base, 0);
    if (keep) o[base + __popc(bal & lanemask_lt())] = pack_key(s, uint32_t(i));
  }
}

// Large k: each run of kRun keys of a row (rows of k keys) sorted descending in shared
// memory; the row's tail past k is padded with zeros, which sort last and are not stored.
__global__ void __launch_bounds__(kRunThreads)
sort_runs_kernel(uint64_t* __restrict__ keys, int64_t k) {
  __shared__ uint64_t s[kRun];
  const int64_t row = blockIdx.y;
  const int64_t r0 = int64_t(blockIdx.x) * kRun;
  const int32_t n = int32_t(min64(int64_t(kRun), k - r0));
  uint64_t* __restrict__ g = keys + row * k + r0;
  for (int32_t i = threadIdx.x; i < kRun; i += blockDim.x) s[i] = i < n ? g[i] : 0ull;
  __syncthreads();
  for (int32_t size = 2; size <= kRun; size <<= 1) {
    for (int32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (int32_t i = threadIdx.x; i < kRun; i += blockDim.x) {
        const int32_t j = i ^ stride;
        if (j > i) {
          const uint64_t a = s[i], c = s[j];
          const bool desc = (i & size) == 0;
          if ((a < c) == desc) {
            s[i] = c;
            s[j] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int32_t i = threadIdx.x; i < n; i += blockDim.x) g[i] = s[i];
}

// Large k: one merge pass.  Every row of k keys consists of descending runs of L keys (the
// last one possibly shorter); each pair of runs becomes one descending run of 2L keys in
// dst.  A thread writes kMergeOut consecutive outputs: it finds how many of them come from
// the first run by a binary search along its merge-path diagonal, then merges.  Keys of a
// row are distinct except for zero padding, so the split is unique.
__global__ void __launch_bounds__(kMergePassThreads)
merge_pass_kernel(const uint64_t* __restrict__ src, uint64_t* __restrict__ dst, int64_t k, int64_t L) {
  const int64_t row = blockIdx.y;
  const int64_t o0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * kMergeOut;
  if (o0 >= k) return;
  const uint64_t* __restrict__ s = src + row * k;
  uint64_t* __restrict__ d = dst + row * k;
  const int64_t pbase = (o0 / (2 * L)) * (2 * L);
  const int64_t lenA = min64(L, k - pbase);
  const int64_t lenB = lenA < L ? 0 : min64(L, k - pbase - L);
  const uint64_t* __restrict__ A = s + pbase;
  const uint64_t* __restrict__ Bv = A + lenA;
  const int64_t diag = o0 - pbase;
  // i = how many of the first `diag` outputs come from A
  int64_t lo = diag > lenB ? diag - lenB : 0, hi = min64(diag, lenA);
  while (lo < hi) {
    const int64_t mid = (lo + hi) >> 1;
    if (A[mid] > Bv[diag - 1 - mid]) lo = mid + 1; else hi = mid;
  }
  int64_t i = lo, j = diag - lo;
  const int64_t end = min64(o0 + kMergeOut, pbase + lenA + lenB);
  for (int64_t o = o0; o < end; ++o) {
    const bool take_a = i < lenA && (j >= lenB || A[i] > Bv[j]);
    d[o] = take_a ? A[i++] : Bv[j++];
  }
}

// Large k: sorted keys -> (score, doc id) and optionally the keys; key 0 is no document.
__global__ void decode_keys_kernel(const uint64_t* __restrict__ keys, int64_t B, int64_t k,
                                   const int32_t* __restrict__ fault, int64_t pad_id,
                                   float* __restrict__ out_s, int64_t* __restrict__ out_i,
                                   uint64_t* __restrict__ out_k) {
  const int64_t n = B * k;
  const bool bad = fault && *fault;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n; e += int64_t(gridDim.x) * blockDim.x) {
    const uint64_t key = bad ? 0ull : keys[e];
    if (bad) {
      if (out_s) out_s[e] = __int_as_float(0x7fc00000);
      if (out_i) out_i[e] = -1;
    } else if (key != 0ull) {
      if (out_s) out_s[e] = key_score(key);
      if (out_i) out_i[e] = int64_t(key_doc(key));
    } else {
      if (out_s) out_s[e] = -INFINITY;
      if (out_i) out_i[e] = pad_id;
    }
    if (out_k) out_k[e] = key;
  }
}

}  // namespace

int64_t large_k_ws_bytes(int64_t B, int64_t k) {
  if (k <= kMaxK) return 0;
  return 2 * (((B * k * 8) + 255) / 256) * 256;
}

int merge_topk_device(const uint64_t* keys, int64_t B, int64_t R, int64_t stride_b, int64_t stride_r,
                      const int32_t* counts_dev, int64_t cstride_b, const int32_t* counts_host,
                      int64_t k, float* out_scores, int64_t* out_ids, uint64_t* out_keys,
                      cudaStream_t st, int64_t pad_id, const int32_t* fault, void* large_ws) {
  GSP_REQUIRE(B >= 0 && R >= 1 && k >= 0, GSP_ERR_ARG, "merge: bad arguments");
  GSP_REQUIRE(k <= kMaxK || large_ws, GSP_ERR_ARG,
              "merge: k %lld above %d needs a workspace of large_k_ws_bytes", (long long)k, kMaxK);
  GSP_REQUIRE(k <= 0x7FFFFFFF && B * k <= (int64_t(1) << 40), GSP_ERR_UNSUPPORTED,
              "merge: B x k = %lld x %lld is too large", (long long)B, (long long)k);
  GSP_REQUIRE(R <= 0x7FFFFFFF, GSP_ERR_ARG, "merge: too many lists");
  if (B == 0 || k == 0) return GSP_OK;
  CountsParam cp{};
  int use_param = 0;
  if (counts_host) {
    GSP_REQUIRE(R <= kMaxParamCounts, GSP_ERR_UNSUPPORTED, "merge: at most %d host-counted lists",
                kMaxParamCounts);
    for (int64_t r = 0; r < R; ++r) cp.c[r] = counts_host[r];
    use_param = 1;
  }
  if (k > kMaxK) {
    // gather each query's k keys into the workspace, sort runs, merge passes, decode
    GSP_REQUIRE(B <= 65535, GSP_ERR_UNSUPPORTED, "merge: at most 65535 queries per call above k = %d",
                kMaxK);
    uint64_t* buf[2] = {static_cast<uint64_t*>(large_ws),
                        reinterpret_cast<uint64_t*>(static_cast<char*>(large_ws) + large_k_ws_bytes(B, k) / 2)};
    merge_kernel<<<unsigned(B), kMergeThreads, 0, st>>>(keys, stride_b, stride_r, int32_t(R), fault, counts_dev,
                                                        cstride_b, cp, use_param, int32_t(k), int32_t(k), 0,
                                                        pad_id, nullptr, nullptr, nullptr, 0, 0, buf[0]);
    GSP_CHECK_LAUNCH();
    const int64_t runs = (k + kRun - 1) / kRun;
    sort_runs_kernel<<<dim3(unsigned(runs), unsigned(B)), kRunThreads, 0, st>>>(buf[0], k);
    GSP_CHECK_LAUNCH();
    int cur = 0;
    const int64_t per_cta = int64_t(kMergePassThreads) * kMergeOut;
    for (int64_t L = kRun; L < k; L *= 2) {
      merge_pass_kernel<<<dim3(unsigned((k + per_cta - 1) / per_cta), unsigned(B)), kMergePassThreads, 0, st>>>(
          buf[cur], buf[cur ^ 1], k, L);
      GSP_CHECK_LAUNCH();
      cur ^= 1;
    }
    const int64_t n = B * k;
    const unsigned grid = unsigned(std::min<int64_t>((n + 255) / 256, int64_t(num_sms()) * 16));
    decode_keys_kernel<<<grid, 256, 0, st>>>(buf[cur], B, k, fault, pad_id, out_scores, out_ids, out_keys);
    GSP_CHECK_LAUNCH();
    return GSP_OK;
  }
  int32_t kpow2 = 1;
  while (kpow2 < k) kpow2 <<= 1;
  const size_t smem = size_t(kpow2) * 8;
  if (int rc = ensure_smem(reinterpret_cast<const void*>(merge_kernel), int(smem))) return rc;
  merge_kernel<<<unsigned(B), kMergeThreads, smem, st>>>(keys, stride_b, stride_r, int32_t(R), fault,
                                                         counts_dev, cstride_b, cp, use_param, int32_t(k),
                                                         int32_t(k), kpow2, pad_id, out_scores, out_ids,
                                                         out_keys, 0, 0, nullptr);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

int merge_tree_level(const uint64_t* lists, int64_t B, int32_t n_in, int32_t slots, int64_t k,
                     float* out_scores, int64_t* out_ids, uint64_t* out_keys, cudaStream_t st,
                     int64_t pad_id) {
  constexpr int32_t R = kTreeFanIn;
  static_assert(kTreeFanIn <= kMaxParamCounts, "tree fan-in above the parameter counts");
  GSP_REQUIRE(B >= 0 && n_in >= 1 && slots >= 1 && k >= 1 && k <= kMaxK, GSP_ERR_ARG,
              "merge tree: bad arguments");
  const int32_t groups = (n_in + R - 1) / R;
  const int64_t rows = B * groups;
  GSP_REQUIRE(rows <= 0x7FFFFFFF, GSP_ERR_UNSUPPORTED, "merge tree: too many lists");
  if (rows == 0) return GSP_OK;
  CountsParam cp{};
  for (int r = 0; r < R; ++r) cp.c[r] = slots;
  int32_t kpow2 = 1;
  while (kpow2 < k) kpow2 <<= 1;
  const size_t smem = size_t(kpow2) * 8;
  if (int rc = ensure_smem(reinterpret_cast<const void*>(merge_kernel), int(smem))) return rc;
  merge_kernel<<<unsigned(rows), kMergeThreads, smem, st>>>(lists, 0, slots, R, nullptr, nullptr, 0, cp, 1,
                                                            int32_t(k), int32_t(k), kpow2, pad_id, out_scores,
                                                            out_ids, out_keys, groups, n_in, nullptr);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

}  // namespace gsp

using namespace gsp;

extern "C" int64_t gsp_merge_ws_bytes(int64_t B, int64_t k) {
  if (B < 0 || k < 0) return -int64_t(GSP_ERR_ARG);
  return large_k_ws_bytes(B, k);
}

extern "C" int gsp_merge_topk(const uint64_t* keys, int64_t B, int64_t R, int64_t stride_b,
                              int64_t stride_r, const int32_t* counts_host, int64_t k, float* out_scores,
                              int64_t* out_ids, uint64_t* out_keys, void* ws, int64_t ws_bytes,
                              void* stream) {
  GSP_REQUIRE(keys && counts_host && out_scores && out_ids, GSP_ERR_ARG, "gsp_merge_topk: null argument");
  int64_t total = 0;
  for (int64_t r = 0; r < R; ++r) {
    GSP_REQUIRE(counts_host[r] >= 0, GSP_ERR_ARG,
                "gsp_merge_topk: count %d of list %lld out of range", counts_host[r], (long long)r);
    total += counts_host[r];
  }
  GSP_REQUIRE(k <= total, GSP_ERR_ARG, "gsp_merge_topk: k %lld exceeds the %lld candidates", (long long)k,
              (long long)total);
  GSP_REQUIRE(ws_bytes >= large_k_ws_bytes(B, k) && (ws || large_k_ws_bytes(B, k) == 0), GSP_ERR_ARG,
              "gsp_merge_topk: workspace too small (%lld < %lld)", (long long)ws_bytes,
              (long long)large_k_ws_bytes(B, k));
  return merge_topk_device(keys, B, R, stride_b, stride_r, nullptr, 0, counts_host, k, out_scores,
                           out_ids, out_keys, as_stream(stream), -1, nullptr, ws);
}

static int64_t compacted_keys_bytes(int64_t B, int64_t L) { return ((B * L * 8 + 255) / 256) * 256; }
static int64_t compacted_counts_bytes(int64_t B) { return ((B * 4 + 255) / 256) * 256; }

extern "C" int64_t gsp_compacted_ws_bytes(int64_t B, int64_t L, int64_t k, int64_t max_cand) {
  (void)max_cand;
  if (B < 0 || L < 0 || k < 0) return -1;
  return compacted_keys_bytes(B, L) + compacted_counts_bytes(B) + large_k_ws_bytes(B, std::min(k, L));
}

extern "C" int gsp_compacted_topk(const float* scores, int64_t B, int64_t L, int64_t stride,
                                  const float* tau, int64_t k, int64_t max_cand, float* out_v,
                                  int64_t* out_i, void* ws, int64_t ws_bytes, void* stream) {
  GSP_REQUIRE(B >= 0 && L >= 0 && stride >= L && k >= 0 && max_cand >= 0, GSP_ERR_ARG,
              "gsp_compacted_topk: bad arguments");
  GSP_REQUIRE(ws_bytes >= gsp_compacted_ws_bytes(B, L, k, max_cand), GSP_ERR_ARG,
              "gsp_compacted_topk: workspace too small");
  const int64_t kk = std::min(k, L);
  if (B == 0 || kk == 0) return GSP_OK;
  GSP_REQUIRE(L <= 0x7FFFFFFFll, GSP_ERR_UNSUPPORTED, "gsp_compacted_topk: row too long");
  cudaStream_t st = as_stream(stream);
  char* w = static_cast<char*>(ws);
  uint64_t* keys = reinterpret_cast<uint64_t*>(w);
  int32_t* counts = reinterpret_cast<int32_t*>(w + compacted_keys_bytes(B, L));
  void* large = w + compacted_keys_bytes(B, L) + compacted_counts_bytes(B);
  GSP_CUDA(cudaMemsetAsync(counts, 0, size_t(B) * 4, st));
  const int64_t per = 256;
  int64_t gx = std::min<int64_t>((L + per - 1) / per, 1024);
  GSP_REQUIRE(B <= 65535, GSP_ERR_UNSUPPORTED, "gsp_compacted_topk: at most 65535 rows per call");
  compact_rows_kernel<<<dim3(unsigned(gx), unsigned(B)), unsigned(per), 0, st>>>(scores, L, stride, tau,
                                                                                keys, counts);
  GSP_CHECK_LAUNCH();
  return merge_topk_device(keys, B, 1, L, L, counts, 1, nullptr, kk, out_v, out_i, nullptr, st, 0, nullptr,
                           large);
}
