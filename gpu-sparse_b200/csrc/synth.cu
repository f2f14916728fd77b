// Seeded synthetic SPLADE-shaped documents / queries generated on the GPU.
//
// The law (the benchmark configs' stand-in for MS MARCO SPLADE): term ids follow a Zipf
// law over the vocabulary (rank r <-> id r-1), each item's number of distinct terms is a
// clipped, rounded log-normal, the distinct terms are drawn by successive sampling
// (i.i.d. Zipf draws, first occurrences kept -- the same law as sampling without
// replacement), and weights are log1p(relu(N(mu, sd))).  All randomness comes from a
// counter-based SplitMix64 stream keyed by (seed, stream, item, counter), so any item
// range can be generated independently (one shard per GPU) and every floating-point step
// is an explicitly rounded IEEE operation: the CPU generator in the test oracle produces
// byte-identical CSR matrices.
#include "common.cuh"

namespace gsp {
namespace {

constexpr int kWtabSegs = 65536;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t item_key(uint64_t seed, uint32_t stream, uint64_t item) {
  uint64_t z = mix64(seed ^ (0x9E3779B97F4A7C15ULL * uint64_t(stream + 1)));
  return mix64(z ^ (item * 0xD1B54A32D192ED03ULL));
}
__device__ __forceinline__ uint64_t draw64(uint64_t key, uint64_t ctr) {
  return mix64(key + (ctr + 1) * 0x9E3779B97F4A7C15ULL);
}
__device__ __forceinline__ double u53(uint64_t x) {
  return __dmul_rn(__ull2double_rn(x >> 11), 1.0 / 9007199254740992.0);
}
// first i in [0, n) with cdf[i] > u
__device__ __forceinline__ int32_t upper_idx(const double* __restrict__ cdf, int32_t n, double u) {
  int32_t lo = 0, hi = n - 1;
  while (lo < hi) {
    int32_t mid = lo + ((hi - lo) >> 1);
    if (__ldg(cdf + mid) > u) hi = mid; else lo = mid + 1;
  }
  return lo;
}
// same answer as upper_idx over the whole table, searched inside the guide interval
// [guide[j], guide[j+1]] of u's 1/65536 slice (guide[j] = upper_idx(j / 65536))
constexpr int kGuide = 65536;
__device__ __forceinline__ int32_t upper_idx_guided(const double* __restrict__ cdf,
                                                    const int32_t* __restrict__ guide, double u) {
  const int32_t j = int32_t(__dmul_rn(u, double(kGuide)));
  int32_t lo = __ldg(guide + j), hi = __ldg(guide + j + 1);
  while (lo < hi) {
    int32_t mid = lo + ((hi - lo) >> 1);
    if (__ldg(cdf + mid) > u) hi = mid; else lo = mid + 1;
  }
  return lo;
}
__device__ __forceinline__ float weight_of(uint64_t x, const double* __restrict__ wtab) {
  double u = u53(x);
  double s = __dmul_rn(u, double(kWtabSegs));
  int32_t i = int32_t(s);
  double f = __dsub_rn(s, double(i));
  double a = __ldg(wtab + i), b = __ldg(wtab + i + 1);
  double w = __dadd_rn(a, __dmul_rn(f, __dsub_rn(b, a)));
  return __double2float_rn(w);
}

__global__ void synth_nnz_kernel(uint64_t seed, uint32_t kind, uint64_t first, int64_t n, int32_t V,
                                 const double* __restrict__ nnz_cdf, int32_t n_nnz, int32_t nnz_lo,
                                 int32_t min0, int32_t* __restrict__ out) {
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint64_t item = first + uint64_t(i);
  double u = u53(draw64(item_key(seed, 3u * kind, item), 0));
  int32_t k = nnz_lo + upper_idx(nnz_cdf, n_nnz, u);
  if (item == 0 && k < min0) k = min0;
  if (k > V) k = V;
  out[i] = k;
}

constexpr int kFillWarps = 8;

// One warp per item; a V-bit "already drawn" bitmap per warp in shared memory.
__global__ void __launch_bounds__(kFillWarps * 32)
synth_fill_kernel(uint64_t seed, uint32_t kind, uint64_t first, int64_t n, int32_t V,
                  const double* __restrict__ term_cdf, const int32_t* __restrict__ guide,
                  const double* __restrict__ wtab, const int64_t* __restrict__ indptr,
                  int32_t* __restrict__ indices,
                  float* __restrict__ data) {
  extern __shared__ uint32_t smem_bits[];
  const int lane = lane_id(), wid = threadIdx.x >> 5;
  const int32_t nwords = (V + 31) >> 5;
  uint32_t* bits = smem_bits + int64_t(wid) * nwords;
  for (int32_t w = lane; w < nwords; w += 32) bits[w] = 0u;
  __syncwarp();
  const int64_t stride = int64_t(gridDim.x) * kFillWarps;
  for (int64_t i = int64_t(blockIdx.x) * kFillWarps + wid; i < n; i += stride) {
    const uint64_t item = first + uint64_t(i);
    const int64_t p0 = indptr[i];
    const int32_t need = int32_t(indptr[i + 1] - p0);
    const uint64_t tkey = item_key(seed, 3u * kind + 1u, item);
    const uint64_t wkey = item_key(seed, 3u * kind + 2u, item);
    int32_t got = 0;
    const int64_t cap = 64 * int64_t(need) + 4096;
    for (int64_t c = 0; c < cap && got < need; c += 32) {
      const int64_t j = c + lane;
      int32_t t = -1;
      bool live = j < cap;
      if (live) t = upper_idx_guided(term_cdf, guide, u53(draw64(tkey, uint64_t(j))));
      // first occurrence within this batch of 32 draws, in draw order
      const uint32_t live_mask = __ballot_sync(FULL, live);
      const uint32_t peers = __match_any_sync(FULL, t);
      const bool first_in_batch = live && ((peers & live_mask & lanemask_lt()) == 0u);
      const bool seen = live && ((bits[t >> 5] >> (t & 31)) & 1u);
      const bool fresh = first_in_batch && !seen;
      const uint32_t bal = __ballot_sync(FULL, fresh);
      const int32_t rank = __popc(bal & lanemask_lt());
      const bool take = fresh && (got + rank < need);
      if (take) {
        indices[p0 + got + rank] = t;
        atomicOr(&bits[t >> 5], 1u << (t & 31));
      }
      got += min(__popc(bal), need - got);
      __syncwarp();
    }
    if (got < need && lane == 0) {
      // deterministic completion when the draw cap was hit: smallest unused ids
      for (int32_t t = 0; got < need && t < V; ++t) {
        if (!((bits[t >> 5] >> (t & 31)) & 1u)) {
          bits[t >> 5] |= 1u << (t & 31);
          indices[p0 + got] = t;
          ++got;
        }
      }
    }
    __syncwarp();
    for (int32_t s = lane; s < need; s += 32) {
      data[p0 + s] = weight_of(draw64(wkey, uint64_t(s)), wtab);
      const int32_t t = indices[p0 + s];
      atomicAnd(&bits[t >> 5], ~(1u << (t & 31)));
    }
    __syncwarp();
  }
}

}  // namespace
}  // namespace gsp

using namespace gsp;

extern "C" int gsp_synth_nnz(uint64_t seed, uint32_t kind, uint64_t first, int64_t n, int32_t V,
                             const double* nnz_cdf, int32_t n_nnz, int32_t nnz_lo,
                             int32_t min_nnz_item0, int32_t* nnz, void* stream) {
  GSP_REQUIRE(n >= 0 && V > 0 && n_nnz > 0 && nnz_cdf && (nnz || n == 0) && kind <= 1,
              GSP_ERR_ARG, "gsp_synth_nnz: bad arguments");
  if (n == 0) return GSP_OK;
  const int threads = 256;
  synth_nnz_kernel<<<unsigned((n + threads - 1) / threads), threads, 0, as_stream(stream)>>>(
      seed, kind, first, n, V, nnz_cdf, n_nnz, nnz_lo, min_nnz_item0, nnz);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

extern "C" int gsp_synth_fill(uint64_t seed, uint32_t kind, uint64_t first, int64_t n, int32_t V,
                              const double* term_cdf, const int32_t* term_guide, const double* wtab,
                              const int64_t* indptr, int32_t* indices, float* data, void* stream) {
  GSP_REQUIRE(n >= 0 && V > 0 && term_cdf && term_guide && wtab && indptr && kind <= 1, GSP_ERR_ARG,
              "gsp_synth_fill: bad arguments");
  if (n == 0) return GSP_OK;
  const size_t smem = size_t(kFillWarps) * ((V + 31) / 32) * sizeof(uint32_t);
  GSP_REQUIRE(smem <= size_t(max_smem_optin()), GSP_ERR_UNSUPPORTED,
              "gsp_synth_fill: vocabulary %d too large for the shared-memory bitmap", V);
  GSP_CUDA(cudaFuncSetAttribute(synth_fill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(smem)));
  int64_t blocks = (n + kFillWarps - 1) / kFillWarps;
  const int64_t max_blocks = int64_t(num_sms()) * 16;
  if (blocks > max_blocks) blocks = max_blocks;
  synth_fill_kernel<<<unsigned(blocks), kFillWarps * 32, smem, as_stream(stream)>>>(
      seed, kind, first, n, V, term_cdf, term_guide, wtab, indptr, indices, data);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}
