// Shared device helpers and error plumbing for libgpusparse (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/gpusparse.h"

namespace gsp {

constexpr uint32_t FULL = 0xFFFFFFFFu;
constexpr int kPostingPad = 32;   // every posting list is padded to a multiple of 32

void set_error(const char* fmt, ...);

// Returns GSP_ERR_CUDA (and records the message) when a runtime call failed.
#define GSP_CUDA(call)                                                                   \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess) {                                                             \
      ::gsp::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                       __LINE__);                                                        \
      return GSP_ERR_CUDA;                                                               \
    }                                                                                    \
  } while (0)

#define GSP_CHECK_LAUNCH() GSP_CUDA(cudaGetLastError())

#define GSP_REQUIRE(cond, code, ...) \
  do {                               \
    if (!(cond)) {                   \
      ::gsp::set_error(__VA_ARGS__); \
      return (code);                 \
    }                                \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int num_sms();
int max_smem_optin();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) only when `bytes` exceeds what was set
// for this kernel on the current device before.
int ensure_smem(const void* func, int bytes);

// Largest k whose keys one CTA sorts in shared memory; above it the selection sorts in
// global memory and needs a workspace of large_k_ws_bytes(B, k).
constexpr int kMaxSmemK = 8192;
int64_t large_k_ws_bytes(int64_t B, int64_t k);

// Exact top-k over packed candidate lists (select.cu); counts either on the device
// (counts_dev[b * cstride_b + r]) or, for at most 64 lists, on the host.  large_ws:
// large_k_ws_bytes(B, k) bytes of device scratch, needed only when k > kMaxSmemK.
int merge_topk_device(const uint64_t* keys, int64_t B, int64_t R, int64_t stride_b,
                      int64_t stride_r, const int32_t* counts_dev, int64_t cstride_b,
                      const int32_t* counts_host, int64_t k, float* out_scores, int64_t* out_ids,
                      uint64_t* out_keys, cudaStream_t st, int64_t pad_id = -1,
                      const int32_t* fault = nullptr, void* large_ws = nullptr);
// Lists per node of the small-batch merge tree.
#ifndef GSP_TREE_FAN_IN
#define GSP_TREE_FAN_IN 8
#endif
constexpr int kTreeFanIn = GSP_TREE_FAN_IN;

// One level of a merge tree: every group of kTreeFanIn consecutive lists (of `slots` keys
// each, unused slots 0) of each of B queries, n_in lists per query, reduced to its k
// largest keys; the output rows are B x ceil(n_in / kTreeFanIn), in order, k keys each.
int merge_tree_level(const uint64_t* lists, int64_t B, int32_t n_in, int32_t slots, int64_t k,
                     float* out_scores, int64_t* out_ids, uint64_t* out_keys, cudaStream_t st,
                     int64_t pad_id);


// ---- order-preserving float <-> uint32 key (-0 folded onto +0) ----------------------
__host__ __device__ __forceinline__ uint32_t fkey(float f) {
#ifdef __CUDA_ARCH__
  uint32_t b = __float_as_uint(__fadd_rn(f, 0.0f));
#else
  float g = f + 0.0f;
  uint32_t b;
  memcpy(&b, &g, 4);
#endif
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__host__ __device__ __forceinline__ float fkey_inv(uint32_t k) {
  uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
#ifdef __CUDA_ARCH__
  return __uint_as_float(b);
#else
  float f;
  memcpy(&f, &b, 4);
  return f;
#endif
}
// packed candidate: larger = better (higher score, then lower doc id)
__host__ __device__ __forceinline__ uint64_t pack_key(float s, uint32_t doc) {
  return (uint64_t(fkey(s)) << 32) | uint64_t(0xFFFFFFFFu - doc);
}
__host__ __device__ __forceinline__ float key_score(uint64_t k) { return fkey_inv(uint32_t(k >> 32)); }
__host__ __device__ __forceinline__ uint32_t key_doc(uint64_t k) {
  return 0xFFFFFFFFu - uint32_t(k & 0xFFFFFFFFu);
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// ---- weight decode -------------------------------------------------------------------
template <typename WT>
struct WDecode;
template <>
struct WDecode<float> {
  __device__ __forceinline__ static float get(const float* w, int64_t i, float) { return __ldg(w + i); }
};
template <>
struct WDecode<__nv_bfloat16> {
  __device__ __forceinline__ static float get(const __nv_bfloat16* w, int64_t i, float) {
    return __bfloat162float(w[i]);
  }
};
template <>
struct WDecode<uint8_t> {
  // weight = q * scale_t with one fp32 rounding, the dequantised value the oracle uses
  __device__ __forceinline__ static float get(const uint8_t* w, int64_t i, float scale) {
    return __fmul_rn(float(__ldg(w + i)), scale);
  }
};

}  // namespace gsp
