// Error reporting, device queries and a device-wide exclusive scan (int32 -> int64).
#include "common.cuh"

#include <map>
#include <mutex>
#include <utility>

#include <string.h>

namespace gsp {

static thread_local char g_err[1024] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int num_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return n;
}

// Raises a kernel's dynamic shared-memory limit only when a launch needs more than was set
// before on this device, so repeated calls (and calls inside a stream capture, after a
// first call outside it) make no attribute call.
int ensure_smem(const void* func, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> done;
  int dev = 0;
  GSP_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> g(mu);
  int& cur = done[{dev, func}];
  if (bytes > cur) {
    GSP_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    cur = bytes;
  }
  return GSP_OK;
}

int max_smem_optin() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 227 * 1024;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return 227 * 1024;
  return n;
}

// ---- scan -----------------------------------------------------------------------------
constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;  // per thread
constexpr int kScanTile = kScanThreads * kScanItems;

__device__ __forceinline__ int64_t block_excl_scan(int64_t v, int64_t* sh, int64_t* total) {
  // warp inclusive scan
  int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int64_t y = __shfl_up_sync(FULL, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sh[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int64_t s = (lane < (int)(blockDim.x >> 5)) ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int64_t y = __shfl_up_sync(FULL, s, o);
      if (lane >= o) s += y;
    }
    sh[lane] = s;  // inclusive warp totals
  }
  __syncthreads();
  int64_t base = wid ? sh[wid - 1] : 0;
  *total = sh[(blockDim.x >> 5) - 1];
  __syncthreads();
  return base + x - v;
}

__global__ void scan_tiles(const int32_t* in, int64_t n, int64_t* out, int64_t* tile_sums) {
  __shared__ int64_t sh[32];
  int64_t t0 = int64_t(blockIdx.x) * kScanTile;
  int64_t v[kScanItems];
  int64_t s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    int64_t j = t0 + int64_t(threadIdx.x) * kScanItems + i;
    v[i] = j < n ? int64_t(in[j]) : 0;
    s += v[i];
  }
  int64_t total;
  int64_t pre = block_excl_scan(s, sh, &total);
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    int64_t j = t0 + int64_t(threadIdx.x) * kScanItems + i;
    if (j < n) out[j] = pre;
    pre += v[i];
  }
  if (threadIdx.x == 0) tile_sums[blockIdx.x] = total;
}

__global__ void scan_sums(int64_t* tile_sums, int64_t n_tiles, int64_t* out, int64_t n) {
  __shared__ int64_t sh[32];
  int64_t carry = 0;
  for (int64_t b = 0; b < n_tiles; b += blockDim.x) {
    int64_t j = b + threadIdx.x;
    int64_t v = j < n_tiles ? tile_sums[j] : 0;
    int64_t total;
    int64_t pre = block_excl_scan(v, sh, &total);
    if (j < n_tiles) tile_sums[j] = carry + pre;
    carry += total;
  }
  if (threadIdx.x == 0) out[n] = carry;
}

__global__ void scan_add(int64_t* out, int64_t n, const int64_t* tile_sums) {
  int64_t j = int64_t(blockIdx.x) * kScanTile + threadIdx.x;
  int64_t add = tile_sums[blockIdx.x];
  for (int i = 0; i < kScanItems; ++i, j += kScanThreads)
    if (j < n) out[j] += add;
}

}  // namespace gsp

using namespace gsp;

extern "C" const char* gsp_last_error(void) { return g_err; }
extern "C" int gsp_version(void) { return 1; }

extern "C" int64_t gsp_scan_ws_bytes(int64_t n) {
  return ((n + kScanTile - 1) / kScanTile + 1) * int64_t(sizeof(int64_t));
}

extern "C" int gsp_scan_i32(const int32_t* in, int64_t n, int64_t* out, void* ws, int64_t ws_bytes,
                            void* stream) {
  GSP_REQUIRE(n >= 0 && out, GSP_ERR_ARG, "gsp_scan_i32: bad arguments");
  GSP_REQUIRE(ws_bytes >= gsp_scan_ws_bytes(n), GSP_ERR_ARG, "gsp_scan_i32: workspace too small");
  cudaStream_t st = as_stream(stream);
  if (n == 0) {
    GSP_CUDA(cudaMemsetAsync(out, 0, sizeof(int64_t), st));
    return GSP_OK;
  }
  int64_t tiles = (n + kScanTile - 1) / kScanTile;
  int64_t* sums = static_cast<int64_t*>(ws);
  scan_tiles<<<unsigned(tiles), kScanThreads, 0, st>>>(in, n, out, sums);
  GSP_CHECK_LAUNCH();
  scan_sums<<<1, kScanThreads, 0, st>>>(sums, tiles, out, n);
  GSP_CHECK_LAUNCH();
  scan_add<<<unsigned(tiles), kScanThreads, 0, st>>>(out, n, sums);
  GSP_CHECK_LAUNCH();
  return GSP_OK;
}

// ---------------------------------------------------------------------------------------
// Threshold boards: one uint64 key per query that other processes (the other doc-range
// shards of a batch, one per GPU) raise through CUDA IPC mappings of it.  Allocated with
// cudaMalloc so that the IPC handle covers exactly the board.
extern "C" int gsp_board_alloc(int64_t n, uint64_t** board, void* ipc_handle) {
  GSP_REQUIRE(n > 0 && board, GSP_ERR_ARG, "gsp_board_alloc: bad arguments");
  void* p = nullptr;
  GSP_CUDA(cudaMalloc(&p, size_t(n) * sizeof(uint64_t)));
  if (cudaMemset(p, 0, size_t(n) * sizeof(uint64_t)) != cudaSuccess) {
    cudaFree(p);
    set_error("gsp_board_alloc: cudaMemset failed");
    return GSP_ERR_CUDA;
  }
  if (ipc_handle) {
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
      cudaFree(p);
      set_error("gsp_board_alloc: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
      return GSP_ERR_CUDA;
    }
    static_assert(sizeof(h) == GSP_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(ipc_handle, &h, sizeof(h));
  }
  *board = static_cast<uint64_t*>(p);
  return GSP_OK;
}

extern "C" int gsp_board_free(uint64_t* board) {
  GSP_REQUIRE(board, GSP_ERR_ARG, "gsp_board_free: null board");
  GSP_CUDA(cudaFree(board));
  return GSP_OK;
}

extern "C" int gsp_board_open(const void* ipc_handle, uint64_t** board) {
  GSP_REQUIRE(ipc_handle && board, GSP_ERR_ARG, "gsp_board_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  GSP_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *board = static_cast<uint64_t*>(p);
  return GSP_OK;
}

extern "C" int gsp_board_close(uint64_t* board) {
  GSP_REQUIRE(board, GSP_ERR_ARG, "gsp_board_close: null board");
  GSP_CUDA(cudaIpcCloseMemHandle(board));
  return GSP_OK;
}

extern "C" int gsp_board_clear(uint64_t* board, int64_t n, void* stream) {
  GSP_REQUIRE(board && n >= 0, GSP_ERR_ARG, "gsp_board_clear: bad arguments");
  GSP_CUDA(cudaMemsetAsync(board, 0, size_t(n) * sizeof(uint64_t), as_stream(stream)));
  return GSP_OK;
}
