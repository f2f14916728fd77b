// Tensor-core head phase of the scorer (included by score.cu inside its anonymous namespace).
//
// The head terms' contribution to a tile is a dense product: for the 1024 documents d of
// a tile and a batch's queries q, H[d, q] = sum over the H head terms h of row[h][d] *
// Qh[q][h], where row are the index's dense head rows and Qh the queries' head weights.  The
// CUDA-core scorer computes it per (tile, query) work item, re-reading each query's head row
// slices; here one tcgen05.mma chain computes it for a "unit" of 64 queries at once, so a
// row slice is read once per 64 queries:
//   D[128 documents x 64 queries] (fp32, tensor memory) += A[128 x 8] * B[8 x 64] (tf32)
// for each of the tile's 8 slices of 128 documents and every 8 head terms.  fp32 operands
// are split into a tf32 "hi" part (the value itself: the tensor core truncates its low 13
// mantissa bits) and a "lo" part (value - truncation, exact in fp32); hi*hi + hi*lo + lo*hi
// keeps the products to about 2^-21 relative (3xTF32).
//
// CTA layout (one persistent CTA per SM, 32 warps):
//   warp 0  : TMA producer.  Claims units (tile, 64-query group) in tile-major order from a
//             global counter, publishes each unit id, and streams per 16-head-term chunk the
//             query weights Qh (hi, lo: [64 x 16], 64-byte swizzle) and, per 128-document
//             slice, the head rows (hi, lo: [128 x 16], 32-byte-atom 128-byte swizzle).
//   warp 1  : owns the 512 tensor-memory columns (8 slices x 64 queries); one lane issues the
//             MMAs of a unit once the previous unit has been drained, frees each smem stage
//             with tcgen05.commit, and publishes the unit as ready.
//   warps 4..31: seven quads of tail warps (one warp per tensor-memory sub-partition).  A
//             quad claims 4 queries of a ready unit, each warp copies its 32-lane quarter of
//             the 4 queries' accumulators (tcgen05.ld) into the 4 warps' shared-memory tiles,
//             and then every warp scores its query's tail runs and selection exactly as the
//             CUDA-core scorer does (item_tail_select).  A warp can only read the tensor-
//             memory lanes of its own sub-partition, so copying one query's 1024 sums takes
//             four warps: the quad works in step.
// Every wait is bounded; one that runs out sets the fault flag (the merge then reports NaN),
// and every role winds down: in-flight copies and MMAs are waited for (bounded) before the
// tensor memory is released.
//
// Measured on B200 (config 2: 8.8M documents, 1000 queries, k = 1000) this path is slower
// than the CUDA-core head phase (48.2 against 33.7 ms per batch), which is why the automatic
// head mode keeps fp32 on the CUDA cores; see gsp_set_head_mode.  The operand stream is the
// limit: a unit's head rows (hi and lo, 1 MB) arrive through TMA at about 20 bytes per clock
// per SM whatever the number of boxes in flight (about 5.9 TB/s over the GPU, L2-resident or
// not), and tf32 MMAs of N = 64 run at two thirds of the tensor rate, so a unit's MMAs take
// about as long as its 64 tails; the single tensor-memory buffer then serialises the two,
// and the quads wait for their slowest warp.

namespace tc {

constexpr int kThreads = 1024;
constexpr int kFirstQuadWarp = 4;
constexpr int kQuads = 7;
constexpr int kUnitQ = 64;                      // queries per unit (MMA N)
constexpr int kGroups = kUnitQ / 4;             // quad-groups per unit
constexpr int kSlices = kTile / 128;            // MMA M = 128 documents
constexpr int kKC = 16;                         // head terms per chunk
constexpr int kNSA = 4, kNSB = 2;               // stage ring depths
constexpr int kAPiece = 128 * kKC * 4;          // bytes of one A piece (hi or lo)
constexpr int kBPiece = kUnitQ * kKC * 4;       // bytes of one B piece
constexpr int kUQ = 4;                          // ring of published unit ids
constexpr int kTmemCols = 512;                  // kSlices * kUnitQ
static_assert(kSlices * kUnitQ == kTmemCols, "one unit fills the tensor memory");
constexpr int kDrainsPerUnit = kGroups * 4;     // one per warp per quad-group

// dynamic shared memory layout (base aligned to 1024 bytes)
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kNSA * 2 * kAPiece;
constexpr int kOffBar = kOffB + kNSB * 2 * kBPiece;
constexpr int kOffCtl = kOffBar + 256;
constexpr int kOffWarps = kOffCtl + 256;
constexpr int kSmem = kOffWarps + kQuads * 4 * WarpLayout::total;
static_assert(kSmem + 1024 <= 232448, "tensor-core scorer exceeds shared memory");

struct Ctl {
  uint32_t tmem_base;
  int32_t units_published;   // units whose id is in unit_id[]
  int32_t units_ready;       // units whose accumulators are complete in tensor memory
  int32_t drained;           // warp drains (kDrainsPerUnit per unit)
  int32_t gclaim;            // quad-group claims
  int32_t k_end;             // index of the end sentinel (INT_MAX until known)
  int32_t fault;
  int32_t unit_id[kUQ];
  int32_t quad_g[kQuads];
};

// ---- PTX helpers -----------------------------------------------------------------------
__device__ __forceinline__ uint32_t su32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t cnt) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(cnt));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok)
               : "r"(su32(b)), "r"(parity)
               : "memory");
  return ok != 0;
}
// waits for the phase of parity `parity` to complete; false if `limit` polls ran out or the
// CTA has faulted
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, int32_t limit, volatile int32_t* fault) {
  for (int32_t i = 0; i <= limit; ++i) {
    if (mbar_test(b, parity)) return true;
    if ((i & 63) == 63 && *fault) return false;
    __nanosleep(32);
  }
  return false;
}
// the same without the fault check and with a fixed bound of its own (about a second; not
// the caller's wait limit, which may be 0): copies and MMAs already issued must land before
// the CTA exits or releases the tensor memory
constexpr int32_t kLandLimit = 1 << 24;
__device__ __forceinline__ bool mbar_wait_landed(uint64_t* b, uint32_t parity) {
  for (int32_t i = 0; i <= kLandLimit; ++i) {
    if (mbar_test(b, parity)) return true;
    __nanosleep(32);
  }
  return false;
}
// waits until *a >= v; false on timeout or fault
__device__ __forceinline__ bool spin_ge(volatile int32_t* a, int32_t v, int32_t limit, volatile int32_t* fault) {
  for (int32_t i = 0; i <= limit; ++i) {
    if (*a >= v) return true;
    if (*fault) return false;
    __nanosleep(64);
  }
  return false;
}

__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          su32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar)) : "memory");
}
__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}
// 32 lanes x 4 columns: thread t gets lane (base lane + t), columns c .. c+3
__device__ __forceinline__ void tc_ld_x4(uint32_t taddr, float (&v)[4]) {
  uint32_t r0, r1, r2, r3;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(taddr));
  v[0] = __uint_as_float(r0);
  v[1] = __uint_as_float(r1);
  v[2] = __uint_as_float(r2);
  v[3] = __uint_as_float(r3);
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptors (tcgen05 "version 1" format: start address, leading and
// stride byte offsets in 16-byte units, layout type in bits 61..63).
// A: MN-major (documents contiguous), 128-byte rows of 32 documents in 4-row atoms with
//    32-byte swizzle granules (the only MN-major layout tf32 allows); MN atoms of 32
//    documents are kKC * 128 bytes apart (LBO), 4-row K groups 512 bytes apart (SBO).
__device__ __forceinline__ uint64_t desc_a(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t((kKC * 128) >> 4) << 16) | (uint64_t(512 >> 4) << 32) |
         (1ull << 46) | (1ull << 61);
}
// B: K-major (head terms contiguous), 64-byte rows (one query's 16 weights), 64-byte swizzle,
//    8-row groups 512 bytes apart (SBO); a K step of 8 terms advances the start by 32 bytes.
__device__ __forceinline__ uint64_t desc_b(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFF) | (1ull << 16) | (uint64_t(512 >> 4) << 32) | (1ull << 46) | (4ull << 61);
}
// instruction descriptor: fp32 accumulate, tf32 A and B, A MN-major, B K-major, N = 64, M = 128
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (1u << 15) | (0u << 16) |
                            (uint32_t(kUnitQ >> 3) << 17) | (uint32_t(128 >> 4) << 24);

}  // namespace tc

struct TcParams {
  CUtensorMap a_hi, a_lo;      // head rows hi / lo: {32 docs, H terms, ld / 32}, box {32, 16, 4}
  CUtensorMap b_hi, b_lo;      // query head weights hi / lo: {128 terms, queries}, box {16, 64}
  int32_t n_kc;                // 16-term chunks covering the head terms
  int32_t n_groups;            // 64-query units per tile
  int32_t n_units;             // tiles * n_groups
  unsigned long long* unit_next;   // unit claim counter (zeroed)
};

// Dense head weights of every query, split for 3xTF32: hi[q][h] = the fp32 sum of the
// query's weights for head term h (its entries in slot order), lo = hi - trunc_tf32(hi).
// Rows of queries >= B (padding of the last unit) are zero.
__global__ void qhead_kernel(ScoreParams p, int32_t B, int32_t n_head, float* __restrict__ qh,
                             float* __restrict__ qh_lo) {
  const int32_t q = blockIdx.x;
  const int32_t h = threadIdx.x;   // 128 threads
  float v = 0.0f;
  if (q < B && h < n_head) {
    const int64_t pbase = int64_t(q) * p.ecap;
    const int32_t nhe = p.n_head_e[q];
    for (int32_t e = 0; e < nhe; ++e) {
      if (int32_t(p.head_h[pbase + e]) == h) v = __fadd_rn(v, p.head_w[pbase + e]);
    }
  }
  const float hi = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
  qh[int64_t(q) * 128 + h] = v;
  qh_lo[int64_t(q) * 128 + h] = __fsub_rn(v, hi);
}

template <typename WT, int kMode>
__global__ void __launch_bounds__(tc::kThreads, 1)
score_tc_kernel(const ScoreParams p, const __grid_constant__ TcParams tp) {
  using namespace tc;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // the runtime aligns dynamic shared memory to at least 16 bytes; the swizzled stages need 1024
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* a_full = bars;              // [kNSA]
  uint64_t* a_empty = bars + kNSA;      // [kNSA]
  uint64_t* b_full = bars + 2 * kNSA;   // [kNSB]
  uint64_t* b_empty = b_full + kNSB;    // [kNSB]
  uint64_t* mma_done = b_empty + kNSB;  // [1]
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + kOffCtl);
  volatile int32_t* vfault = &ctl->fault;
  const int wid = threadIdx.x >> 5, lane = lane_id();
  const int32_t limit = p.wait_limit;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNSA; ++i) {
      mbar_init(a_full + i, 1);
      mbar_init(a_empty + i, 1);
    }
    for (int i = 0; i < kNSB; ++i) {
      mbar_init(b_full + i, 1);
      mbar_init(b_empty + i, 1);
    }
    mbar_init(mma_done, 1);
    ctl->units_published = 0;
    ctl->units_ready = 0;
    ctl->drained = 0;
    ctl->gclaim = 0;
    ctl->k_end = 0x7FFFFFFF;
    ctl->fault = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (wid == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&ctl->tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (wid == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t a_it = 0, b_it = 0;
      bool ok = true;
      for (int32_t k = 0; ok; ++k) {
        int32_t u = int32_t(atomicAdd(tp.unit_next, 1ull));
        if (u >= tp.n_units) u = -1;
        // slot k % kUQ is free once unit k - kUQ has been drained
        if (k >= kUQ) ok = spin_ge(&ctl->drained, kDrainsPerUnit * (k - kUQ + 1), limit, vfault);
        if (!ok) break;
        ctl->unit_id[k % kUQ] = u;
        __threadfence_block();
        *reinterpret_cast<volatile int32_t*>(&ctl->units_published) = k + 1;
        if (u < 0) break;
        const int32_t tile = u / tp.n_groups;
        const int32_t q0 = p.q_lo + (u - tile * tp.n_groups) * kUnitQ;
        for (int32_t kc = 0; kc < tp.n_kc && ok; ++kc) {
          const uint32_t bs = b_it % kNSB, bn = b_it / kNSB;
          if (bn > 0) ok = mbar_wait(b_empty + bs, (bn - 1) & 1, limit, vfault);
          if (!ok) break;
          unsigned char* bdst = smem + kOffB + bs * 2 * kBPiece;
          mbar_expect_tx(b_full + bs, 2 * kBPiece);
          tma_2d(bdst, &tp.b_hi, kc * kKC, q0, b_full + bs);
          tma_2d(bdst + kBPiece, &tp.b_lo, kc * kKC, q0, b_full + bs);
          ++b_it;
          for (int32_t j = 0; j < kSlices && ok; ++j) {
            const uint32_t as = a_it % kNSA, an = a_it / kNSA;
            if (an > 0) ok = mbar_wait(a_empty + as, (an - 1) & 1, limit, vfault);
            if (!ok) break;
            unsigned char* adst = smem + kOffA + as * 2 * kAPiece;
            mbar_expect_tx(a_full + as, 2 * kAPiece);
            tma_3d(adst, &tp.a_hi, 0, kc * kKC, tile * (kTile / 32) + j * 4, a_full + as);
            tma_3d(adst + kAPiece, &tp.a_lo, 0, kc * kKC, tile * (kTile / 32) + j * 4, a_full + as);
            ++a_it;
          }
        }
      }
      if (!ok) {
        atomicOr(p.fault, 1);
        *vfault = 1;
      }
      // copies still in flight land before the CTA may exit: wait for the last stages' arrivals
      for (uint32_t i = 0; i < kNSA && i < a_it; ++i) {
        const uint32_t it = a_it - 1 - i;
        mbar_wait_landed(a_full + it % kNSA, (it / kNSA) & 1);
      }
      for (uint32_t i = 0; i < kNSB && i < b_it; ++i) {
        const uint32_t it = b_it - 1 - i;
        mbar_wait_landed(b_full + it % kNSB, (it / kNSB) & 1);
      }
    }
  } else if (wid == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t a_it = 0, b_it = 0;
      bool ok = true;
      int32_t k = 0;
      for (;; ++k) {
        ok = spin_ge(&ctl->units_published, k + 1, limit, vfault);
        if (!ok) break;
        __threadfence_block();
        const int32_t u = *reinterpret_cast<volatile int32_t*>(&ctl->unit_id[k % kUQ]);
        if (u < 0) break;
        // the previous unit's accumulators have been copied out of tensor memory
        ok = spin_ge(&ctl->drained, kDrainsPerUnit * k, limit, vfault);
        if (!ok) break;
        tc_fence_after();
        for (int32_t kc = 0; kc < tp.n_kc && ok; ++kc) {
          const uint32_t bs = b_it % kNSB, bn = b_it / kNSB;
          ok = mbar_wait(b_full + bs, bn & 1, limit, vfault);
          if (!ok) break;
          const uint32_t b_base = su32(smem + kOffB + bs * 2 * kBPiece);
          for (int32_t j = 0; j < kSlices && ok; ++j) {
            const uint32_t as = a_it % kNSA, an = a_it / kNSA;
            ok = mbar_wait(a_full + as, an & 1, limit, vfault);
            if (!ok) break;
            tc_fence_after();
            const uint32_t a_base = su32(smem + kOffA + as * 2 * kAPiece);
            const uint32_t d = tmem + uint32_t(j * kUnitQ);
#pragma unroll
            for (int t = 0; t < kKC / 8; ++t) {
              const uint64_t ah = desc_a(a_base + t * 1024), al = desc_a(a_base + kAPiece + t * 1024);
              const uint64_t bh = desc_b(b_base + t * 32), bl = desc_b(b_base + kBPiece + t * 32);
              tc_mma_tf32(d, ah, bh, kIdesc, (kc > 0 || t > 0) ? 1u : 0u);
              tc_mma_tf32(d, ah, bl, kIdesc, 1u);
              tc_mma_tf32(d, al, bh, kIdesc, 1u);
            }
            tc_commit(a_empty + as);   // the stage is free once these MMAs have read it
            ++a_it;
          }
          tc_commit(b_empty + bs);
          ++b_it;
        }
        if (!ok) break;
        tc_commit(mma_done);
        ok = mbar_wait(mma_done, uint32_t(k) & 1, limit, vfault);
        if (!ok) break;
        tc_fence_before();
        __threadfence_block();
        *reinterpret_cast<volatile int32_t*>(&ctl->units_ready) = k + 1;
      }
      if (ok) {
        *reinterpret_cast<volatile int32_t*>(&ctl->k_end) = k;
      } else {
        atomicOr(p.fault, 1);
        *vfault = 1;
        // MMAs already issued finish before the tensor memory is released
        tc_commit(mma_done);
        mbar_wait_landed(mma_done, uint32_t(k) & 1);
      }
    }
  } else if (wid >= kFirstQuadWarp) {
    // ------------------------------------------------------------------ quads of tail warps
    const int qw = wid - kFirstQuadWarp;
    const int quad = qw >> 2, s = qw & 3;   // s == wid % 4: this warp's tensor-memory sub-partition
    unsigned char* wbase = smem + kOffWarps;
    float* acc = reinterpret_cast<float*>(wbase + size_t(qw) * WarpLayout::total + WarpLayout::acc);
    uint32_t* hist = reinterpret_cast<uint32_t*>(wbase + size_t(qw) * WarpLayout::total + WarpLayout::hist);
    const uint32_t bar_id = 1 + quad;
    for (;;) {
      asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(128) : "memory");   // the quad's tiles are free
      if (s == 0 && lane == 0) {
        // claim 4 queries of unit k and wait until unit k is in tensor memory (or the end);
        // the leader decides for the whole quad (quad_g < 0: stop)
        const int32_t G = atomicAdd(&ctl->gclaim, 1);
        const int32_t k = G / kGroups;
        bool ready = false;
        for (int32_t i = 0; i <= limit; ++i) {
          if (*reinterpret_cast<volatile int32_t*>(&ctl->units_ready) > k) {
            ready = true;
            break;
          }
          if (*reinterpret_cast<volatile int32_t*>(&ctl->k_end) <= k || *vfault) break;
          __nanosleep(64);
        }
        if (!ready && *reinterpret_cast<volatile int32_t*>(&ctl->k_end) > k && !*vfault) {
          atomicOr(p.fault, 1);
          *vfault = 1;
        }
        __threadfence_block();
        ctl->quad_g[quad] = ready ? G : -1;
      }
      asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(128) : "memory");
      const int32_t G = *reinterpret_cast<volatile int32_t*>(&ctl->quad_g[quad]);
      if (G < 0) break;
      const int32_t k = G / kGroups, grp = G - k * kGroups;
      const int32_t u = *reinterpret_cast<volatile int32_t*>(&ctl->unit_id[k % kUQ]);
      const int32_t tile = u / tp.n_groups;
      const int32_t q0 = p.q_lo + (u - tile * tp.n_groups) * kUnitQ + grp * 4;
      tc_fence_after();
      float v[kSlices][4];
      const uint32_t tl = tmem + (uint32_t(32 * s) << 16) + uint32_t(grp * 4);
#pragma unroll
      for (int j = 0; j < kSlices; ++j) tc_ld_x4(tl + uint32_t(j * kUnitQ), v[j]);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) atomicAdd(&ctl->drained, 1);   // this warp's share of unit k is out
      // document 128 j + 32 s + lane of query q0 + c goes to quad member c's tile
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float* dst = reinterpret_cast<float*>(wbase + size_t(quad * 4 + c) * WarpLayout::total + WarpLayout::acc);
#pragma unroll
        for (int j = 0; j < kSlices; ++j) dst[128 * j + 32 * s + lane] = v[j][c];
      }
      asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(128) : "memory");
      const int32_t q = q0 + s;
      if (q < p.q_lo + p.q_n) item_tail_select<WT, kMode>(p, q, tile, acc, hist);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (wid == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}
