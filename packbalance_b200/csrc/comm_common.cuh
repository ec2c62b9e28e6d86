// Device helpers shared by the peer-memory collectives (all-reduce, reduce-scatter,
// sharded optimizer): peer pointer tables, per-CTA cross-rank barriers through
// signal pads in symmetric memory (release/acquire at system scope, epoch-tagged so
// pads never need resetting, bounded waits) and the per-CTA split of a range.
#pragma once

#include "common.cuh"

namespace pb {

struct ArArgs {
  float* const* ptrs;   // [W] peer buffer base pointers (device array)
  uint32_t* const* pads;  // [W] peer signal pads (device array)
  long lo, hi;
  int rank, world;
  uint32_t epoch;
  // When set, the launch's epoch is epoch + *epoch_base: the base is bumped on the
  // device once per training step, so a captured CUDA graph replays with fresh epochs.
  const uint32_t* epoch_base;
  float scale;
  float* sumsq;
  int* status;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t launch_epoch(const ArArgs& a) {
  return a.epoch + (a.epoch_base != nullptr ? *a.epoch_base : 0u);
}

// Barrier ``k`` between CTA ``blockIdx.x`` of every rank.  Slot (k, b, p) of rank r's pad
// holds the last epoch in which rank p reached barrier k with CTA b.
__device__ __forceinline__ bool cta_barrier(const ArArgs& a, int k, volatile int* abort) {
  __syncthreads();
  const int b = blockIdx.x;
  const int W = a.world;
  bool ok = true;
  if (threadIdx.x < W) {
    const int p = threadIdx.x;
    const long slot_mine = (static_cast<long>(k) * gridDim.x + b) * W + a.rank;
    const uint32_t ep = launch_epoch(a);
    __threadfence_system();
    st_release_sys(a.pads[p] + slot_mine, ep);
    const uint32_t* watch = a.pads[a.rank] + (static_cast<long>(k) * gridDim.x + b) * W + p;
    const uint64_t t0 = globaltimer();
    while (static_cast<int>(ld_acquire_sys(watch) - ep) < 0) {
      if (*abort) {
        ok = false;
        break;
      }
      if (globaltimer() - t0 > PB_WAIT_TIMEOUT_NS / 2) {
        report_error(a.status, 401 + 1000 * p);
        *abort = 1;
        ok = false;
        break;
      }
    }
  }
  __syncthreads();
  return ok && !*abort;
}

constexpr int kMaxWorld = 8;

// Collective kernels run beside the compute kernels of the backward pass.  Small CTAs
// with a capped register budget (128 threads x <= 64 registers = 8 K registers) fit
// next to a resident GEMM or attention CTA on the same SM, so communication never
// evicts compute from an SM; bandwidth comes from many such CTAs.
constexpr int kCommThreads = 128;
constexpr int kCommMinBlocks = 8;

// Sub-range of chunk ``c`` owned by this CTA (same split on every rank).
__device__ __forceinline__ void sub_range(const ArArgs& a, long cs, long sub, int c, long& s0, long& s1) {
  const long c0 = a.lo + c * cs;
  const long c1 = min(c0 + cs, a.hi);
  s0 = min(c0 + static_cast<long>(blockIdx.x) * sub, c1);
  s1 = min(s0 + sub, c1);
}

// NVLink multicast (NVLS) through the NVSwitch: ``mc`` addresses a multicast object
// bound over every rank's buffer.  ld_reduce returns the sum over all ranks, st writes
// every rank, red adds into every rank.
__device__ __forceinline__ float4 mm_ld_reduce(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void mm_st(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void mm_red_add(float* mc, float v) {
  asm volatile("multimem.red.relaxed.sys.global.add.f32 [%0], %1;" ::"l"(mc), "f"(v) : "memory");
}

}  // namespace pb
