// Parameter all-gather over NVSwitch peer memory, as a role inside a consumer kernel.
//
// Sharded training keeps every sharded unit (a decoder layer's projection weights, the
// embedding, the LM head) as one contiguous range of a bf16 "gathered" buffer that
// every rank allocates in symmetric memory with the same layout.  Rank p owns elements
// [unit0 + p * cs, unit0 + (p + 1) * cs) of a unit and writes them after its optimizer
// step; the others fetch them before use.
//
// A fetch is split into pieces of 2^piece_shift elements.  Copy warps of the consumer
// kernel (the GEMM that first reads the weights) take pieces from a dispenser (an
// atomic counter zeroed before the launch), copy the peer-owned parts with 16-byte
// loads from the owner's buffer and 16-byte stores into this GPU's buffer, then publish
// the piece with a release store of the launch's epoch into a per-piece flag.  The
// consumer's TMA producer waits (bounded) for the flags of the pieces a B tile covers
// and then loads the tile from local memory, so the NVLink transfer of later pieces
// overlaps the MMAs on earlier ones.  TMA never reads peer memory here.
//
// Progress does not depend on which CTAs are resident: pieces are handed out only to
// copy warps that are running, and copy warps never wait, so a waiting producer's piece
// is either being copied or will be taken by its own CTA's copy warps.
#pragma once

#include "common.cuh"

namespace pb {

struct AgSpec {
  const __nv_bfloat16* const* src;  // [W] device array: every rank's gathered-buffer base
  __nv_bfloat16* dst;               // this rank's gathered-buffer base
  long lo, hi;                      // element range of the gathered buffer to fill
  long unit0, cs;                   // element e belongs to rank (e - unit0) / cs
  long b0;                          // consumer GEMM: element offset of B row 0
  int rank, world;                  // world == 0: no gather in this launch
  int piece_shift;
  int rot;                          // first piece handed out (the dispenser wraps around)
  uint32_t* flags;                  // per piece: the epoch of the launch that filled it
  int* counter;
  uint32_t epoch;
};

__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Orders this thread's generic-proxy global accesses with later async-proxy (TMA)
// accesses and vice versa.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ int ag_num_pieces(const AgSpec& s) {
  return static_cast<int>((s.hi - s.lo + (1L << s.piece_shift) - 1) >> s.piece_shift);
}

// Warp copy of n bf16 (n % 8 == 0, both ends 16-byte aligned), 8 loads in flight per lane.
__device__ __forceinline__ void ag_copy_span(const __nv_bfloat16* src, __nv_bfloat16* dst, long n) {
  const int4* s4 = reinterpret_cast<const int4*>(src);
  int4* d4 = reinterpret_cast<int4*>(dst);
  const long nv = n >> 3;
  const int lane = threadIdx.x & 31;
  for (long i = lane; i < nv; i += 32 * 8) {
    int4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i + u * 32 < nv) v[u] = __ldcg(s4 + i + u * 32);
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (i + u * 32 < nv) d4[i + u * 32] = v[u];
  }
}

// Copy-warp role: take pieces until the dispenser is empty.
__device__ __forceinline__ void ag_copy_warp(const AgSpec& s) {
  const int npieces = ag_num_pieces(s);
  const int lane = threadIdx.x & 31;
  while (true) {
    int t = 0;
    if (lane == 0) t = atomicAdd(s.counter, 1);
    t = __shfl_sync(0xffffffff, t, 0);
    if (t >= npieces) break;
    int g = t + s.rot;
    if (g >= npieces) g -= npieces;
    const long e0 = s.lo + (static_cast<long>(g) << s.piece_shift);
    const long e1 = min(e0 + (1L << s.piece_shift), s.hi);
    for (long e = e0; e < e1;) {
      const int p = static_cast<int>((e - s.unit0) / s.cs);
      const long seg_end = min(e1, s.unit0 + (p + 1) * s.cs);
      if (p != s.rank) ag_copy_span(s.src[p] + e, s.dst + e, seg_end - e);
      e = seg_end;
    }
    fence_proxy_async_global();
    __threadfence();
    __syncwarp();
    if (lane == 0) st_release_gpu(s.flags + g, s.epoch);
  }
}

// Producer side: wait until elements [e0, e1) of the gathered buffer are local.
// Returns false (after recording ``code``) on timeout or when the CTA aborts.
__device__ __forceinline__ bool ag_wait_range(const AgSpec& s, long e0, long e1, int* status, int code,
                                              volatile int* abort) {
  e0 = max(e0, s.lo);
  e1 = min(e1, s.hi);
  if (e0 >= e1) return true;
  const int g0 = static_cast<int>((e0 - s.lo) >> s.piece_shift);
  const int g1 = static_cast<int>((e1 - 1 - s.lo) >> s.piece_shift);
  for (int g = g0; g <= g1; ++g) {
    if (static_cast<int>(ld_acquire_gpu(s.flags + g) - s.epoch) >= 0) continue;
    const uint64_t t0 = globaltimer();
    while (static_cast<int>(ld_acquire_gpu(s.flags + g) - s.epoch) < 0) {
      if (abort != nullptr && *abort) return false;
      if (globaltimer() - t0 > PB_WAIT_TIMEOUT_NS) {
        report_error(status, code);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
  fence_proxy_async_global();
  return true;
}

}  // namespace pb
