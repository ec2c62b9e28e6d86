// Parameter all-gather over NVSwitch peer memory, as a role inside a consumer kernel.
//
// Sharded training addresses every sharded unit (a decoder layer's projection weights,
// the embedding, the LM head) in "gathered coordinates": elements [unit0, unit0 + W cs),
// of which rank p owns [unit0 + p cs, unit0 + (p + 1) cs).  The owner writes the bf16
// copy of its chunk into its symmetric "owned" buffer after its optimizer step; a fetch
// copies the chunks into this rank's gathered storage (the unit's fixed place, or a
// rotating window).  The spec carries per-owner source bases and a destination base
// already offset by the unit's placement, so element e of owner p is read at src[p] + e
// and written at dst + e.  ``copy_own`` also copies this rank's own chunk (local memory).
//
// A fetch of [lo, hi) is cut into pieces of 2^piece_shift elements (8 KB: one round of
// 16-byte loads of a warp).  Copy warps of the consumer kernel (the GEMM that first reads
// the weights) take pieces from a dispenser (an atomic ticket counter), copy the
// peer-owned parts with 16-byte loads from the owner's buffer and 16-byte stores into
// this GPU's buffer, and then add the number of elements they made local to the counter
// of every block of 2^block_shift elements the piece overlaps (release).  The consumer's
// TMA producer waits (bounded) until the blocks a B tile covers are complete and then
// loads the tile from local memory, so the NVLink transfer of later blocks overlaps the
// MMAs on earlier ones.  TMA never reads peer memory here.
//
// Dispense order follows the consumer: with ``split`` > 0 the regions [lo, lo + split)
// and [lo + split, lo + 2 split) (the gate and up rows a SwiGLU tile reads together) are
// handed out interleaved piece by piece, then the rest in order; otherwise the range is
// handed out from piece ``rot`` on, wrapping around.
//
// The ticket and block counters are zeroed before each launch.  Progress does not depend
// on which CTAs are resident: pieces are handed out only to copy warps that are running,
// and copy warps never wait, so a waiting producer's block is either being copied or will
// be completed by its own CTA's copy warps.
#pragma once

#include "common.cuh"

namespace pb {

struct AgSpec {
  const __nv_bfloat16* const* src;  // [W] device array: every rank's gathered-buffer base
  __nv_bfloat16* dst;               // this rank's gathered-buffer base
  long lo, hi;                      // element range of the gathered buffer to fill
  long unit0, cs;                   // element e belongs to rank (e - unit0) / cs
  long b0;                          // consumer GEMM: element offset of B row 0
  long split;                       // > 0: interleave [lo, lo+split) with [lo+split, lo+2 split)
  int rank, world;                  // world == 0: no gather in this launch
  int piece_shift, block_shift;
  int rot;                          // first piece handed out (no split)
  int copy_own;                     // 1: copy this rank's chunk too (from src[rank])
  uint32_t* counters;               // [0]: tickets, [1 + b]: elements of block b made local
};

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_release_add_gpu(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// Orders this thread's generic-proxy global accesses with later async-proxy (TMA)
// accesses and vice versa.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ long ag_pieces(long n, int shift) { return (n + (1L << shift) - 1) >> shift; }

// Elements of block b that lie in [lo, hi).
__device__ __forceinline__ uint32_t ag_block_len(const AgSpec& s, long b) {
  const long a = s.lo + (b << s.block_shift);
  return static_cast<uint32_t>(min(a + (1L << s.block_shift), s.hi) - a);
}

// Warp copy of n bf16 (n % 8 == 0, both ends 16-byte aligned), 16 loads in flight per lane.
__device__ __forceinline__ void ag_copy_span(const __nv_bfloat16* src, __nv_bfloat16* dst, long n) {
  constexpr int U = 16;
  const int4* s4 = reinterpret_cast<const int4*>(src);
  int4* d4 = reinterpret_cast<int4*>(dst);
  const long nv = n >> 3;
  const int lane = threadIdx.x & 31;
  for (long i = lane; i < nv; i += 32 * U) {
    int4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i + u * 32 < nv) v[u] = __ldcg(s4 + i + u * 32);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i + u * 32 < nv) d4[i + u * 32] = v[u];
  }
}

// Ticket -> element range of the piece, in dispense order.  False when out of tickets.
__device__ __forceinline__ bool ag_piece_of(const AgSpec& s, long t, long& e0, long& e1) {
  const long P = 1L << s.piece_shift;
  if (s.split > 0) {
    const long na = ag_pieces(s.split, s.piece_shift);
    if (t < 2 * na) {
      const long base = s.lo + (t & 1) * s.split + (t >> 1) * P;
      e0 = base;
      e1 = min(base + P, s.lo + ((t & 1) + 1) * s.split);
      return true;
    }
    t -= 2 * na;
    const long r0 = s.lo + 2 * s.split;
    if (t >= ag_pieces(s.hi - r0, s.piece_shift)) return false;
    e0 = r0 + t * P;
    e1 = min(e0 + P, s.hi);
    return true;
  }
  const long np = ag_pieces(s.hi - s.lo, s.piece_shift);
  if (t >= np) return false;
  long g = t + s.rot;
  if (g >= np) g -= np;
  e0 = s.lo + g * P;
  e1 = min(e0 + P, s.hi);
  return true;
}

// Copy-warp role: take pieces until the dispenser is empty.
__device__ __forceinline__ void ag_copy_warp(const AgSpec& s) {
  const int lane = threadIdx.x & 31;
  while (true) {
    uint32_t t = 0;
    if (lane == 0) t = atomicAdd(s.counters, 1u);
    t = __shfl_sync(0xffffffff, t, 0);
    long e0, e1;
    if (!ag_piece_of(s, t, e0, e1)) break;
    for (long e = e0; e < e1;) {
      const int p = static_cast<int>((e - s.unit0) / s.cs);
      const long seg_end = min(e1, s.unit0 + (p + 1) * s.cs);
      if ((p != s.rank || s.copy_own) && PB_BOUNDS_OK(p >= 0 && p < s.world, nullptr, 0))
        ag_copy_span(s.src[p] + e, s.dst + e, seg_end - e);
      e = seg_end;
    }
    fence_proxy_async_global();
    __threadfence();
    __syncwarp();
    if (lane == 0) {
      for (long e = e0; e < e1;) {
        const long b = (e - s.lo) >> s.block_shift;
        const long b_end = min(e1, s.lo + ((b + 1) << s.block_shift));
        red_release_add_gpu(s.counters + 1 + b, static_cast<uint32_t>(b_end - e));
        e = b_end;
      }
    }
  }
}

// Producer side: wait until elements [e0, e1) of the gathered buffer are local.
// Returns false (after recording ``code``) on timeout or when the CTA aborts.
__device__ __forceinline__ bool ag_wait_range(const AgSpec& s, long e0, long e1, int* status, int code,
                                              volatile int* abort) {
  e0 = max(e0, s.lo);
  e1 = min(e1, s.hi);
  if (e0 >= e1) return true;
  const long b0 = (e0 - s.lo) >> s.block_shift;
  const long b1 = (e1 - 1 - s.lo) >> s.block_shift;
  for (long b = b0; b <= b1; ++b) {
    const uint32_t need = ag_block_len(s, b);
    if (ld_relaxed_gpu(s.counters + 1 + b) >= need) continue;
    const uint64_t t0 = globaltimer();
    while (ld_relaxed_gpu(s.counters + 1 + b) < need) {
      if (abort != nullptr && *abort) return false;
      if (globaltimer() - t0 > PB_WAIT_TIMEOUT_NS) {
        report_error(status, code);
        if (abort != nullptr) *abort = 1;
        return false;
      }
    }
  }
  // The relaxed loads above observed the copy warps' release additions; this fence
  // makes that an acquire, and the proxy fence extends it to the TMA loads that follow.
  fence_acq_rel_gpu();
  fence_proxy_async_global();
  return true;
}

}  // namespace pb
