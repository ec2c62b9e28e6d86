// Device kernels of the LM-head cross-entropy shared by the extension and the
// allocation-free C entry point.
#pragma once

#include "common.cuh"

namespace pb {

// ------------------------------- LM-head CE row reduction -------------------------
// Combines the per-tile (max, sum exp) partials of each row into lse, and the summed
// loss  lse - logit[target] + z * lse^2  over labelled rows.  A 256-thread block covers
// kCeRows rows with kCeGroups threads per row: thread (g, r) folds tiles g, g + 8, ...
// of row r with the online (max, sum) recurrence (adjacent threads read adjacent rows
// of a tile: coalesced), then the 8 partials of a row are merged through shared memory.
constexpr int kCeRows = 32;
constexpr int kCeGroups = 8;

__device__ __forceinline__ void ce_merge(float& m, float& s, float pm, float ps) {
  const float mn = fmaxf(m, pm);
  if (mn == -INFINITY) return;
  s = s * __expf(m - mn) + ps * __expf(pm - mn);
  m = mn;
}

static __global__ void __launch_bounds__(kCeRows * kCeGroups) ce_finalize_kernel(
    const float* __restrict__ pmax, const float* __restrict__ psum, int ntiles, int rows,
    const float* __restrict__ tlogit, const int64_t* __restrict__ targets, int64_t ignore_index, float z,
    float* __restrict__ lse, float* __restrict__ loss) {
  __shared__ float sm[kCeGroups][kCeRows], ss[kCeGroups][kCeRows];
  const int rl = threadIdx.x % kCeRows, grp = threadIdx.x / kCeRows;
  const int r = blockIdx.x * kCeRows + rl;
  float m = -INFINITY, s = 0.f;
  if (r < rows) {
    for (int t = grp; t < ntiles; t += kCeGroups) {
      const long o = static_cast<long>(t) * rows + r;
      ce_merge(m, s, pmax[o], psum[o]);
    }
  }
  sm[grp][rl] = m;
  ss[grp][rl] = s;
  __syncthreads();
  if (grp == 0) {
    float l = 0.f;
    if (r < rows) {
      for (int q = 1; q < kCeGroups; ++q) ce_merge(m, s, sm[q][rl], ss[q][rl]);
      const float ls = m + logf(s);
      lse[r] = ls;
      if (targets[r] != ignore_index) l = ls - tlogit[r] + z * ls * ls;
    }
    l = warp_sum(l);
    if (rl == 0) atomicAdd(loss, l);
  }
}

inline unsigned ce_finalize_blocks(int rows) { return static_cast<unsigned>((rows + kCeRows - 1) / kCeRows); }

}  // namespace pb
