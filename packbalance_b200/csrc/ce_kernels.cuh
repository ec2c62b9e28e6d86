// Device kernels of the LM-head cross-entropy shared by the extension and the
// allocation-free C entry point.
#pragma once

#include "common.cuh"

namespace pb {

// ------------------------------- LM-head CE row reduction -------------------------
// Combines the per-tile (max, sum exp) partials of each row into lse, and the summed
// loss  lse - logit[target] + z * lse^2  over labelled rows.
static __global__ void ce_finalize_kernel(const float* __restrict__ pmax, const float* __restrict__ psum, int ntiles,
                                   int rows, const float* __restrict__ tlogit, const int64_t* __restrict__ targets,
                                   int64_t ignore_index, float z, float* __restrict__ lse, float* __restrict__ loss) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  float l = 0.f;
  if (r < rows) {
    float mx = -INFINITY;
    for (int t = 0; t < ntiles; ++t) mx = fmaxf(mx, pmax[static_cast<long>(t) * rows + r]);
    float se = 0.f;
    for (int t = 0; t < ntiles; ++t) se += psum[static_cast<long>(t) * rows + r] * __expf(pmax[static_cast<long>(t) * rows + r] - mx);
    const float ls = mx + logf(se);
    lse[r] = ls;
    if (targets[r] != ignore_index) l = ls - tlogit[r] + z * ls * ls;
  }
  l = warp_sum(l);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = l;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(loss, v);
  }
}

}  // namespace pb
