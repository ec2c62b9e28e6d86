// Fused gradient all-reduce over NVSwitch peer memory (sm_100a).
//
// The flat fp32 gradient buffer of every rank lives in symmetric memory (one
// allocation per rank, mapped into every peer), so a bucket [lo, hi) can be averaged
// by one kernel without staging copies:
//
//   barrier 0   every rank's bucket is final (its backward kernels precede this launch)
//   phase 1     reduce-scatter: rank r sums chunk r of the bucket over all ranks with
//               16-byte peer loads, scales by 1/W (the average), writes it back into its
//               own buffer and accumulates the squared norm of the result
//   barrier 1   reduced chunks visible
//   phase 2     all-gather: rank r copies chunk p (p != r) from rank p's buffer into its
//               own, accumulating the squared norm of those chunks too
//   barrier 2   no rank still reads this rank's buffer (its next backward may write it)
//
// Each chunk is split into one sub-range per CTA with the same split on every rank, so
// CTA b of rank q only reads data produced by CTA b of rank p: barriers are per CTA
// (flags in the peers' signal pads, release/acquire at system scope).  Per rank the
// bucket crosses NVLink 2 (W - 1) / W times, the bandwidth optimum for an all-reduce
// without in-switch reduction.  Every wait is bounded: on timeout the kernel records
// status 401 (and the peer that did not arrive, +1000 * peer) and returns.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "host_utils.h"

namespace pb {

struct ArArgs {
  float* const* ptrs;   // [W] peer buffer base pointers (device array)
  uint32_t* const* pads;  // [W] peer signal pads (device array)
  long lo, hi;
  int rank, world;
  uint32_t epoch;
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
    __threadfence_system();
    st_release_sys(a.pads[p] + slot_mine, a.epoch);
    const uint32_t* watch = a.pads[a.rank] + (static_cast<long>(k) * gridDim.x + b) * W + p;
    const uint64_t t0 = globaltimer();
    while (static_cast<int>(ld_acquire_sys(watch) - a.epoch) < 0) {
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

__global__ void __launch_bounds__(512) fused_allreduce_kernel(const ArArgs a) {
  __shared__ volatile int abort_sh;
  __shared__ float red[32];
  if (threadIdx.x == 0) abort_sh = 0;
  __syncthreads();
  const int W = a.world;
  const long n = a.hi - a.lo;
  // chunk and per-CTA sub-range sizes (multiples of 4 floats for 16-byte accesses)
  const long cs = ((n + W - 1) / W + 3) / 4 * 4;
  const long sub = ((cs + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
  float ss = 0.f;
  if (!cta_barrier(a, 0, &abort_sh)) return;
  {
    const long c0 = a.lo + a.rank * cs;
    const long s0 = min(c0 + static_cast<long>(blockIdx.x) * sub, min(c0 + cs, a.hi));
    const long s1 = min(s0 + sub, min(c0 + cs, a.hi));
    float* mine = a.ptrs[a.rank];
    for (long i = s0 + threadIdx.x * 4; i < s1; i += blockDim.x * 4) {
      if (i + 3 < s1) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < W; ++p) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(a.ptrs[p] + i));
          acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        acc.x *= a.scale; acc.y *= a.scale; acc.z *= a.scale; acc.w *= a.scale;
        *reinterpret_cast<float4*>(mine + i) = acc;
        ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
      } else {
        for (long e = i; e < s1; ++e) {
          float acc = 0.f;
          for (int p = 0; p < W; ++p) acc += __ldcg(a.ptrs[p] + e);
          acc *= a.scale;
          mine[e] = acc;
          ss += acc * acc;
        }
      }
    }
  }
  if (!cta_barrier(a, 1, &abort_sh)) return;
  for (int step = 1; step < W; ++step) {
    const int p = (a.rank + step) % W;
    const long c0 = a.lo + p * cs;
    const long s0 = min(c0 + static_cast<long>(blockIdx.x) * sub, min(c0 + cs, a.hi));
    const long s1 = min(s0 + sub, min(c0 + cs, a.hi));
    const float* src = a.ptrs[p];
    float* dst = a.ptrs[a.rank];
    for (long i = s0 + threadIdx.x * 4; i < s1; i += blockDim.x * 4) {
      if (i + 3 < s1) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src + i));
        *reinterpret_cast<float4*>(dst + i) = v;
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      } else {
        for (long e = i; e < s1; ++e) {
          const float v = __ldcg(src + e);
          dst[e] = v;
          ss += v * v;
        }
      }
    }
  }
  if (!cta_barrier(a, 2, &abort_sh)) return;
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(a.sumsq, v);
  }
}

// ptrs_dev / pads_dev: device arrays of W uint64 addresses (from the symmetric-memory
// rendezvous).  ``pad_words`` is the signal pad size in uint32 words.
void fused_allreduce(int64_t ptrs_dev, int64_t pads_dev, int64_t pad_words, int64_t lo, int64_t hi, int64_t rank,
                     int64_t world, int64_t epoch, double scale, at::Tensor sumsq, int64_t ctas) {
  TORCH_CHECK(sumsq.is_cuda() && sumsq.scalar_type() == at::kFloat);
  TORCH_CHECK(lo % 4 == 0, "fused_allreduce: bucket start must be 16-byte aligned");
  TORCH_CHECK(3 * ctas * world <= pad_words, "fused_allreduce: signal pad too small for ", ctas, " CTAs");
  const c10::cuda::CUDAGuard guard(sumsq.device());
  ArArgs a{};
  a.ptrs = reinterpret_cast<float* const*>(ptrs_dev);
  a.pads = reinterpret_cast<uint32_t* const*>(pads_dev);
  a.lo = lo;
  a.hi = hi;
  a.rank = (int)rank;
  a.world = (int)world;
  a.epoch = static_cast<uint32_t>(epoch);
  a.scale = (float)scale;
  a.sumsq = sumsq.data_ptr<float>();
  a.status = status_ptr(sumsq.device().index());
  fused_allreduce_kernel<<<(int)ctas, 512, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  PB_CUDA_CHECK(cudaGetLastError());
}

void comm_bindings(pybind11::module& m) { m.def("fused_allreduce", &fused_allreduce); }

}  // namespace pb
