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

#include "comm_common.cuh"
#include "common.cuh"
#include "host_utils.h"

namespace pb {

template <int W>
__device__ __forceinline__ float reduce_phase(const ArArgs& a, long s0, long s1) {
  // All W peer loads of a 16-byte group are issued before any is used, G groups per
  // thread per iteration (G W <= 8 keeps the data in 32 registers), so each thread keeps
  // G W loads in flight over NVLink.
  constexpr int G = W <= 4 ? 2 : 1;
  float ss = 0.f;
  float* mine = a.ptrs[a.rank];
  const long step = static_cast<long>(blockDim.x) * 4 * G;
  for (long i = s0 + threadIdx.x * 4; i < s1; i += step) {
    float4 v[G][W];
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const long j = i + u * blockDim.x * 4;
      if (j + 3 < s1) {
#pragma unroll
        for (int p = 0; p < W; ++p) v[u][p] = __ldcg(reinterpret_cast<const float4*>(a.ptrs[p] + j));
      }
    }
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const long j = i + u * blockDim.x * 4;
      if (j + 3 < s1) {
        float4 acc = v[u][0];
#pragma unroll
        for (int p = 1; p < W; ++p) {
          acc.x += v[u][p].x; acc.y += v[u][p].y; acc.z += v[u][p].z; acc.w += v[u][p].w;
        }
        acc.x *= a.scale; acc.y *= a.scale; acc.z *= a.scale; acc.w *= a.scale;
        *reinterpret_cast<float4*>(mine + j) = acc;
        ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
      } else if (j < s1) {
        for (long e = j; e < s1; ++e) {
          float acc = 0.f;
          for (int p = 0; p < W; ++p) acc += __ldcg(a.ptrs[p] + e);
          acc *= a.scale;
          mine[e] = acc;
          ss += acc * acc;
        }
      }
    }
  }
  return ss;
}

template <int W>
__device__ __forceinline__ float gather_phase(const ArArgs& a, long cs, long sub) {
  // Copy the other ranks' reduced chunks; for each position the W - 1 peer loads are
  // in flight together.
  float ss = 0.f;
  float* mine = a.ptrs[a.rank];
  long s0[W], s1[W];
#pragma unroll
  for (int p = 0; p < W; ++p) sub_range(a, cs, sub, p, s0[p], s1[p]);
  for (long off = threadIdx.x * 4; off < sub; off += static_cast<long>(blockDim.x) * 4) {
    float4 v[W];
#pragma unroll
    for (int p = 0; p < W; ++p)
      if (p != a.rank && s0[p] + off + 3 < s1[p]) v[p] = __ldcg(reinterpret_cast<const float4*>(a.ptrs[p] + s0[p] + off));
#pragma unroll
    for (int p = 0; p < W; ++p) {
      if (p == a.rank) continue;
      const long j = s0[p] + off;
      if (j + 3 < s1[p]) {
        *reinterpret_cast<float4*>(mine + j) = v[p];
        ss += v[p].x * v[p].x + v[p].y * v[p].y + v[p].z * v[p].z + v[p].w * v[p].w;
      } else {
        for (long e = j; e < s1[p]; ++e) {
          const float x = __ldcg(a.ptrs[p] + e);
          mine[e] = x;
          ss += x * x;
        }
      }
    }
  }
  return ss;
}

template <int W>
__global__ void __launch_bounds__(kCommThreads, kCommMinBlocks) fused_allreduce_kernel(const ArArgs a) {
  __shared__ volatile int abort_sh;
  __shared__ float red[32];
  if (threadIdx.x == 0) abort_sh = 0;
  __syncthreads();
  const long n = a.hi - a.lo;
  // chunk and per-CTA sub-range sizes (multiples of 4 floats for 16-byte accesses)
  const long cs = ((n + W - 1) / W + 3) / 4 * 4;
  const long sub = ((cs + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
  if (!cta_barrier(a, 0, &abort_sh)) return;
  long s0, s1;
  sub_range(a, cs, sub, a.rank, s0, s1);
  float ss = reduce_phase<W>(a, s0, s1);
  if (!cta_barrier(a, 1, &abort_sh)) return;
  ss += gather_phase<W>(a, cs, sub);
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

// ----------------------------- NVLS (multimem) variant ----------------------------
// With an NVLink multicast object bound over the symmetric buffers, one
// multimem.ld_reduce returns the sum over all ranks (reduced inside the NVSwitch) and
// one multimem.st writes the result into every rank's buffer.  Rank r handles chunk r:
//   barrier 0 -> ld_reduce / scale / st over its chunk -> multimem.red of its squared
//   norm into every rank's accumulator -> barrier 1
// Per rank NVLink carries about (W - 1) / W of the bucket in each direction.
__global__ void __launch_bounds__(kCommThreads, kCommMinBlocks) nvls_allreduce_kernel(const ArArgs a, float* mc,
                                                                                     float* mc_sumsq) {
  __shared__ volatile int abort_sh;
  __shared__ float red[32];
  if (threadIdx.x == 0) abort_sh = 0;
  __syncthreads();
  const int W = a.world;
  const long n = a.hi - a.lo;
  const long cs = ((n + W - 1) / W + 3) / 4 * 4;
  const long sub = ((cs + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
  if (!cta_barrier(a, 0, &abort_sh)) return;
  long s0, s1;
  sub_range(a, cs, sub, a.rank, s0, s1);
  // Eight 16-byte multimem loads in flight per thread: a narrow launch (a few CTAs beside
  // the backward pass's kernels) still keeps enough bytes in flight over NVLink.
  constexpr int U = 8;
  float ss = 0.f;
  const long step = static_cast<long>(blockDim.x) * 4 * U;
  for (long i = s0 + threadIdx.x * 4; i < s1; i += step) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long j = i + u * blockDim.x * 4;
      if (j + 3 < s1) v[u] = mm_ld_reduce(mc + j);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long j = i + u * blockDim.x * 4;
      if (j + 3 < s1) {
        float4 x = v[u];
        x.x *= a.scale; x.y *= a.scale; x.z *= a.scale; x.w *= a.scale;
        mm_st(mc + j, x);
        ss += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
      } else if (j < s1) {
        // ragged tail (bucket end not a multiple of 4): plain peer loads and stores
        for (long e = j; e < s1; ++e) {
          float acc = 0.f;
          for (int p = 0; p < W; ++p) acc += __ldcg(a.ptrs[p] + e);
          acc *= a.scale;
          for (int p = 0; p < W; ++p) a.ptrs[p][e] = acc;
          ss += acc * acc;
        }
      }
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) mm_red_add(mc_sumsq, v);
  }
  cta_barrier(a, 1, &abort_sh);
}

void nvls_allreduce(int64_t ptrs_dev, int64_t pads_dev, int64_t pad_words, int64_t mc_ptr, int64_t mc_sumsq,
                    int64_t lo, int64_t hi, int64_t rank, int64_t world, int64_t epoch, double scale,
                    at::Tensor local_sumsq, int64_t ctas, int64_t epoch_base) {
  TORCH_CHECK(lo % 4 == 0, "nvls_allreduce: bucket start must be 16-byte aligned");
  TORCH_CHECK(2 * ctas * world <= pad_words, "nvls_allreduce: signal pad too small");
  const c10::cuda::CUDAGuard guard(local_sumsq.device());
  ArArgs a{};
  a.ptrs = reinterpret_cast<float* const*>(ptrs_dev);
  a.pads = reinterpret_cast<uint32_t* const*>(pads_dev);
  a.lo = lo;
  a.hi = hi;
  a.rank = (int)rank;
  a.world = (int)world;
  a.epoch = static_cast<uint32_t>(epoch);
  a.epoch_base = reinterpret_cast<const uint32_t*>(epoch_base);
  a.scale = (float)scale;
  a.sumsq = local_sumsq.data_ptr<float>();
  a.status = status_ptr(local_sumsq.device().index());
  nvls_allreduce_kernel<<<pb::smem_max(nvls_allreduce_kernel, (int)ctas), kCommThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      a, reinterpret_cast<float*>(mc_ptr), reinterpret_cast<float*>(mc_sumsq));
  PB_CUDA_CHECK(cudaGetLastError());
}

// ptrs_dev / pads_dev: device arrays of W uint64 addresses (from the symmetric-memory
// rendezvous).  ``pad_words`` is the signal pad size in uint32 words.
void fused_allreduce(int64_t ptrs_dev, int64_t pads_dev, int64_t pad_words, int64_t lo, int64_t hi, int64_t rank,
                     int64_t world, int64_t epoch, double scale, at::Tensor sumsq, int64_t ctas, int64_t epoch_base) {
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
  a.epoch_base = reinterpret_cast<const uint32_t*>(epoch_base);
  a.scale = (float)scale;
  a.sumsq = sumsq.data_ptr<float>();
  a.status = status_ptr(sumsq.device().index());
  auto st = at::cuda::getCurrentCUDAStream();
  switch (world) {
    case 2: fused_allreduce_kernel<2><<<pb::smem_max(fused_allreduce_kernel<2>, (int)ctas), kCommThreads, 0, st>>>(a); break;
    case 3: fused_allreduce_kernel<3><<<pb::smem_max(fused_allreduce_kernel<3>, (int)ctas), kCommThreads, 0, st>>>(a); break;
    case 4: fused_allreduce_kernel<4><<<pb::smem_max(fused_allreduce_kernel<4>, (int)ctas), kCommThreads, 0, st>>>(a); break;
    case 5: fused_allreduce_kernel<5><<<pb::smem_max(fused_allreduce_kernel<5>, (int)ctas), kCommThreads, 0, st>>>(a); break;
    case 6: fused_allreduce_kernel<6><<<pb::smem_max(fused_allreduce_kernel<6>, (int)ctas), kCommThreads, 0, st>>>(a); break;
    case 7: fused_allreduce_kernel<7><<<pb::smem_max(fused_allreduce_kernel<7>, (int)ctas), kCommThreads, 0, st>>>(a); break;
    case 8: fused_allreduce_kernel<8><<<pb::smem_max(fused_allreduce_kernel<8>, (int)ctas), kCommThreads, 0, st>>>(a); break;
    default: TORCH_CHECK(false, "fused_allreduce: world size 2..8 on one node");
  }
  PB_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------ bf16 wire (two-shot) ---------------------------------
// The bucket crosses NVLink as bf16, half the bytes of the fp32 kernel; every sum is fp32.
//   phase 0   each CTA casts its sub-range of every chunk of this rank's bucket to bf16
//             into this rank's wire buffer (symmetric, same element indexing)
//   barrier 0
//   phase 1   rank r sums its chunk over the ranks' wires in rank order (fp32), scales,
//             rounds to bf16, and writes the rounded value to its wire (for the peers)
//             and, as fp32, to its gradient
//   barrier 1
//   phase 2   rank r copies the other ranks' reduced chunks from their wires (bf16 -> fp32)
//   barrier 2
// Every rank ends with the same (bf16-rounded) average, so the replicas stay identical.
// Chunk and sub-range sizes are multiples of 8 elements (16-byte bf16 vectors).
__device__ __forceinline__ void bf16x8_to_f32(uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <int W>
__global__ void __launch_bounds__(kCommThreads, kCommMinBlocks)
    fused_allreduce_bf16_kernel(const ArArgs a, __nv_bfloat16* const* wires) {
  __shared__ volatile int abort_sh;
  __shared__ float red[32];
  if (threadIdx.x == 0) abort_sh = 0;
  __syncthreads();
  const long n = a.hi - a.lo;
  const long cs = ((n + W - 1) / W + 7) / 8 * 8;
  const long sub = ((cs + gridDim.x - 1) / gridDim.x + 7) / 8 * 8;
  float* mine = a.ptrs[a.rank];
  __nv_bfloat16* wmine = wires[a.rank];
  const long step = static_cast<long>(blockDim.x) * 8;
  // phase 0: cast this CTA's sub-range of every chunk
#pragma unroll 1
  for (int c = 0; c < W; ++c) {
    long s0, s1;
    sub_range(a, cs, sub, c, s0, s1);
    for (long i = s0 + threadIdx.x * 8; i < s1; i += step) {
      if (i + 7 < s1) {
        const float4 x0 = *reinterpret_cast<const float4*>(mine + i);
        const float4 x1 = *reinterpret_cast<const float4*>(mine + i + 4);
        *reinterpret_cast<uint4*>(wmine + i) = make_uint4(pack_bf16x2(x0.x, x0.y), pack_bf16x2(x0.z, x0.w),
                                                          pack_bf16x2(x1.x, x1.y), pack_bf16x2(x1.z, x1.w));
      } else {
        for (long e = i; e < s1; ++e) wmine[e] = __float2bfloat16(mine[e]);
      }
    }
  }
  if (!cta_barrier(a, 0, &abort_sh)) return;
  // phase 1: reduce this rank's chunk (fp32 sums in rank order)
  float ss = 0.f;
  {
    long s0, s1;
    sub_range(a, cs, sub, a.rank, s0, s1);
    for (long i = s0 + threadIdx.x * 8; i < s1; i += step) {
      if (i + 7 < s1) {
        uint4 v[W];
#pragma unroll
        for (int p = 0; p < W; ++p) v[p] = __ldcg(reinterpret_cast<const uint4*>(wires[p] + i));
        float acc[8], t[8];
        bf16x8_to_f32(v[0], acc);
#pragma unroll
        for (int p = 1; p < W; ++p) {
          bf16x8_to_f32(v[p], t);
#pragma unroll
          for (int k = 0; k < 8; ++k) acc[k] += t[k];
        }
        uint32_t pk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) pk[k] = pack_bf16x2(acc[2 * k] * a.scale, acc[2 * k + 1] * a.scale);
        const uint4 out = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(wmine + i) = out;
        float r[8];
        bf16x8_to_f32(out, r);
        *reinterpret_cast<float4*>(mine + i) = make_float4(r[0], r[1], r[2], r[3]);
        *reinterpret_cast<float4*>(mine + i + 4) = make_float4(r[4], r[5], r[6], r[7]);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += r[k] * r[k];
      } else {
        for (long e = i; e < s1; ++e) {
          float acc = 0.f;
          for (int p = 0; p < W; ++p) acc += __bfloat162float(__ldcg(wires[p] + e));
          const __nv_bfloat16 b = __float2bfloat16(acc * a.scale);
          wmine[e] = b;
          const float r = __bfloat162float(b);
          mine[e] = r;
          ss += r * r;
        }
      }
    }
  }
  if (!cta_barrier(a, 1, &abort_sh)) return;
  // phase 2: the other ranks' reduced chunks
#pragma unroll 1
  for (int p = 0; p < W; ++p) {
    if (p == a.rank) continue;
    long s0, s1;
    sub_range(a, cs, sub, p, s0, s1);
    for (long i = s0 + threadIdx.x * 8; i < s1; i += step) {
      if (i + 7 < s1) {
        float r[8];
        bf16x8_to_f32(__ldcg(reinterpret_cast<const uint4*>(wires[p] + i)), r);
        *reinterpret_cast<float4*>(mine + i) = make_float4(r[0], r[1], r[2], r[3]);
        *reinterpret_cast<float4*>(mine + i + 4) = make_float4(r[4], r[5], r[6], r[7]);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += r[k] * r[k];
      } else {
        for (long e = i; e < s1; ++e) {
          const float r = __bfloat162float(__ldcg(wires[p] + e));
          mine[e] = r;
          ss += r * r;
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

// wires_dev: device array of W bf16 wire buffers (symmetric; same indexing as the fp32
// gradient buffers).  ``lo`` must be a multiple of 8 elements.
void fused_allreduce_bf16(int64_t ptrs_dev, int64_t wires_dev, int64_t pads_dev, int64_t pad_words, int64_t lo,
                          int64_t hi, int64_t rank, int64_t world, int64_t epoch, double scale, at::Tensor sumsq,
                          int64_t ctas, int64_t epoch_base) {
  TORCH_CHECK(sumsq.is_cuda() && sumsq.scalar_type() == at::kFloat);
  TORCH_CHECK(lo % 8 == 0, "fused_allreduce_bf16: bucket start must be a multiple of 8 elements");
  TORCH_CHECK(3 * ctas * world <= pad_words, "fused_allreduce_bf16: signal pad too small for ", ctas, " CTAs");
  const c10::cuda::CUDAGuard guard(sumsq.device());
  ArArgs a{};
  a.ptrs = reinterpret_cast<float* const*>(ptrs_dev);
  a.pads = reinterpret_cast<uint32_t* const*>(pads_dev);
  a.lo = lo;
  a.hi = hi;
  a.rank = (int)rank;
  a.world = (int)world;
  a.epoch = static_cast<uint32_t>(epoch);
  a.epoch_base = reinterpret_cast<const uint32_t*>(epoch_base);
  a.scale = (float)scale;
  a.sumsq = sumsq.data_ptr<float>();
  a.status = status_ptr(sumsq.device().index());
  auto wires = reinterpret_cast<__nv_bfloat16* const*>(wires_dev);
  auto st = at::cuda::getCurrentCUDAStream();
  switch (world) {
#define PB_AR16(w) \
  case w: fused_allreduce_bf16_kernel<w><<<pb::smem_max(fused_allreduce_bf16_kernel<w>, (int)ctas), kCommThreads, 0, st>>>(a, wires); break;
    PB_AR16(2) PB_AR16(3) PB_AR16(4) PB_AR16(5) PB_AR16(6) PB_AR16(7) PB_AR16(8)
#undef PB_AR16
    default: TORCH_CHECK(false, "fused_allreduce_bf16: world size 2..8 on one node");
  }
  PB_CUDA_CHECK(cudaGetLastError());
}

__global__ void epoch_bump_kernel(uint32_t* base, uint32_t inc) { *base += inc; }

// Adds ``inc`` to the device epoch base (stream-ordered, capturable in a CUDA graph).
void epoch_bump(at::Tensor base, int64_t inc) {
  TORCH_CHECK(base.is_cuda() && base.scalar_type() == at::kInt && base.numel() >= 1, "epoch_bump: int32 CUDA tensor");
  const c10::cuda::CUDAGuard guard(base.device());
  epoch_bump_kernel<<<pb::smem_max(epoch_bump_kernel, 1), 1, 0, at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<uint32_t*>(base.data_ptr()),
                                                                     static_cast<uint32_t>(inc));
  PB_CUDA_CHECK(cudaGetLastError());
}

void comm_bindings(pybind11::module& m) {
  m.def("epoch_bump", &epoch_bump);
  m.def("fused_allreduce", &fused_allreduce);
  m.def("fused_allreduce_bf16", &fused_allreduce_bf16);
  m.def("nvls_allreduce", &nvls_allreduce);
}

}  // namespace pb
