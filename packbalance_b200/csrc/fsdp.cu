// Sharded data parallelism (FSDP) over NVSwitch peer memory (sm_100a).
//
// Layout (built by packbalance_b200/parallel/sharded.py).  A sharded unit (one decoder
// layer's projections, the embedding, the LM head) covers gathered coordinates
// [unit0, unit0 + W * cs); rank p owns [unit0 + p * cs, unit0 + (p + 1) * cs) and keeps
// the fp32 master, Adam moments, reduced gradient and bf16 copy ("owned") of that chunk
// at offset soff + (e - unit0 - p * cs) of its shard buffers (soff is the same on every
// rank; master and owned are symmetric memory).  Gradients live in symmetric fp32
// buffers (fixed places and rotating per-layer windows); the gathered bf16 weights in
// local storage that the fetches of ag_copy.cuh fill from the owners' bf16 chunks.
// RMSNorm weights are few and small: they stay replicated in fp32 and their gradient
// is averaged with the fused all-reduce (comm.cu).
//
// Kernels:
//   fsdp_reduce_scatter   rank r sums chunk r of a unit's gradient over all ranks (W
//                         16-byte peer loads in flight per position), scales by 1/W,
//                         writes the shard gradient and adds its squared norm to a
//                         device accumulator.  Issued per unit as soon as the backward
//                         pass has finished the unit, on the communication stream.
//                         With an NVLink multicast object over the gradient buffers the
//                         sum is one multimem.ld_reduce per 16 bytes, done in the switch.
//   fsdp_adamw            the step's last reduce-scatter (the embedding unit, finished
//                         last) fused with the optimizer: barrier, reduce-scatter, the
//                         squared norms of all ranks' shards exchanged through peer
//                         memory, clip coefficient, AdamW over the whole shard and the
//                         replicated norms, bf16 copy of the updated shard written into
//                         this rank's owned buffer, closing barrier (no rank fetches a
//                         chunk before its owner has written it).
//                         Cooperative launch: the CTAs wait for one another once.
//   fsdp_embedding_fwd    the embedding lookup reads each token's row straight from
//                         the owners' fp32 master shards, so the table is never gathered
//                         for the lookup.
//   fsdp_all_gather       the copy-warp role of ag_copy.cuh as a kernel of its own, for
//                         consumers that are not a GEMM.
// Every wait is bounded; a timeout records status 4xx and the kernel returns.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "ag_copy.cuh"
#include "comm_common.cuh"
#include "common.cuh"
#include "host_utils.h"

namespace pb {

struct OptSeg {  // one contiguous span of the optimizer's domain
  float* p;
  float* m;
  float* v;
  const float* g;
  __nv_bfloat16* out;  // bf16 copy of the updated values (nullptr: none)
  long n;              // multiple of 4
};

// Chunk [c0, c1) of the gradient summed over all ranks, scaled, into out[0 .. c1 - c0).
// This CTA takes its own sub-range (same split on every rank).  Returns the CTA-local
// squared norm contribution of this thread.
template <int W>
__device__ __forceinline__ float rs_chunk(float* const* ptrs, long c0, long c1, float* out, float scale) {
  const long n = c1 - c0;
  const long sub = ((n + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
  const long s0 = min(c0 + static_cast<long>(blockIdx.x) * sub, c1);
  const long s1 = min(s0 + sub, c1);
  constexpr int G = W <= 4 ? 2 : 1;  // G W <= 8 loads of 16 bytes in flight per thread
  float ss = 0.f;
  const long stride = static_cast<long>(blockDim.x) * 4;
  for (long i = s0 + threadIdx.x * 4; i < s1; i += G * stride) {
    float4 v[G][W];
#pragma unroll
    for (int u = 0; u < G; ++u)
#pragma unroll
      for (int p = 0; p < W; ++p)
        if (i + u * stride < s1) v[u][p] = __ldcg(reinterpret_cast<const float4*>(ptrs[p] + i + u * stride));
#pragma unroll
    for (int u = 0; u < G; ++u) {
      const long j = i + u * stride;
      if (j < s1) {
        float4 acc = v[u][0];
#pragma unroll
        for (int p = 1; p < W; ++p) {
          acc.x += v[u][p].x;
          acc.y += v[u][p].y;
          acc.z += v[u][p].z;
          acc.w += v[u][p].w;
        }
        acc.x *= scale;
        acc.y *= scale;
        acc.z *= scale;
        acc.w *= scale;
        *reinterpret_cast<float4*>(out + (j - c0)) = acc;
        ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
      }
    }
  }
  return ss;
}

// Same as rs_chunk, with the sum done in the NVSwitch: one multimem.ld_reduce per 16
// bytes over the gradient buffer's multicast address.
__device__ __forceinline__ float rs_chunk_mc(const float* mc, long c0, long c1, float* out, float scale) {
  const long n = c1 - c0;
  const long sub = ((n + gridDim.x - 1) / gridDim.x + 3) / 4 * 4;
  const long s0 = min(c0 + static_cast<long>(blockIdx.x) * sub, c1);
  const long s1 = min(s0 + sub, c1);
  // eight 16-byte multimem loads in flight per thread (narrow launches beside compute)
  constexpr int U = 8;
  float ss = 0.f;
  const long stride = static_cast<long>(blockDim.x) * 4;
  for (long i = s0 + threadIdx.x * 4; i < s1; i += U * stride) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i + u * stride < s1) v[u] = mm_ld_reduce(mc + i + u * stride);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const long j = i + u * stride;
      if (j < s1) {
        float4 acc = v[u];
        acc.x *= scale;
        acc.y *= scale;
        acc.z *= scale;
        acc.w *= scale;
        *reinterpret_cast<float4*>(out + (j - c0)) = acc;
        ss += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
      }
    }
  }
  return ss;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
  if (threadIdx.x < 32) t = warp_sum(t);
  return t;  // valid in thread 0
}

template <int W>
__global__ void __launch_bounds__(kCommThreads, kCommMinBlocks) fsdp_reduce_scatter_kernel(const ArArgs a, float* out,
                                                                                          const float* mc) {
  __shared__ volatile int abort_sh;
  __shared__ float red[32];
  if (threadIdx.x == 0) abort_sh = 0;
  __syncthreads();
  if (!cta_barrier(a, 0, &abort_sh)) return;
  const float ss = mc != nullptr ? rs_chunk_mc(mc, a.lo, a.hi, out, a.scale) : rs_chunk<W>(a.ptrs, a.lo, a.hi, out, a.scale);
  const float t = block_sum(ss, red);
  if (threadIdx.x == 0) atomicAdd(a.sumsq, t);
}

struct FinalArgs {
  ArArgs a;                // peers' gradient buffers + sync pads; lo/hi: last unit's chunk
  const float* mc;         // multicast address of the gradient buffer (NVLS), or null
  float* rs_out;           // shard gradient of that chunk
  const float* rep_sumsq;  // squared norm of the replicated (already averaged) grads, or null
  float* const* xchg;      // [W] every rank's exchange slots (W floats each)
  unsigned* arrive;        // arrival counter of this GPU's CTAs (never reset)
  unsigned arrive_target;
  uint32_t* go;            // this GPU: epoch once the global norm is published
  float* norm_out;
  int* skipped;
  const OptSeg* segs;
  int nseg;
  float lr, b1, b2, eps, wd, bc1, bc2, max_norm;
};

__device__ __forceinline__ bool spin_until(const uint32_t* p, uint32_t target, int* status, int code) {
  const uint64_t t0 = globaltimer();
  while (static_cast<int>(ld_acquire_gpu(p) - target) < 0) {
    if (globaltimer() - t0 > PB_WAIT_TIMEOUT_NS / 2) {
      report_error(status, code);
      return false;
    }
  }
  return true;
}

template <int W>
__global__ void __launch_bounds__(512) fsdp_adamw_kernel(const FinalArgs f) {
  __shared__ volatile int abort_sh;
  __shared__ float red[32];
  __shared__ float norm_sh;
  __shared__ int go_ok;
  const ArArgs& a = f.a;
  if (threadIdx.x == 0) abort_sh = 0;
  __syncthreads();
  // 0: every rank has finished its backward pass and its earlier reduce-scatters.
  if (!cta_barrier(a, 0, &abort_sh)) return;
  float ss = 0.f;
  if (a.hi > a.lo)
    ss = f.mc != nullptr ? rs_chunk_mc(f.mc, a.lo, a.hi, f.rs_out, a.scale) : rs_chunk<W>(a.ptrs, a.lo, a.hi, f.rs_out, a.scale);
  const float t = block_sum(ss, red);
  if (threadIdx.x == 0) {
    if (t != 0.f) atomicAdd(a.sumsq, t);
    __threadfence();
    atomicAdd(f.arrive, 1u);
  }
  // 1: CTA 0 collects this GPU's total, exchanges it with the peers, publishes the norm.
  if (blockIdx.x == 0) {
    if (threadIdx.x == 0) {
      bool ok = spin_until(reinterpret_cast<const uint32_t*>(f.arrive), f.arrive_target, a.status, 402);
      const float mine = ok ? *reinterpret_cast<volatile float*>(a.sumsq) : __int_as_float(0x7fc00000);
      for (int p = 0; p < W; ++p) reinterpret_cast<volatile float*>(f.xchg[p])[a.rank] = mine;
    }
    const bool ok = cta_barrier(a, 1, &abort_sh);
    if (threadIdx.x == 0) {
      float tot = f.rep_sumsq != nullptr ? *f.rep_sumsq : 0.f;
      const volatile float* x = f.xchg[a.rank];
      for (int p = 0; p < W; ++p) tot += x[p];
      const float nv = ok ? sqrtf(tot) : __int_as_float(0x7fc00000);
      *f.norm_out = nv;
      *f.skipped = isfinite(nv) ? 0 : 1;
      __threadfence();
      st_release_gpu(f.go, launch_epoch(a));
    }
  }
  if (threadIdx.x == 0) {
    go_ok = spin_until(f.go, launch_epoch(a), a.status, 403) ? 1 : 0;
    norm_sh = *reinterpret_cast<volatile float*>(f.norm_out);
  }
  __syncthreads();
  const float nv = norm_sh;
  if (go_ok && isfinite(nv)) {
    const float gs = f.max_norm > 0.f ? fminf(1.f, f.max_norm / (nv + 1e-6f)) : 1.f;
    const float step = f.lr / f.bc1;
    const float inv_sqrt_bc2 = rsqrtf(f.bc2);
    const float decay = 1.f - f.lr * f.wd;
    const long tid = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const long nthreads = static_cast<long>(gridDim.x) * blockDim.x;
    for (int s = 0; s < f.nseg; ++s) {
      const OptSeg sg = f.segs[s];
      for (long i = tid; i < sg.n / 4; i += nthreads) {
        float4 pv = reinterpret_cast<float4*>(sg.p)[i];
        const float4 gv = reinterpret_cast<const float4*>(sg.g)[i];
        float4 mv = reinterpret_cast<float4*>(sg.m)[i];
        float4 vv = reinterpret_cast<float4*>(sg.v)[i];
        float* pp = &pv.x;
        const float* gg = &gv.x;
        float* mm = &mv.x;
        float* ww = &vv.x;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float gk = gg[k] * gs;
          mm[k] = f.b1 * mm[k] + (1.f - f.b1) * gk;
          ww[k] = f.b2 * ww[k] + (1.f - f.b2) * gk * gk;
          pp[k] = pp[k] * decay - step * mm[k] / (sqrtf(ww[k]) * inv_sqrt_bc2 + f.eps);
        }
        reinterpret_cast<float4*>(sg.p)[i] = pv;
        reinterpret_cast<float4*>(sg.m)[i] = mv;
        reinterpret_cast<float4*>(sg.v)[i] = vv;
        if (sg.out != nullptr)
          reinterpret_cast<uint2*>(sg.out)[i] = make_uint2(pack_bf16x2(pv.x, pv.y), pack_bf16x2(pv.z, pv.w));
      }
    }
  }
  // 2: this CTA's writes are done on every rank before anyone fetches a chunk.
  cta_barrier(a, 2, &abort_sh);
}

__global__ void fsdp_embedding_kernel(const int64_t* __restrict__ ids, long T, float* const* masters, long row0,
                                      long unit0, long cs, long soff, int d, long vocab, float* __restrict__ out,
                                      int* status) {
  const long row = static_cast<long>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
  if (row >= T) return;
  const int lane = threadIdx.x & 31;
  const int64_t id = ids[row];
  float* o = out + row * d;
  if (id < 0 || id >= vocab) {
    if (lane == 0) report_error(status, 501);
    for (int j = lane * 4; j < d; j += 128) *reinterpret_cast<float4*>(o + j) = make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }
  for (int j = lane * 4; j < d; j += 128) {
    const long e = row0 + id * d + j;
    const int p = static_cast<int>((e - unit0) / cs);
    if (!PB_BOUNDS_OK(p >= 0 && p < kMaxWorld, status, 502)) continue;
    const float* src = masters[p] + soff + (e - unit0 - p * cs);
    *reinterpret_cast<float4*>(o + j) = __ldcg(reinterpret_cast<const float4*>(src));
  }
}

__global__ void __launch_bounds__(128) fsdp_all_gather_kernel(const AgSpec s) { ag_copy_warp(s); }

// ------------------------------------ host ----------------------------------------
static ArArgs make_args(int64_t ptrs_dev, int64_t pads_dev, int64_t lo, int64_t hi, int64_t rank, int64_t world,
                        int64_t epoch, double scale, float* sumsq, int dev) {
  ArArgs a{};
  a.ptrs = reinterpret_cast<float* const*>(ptrs_dev);
  a.pads = reinterpret_cast<uint32_t* const*>(pads_dev);
  a.lo = lo;
  a.hi = hi;
  a.rank = (int)rank;
  a.world = (int)world;
  a.epoch = static_cast<uint32_t>(epoch);
  a.scale = (float)scale;
  a.sumsq = sumsq;
  a.status = status_ptr(dev);
  return a;
}

// ``mc``: multicast address of the gradient buffer (0: peer loads).
void fsdp_reduce_scatter(int64_t gptrs_dev, int64_t pads_dev, int64_t pad_words, int64_t lo, int64_t hi, int64_t out,
                         int64_t rank, int64_t world, int64_t epoch, double scale, at::Tensor sumsq, int64_t ctas,
                         int64_t mc) {
  TORCH_CHECK(sumsq.is_cuda() && sumsq.scalar_type() == at::kFloat, "fsdp_reduce_scatter: fp32 CUDA accumulator");
  TORCH_CHECK(lo % 4 == 0 && hi % 4 == 0 && out % 16 == 0, "fsdp_reduce_scatter: 16-byte aligned chunk");
  TORCH_CHECK(ctas * world <= pad_words, "fsdp_reduce_scatter: sync pad too small");
  const c10::cuda::CUDAGuard guard(sumsq.device());
  const ArArgs a = make_args(gptrs_dev, pads_dev, lo, hi, rank, world, epoch, scale, sumsq.data_ptr<float>(),
                             sumsq.device().index());
  float* o = reinterpret_cast<float*>(out);
  const float* m = reinterpret_cast<const float*>(mc);
  auto st = at::cuda::getCurrentCUDAStream();
  switch (world) {
    case 2: fsdp_reduce_scatter_kernel<2><<<pb::smem_max(fsdp_reduce_scatter_kernel<2>, (int)ctas), kCommThreads, 0, st>>>(a, o, m); break;
    case 3: fsdp_reduce_scatter_kernel<3><<<pb::smem_max(fsdp_reduce_scatter_kernel<3>, (int)ctas), kCommThreads, 0, st>>>(a, o, m); break;
    case 4: fsdp_reduce_scatter_kernel<4><<<pb::smem_max(fsdp_reduce_scatter_kernel<4>, (int)ctas), kCommThreads, 0, st>>>(a, o, m); break;
    case 5: fsdp_reduce_scatter_kernel<5><<<pb::smem_max(fsdp_reduce_scatter_kernel<5>, (int)ctas), kCommThreads, 0, st>>>(a, o, m); break;
    case 6: fsdp_reduce_scatter_kernel<6><<<pb::smem_max(fsdp_reduce_scatter_kernel<6>, (int)ctas), kCommThreads, 0, st>>>(a, o, m); break;
    case 7: fsdp_reduce_scatter_kernel<7><<<pb::smem_max(fsdp_reduce_scatter_kernel<7>, (int)ctas), kCommThreads, 0, st>>>(a, o, m); break;
    case 8: fsdp_reduce_scatter_kernel<8><<<pb::smem_max(fsdp_reduce_scatter_kernel<8>, (int)ctas), kCommThreads, 0, st>>>(a, o, m); break;
    default: TORCH_CHECK(false, "fsdp_reduce_scatter: world size 2..8 on one node");
  }
  PB_CUDA_CHECK(cudaGetLastError());
}

template <int W>
static void launch_final(FinalArgs& f, int ctas, cudaStream_t st) {
  auto kern = fsdp_adamw_kernel<W>;
  void* args[] = {&f};
  PB_CUDA_CHECK(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(kern), pb::smem_max(kern, dim3(ctas)), dim3(512),
                                            args, 0, st));
}

// Largest grid of the cooperative optimizer kernel on this device.
int64_t fsdp_adamw_max_ctas(int64_t world) {
  int per_sm = 0;
  switch (world) {
#define PB_OCC(w) \
  case w: PB_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fsdp_adamw_kernel<w>, 512, 0)); break;
    PB_OCC(2) PB_OCC(3) PB_OCC(4) PB_OCC(5) PB_OCC(6) PB_OCC(7) PB_OCC(8)
#undef PB_OCC
    default: TORCH_CHECK(false, "fsdp_adamw: world size 2..8 on one node");
  }
  int dev = 0;
  PB_CUDA_CHECK(cudaGetDevice(&dev));
  return static_cast<int64_t>(per_sm) * num_sms(dev);
}

// ``p``: {gptrs_dev, pads_dev, pad_words, rank, world, epoch, rs_lo, rs_hi, rs_out,
//         rep_sumsq, xchg_ptrs_dev, arrive, arrive_target, go, segs, nseg, ctas, mc}
// ``h``: {scale, lr, b1, b2, eps, wd, bc1, bc2, max_norm}
void fsdp_adamw(std::vector<int64_t> p, std::vector<double> h, at::Tensor sumsq, at::Tensor norm_out,
                at::Tensor skipped) {
  TORCH_CHECK(p.size() == 18 && h.size() == 9, "fsdp_adamw: argument vectors");
  TORCH_CHECK(sumsq.is_cuda() && norm_out.is_cuda() && skipped.is_cuda(), "fsdp_adamw: CUDA tensors");
  const c10::cuda::CUDAGuard guard(sumsq.device());
  const int64_t world = p[4], ctas = p[16];
  TORCH_CHECK(3 * ctas * world <= p[2], "fsdp_adamw: sync pad too small");
  TORCH_CHECK(p[6] % 4 == 0 && p[7] % 4 == 0 && p[8] % 16 == 0, "fsdp_adamw: 16-byte aligned chunk");
  TORCH_CHECK(ctas >= 1 && ctas <= fsdp_adamw_max_ctas(world), "fsdp_adamw: grid larger than one co-resident wave");
  FinalArgs f{};
  f.a = make_args(p[0], p[1], p[6], p[7], p[3], world, p[5], h[0], sumsq.data_ptr<float>(), sumsq.device().index());
  f.rs_out = reinterpret_cast<float*>(p[8]);
  f.mc = reinterpret_cast<const float*>(p[17]);
  f.rep_sumsq = reinterpret_cast<const float*>(p[9]);
  f.xchg = reinterpret_cast<float* const*>(p[10]);
  f.arrive = reinterpret_cast<unsigned*>(p[11]);
  f.arrive_target = static_cast<unsigned>(p[12]);
  f.go = reinterpret_cast<uint32_t*>(p[13]);
  f.segs = reinterpret_cast<const OptSeg*>(p[14]);
  f.nseg = (int)p[15];
  f.norm_out = norm_out.data_ptr<float>();
  f.skipped = skipped.data_ptr<int>();
  f.lr = (float)h[1];
  f.b1 = (float)h[2];
  f.b2 = (float)h[3];
  f.eps = (float)h[4];
  f.wd = (float)h[5];
  f.bc1 = (float)h[6];
  f.bc2 = (float)h[7];
  f.max_norm = (float)h[8];
  auto st = at::cuda::getCurrentCUDAStream();
  switch (world) {
    case 2: launch_final<2>(f, (int)ctas, st); break;
    case 3: launch_final<3>(f, (int)ctas, st); break;
    case 4: launch_final<4>(f, (int)ctas, st); break;
    case 5: launch_final<5>(f, (int)ctas, st); break;
    case 6: launch_final<6>(f, (int)ctas, st); break;
    case 7: launch_final<7>(f, (int)ctas, st); break;
    case 8: launch_final<8>(f, (int)ctas, st); break;
    default: TORCH_CHECK(false, "fsdp_adamw: world size 2..8 on one node");
  }
}

at::Tensor fsdp_embedding_fwd(at::Tensor ids, int64_t masters_dev, int64_t row0, int64_t unit0, int64_t cs,
                              int64_t soff, int64_t d, int64_t vocab) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == at::kLong && ids.is_contiguous(), "fsdp_embedding_fwd: ids");
  TORCH_CHECK(d % 4 == 0 && (row0 - unit0) % 4 == 0 && cs % 4 == 0 && soff % 4 == 0,
              "fsdp_embedding_fwd: 16-byte aligned rows");
  const c10::cuda::CUDAGuard guard(ids.device());
  const long T = ids.numel();
  auto out = at::empty({T, d}, ids.options().dtype(at::kFloat));
  if (T > 0) {
    fsdp_embedding_kernel<<<pb::smem_max(fsdp_embedding_kernel, (unsigned)((T + 7) / 8)), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        ids.data_ptr<int64_t>(), T, reinterpret_cast<float* const*>(masters_dev), row0, unit0, cs, soff, (int)d, vocab,
        out.data_ptr<float>(), status_ptr(ids.device().index()));
    PB_CUDA_CHECK(cudaGetLastError());
  }
  return out;
}

// ``ag``: the spec of gemm_tc's fused all-gather (b0 unused).
void parse_ag_spec(const std::vector<int64_t>& ag, AgSpec& s);

void fsdp_all_gather(std::vector<int64_t> ag, int64_t ctas) {
  AgSpec s{};
  parse_ag_spec(ag, s);
  if (s.hi <= s.lo) return;
  auto st = at::cuda::getCurrentCUDAStream();
  const long nblocks = (s.hi - s.lo + (1L << s.block_shift) - 1) >> s.block_shift;
  PB_CUDA_CHECK(cudaMemsetAsync(s.counters, 0, sizeof(uint32_t) * (1 + nblocks), st));
  fsdp_all_gather_kernel<<<pb::smem_max(fsdp_all_gather_kernel, (int)ctas), 128, 0, st>>>(s);
  PB_CUDA_CHECK(cudaGetLastError());
}

void fsdp_bindings(pybind11::module& m) {
  m.def("fsdp_reduce_scatter", &fsdp_reduce_scatter);
  m.def("fsdp_adamw", &fsdp_adamw);
  m.def("fsdp_adamw_max_ctas", &fsdp_adamw_max_ctas);
  m.def("fsdp_embedding_fwd", &fsdp_embedding_fwd);
  m.def("fsdp_all_gather", &fsdp_all_gather);
}

}  // namespace pb
