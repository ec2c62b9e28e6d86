// Memory-bound kernels of the training step (sm_100a): RMSNorm forward/backward,
// SwiGLU forward/backward on separate tensors, in-place RoPE (forward or inverse),
// embedding gather / scatter-add, the LM-head CE row reduction, the flat-buffer
// AdamW update, and a squared L2 norm.  All use 16-byte vector accesses; none
// allocates memory.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <ATen/ATen.h>

#include "ce_kernels.cuh"
#include "common.cuh"
#include "host_utils.h"

namespace pb {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// ------------------------------- RMSNorm ------------------------------------------
// Vector helpers: 4 consecutive elements as fp32.
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void st4(__nv_bfloat16* p, float4 v) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

// One warp per row (n % 4 == 0).  x = x_prev (+ delta); y = x * rstd * w with
// rstd = 1/sqrt(mean(x^2) + eps).  ``x_out`` receives x when a delta is added.
template <typename TI, typename TO>
__global__ void add_rmsnorm_kernel(const TI* __restrict__ xp, const __nv_bfloat16* __restrict__ delta,
                                   const float* __restrict__ w, float* __restrict__ x_out, TO* __restrict__ y,
                                   float* __restrict__ rstd, int rows, int n, float eps) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (row >= rows) return;
  const long off = static_cast<long>(row) * n;
  float ss = 0.f;
  for (int c = lane * 4; c < n; c += 128) {
    float4 v = ld4(xp + off + c);
    if (delta != nullptr) {
      const float4 d = ld4(delta + off + c);
      v.x += d.x; v.y += d.y; v.z += d.z; v.w += d.w;
      st4(x_out + off + c, v);
    }
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / n + eps);
  if (lane == 0) rstd[row] = r;
  __syncwarp();
  for (int c = lane * 4; c < n; c += 128) {
    float4 v = delta != nullptr ? ld4(x_out + off + c) : ld4(xp + off + c);
    const float4 g = ld4(w + c);
    st4(y + off + c, make_float4(v.x * r * g.x, v.y * r * g.y, v.z * r * g.z, v.w * r * g.w));
  }
}

// dx = rstd * (g - xhat * mean(g * xhat)) [+ dres], g = dy * w.  Each warp keeps its
// own dw partial row in shared memory (lane-owned columns: no atomics, no bank
// conflicts); the block's partial is added to dw_out with one atomic per column.
template <typename TI, typename TD>
__global__ void rmsnorm_bwd_kernel(const TD* __restrict__ dy, const TI* __restrict__ x, const float* __restrict__ w,
                                   const float* __restrict__ rstd, const float* __restrict__ dres,
                                   float* __restrict__ dx, __nv_bfloat16* __restrict__ dx_bf16,
                                   float* __restrict__ dw_out, int rows, int n, float* __restrict__ dw_part) {
  extern __shared__ float sdw[];  // [warps][n]
  const int warps = blockDim.x / 32;
  const int wid = threadIdx.x / 32, lane = threadIdx.x % 32;
  float* mine = sdw + static_cast<long>(wid) * n;
  for (int c = lane * 4; c < n; c += 128) st4(mine + c, make_float4(0.f, 0.f, 0.f, 0.f));
  for (int row = blockIdx.x * warps + wid; row < rows; row += gridDim.x * warps) {
    const long off = static_cast<long>(row) * n;
    const float r = rstd[row];
    float dot = 0.f;
    for (int c = lane * 4; c < n; c += 128) {
      const float4 g = ld4(dy + off + c), xv = ld4(x + off + c), wv = ld4(w + c);
      dot += g.x * wv.x * xv.x + g.y * wv.y * xv.y + g.z * wv.z * xv.z + g.w * wv.w * xv.w;
    }
    dot = warp_sum(dot) * r / n;
    for (int c = lane * 4; c < n; c += 128) {
      const float4 g = ld4(dy + off + c), xv = ld4(x + off + c), wv = ld4(w + c);
      float4 d = make_float4(r * (g.x * wv.x - xv.x * r * dot), r * (g.y * wv.y - xv.y * r * dot),
                             r * (g.z * wv.z - xv.z * r * dot), r * (g.w * wv.w - xv.w * r * dot));
      if (dres != nullptr) {
        const float4 e = ld4(dres + off + c);
        d.x += e.x; d.y += e.y; d.z += e.z; d.w += e.w;
      }
      st4(dx + off + c, d);
      if (dx_bf16 != nullptr) st4(dx_bf16 + off + c, d);
      float4 p = ld4(mine + c);
      p.x += g.x * xv.x * r; p.y += g.y * xv.y * r; p.z += g.z * xv.z * r; p.w += g.w * xv.w * r;
      st4(mine + c, p);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < n; c += blockDim.x) {
    float t = 0.f;
    for (int k = 0; k < warps; ++k) t += sdw[static_cast<long>(k) * n + c];
    if (dw_part != nullptr) dw_part[static_cast<long>(blockIdx.x) * n + c] = t;  // summed in block order later
    else atomicAdd(dw_out + c, t);
  }
}

// Register-resident variants for n = 128 * CH (the common model widths): each warp
// holds its row in registers, so x (and dy, dres) are read from HBM exactly once and
// all loads of a row are issued before the first reduction; rows are strided over a
// persistent grid.  The backward keeps each lane's dw partial (4 CH columns) in
// registers across the warp's rows.
template <int CH, typename TI, typename TO>
__global__ void __launch_bounds__(256) add_rmsnorm_reg_kernel(const TI* __restrict__ xp,
                                                               const __nv_bfloat16* __restrict__ delta,
                                                               const float* __restrict__ w, float* __restrict__ x_out,
                                                               TO* __restrict__ y, float* __restrict__ rstd, int rows,
                                                               float eps) {
  constexpr int n = 128 * CH;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x / 32;
  for (int row = blockIdx.x * warps + threadIdx.x / 32; row < rows; row += gridDim.x * warps) {
    const long off = static_cast<long>(row) * n;
    float4 v[CH];
#pragma unroll
    for (int k = 0; k < CH; ++k) v[k] = ld4(xp + off + lane * 4 + k * 128);
    if (delta != nullptr) {
#pragma unroll
      for (int k = 0; k < CH; ++k) {
        const float4 d = ld4(delta + off + lane * 4 + k * 128);
        v[k].x += d.x; v[k].y += d.y; v[k].z += d.z; v[k].w += d.w;
        st4(x_out + off + lane * 4 + k * 128, v[k]);
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < CH; ++k) ss += v[k].x * v[k].x + v[k].y * v[k].y + v[k].z * v[k].z + v[k].w * v[k].w;
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / n + eps);
    if (lane == 0) rstd[row] = r;
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const float4 g = ld4(w + lane * 4 + k * 128);
      st4(y + off + lane * 4 + k * 128, make_float4(v[k].x * r * g.x, v[k].y * r * g.y, v[k].z * r * g.z, v[k].w * r * g.w));
    }
  }
}

template <int CH, typename TI, typename TD>
__global__ void __launch_bounds__(256) rmsnorm_bwd_reg_kernel(const TD* __restrict__ dy, const TI* __restrict__ x,
                                                               const float* __restrict__ w,
                                                               const float* __restrict__ rstd,
                                                               const float* __restrict__ dres, float* __restrict__ dx,
                                                               __nv_bfloat16* __restrict__ dx_bf16,
                                                               float* __restrict__ dw_out, int rows,
                                                               float* __restrict__ dw_part) {
  constexpr int n = 128 * CH;
  __shared__ float sdw[8][n];
  const int lane = threadIdx.x & 31, wid = threadIdx.x / 32;
  const int warps = blockDim.x / 32;
  float4 acc[CH];
#pragma unroll
  for (int k = 0; k < CH; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int row = blockIdx.x * warps + wid; row < rows; row += gridDim.x * warps) {
    const long off = static_cast<long>(row) * n;
    float4 g[CH], xv[CH], e[CH];
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      g[k] = ld4(dy + off + lane * 4 + k * 128);
      xv[k] = ld4(x + off + lane * 4 + k * 128);
    }
    if (dres != nullptr) {
#pragma unroll
      for (int k = 0; k < CH; ++k) e[k] = ld4(dres + off + lane * 4 + k * 128);
    }
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const float4 wv = ld4(w + lane * 4 + k * 128);
      dot += g[k].x * wv.x * xv[k].x + g[k].y * wv.y * xv[k].y + g[k].z * wv.z * xv[k].z + g[k].w * wv.w * xv[k].w;
    }
    dot = warp_sum(dot) * r / n;
#pragma unroll
    for (int k = 0; k < CH; ++k) {
      const float4 wv = ld4(w + lane * 4 + k * 128);
      float4 d = make_float4(r * (g[k].x * wv.x - xv[k].x * r * dot), r * (g[k].y * wv.y - xv[k].y * r * dot),
                             r * (g[k].z * wv.z - xv[k].z * r * dot), r * (g[k].w * wv.w - xv[k].w * r * dot));
      if (dres != nullptr) {
        d.x += e[k].x; d.y += e[k].y; d.z += e[k].z; d.w += e[k].w;
      }
      st4(dx + off + lane * 4 + k * 128, d);
      if (dx_bf16 != nullptr) st4(dx_bf16 + off + lane * 4 + k * 128, d);
      acc[k].x += g[k].x * xv[k].x * r;
      acc[k].y += g[k].y * xv[k].y * r;
      acc[k].z += g[k].z * xv[k].z * r;
      acc[k].w += g[k].w * xv[k].w * r;
    }
  }
#pragma unroll
  for (int k = 0; k < CH; ++k) st4(&sdw[wid][lane * 4 + k * 128], acc[k]);
  __syncthreads();
  for (int c = threadIdx.x; c < n; c += blockDim.x) {
    float t = 0.f;
    for (int q = 0; q < warps; ++q) t += sdw[q][c];
    if (dw_part != nullptr) dw_part[static_cast<long>(blockIdx.x) * n + c] = t;  // summed in block order later
    else atomicAdd(dw_out + c, t);
  }
}

// Deterministic mode: dw_out[c] (+)= sum over blocks b = 0, 1, ... of part[b, c], always in
// that order.
__global__ void dw_reduce_kernel(const float* __restrict__ part, int blocks, int n, float* __restrict__ dw_out) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += gridDim.x * blockDim.x) {
    float t = 0.f;
    for (int b = 0; b < blocks; ++b) t += part[static_cast<long>(b) * n + c];
    dw_out[c] += t;
  }
}

// Reductions whose order depends on scheduling (fp32 atomics) are replaced, while this is
// set, by ones with a fixed order: RMSNorm dw through per-block partials summed in block
// order, the embedding gradient through a stable sort of the token ids.
static bool g_deterministic = false;

bool set_deterministic(bool on) {
  const bool prev = g_deterministic;
  g_deterministic = on;
  return prev;
}

std::vector<at::Tensor> add_rmsnorm_fwd(at::Tensor x, c10::optional<at::Tensor> delta, at::Tensor w, double eps,
                                        bool out_bf16) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && w.is_contiguous() && w.scalar_type() == at::kFloat);
  const c10::cuda::CUDAGuard guard(x.device());
  const int n = x.size(-1);
  TORCH_CHECK(n % 4 == 0, "rmsnorm: feature dim must be a multiple of 4");
  const int rows = x.numel() / n;
  auto y = at::empty(x.sizes(), x.options().dtype(out_bf16 ? at::kBFloat16 : x.scalar_type()));
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor xo = x;
  const __nv_bfloat16* dp = nullptr;
  if (delta.has_value()) {
    TORCH_CHECK(x.scalar_type() == at::kFloat && delta->scalar_type() == at::kBFloat16 && delta->is_contiguous() &&
                    delta->numel() == x.numel(),
                "add_rmsnorm: fp32 x and bf16 delta of the same shape");
    xo = at::empty_like(x);
    dp = reinterpret_cast<const __nv_bfloat16*>(delta->data_ptr());
  }
  if (rows == 0) return {xo, y, rstd};
  const int warps = 8;
  dim3 grid((rows + warps - 1) / warps);
  auto s = at::cuda::getCurrentCUDAStream();
  float* xop = delta.has_value() ? xo.data_ptr<float>() : nullptr;
  if (x.scalar_type() == at::kFloat && out_bf16 && n % 128 == 0 && n / 128 <= 32) {
    const int g2 = std::min<int>((rows + warps - 1) / warps, 4 * num_sms(x.device().index()));
    const float* xp = x.data_ptr<float>();
    auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr());
    bool done = true;
    switch (n / 128) {
#define PB_FWD_CH(C) \
  case C: add_rmsnorm_reg_kernel<C, float, __nv_bfloat16><<<g2, 256, 0, s>>>(xp, dp, w.data_ptr<float>(), xop, yp, rstd.data_ptr<float>(), rows, (float)eps); break;
      PB_FWD_CH(2) PB_FWD_CH(4) PB_FWD_CH(6) PB_FWD_CH(8) PB_FWD_CH(12) PB_FWD_CH(16) PB_FWD_CH(32)
#undef PB_FWD_CH
      default: done = false;
    }
    if (done) {
      PB_CUDA_CHECK(cudaGetLastError());
      return {xo, y, rstd};
    }
  }
  if (x.scalar_type() == at::kFloat) {
    if (out_bf16)
      add_rmsnorm_kernel<float, __nv_bfloat16><<<grid, warps * 32, 0, s>>>(
          x.data_ptr<float>(), dp, w.data_ptr<float>(), xop, reinterpret_cast<__nv_bfloat16*>(y.data_ptr()),
          rstd.data_ptr<float>(), rows, n, (float)eps);
    else
      add_rmsnorm_kernel<float, float><<<grid, warps * 32, 0, s>>>(x.data_ptr<float>(), dp, w.data_ptr<float>(), xop,
                                                                   y.data_ptr<float>(), rstd.data_ptr<float>(), rows,
                                                                   n, (float)eps);
  } else {
    TORCH_CHECK(x.scalar_type() == at::kBFloat16 && !delta.has_value(), "rmsnorm: fp32 or bf16 input");
    add_rmsnorm_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, warps * 32, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), nullptr, w.data_ptr<float>(), nullptr,
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), rstd.data_ptr<float>(), rows, n, (float)eps);
  }
  PB_CUDA_CHECK(cudaGetLastError());
  return {xo, y, rstd};
}

std::vector<at::Tensor> rmsnorm_fwd(at::Tensor x, at::Tensor w, double eps, bool out_bf16) {
  auto r = add_rmsnorm_fwd(x, c10::nullopt, w, eps, out_bf16);
  return {r[1], r[2]};
}

// Returns dx (fp32).  dw is written (or accumulated) into ``dw_out``.
at::Tensor rmsnorm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, c10::optional<at::Tensor> dres,
                       c10::optional<at::Tensor> dx_bf16, at::Tensor dw_out, bool accumulate_dw) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dy.numel() == x.numel());
  const c10::cuda::CUDAGuard guard(x.device());
  const int n = x.size(-1);
  TORCH_CHECK(n % 4 == 0, "rmsnorm: feature dim must be a multiple of 4");
  const int rows = x.numel() / n;
  auto dx = at::empty(x.sizes(), x.options().dtype(at::kFloat));
  auto s = at::cuda::getCurrentCUDAStream();
  if (!accumulate_dw) PB_CUDA_CHECK(cudaMemsetAsync(dw_out.data_ptr(), 0, n * sizeof(float), s));
  if (rows == 0) return dx;
  // deterministic mode: per-block dw partials, then one ordered sum (dw_reduce_kernel)
  auto reduce_parts = [&](const at::Tensor& part, int blocks) {
    dw_reduce_kernel<<<(n + 255) / 256, 256, 0, s>>>(part.data_ptr<float>(), blocks, n, dw_out.data_ptr<float>());
  };
  if (x.scalar_type() == at::kFloat && dy.scalar_type() == at::kFloat && n % 128 == 0 && n / 128 <= 8) {
    // one persistent wave: 1 CTA of 8 warps per SM for CH >= 6 (register-bound), else 2
    const int g2 = std::min<int>((rows + 7) / 8, (n / 128 >= 6 ? 1 : 2) * num_sms(x.device().index()));
    const float* dres_q = dres.has_value() ? dres->data_ptr<float>() : nullptr;
    __nv_bfloat16* dxq = dx_bf16.has_value() ? reinterpret_cast<__nv_bfloat16*>(dx_bf16->data_ptr()) : nullptr;
    at::Tensor part;
    if (g_deterministic) part = at::empty({g2, n}, x.options().dtype(at::kFloat));
    float* pp = g_deterministic ? part.data_ptr<float>() : nullptr;
    bool done = true;
    switch (n / 128) {
#define PB_BWD_CH(C) \
  case C: rmsnorm_bwd_reg_kernel<C, float, float><<<g2, 256, 0, s>>>(dy.data_ptr<float>(), x.data_ptr<float>(), w.data_ptr<float>(), rstd.data_ptr<float>(), dres_q, dx.data_ptr<float>(), dxq, dw_out.data_ptr<float>(), rows, pp); break;
      PB_BWD_CH(2) PB_BWD_CH(4) PB_BWD_CH(6) PB_BWD_CH(8)
#undef PB_BWD_CH
      default: done = false;
    }
    if (done) {
      if (g_deterministic) reduce_parts(part, g2);
      PB_CUDA_CHECK(cudaGetLastError());
      return dx;
    }
  }
  const int warps = 4;
  const int nb = std::min((rows + warps - 1) / warps, 2 * num_sms(x.device().index()));
  const float* dres_p = dres.has_value() ? dres->data_ptr<float>() : nullptr;
  __nv_bfloat16* dxb = dx_bf16.has_value() ? reinterpret_cast<__nv_bfloat16*>(dx_bf16->data_ptr()) : nullptr;
  const size_t smem = static_cast<size_t>(warps) * n * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "rmsnorm_bwd: feature dim too large");
  at::Tensor part;
  if (g_deterministic) part = at::empty({nb, n}, x.options().dtype(at::kFloat));
  float* pp = g_deterministic ? part.data_ptr<float>() : nullptr;
#define PB_RMS_BWD(TI, TD)                                                                                    \
  do {                                                                                                        \
    auto k = rmsnorm_bwd_kernel<TI, TD>;                                                                      \
    if (smem > 48 * 1024) PB_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)); \
    k<<<nb, warps * 32, smem, s>>>(reinterpret_cast<const TD*>(dy.data_ptr()), reinterpret_cast<const TI*>(x.data_ptr()), \
                                   w.data_ptr<float>(), rstd.data_ptr<float>(), dres_p, dx.data_ptr<float>(), dxb,      \
                                   dw_out.data_ptr<float>(), rows, n, pp);                                    \
  } while (0)
  const bool xf = x.scalar_type() == at::kFloat, df = dy.scalar_type() == at::kFloat;
  if (xf && df) PB_RMS_BWD(float, float);
  else if (xf && !df) PB_RMS_BWD(float, __nv_bfloat16);
  else if (!xf && df) PB_RMS_BWD(__nv_bfloat16, float);
  else PB_RMS_BWD(__nv_bfloat16, __nv_bfloat16);
#undef PB_RMS_BWD
  if (g_deterministic) reduce_parts(part, nb);
  PB_CUDA_CHECK(cudaGetLastError());
  return dx;
}

// SwiGLU backward on the packed layout: gu = [g | u] (bf16 [M, 2F]), dh (bf16 [M, F])
// -> dgu = [dg | du] (bf16 [M, 2F]).  8 elements per thread.
__global__ void swiglu_bwd_packed_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ gu,
                                         __nv_bfloat16* __restrict__ dgu, long rows, int F) {
  const int f8 = F / 8;
  const long total = rows * f8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long r = i / f8;
    const int c = static_cast<int>(i % f8) * 8;
    const uint4 hv = *reinterpret_cast<const uint4*>(dh + r * F + c);
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + r * 2 * F + c);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + r * 2 * F + F + c);
    const uint32_t* hp = &hv.x;
    const uint32_t* gp = &gv.x;
    const uint32_t* up = &uv.x;
    uint32_t dgo[4], duo[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 d = unpack_bf16x2(hp[k]), g = unpack_bf16x2(gp[k]), u = unpack_bf16x2(up[k]);
      const float s0 = sigmoidf_(g.x), s1 = sigmoidf_(g.y);
      dgo[k] = pack_bf16x2(d.x * u.x * s0 * (1.f + g.x * (1.f - s0)), d.y * u.y * s1 * (1.f + g.y * (1.f - s1)));
      duo[k] = pack_bf16x2(d.x * g.x * s0, d.y * g.y * s1);
    }
    *reinterpret_cast<uint4*>(dgu + r * 2 * F + c) = make_uint4(dgo[0], dgo[1], dgo[2], dgo[3]);
    *reinterpret_cast<uint4*>(dgu + r * 2 * F + F + c) = make_uint4(duo[0], duo[1], duo[2], duo[3]);
  }
}

void swiglu_bwd_packed(at::Tensor dh, at::Tensor gu, at::Tensor dgu) {
  TORCH_CHECK(dh.is_contiguous() && gu.is_contiguous() && dgu.is_contiguous());
  const c10::cuda::CUDAGuard guard(dh.device());
  const long rows = dh.size(0);
  const int F = dh.size(1);
  TORCH_CHECK(F % 8 == 0 && gu.size(1) == 2 * F && dgu.size(1) == 2 * F);
  const long total = rows * (F / 8);
  if (total == 0) return;
  swiglu_bwd_packed_kernel<<<(int)std::min<long>((total + 255) / 256, 16L * num_sms(dh.device().index())), 256, 0,
                             at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(gu.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(dgu.data_ptr()), rows, F);
  PB_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------- SwiGLU -------------------------------------------
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ h, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float gv = to_f(g[i]);
    h[i] = from_f<T>(gv * sigmoidf_(gv) * to_f(u[i]));
  }
}
template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ g, const T* __restrict__ u, const T* __restrict__ dh,
                                  T* __restrict__ dg, T* __restrict__ du, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float gv = to_f(g[i]), uv = to_f(u[i]), d = to_f(dh[i]);
    const float s = sigmoidf_(gv);
    dg[i] = from_f<T>(d * uv * (s * (1.f + gv * (1.f - s))));
    du[i] = from_f<T>(d * gv * s);
  }
}

static int ew_grid(long n, int dev) { return (int)std::max<long>(1, std::min<long>((n + 255) / 256, 8L * num_sms(dev))); }

at::Tensor swiglu_fwd(at::Tensor g, at::Tensor u) {
  TORCH_CHECK(g.is_contiguous() && u.is_contiguous() && g.sizes() == u.sizes() && g.scalar_type() == u.scalar_type());
  const c10::cuda::CUDAGuard guard(g.device());
  auto h = at::empty_like(g);
  const long n = g.numel();
  if (n == 0) return h;
  auto s = at::cuda::getCurrentCUDAStream();
  const int grid = ew_grid(n, g.device().index());
  if (g.scalar_type() == at::kFloat)
    swiglu_fwd_kernel<float><<<grid, 256, 0, s>>>(g.data_ptr<float>(), u.data_ptr<float>(), h.data_ptr<float>(), n);
  else
    swiglu_fwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(u.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), n);
  PB_CUDA_CHECK(cudaGetLastError());
  return h;
}

std::vector<at::Tensor> swiglu_bwd(at::Tensor g, at::Tensor u, at::Tensor dh) {
  const c10::cuda::CUDAGuard guard(g.device());
  dh = dh.contiguous().to(g.scalar_type());
  auto dg = at::empty_like(g), du = at::empty_like(u);
  const long n = g.numel();
  if (n == 0) return {dg, du};
  auto s = at::cuda::getCurrentCUDAStream();
  const int grid = ew_grid(n, g.device().index());
  if (g.scalar_type() == at::kFloat)
    swiglu_bwd_kernel<float><<<grid, 256, 0, s>>>(g.data_ptr<float>(), u.data_ptr<float>(), dh.data_ptr<float>(),
                                                  dg.data_ptr<float>(), du.data_ptr<float>(), n);
  else
    swiglu_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        reinterpret_cast<const __nv_bfloat16*>(g.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(u.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(dh.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dg.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(du.data_ptr()), n);
  PB_CUDA_CHECK(cudaGetLastError());
  return {dg, du};
}

// ------------------------------- RoPE ---------------------------------------------
// In place on x [T, ncols] (row pitch ld): every head of ``head_dim`` columns below
// ``n_rope_cols`` is rotated by angle(pos[t], i); inverse = rotate by -angle.
template <typename T>
__global__ void rope_kernel(T* __restrict__ x, long ld, const int* __restrict__ pos, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, int rows, int n_rope_cols, int head_dim, int inverse,
                            int n_pos) {
  const int half = head_dim / 2;
  const long pairs_per_row = n_rope_cols / 2;
  const long total = static_cast<long>(rows) * pairs_per_row;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int row = static_cast<int>(i / pairs_per_row);
    const int pr = static_cast<int>(i % pairs_per_row);
    const int head = pr / half, j = pr % half;
    const int p = min(max(pos[row], 0), n_pos - 1);
    const float c = cos_t[static_cast<long>(p) * half + j];
    const float s = inverse ? -sin_t[static_cast<long>(p) * half + j] : sin_t[static_cast<long>(p) * half + j];
    T* base = x + row * ld + head * head_dim;
    const float x1 = to_f(base[j]), x2 = to_f(base[j + half]);
    base[j] = from_f<T>(x1 * c - x2 * s);
    base[j + half] = from_f<T>(x2 * c + x1 * s);
  }
}

void rope_apply(at::Tensor x, at::Tensor pos, at::Tensor cos_t, at::Tensor sin_t, int64_t n_rope_cols,
                int64_t head_dim, bool inverse) {
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && pos.scalar_type() == at::kInt);
  const c10::cuda::CUDAGuard guard(x.device());
  const int rows = x.size(0);
  const long total = (long)rows * (n_rope_cols / 2);
  if (total == 0) return;
  auto s = at::cuda::getCurrentCUDAStream();
  const int grid = ew_grid(total, x.device().index());
  if (x.scalar_type() == at::kFloat)
    rope_kernel<float><<<grid, 256, 0, s>>>(x.data_ptr<float>(), x.stride(0), pos.data_ptr<int>(),
                                            cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), rows, (int)n_rope_cols,
                                            (int)head_dim, inverse, (int)cos_t.size(0));
  else
    rope_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), x.stride(0),
                                                    pos.data_ptr<int>(), cos_t.data_ptr<float>(),
                                                    sin_t.data_ptr<float>(), rows, (int)n_rope_cols, (int)head_dim,
                                                    inverse, (int)cos_t.size(0));
  PB_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------- embedding ----------------------------------------
// Ids outside [0, vocab) read row 0 and record status 501 (no out-of-range access).
__device__ __forceinline__ int64_t checked_id(int64_t id, int64_t vocab, int* status) {
  if (id < 0 || id >= vocab) {
    report_error(status, 501);
    return 0;
  }
  return id;
}

__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ w,
                                     float* __restrict__ out, int rows, int d, int64_t vocab, int* status) {
  const int d4 = d / 4;
  const long total = static_cast<long>(rows) * d4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = static_cast<int>(i / d4), c = static_cast<int>(i % d4);
    reinterpret_cast<float4*>(out)[i] = reinterpret_cast<const float4*>(w + checked_id(ids[r], vocab, status) * d)[c];
  }
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, const float* __restrict__ dx,
                                     float* __restrict__ grad, int rows, int d, int64_t vocab, int* status) {
  const int d4 = d / 4;
  const long total = static_cast<long>(rows) * d4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = static_cast<int>(i / d4), c = static_cast<int>(i % d4);
    atomicAdd(reinterpret_cast<float4*>(grad + checked_id(ids[r], vocab, status) * d) + c,
              reinterpret_cast<const float4*>(dx)[i]);
  }
}

// Deterministic embedding gradient: token positions sorted stably by id; one thread per
// (run of equal ids, 4 columns) sums the run's rows in position order and adds the sum to
// the row of the table.  ``starts``: first sorted position of every run, then the total.
__global__ void embedding_bwd_sorted_kernel(const int64_t* __restrict__ sorted_ids, const int64_t* __restrict__ pos,
                                            const int64_t* __restrict__ starts, int runs, const float* __restrict__ dx,
                                            float* __restrict__ grad, int d, int64_t vocab, int* status) {
  const int d4 = d / 4;
  const long total = static_cast<long>(runs) * d4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int run = static_cast<int>(i / d4), c = static_cast<int>(i % d4);
    const long a = starts[run], b = starts[run + 1];
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
    for (long k = a; k < b; ++k) {
      const float4 v = reinterpret_cast<const float4*>(dx + pos[k] * d)[c];
      t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
    }
    float4* g = reinterpret_cast<float4*>(grad + checked_id(sorted_ids[a], vocab, status) * d) + c;
    float4 o = *g;
    o.x += t.x; o.y += t.y; o.z += t.z; o.w += t.w;
    *g = o;
  }
}

at::Tensor embedding_fwd(at::Tensor ids, at::Tensor w) {
  TORCH_CHECK(ids.scalar_type() == at::kLong && w.scalar_type() == at::kFloat && w.size(1) % 4 == 0);
  const c10::cuda::CUDAGuard guard(w.device());
  ids = ids.contiguous();
  const int rows = ids.numel(), d = w.size(1);
  auto out = at::empty({rows, d}, w.options());
  if (rows == 0) return out;
  const long total = (long)rows * d / 4;
  embedding_fwd_kernel<<<ew_grid(total, w.device().index()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), w.data_ptr<float>(), out.data_ptr<float>(), rows, d, w.size(0),
      status_ptr(w.device().index()));
  PB_CUDA_CHECK(cudaGetLastError());
  return out;
}

// grad (+)= scatter of dx rows; ``accumulate`` false zeroes ``grad`` first.
void embedding_bwd(at::Tensor ids, at::Tensor dx, at::Tensor grad, bool accumulate) {
  const c10::cuda::CUDAGuard guard(grad.device());
  ids = ids.contiguous();
  dx = dx.contiguous();
  if (!accumulate) grad.zero_();
  const int rows = ids.numel(), d = grad.size(1);
  if (rows == 0) return;
  if (g_deterministic) {
    auto flat_ids = ids.reshape(-1);
    auto sorted = at::sort(flat_ids, /*stable=*/true, /*dim=*/0, /*descending=*/false);
    auto sid = std::get<0>(sorted), pos = std::get<1>(sorted);
    auto uc = at::unique_consecutive(sid, /*return_inverse=*/false, /*return_counts=*/true);
    auto counts = std::get<2>(uc);
    auto starts = at::cat({at::zeros({1}, counts.options()), at::cumsum(counts, 0)});
    const int runs = static_cast<int>(counts.numel());
    const long total = (long)runs * d / 4;
    embedding_bwd_sorted_kernel<<<ew_grid(total, grad.device().index()), 256, 0,
                                  at::cuda::getCurrentCUDAStream()>>>(
        sid.data_ptr<int64_t>(), pos.data_ptr<int64_t>(), starts.data_ptr<int64_t>(), runs, dx.data_ptr<float>(),
        grad.data_ptr<float>(), d, grad.size(0), status_ptr(grad.device().index()));
    PB_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const long total = (long)rows * d / 4;
  embedding_bwd_kernel<<<ew_grid(total, grad.device().index()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ids.data_ptr<int64_t>(), dx.data_ptr<float>(), grad.data_ptr<float>(), rows, d, grad.size(0),
      status_ptr(grad.device().index()));
  PB_CUDA_CHECK(cudaGetLastError());
}

void ce_finalize(at::Tensor pmax, at::Tensor psum, at::Tensor tlogit, at::Tensor targets, int64_t ignore_index,
                 double z, at::Tensor lse, at::Tensor loss) {
  const c10::cuda::CUDAGuard guard(pmax.device());
  const int ntiles = pmax.size(0), rows = pmax.size(1);
  if (rows == 0) return;
  ce_finalize_kernel<<<ce_finalize_blocks(rows), kCeRows * kCeGroups, 0, at::cuda::getCurrentCUDAStream()>>>(
      pmax.data_ptr<float>(), psum.data_ptr<float>(), ntiles, rows, tlogit.data_ptr<float>(),
      targets.data_ptr<int64_t>(), ignore_index, (float)z, lse.data_ptr<float>(), loss.data_ptr<float>());
  PB_CUDA_CHECK(cudaGetLastError());
}

__global__ void ce_row_scale_kernel(const int64_t* __restrict__ targets, int64_t ignore_index,
                                    const float* __restrict__ g, float* __restrict__ scale, int rows) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows) scale[r] = targets[r] != ignore_index ? *g : 0.f;
}

void ce_row_scale(at::Tensor targets, int64_t ignore_index, at::Tensor grad_out, at::Tensor scale) {
  const c10::cuda::CUDAGuard guard(targets.device());
  const int rows = targets.numel();
  if (rows == 0) return;
  ce_row_scale_kernel<<<(rows + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      targets.data_ptr<int64_t>(), ignore_index, grad_out.data_ptr<float>(), scale.data_ptr<float>(), rows);
  PB_CUDA_CHECK(cudaGetLastError());
}

// dlogits = (softmax * (1 + 2 z lse) - onehot(target)) * scale[row], in place over the
// bf16 logits kept by the forward GEMM; 8 columns per thread, blockIdx.y = row.
__global__ void ce_dlogits_kernel(__nv_bfloat16* __restrict__ lg, const float* __restrict__ lse,
                                  const int64_t* __restrict__ targets, const float* __restrict__ scale, float z, int V) {
  const long r = blockIdx.y;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= V) return;
  const float sc = scale[r];
  uint4* p = reinterpret_cast<uint4*>(lg + r * V + c);
  if (sc == 0.f) {
    *p = make_uint4(0, 0, 0, 0);
    return;
  }
  const float l = lse[r];
  const float zf = 1.f + 2.f * z * l;
  const int64_t t = targets[r] - c;
  uint4 v = *p;
  uint32_t* w = &v.x;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 x = unpack_bf16x2(w[k]);
    const float g0 = (__expf(x.x - l) * zf - (t == 2 * k ? 1.f : 0.f)) * sc;
    const float g1 = (__expf(x.y - l) * zf - (t == 2 * k + 1 ? 1.f : 0.f)) * sc;
    w[k] = pack_bf16x2(g0, g1);
  }
  *p = v;
}

void ce_dlogits(at::Tensor logits, at::Tensor lse, at::Tensor targets, at::Tensor scale, double z) {
  TORCH_CHECK(logits.is_contiguous() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2);
  const int rows = logits.size(0), V = logits.size(1);
  TORCH_CHECK(V % 8 == 0, "ce_dlogits: vocabulary must be a multiple of 8");
  TORCH_CHECK(lse.numel() == rows && targets.numel() == rows && scale.numel() == rows);
  TORCH_CHECK(targets.scalar_type() == at::kLong && lse.scalar_type() == at::kFloat && scale.scalar_type() == at::kFloat);
  const c10::cuda::CUDAGuard guard(logits.device());
  if (rows == 0) return;
  const dim3 grid((V / 8 + 255) / 256, rows);
  ce_dlogits_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), lse.data_ptr<float>(), targets.data_ptr<int64_t>(),
      scale.data_ptr<float>(), (float)z, V);
  PB_CUDA_CHECK(cudaGetLastError());
}

// ------------------------------- optimizer ----------------------------------------
// AdamW over flat fp32 buffers; the gradient is scaled by min(1, max_norm/(norm+1e-6))
// when max_norm > 0, and nothing changes when the norm is not finite.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ shadow, long n,
                             const float* __restrict__ norm, int* __restrict__ skipped, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2, float max_norm, const float* __restrict__ hp) {
  if (hp != nullptr) {  // per-step values from device memory (CUDA-graph replay)
    lr = hp[0];
    bc1 = hp[1];
    bc2 = hp[2];
  }
  const float nv = *norm;
  const bool bad = !isfinite(nv);
  if (blockIdx.x == 0 && threadIdx.x == 0) *skipped = bad ? 1 : 0;
  if (bad) return;
  float gs = 1.f;
  if (max_norm > 0.f) gs = fminf(1.f, max_norm / (nv + 1e-6f));
  const float step = lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const float decay = 1.f - lr * wd;
  const long n4 = n / 4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    float4 pv = reinterpret_cast<float4*>(p)[i];
    const float4 gv = reinterpret_cast<const float4*>(g)[i];
    float4 mv = reinterpret_cast<float4*>(m)[i];
    float4 vv = reinterpret_cast<float4*>(v)[i];
    float* pp = &pv.x;
    const float* gg = &gv.x;
    float* mm = &mv.x;
    float* ww = &vv.x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gk = gg[k] * gs;
      mm[k] = b1 * mm[k] + (1.f - b1) * gk;
      ww[k] = b2 * ww[k] + (1.f - b2) * gk * gk;
      pp[k] = pp[k] * decay - step * mm[k] / (sqrtf(ww[k]) * inv_sqrt_bc2 + eps);
    }
    reinterpret_cast<float4*>(p)[i] = pv;
    reinterpret_cast<float4*>(m)[i] = mv;
    reinterpret_cast<float4*>(v)[i] = vv;
    if (shadow != nullptr) {
      uint2 o = make_uint2(pack_bf16x2(pv.x, pv.y), pack_bf16x2(pv.z, pv.w));
      reinterpret_cast<uint2*>(shadow)[i] = o;
    }
  }
  for (long i = n4 * 4 + blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float gk = g[i] * gs;
    m[i] = b1 * m[i] + (1.f - b1) * gk;
    v[i] = b2 * v[i] + (1.f - b2) * gk * gk;
    p[i] = p[i] * decay - step * m[i] / (sqrtf(v[i]) * inv_sqrt_bc2 + eps);
    if (shadow != nullptr) shadow[i] = __float2bfloat16_rn(p[i]);
  }
}

// ``hparams`` (optional, device fp32 [3]): lr, bc1, bc2 read by the kernel instead of
// the host values, so a captured CUDA graph picks up each step's schedule.
void adamw_step(at::Tensor p, at::Tensor g, at::Tensor m, at::Tensor v, at::Tensor shadow, at::Tensor norm,
                at::Tensor skipped, double lr, double b1, double b2, double eps, double wd, double bc1, double bc2,
                double max_norm, bool write_shadow, c10::optional<at::Tensor> hparams) {
  const c10::cuda::CUDAGuard guard(p.device());
  const long n = p.numel();
  TORCH_CHECK(reinterpret_cast<uintptr_t>(p.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(g.data_ptr()) % 16 == 0);
  adamw_kernel<<<4 * num_sms(p.device().index()), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(),
      write_shadow ? reinterpret_cast<__nv_bfloat16*>(shadow.data_ptr()) : nullptr, n, norm.data_ptr<float>(),
      skipped.data_ptr<int>(), (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1, (float)bc2,
      (float)max_norm, hparams.has_value() ? hparams->data_ptr<float>() : nullptr);
  PB_CUDA_CHECK(cudaGetLastError());
}

__global__ void sumsq_kernel(const float* __restrict__ x, long n, float* __restrict__ out, float* __restrict__ part) {
  float s = 0.f;
  const long n4 = n / 4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long i = n4 * 4 + blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    s += x[i] * x[i];
  s = warp_sum(s);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) {
      if (part != nullptr) part[blockIdx.x] = t;  // deterministic mode: summed in block order
      else atomicAdd(out, t);
    }
  }
}

at::Tensor l2_norm(at::Tensor x) {
  const c10::cuda::CUDAGuard guard(x.device());
  auto acc = at::zeros({}, x.options().dtype(at::kFloat));
  const long n = x.numel();
  const int blocks = 2 * num_sms(x.device().index());
  at::Tensor part;
  if (g_deterministic) part = at::empty({blocks}, x.options().dtype(at::kFloat));
  if (n > 0) {
    sumsq_kernel<<<blocks, 512, 0, at::cuda::getCurrentCUDAStream()>>>(
        x.data_ptr<float>(), n, acc.data_ptr<float>(), g_deterministic ? part.data_ptr<float>() : nullptr);
    if (g_deterministic)
      dw_reduce_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(part.data_ptr<float>(), blocks, 1,
                                                                         acc.data_ptr<float>());
  }
  PB_CUDA_CHECK(cudaGetLastError());
  return acc.sqrt();
}

}  // namespace pb
