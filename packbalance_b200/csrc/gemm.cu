// tcgen05 GEMM for sm_100a with fused epilogues.
//
//   D[m, n] = sum_k A(m, k) * B(n, k)      bf16 operands, fp32 accumulation in TMEM
//
// A is K-major ([M, K] row-major) or MN-major ([K, M] row-major); same for B.  This
// covers every GEMM of a Linear layer without transposes:
//   forward  y  = x  W^T : A = x  (K-major), B = W (K-major)
//   dgrad    dx = dy W   : A = dy (K-major), B = W (MN-major)
//   wgrad    dW = dy^T x : A = dy (MN-major), B = x (MN-major)
//
// Kernel structure (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0      TMA producer: 128B-swizzled A/B tiles into a STAGES-deep smem ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16)
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (thread = row), fused math,
//               global stores; two TMEM accumulators so tile i's epilogue overlaps
//               tile i+1's MMAs.
// Every mbarrier wait is bounded (common.cuh); a timeout records an error code in
// the status word, the other roles stop, in-flight copies and MMAs are drained and
// TMEM is freed before the CTA exits.
//
// Epilogues (runtime-selected, uniform per launch):
//   BF16        out(bf16) = alpha * acc
//   F32         out(f32)  = alpha * acc (+ out when beta != 0)
//   RESID       out(f32)  = res(f32) + acc                 (residual stream update)
//   SWIGLU      B tile = [gate rows | up rows]; h = silu(g) * u (bf16) and the
//               pre-activations are saved (bf16) for the backward pass
//   ROPE        out(bf16) = acc with half-split RoPE on the first n_rope_cols columns
//               (per-row positions, fp32 cos/sin tables)
//   SWIGLU_BWD  acc = dh; reads saved g|u and writes dg|du (bf16)
//   ATOMIC_F32  out(f32) += acc via vector atomics (split-K partial sums)
//   CE_FWD      per-row max / sum(exp) partials of the logits tile + target logit
//   CE_BWD      dlogits(bf16) = (softmax(logit) * (1 + 2 z lse) - onehot) * row_scale
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <ATen/ATen.h>

#include "common.cuh"
#include "host_utils.h"

namespace pb {

enum GemmEpi : int {
  EPI_BF16 = 0,
  EPI_F32 = 1,
  EPI_RESID = 2,
  EPI_SWIGLU = 3,
  EPI_ROPE = 4,
  EPI_SWIGLU_BWD = 5,
  EPI_ATOMIC_F32 = 6,
  EPI_CE_FWD = 7,
  EPI_CE_BWD = 8,
};

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles, splits, kb_per_split, k_blocks;
  int epi;
  float alpha;
  int beta;
  void* out;
  long ldo;
  const float* res;
  long ldr;
  void* aux;  // SWIGLU: saved g|u (out); SWIGLU_BWD: saved g|u (in)
  long ldaux;
  void* aux2;  // SWIGLU_BWD: dg|du (out)
  long ldaux2;
  int F;  // half width of the gate|up matrices
  const int* pos;
  const float* cos_t;
  const float* sin_t;
  int head_dim;
  int n_rope_cols;
  int n_pos;  // rows of the cos/sin tables; positions are clamped into range
  const int64_t* targets;
  float* pmax;
  float* psum;
  float* tlogit;
  const float* lse;
  const float* row_scale;
  float z_coeff;
  int* status;
};

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
};

__device__ __forceinline__ void tile_coords(const GemmArgs& a, int tile, int& mb, int& nb, int& sp) {
  sp = tile % a.splits;
  const int t = tile / a.splits;
  mb = t % a.m_tiles;
  nb = t / a.m_tiles;
}

// ------------------------------- epilogue helpers ---------------------------------
__device__ __forceinline__ void store_bf16_32(__nv_bfloat16* dst, const float* v, int valid) {
  uint32_t p[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) p[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  if (valid >= 32) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
  } else {
    for (int i = 0; i < valid; ++i) dst[i] = __float2bfloat16_rn(v[i]);
  }
}

__device__ __forceinline__ void load_bf16_32(const __nv_bfloat16* src, float* v, int valid) {
  if (valid >= 32) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 q = s[i];
      float2 f0 = unpack_bf16x2(q.x), f1 = unpack_bf16x2(q.y), f2 = unpack_bf16x2(q.z), f3 = unpack_bf16x2(q.w);
      v[8 * i + 0] = f0.x; v[8 * i + 1] = f0.y; v[8 * i + 2] = f1.x; v[8 * i + 3] = f1.y;
      v[8 * i + 4] = f2.x; v[8 * i + 5] = f2.y; v[8 * i + 6] = f3.x; v[8 * i + 7] = f3.y;
    }
  } else {
    for (int i = 0; i < 32; ++i) v[i] = i < valid ? __bfloat162float(src[i]) : 0.f;
  }
}

__device__ __forceinline__ void tmem_load_f32(uint32_t taddr, float* v) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN>
__device__ void run_epilogue(const GemmArgs& a, uint32_t tacc, int row, int mb, int nb) {
  const bool row_ok = row < a.M;
  float v[32];
  switch (a.epi) {
    case EPI_BF16:
    case EPI_F32:
    case EPI_RESID:
    case EPI_ATOMIC_F32: {
      const int n0 = nb * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        tmem_load_f32(tacc + c, v);
        const int col = n0 + c;
        const int valid = min(32, a.N - col);
        if (!row_ok || valid <= 0) continue;
        if (a.epi == EPI_BF16) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= a.alpha;
          store_bf16_32(reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col, v, valid);
        } else if (a.epi == EPI_ATOMIC_F32) {
          float* dst = reinterpret_cast<float*>(a.out) + row * a.ldo + col;
          if (valid >= 32) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              atomicAdd(reinterpret_cast<float4*>(dst) + i,
                        make_float4(a.alpha * v[4 * i], a.alpha * v[4 * i + 1], a.alpha * v[4 * i + 2],
                                    a.alpha * v[4 * i + 3]));
          } else {
            for (int i = 0; i < valid; ++i) atomicAdd(dst + i, a.alpha * v[i]);
          }
        } else {
          float* dst = reinterpret_cast<float*>(a.out) + row * a.ldo + col;
          const float* add = nullptr;
          if (a.epi == EPI_RESID) add = a.res + row * a.ldr + col;
          else if (a.beta) add = dst;
          const float s = a.epi == EPI_RESID ? 1.f : a.alpha;
          if (valid >= 32) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float4 o = make_float4(s * v[4 * i], s * v[4 * i + 1], s * v[4 * i + 2], s * v[4 * i + 3]);
              if (add != nullptr) {
                float4 b = reinterpret_cast<const float4*>(add)[i];
                o.x += b.x; o.y += b.y; o.z += b.z; o.w += b.w;
              }
              reinterpret_cast<float4*>(dst)[i] = o;
            }
          } else {
            for (int i = 0; i < valid; ++i) dst[i] = s * v[i] + (add != nullptr ? add[i] : 0.f);
          }
        }
      }
      break;
    }
    case EPI_SWIGLU: {
      // acc columns [0, BN/2) = gate, [BN/2, BN) = up, for output columns
      // [nb*BN/2, (nb+1)*BN/2) of h.
      constexpr int HB = BN / 2;
      float u[32];
#pragma unroll 1
      for (int c = 0; c < HB; c += 32) {
        tmem_load_f32(tacc + c, v);
        tmem_load_f32(tacc + HB + c, u);
        const int col = nb * HB + c;
        const int valid = min(32, a.F - col);
        if (!row_ok || valid <= 0) continue;
        __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(a.aux) + row * a.ldaux;
        // Round the pre-activations once and compute h from the rounded values, so
        // the backward pass (which reads the saved bf16 values) sees the same inputs.
        store_bf16_32(gu + col, v, valid);
        store_bf16_32(gu + a.F + col, u, valid);
        float h[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float g = __bfloat162float(__float2bfloat16_rn(v[i]));
          const float up = __bfloat162float(__float2bfloat16_rn(u[i]));
          h[i] = g * sigmoidf_(g) * up;
        }
        store_bf16_32(reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col, h, valid);
      }
      break;
    }
    case EPI_SWIGLU_BWD: {
      const int n0 = nb * BN;
      float g[32], u[32];
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        tmem_load_f32(tacc + c, v);
        const int col = n0 + c;
        const int valid = min(32, a.F - col);
        if (!row_ok || valid <= 0) continue;
        const __nv_bfloat16* gu = reinterpret_cast<const __nv_bfloat16*>(a.aux) + row * a.ldaux;
        load_bf16_32(gu + col, g, valid);
        load_bf16_32(gu + a.F + col, u, valid);
        float dg[32], du[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float s = sigmoidf_(g[i]);
          const float silu = g[i] * s;
          du[i] = v[i] * silu;
          dg[i] = v[i] * u[i] * (s * (1.f + g[i] * (1.f - s)));
        }
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.aux2) + row * a.ldaux2;
        store_bf16_32(out + col, dg, valid);
        store_bf16_32(out + a.F + col, du, valid);
      }
      break;
    }
    case EPI_ROPE: {
      const int n0 = nb * BN;
      const int half = a.head_dim / 2;
      const int p = row_ok ? min(max(a.pos[row], 0), a.n_pos - 1) : 0;
      float w[32];
#pragma unroll 1
      for (int hb = 0; hb < BN; hb += a.head_dim) {
        const int hcol = n0 + hb;
        const bool rot = hcol < a.n_rope_cols;
#pragma unroll 1
        for (int j = 0; j < half; j += 32) {
          tmem_load_f32(tacc + hb + j, v);
          tmem_load_f32(tacc + hb + half + j, w);
          if (!row_ok || hcol >= a.N) continue;
          if (rot) {
            const float* cr = a.cos_t + (long)p * half + j;
            const float* sr = a.sin_t + (long)p * half + j;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float c = cr[i], s = sr[i];
              const float x1 = v[i], x2 = w[i];
              v[i] = x1 * c - x2 * s;
              w[i] = x2 * c + x1 * s;
            }
          }
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + hcol;
          store_bf16_32(dst + j, v, 32);
          store_bf16_32(dst + half + j, w, 32);
        }
      }
      break;
    }
    case EPI_CE_FWD: {
      const int n0 = nb * BN;
      float mx = -INFINITY, se = 0.f;
      const int64_t tgt = row_ok ? a.targets[row] : -1;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        tmem_load_f32(tacc + c, v);
        const int col = n0 + c;
        const int valid = min(32, a.N - col);
        if (!row_ok || valid <= 0) continue;
        float cm = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < valid) cm = fmaxf(cm, v[i]);
        const float nm = fmaxf(mx, cm);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < valid) s += __expf(v[i] - nm);
        se = se * __expf(mx - nm) + s;
        mx = nm;
        if (tgt >= col && tgt < col + valid) {
          float t = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (tgt == col + i) t = v[i];
          a.tlogit[row] = t;
        }
      }
      if (row_ok) {
        a.pmax[(long)nb * a.M + row] = mx;
        a.psum[(long)nb * a.M + row] = se;
      }
      break;
    }
    case EPI_CE_BWD: {
      const int n0 = nb * BN;
      float l = 0.f, scale = 0.f, zf = 1.f;
      int64_t tgt = -1;
      if (row_ok) {
        l = a.lse[row];
        scale = a.row_scale[row];
        tgt = a.targets[row];
        zf = 1.f + 2.f * a.z_coeff * l;
      }
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        tmem_load_f32(tacc + c, v);
        const int col = n0 + c;
        const int valid = min(32, a.N - col);
        if (!row_ok || valid <= 0) continue;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float g = __expf(v[i] - l) * zf;
          if (tgt == col + i) g -= 1.f;
          v[i] = g * scale;
        }
        store_bf16_32(reinterpret_cast<__nv_bfloat16*>(a.out) + row * a.ldo + col, v, valid);
      }
      break;
    }
    default:
      break;
  }
}

// ------------------------------------ kernel --------------------------------------
template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const GemmArgs args) {
  using C = GemmCfg<BN>;
  constexpr uint32_t IDESC = idesc_bf16_f32(C::BM, BN, A_MN, B_MN);
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t accf_bar[2];
  __shared__ __align__(8) uint64_t acce_bar[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&accf_bar[s], 1);
      mbar_init(&acce_bar[s], 4);
    }
    mbar_init(&drain_bar, 1);
    abort_sh = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tma_a);
    tma_prefetch_desc(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  const int num_tiles = args.m_tiles * args.n_tiles * args.splits;
  const bool swiglu = args.epi == EPI_SWIGLU;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued[C::STAGES];
      for (int s = 0; s < C::STAGES; ++s) issued[s] = -1;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb, sp;
        tile_coords(args, tile, mb, nb, sp);
        const int kb0 = sp * args.kb_per_split;
        const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, args.status, 101, &abort_sh)) {
            ok = false;
            break;
          }
          uint64_t* bar = &full_bar[stage];
          mbar_arrive_expect_tx(bar, C::STAGE_BYTES);
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          const int k0 = kb * C::BK;
          if (!A_MN) {
            tma_load_2d(sa, &tma_a, bar, k0, mb * C::BM);
          } else {
            tma_load_2d(sa, &tma_a, bar, mb * C::BM, k0);
            tma_load_2d(sa + 8192, &tma_a, bar, mb * C::BM + 64, k0);
          }
          if (!B_MN) {
            if (swiglu) {
              tma_load_2d(sb, &tma_b, bar, k0, nb * (BN / 2));
              tma_load_2d(sb + (BN / 2) * 128, &tma_b, bar, k0, args.F + nb * (BN / 2));
            } else {
              tma_load_2d(sb, &tma_b, bar, k0, nb * BN);
            }
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, &tma_b, bar, nb * BN + j * 64, k0);
          }
          issued[stage] = phase;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded, once more) for the copies this thread issued.
        for (int s = 0; s < C::STAGES; ++s)
          if (issued[s] >= 0) mbar_wait(&full_bar[s], issued[s], args.status, 102, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb, sp;
        tile_coords(args, tile, mb, nb, sp);
        const int kb0 = sp * args.kb_per_split;
        const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1, args.status, 103, &abort_sh)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, args.status, 104, &abort_sh)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sdesc_sw128(sa + kk * 2048, 8192, 1024) : sdesc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(sb + kk * 2048, 8192, 1024) : sdesc_sw128(sb + kk * 32, 16, 1024);
            umma_ss(d_tmem, ad, bd, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&accf_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // All MMAs issued by this thread must finish before TMEM is released.
      umma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, args.status, 105, nullptr);
    }
  } else {
    const int q = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb, sp;
      tile_coords(args, tile, mb, nb, sp);
      if (!mbar_wait_warp(&accf_bar[acc], acc_phase, args.status, 106, &abort_sh)) break;
      tc_fence_after();
      const int row = mb * C::BM + q * 32 + lane;
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      run_epilogue<BN>(args, tacc, row, mb, nb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ------------------------------------ host ----------------------------------------
template <int BN, bool A_MN, bool B_MN>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, int grid,
                        cudaStream_t stream) {
  using C = GemmCfg<BN>;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!configured[dev]) {
    PB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    configured[dev] = true;
  }
  kern<<<grid, 192, C::SMEM_BYTES, stream>>>(ta, tb, args);
  PB_CUDA_CHECK(cudaGetLastError());
}

template <int BN>
static void dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                           const GemmArgs& args, int grid, cudaStream_t s) {
  if (!a_mn && !b_mn) launch_gemm<BN, false, false>(ta, tb, args, grid, s);
  else if (!a_mn && b_mn) launch_gemm<BN, false, true>(ta, tb, args, grid, s);
  else if (a_mn && b_mn) launch_gemm<BN, true, true>(ta, tb, args, grid, s);
  else launch_gemm<BN, true, false>(ta, tb, args, grid, s);
}

static const void* opt_ptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

// Python-facing entry.  ``a``/``b`` are 2-D bf16 views with unit inner stride; M, N, K
// are the logical GEMM sizes (for SWIGLU N = 2F and ``b`` is the [2F, K] gate|up matrix).
void gemm_tc(at::Tensor a, at::Tensor b, at::Tensor out, int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn,
             int64_t epi, int64_t bn, int64_t splits, int64_t max_ctas, double alpha, bool beta,
             c10::optional<at::Tensor> res, c10::optional<at::Tensor> aux, c10::optional<at::Tensor> aux2,
             c10::optional<at::Tensor> pos, c10::optional<at::Tensor> cos_t, c10::optional<at::Tensor> sin_t,
             int64_t head_dim, int64_t n_rope_cols, c10::optional<at::Tensor> targets,
             c10::optional<at::Tensor> pmax, c10::optional<at::Tensor> psum, c10::optional<at::Tensor> tlogit,
             c10::optional<at::Tensor> lse, c10::optional<at::Tensor> row_scale, double z_coeff) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda(), "gemm_tc: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_tc: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "gemm_tc: 2-D row-major");
  TORCH_CHECK(bn == 64 || bn == 128 || bn == 256, "gemm_tc: bn must be 64/128/256");
  const c10::cuda::CUDAGuard guard(a.device());
  const bool swiglu = epi == EPI_SWIGLU;
  if (!a_mn) {
    TORCH_CHECK(a.size(0) == M && a.size(1) == K, "gemm_tc: A shape");
  } else {
    TORCH_CHECK(a.size(0) == K && a.size(1) == M, "gemm_tc: A shape (MN-major)");
  }
  if (!b_mn) {
    TORCH_CHECK(b.size(0) == N && b.size(1) == K, "gemm_tc: B shape");
  } else {
    TORCH_CHECK(b.size(0) == K && b.size(1) == N, "gemm_tc: B shape (MN-major)");
  }
  TORCH_CHECK((a.stride(0) * 2) % 16 == 0 && (b.stride(0) * 2) % 16 == 0, "gemm_tc: row strides must be 16B multiples");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0,
              "gemm_tc: operands must be 16B aligned");
  TORCH_CHECK(!(swiglu && b_mn), "gemm_tc: SWIGLU needs a K-major B");

  GemmArgs g{};
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.F = swiglu || epi == EPI_SWIGLU_BWD ? (int)(swiglu ? N / 2 : N) : 0;
  g.m_tiles = (int)((M + 127) / 128);
  g.n_tiles = swiglu ? (int)((N / 2 + bn / 2 - 1) / (bn / 2)) : (int)((N + bn - 1) / bn);
  g.k_blocks = (int)((K + 63) / 64);
  g.splits = (int)std::max<int64_t>(1, std::min<int64_t>(splits, g.k_blocks));
  g.kb_per_split = (g.k_blocks + g.splits - 1) / g.splits;
  g.splits = (g.k_blocks + g.kb_per_split - 1) / g.kb_per_split;
  g.epi = (int)epi;
  g.alpha = (float)alpha;
  g.beta = beta ? 1 : 0;
  g.out = out.data_ptr();
  g.ldo = out.dim() == 2 ? out.stride(0) : 0;
  g.res = static_cast<const float*>(opt_ptr(res));
  g.ldr = res.has_value() ? res->stride(0) : 0;
  g.aux = const_cast<void*>(opt_ptr(aux));
  g.ldaux = aux.has_value() ? aux->stride(0) : 0;
  g.aux2 = const_cast<void*>(opt_ptr(aux2));
  g.ldaux2 = aux2.has_value() ? aux2->stride(0) : 0;
  g.pos = static_cast<const int*>(opt_ptr(pos));
  g.cos_t = static_cast<const float*>(opt_ptr(cos_t));
  g.sin_t = static_cast<const float*>(opt_ptr(sin_t));
  g.head_dim = (int)head_dim;
  g.n_rope_cols = (int)n_rope_cols;
  g.n_pos = cos_t.has_value() ? (int)cos_t->size(0) : 1;
  g.targets = static_cast<const int64_t*>(opt_ptr(targets));
  g.pmax = static_cast<float*>(const_cast<void*>(opt_ptr(pmax)));
  g.psum = static_cast<float*>(const_cast<void*>(opt_ptr(psum)));
  g.tlogit = static_cast<float*>(const_cast<void*>(opt_ptr(tlogit)));
  g.lse = static_cast<const float*>(opt_ptr(lse));
  g.row_scale = static_cast<const float*>(opt_ptr(row_scale));
  g.z_coeff = (float)z_coeff;
  g.status = status_ptr(a.device().index());
  if (epi == EPI_ROPE) {
    TORCH_CHECK(head_dim % 64 == 0 && bn % head_dim == 0, "gemm_tc: RoPE needs head_dim % 64 == 0 and bn % head_dim == 0");
    TORCH_CHECK(N % head_dim == 0, "gemm_tc: RoPE output width must be whole heads");
  }
  if (epi == EPI_SWIGLU) TORCH_CHECK((N / 2) % 8 == 0, "gemm_tc: SWIGLU F must be a multiple of 8");
  if (g.splits > 1) TORCH_CHECK(epi == EPI_ATOMIC_F32, "gemm_tc: split-K needs the ATOMIC_F32 epilogue");
  TORCH_CHECK(epi == EPI_CE_FWD || epi == EPI_ATOMIC_F32 || out.stride(-1) == 1, "gemm_tc: output must be row-major");

  // TMA descriptors: 128-byte swizzle, 64-element (128 B) inner box.
  const int bm_box = 128;
  CUtensorMap ta = a_mn ? make_tmap_bf16_2d(a.data_ptr(), M, K, a.stride(0) * 2, 64, 64)
                        : make_tmap_bf16_2d(a.data_ptr(), K, M, a.stride(0) * 2, 64, bm_box);
  CUtensorMap tb;
  if (b_mn) tb = make_tmap_bf16_2d(b.data_ptr(), N, K, b.stride(0) * 2, 64, 64);
  else tb = make_tmap_bf16_2d(b.data_ptr(), K, N, b.stride(0) * 2, 64, swiglu ? bn / 2 : bn);

  const int tiles = g.m_tiles * g.n_tiles * g.splits;
  int grid = std::min<int>(tiles, num_sms(a.device().index()));
  if (max_ctas > 0) grid = std::min<int>(grid, (int)max_ctas);
  grid = std::max(grid, 1);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (bn == 256) dispatch_major<256>(a_mn, b_mn, ta, tb, g, grid, stream);
  else if (bn == 128) dispatch_major<128>(a_mn, b_mn, ta, tb, g, grid, stream);
  else dispatch_major<64>(a_mn, b_mn, ta, tb, g, grid, stream);
}

}  // namespace pb
