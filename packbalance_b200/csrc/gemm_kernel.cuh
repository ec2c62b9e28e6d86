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
//   warps 6..7  (only in launches with a fused all-gather, 256 threads) copy warps that
//               fetch the peer-owned parts of the sharded B operand into this GPU's
//               gathered buffer while the MMAs run (ag_copy.cuh); the producer waits
//               per B tile for the pieces it covers
//   warps 2..5  epilogue, warp q owns TMEM lanes [32q, 32q+32) (= tile rows): each
//               32-column chunk goes tcgen05.ld -> registers -> fused math -> swizzled
//               smem staging slot -> TMA store (or TMA fp32 reduce-add), so global
//               writes are full coalesced boxes issued asynchronously; two staging
//               slots per warp and two TMEM accumulators overlap the epilogue of
//               tile i with the MMAs of tile i+1.
// Every mbarrier wait is bounded (common.cuh); a timeout records an error code in
// the status word, the other roles stop, in-flight copies and MMAs are drained and
// TMEM is freed before the CTA exits.
//
// Epilogues (runtime-selected, uniform per launch; none reads global memory except
// the CE row vectors and the RoPE tables):
//   BF16        out(bf16) = alpha * acc
//   F32         out(f32)  = alpha * acc
//   ADD_F32     out(f32) += alpha * acc   (TMA reduce-add: accumulation and split-K)
//   SWIGLU      B tile = [gate rows | up rows]; h = silu(g) * u and the rounded
//               pre-activations g|u are stored (bf16) for the backward pass
//   ROPE        out(bf16) = acc with half-split RoPE on the first n_rope_cols columns
//               (per-row positions, fp32 cos/sin tables)
//   CE_FWD      per-row max / sum(exp) partials of the logits tile + target logit
//   CE_BWD      dlogits(bf16) = (softmax(logit) * (1 + 2 z lse) - onehot) * row_scale
#pragma once

#include <cudaTypedefs.h>

#include "ag_copy.cuh"
#include "common.cuh"

namespace pb {

enum GemmEpi : int {
  EPI_BF16 = 0,
  EPI_F32 = 1,
  EPI_ADD_F32 = 2,
  EPI_SWIGLU = 3,
  EPI_ROPE = 4,
  EPI_SWIGLU_BWD = 5,
  EPI_CE_FWD = 7,
  EPI_CE_BWD = 8,
};

struct GemmArgs {
  int M, N, K;
  int m_tiles, n_tiles, splits, kb_per_split, k_blocks;
  int epi;
  float alpha;
  int F;  // SWIGLU: width of h (gate|up matrices have 2F rows); SWIGLU_BWD: N
  const __nv_bfloat16* gu;  // SWIGLU_BWD: saved [g | u] pre-activations, bf16 [M, 2F]
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
  int keep_logits;  // CE_FWD: also store the bf16 logits through tm_aux
  // Tests of the pair kernel's abort path only (0 = off): the even CTA's producer stops
  // after arming this many k-blocks, as if it had stalled, without stopping the odd CTA,
  // whose own bounded waits then run out.
  int test_arm_limit;
  AgSpec ag;  // ag.world == 0: B is already local
  int n_rot;  // n-blocks are visited starting at this one (wrapping)
};

constexpr int kEpiWarpBytes = 8192;  // staging ring of one epilogue warp (Stager)

template <int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN >= 192 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr uint32_t TMEM_COLS = BN == 192 ? 512 : 2 * BN;  // allocations are powers of two
  static constexpr int SMEM_BYTES = EPI_OFF + 4 * kEpiWarpBytes + 1024;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

__device__ __forceinline__ void tile_coords(const GemmArgs& a, int tile, int& mb, int& nb, int& sp) {
  sp = tile % a.splits;
  const int t = tile / a.splits;
  mb = t % a.m_tiles;
  nb = t / a.m_tiles + a.n_rot;
  if (nb >= a.n_tiles) nb -= a.n_tiles;
}

// ------------------------------- epilogue helpers ---------------------------------
// Per-warp staging ring in shared memory for the epilogue's TMA stores: NSLOT slots of
// 2 KB (a 32 x 32 bf16 box) or NSLOT / 2 slots of 4 KB (a 32 x 32 fp32 box), so up to
// NSLOT - 1 (or NSLOT / 2 - 1) stores are in flight while the next box is staged.
template <int NSLOT>
struct StagerT {
  static constexpr int kBytes = NSLOT * 2048;
  uint8_t* base;  // this warp's kBytes
  int slot;
  bool wide;  // fp32 boxes
  __device__ __forceinline__ uint8_t* acquire() {
    // The store that last used this slot must have finished reading it.
    if ((threadIdx.x & 31) == 0) {
      if (wide) bulk_wait_read<NSLOT / 2 - 1>();
      else bulk_wait_read<NSLOT - 1>();
    }
    __syncwarp();
    return base + slot * (wide ? 4096 : 2048);
  }
  __device__ __forceinline__ void release() { slot = (slot + 1) & (wide ? NSLOT / 2 - 1 : NSLOT - 1); }
};
using Stager = StagerT<4>;

// 32 fp32 of this lane's row -> 128-byte row of a 128B-swizzled [32 x 32] fp32 box.
__device__ __forceinline__ void stage_f32(uint8_t* s, const float (&v)[32], float scale) {
  const int r = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float4 q = make_float4(v[4 * j] * scale, v[4 * j + 1] * scale, v[4 * j + 2] * scale, v[4 * j + 3] * scale);
    *reinterpret_cast<float4*>(s + r * 128 + ((j ^ (r & 7)) << 4)) = q;
  }
}

// 32 bf16 of this lane's row -> 64-byte row of a 64B-swizzled [32 x 32] bf16 box.
__device__ __forceinline__ void stage_bf16(uint8_t* s, const float (&v)[32], float scale) {
  const int r = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 q = make_uint4(pack_bf16x2(v[8 * j] * scale, v[8 * j + 1] * scale),
                         pack_bf16x2(v[8 * j + 2] * scale, v[8 * j + 3] * scale),
                         pack_bf16x2(v[8 * j + 4] * scale, v[8 * j + 5] * scale),
                         pack_bf16x2(v[8 * j + 6] * scale, v[8 * j + 7] * scale));
    *reinterpret_cast<uint4*>(s + r * 64 + ((j ^ ((r >> 1) & 3)) << 4)) = q;
  }
}

enum StoreKind { ST_STORE = 0, ST_ADD = 1 };

__device__ __forceinline__ void issue_store(const CUtensorMap* map, const uint8_t* s, int col, int row, int kind) {
  fence_async_smem();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    if (kind == ST_ADD) tma_reduce_add_2d(map, s, col, row);
    else tma_store_2d(map, s, col, row);
    bulk_commit();
  }
}

__device__ __forceinline__ void tmem_load_f32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Two 32-column TMEM loads behind one wait.
__device__ __forceinline__ void tmem_load_f32x2(uint32_t ta, float (&v)[32], uint32_t tb, float (&w)[32]) {
  uint32_t r[32], q[32];
  tmem_ld32(ta, r);
  tmem_ld32(tb, q);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = __uint_as_float(r[i]);
    w[i] = __uint_as_float(q[i]);
  }
}

// Visits the 32-column chunks [0, ncols) of this warp's accumulator lanes in order,
// fn(c, v) with v the chunk's 32 fp32 values; the TMEM load of chunk c + 32 is in
// flight while fn processes chunk c.
template <class Fn>
__device__ __forceinline__ void tmem_walk(uint32_t tacc, int ncols, Fn&& fn) {
  uint32_t ra[32], rb[32];
  float v[32];
  tmem_ld32(tacc, ra);
  tmem_wait_ld_regs(ra);
#pragma unroll 1
  for (int c = 0; c < ncols; c += 64) {
    const bool has_b = c + 32 < ncols;
    if (has_b) tmem_ld32(tacc + c + 32, rb);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(ra[i]);
    fn(c, v);
    if (has_b) {
      tmem_wait_ld_regs(rb);
      const bool has_a = c + 64 < ncols;
      if (has_a) tmem_ld32(tacc + c + 64, ra);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(rb[i]);
      fn(c + 32, v);
      if (has_a) tmem_wait_ld_regs(ra);
    }
  }
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Called by an epilogue warp before it waits for the tile's accumulator: inputs of the
// epilogue that do not depend on the MMAs start moving towards the SM (into L2) while
// the MMAs run.
template <int BN>
__device__ __forceinline__ void prefetch_epilogue(const GemmArgs& a, int row0, int nb) {
  if (a.epi != EPI_SWIGLU_BWD) return;
  const int row = row0 + (threadIdx.x & 31);
  if (row >= a.M) return;
  const int c0 = nb * BN, c1 = min(c0 + BN, a.N);
  const __nv_bfloat16* gr = a.gu + static_cast<long>(row) * 2 * a.F;
  for (int c = c0; c < c1; c += 64) {  // 128-byte lines of g and of u
    asm volatile("prefetch.global.L2 [%0];" ::"l"(gr + c));
    asm volatile("prefetch.global.L2 [%0];" ::"l"(gr + a.F + c));
  }
}

// Epilogue of one 128 x BN tile for the 32 rows [row0, row0 + 32) owned by this warp.
template <int BN, class Stg>
__device__ __forceinline__ void run_epilogue(const GemmArgs& a, const CUtensorMap* tm_out, const CUtensorMap* tm_aux,
                                             Stg& st, uint32_t tacc, int row0, int nb) {
  const int lane = threadIdx.x & 31;
  const int row = row0 + lane;
  const bool row_ok = row < a.M;
  float v[32];
  switch (a.epi) {
    case EPI_BF16:
    case EPI_F32:
    case EPI_ADD_F32: {
      tmem_walk(tacc, BN, [&](int c, float (&x)[32]) {
        const int col = nb * BN + c;
        if (col >= a.N) return;  // uniform across the warp
        uint8_t* s = st.acquire();
        if (a.epi == EPI_BF16) stage_bf16(s, x, a.alpha);
        else stage_f32(s, x, a.alpha);
        issue_store(tm_out, s, col, row0, a.epi == EPI_ADD_F32 ? ST_ADD : ST_STORE);
        st.release();
      });
      break;
    }
    case EPI_SWIGLU: {
      // acc columns [0, BN/2) = gate, [BN/2, BN) = up, for h columns [nb*BN/2, ...).
      constexpr int HB = BN / 2;
      float u[32];
#pragma unroll 1
      for (int c = 0; c < HB; c += 32) {
        tmem_load_f32x2(tacc + c, v, tacc + HB + c, u);
        const int col = nb * HB + c;
        if (col >= a.F) continue;
        // Round the pre-activations once and compute h from the rounded values, so
        // the backward pass (which reads the saved bf16 values) sees the same inputs.
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = bf16_round(v[i]);
          u[i] = bf16_round(u[i]);
        }
        uint8_t* s = st.acquire();
        stage_bf16(s, v, 1.f);
        issue_store(tm_aux, s, col, row0, ST_STORE);
        st.release();
        s = st.acquire();
        stage_bf16(s, u, 1.f);
        issue_store(tm_aux, s, a.F + col, row0, ST_STORE);
        st.release();
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __fdividef(v[i] * u[i], 1.f + __expf(-v[i]));
        s = st.acquire();
        stage_bf16(s, v, 1.f);
        issue_store(tm_out, s, col, row0, ST_STORE);
        st.release();
      }
      break;
    }
    case EPI_SWIGLU_BWD: {
      // The accumulator is dh = dL/dh for h columns [nb*BN, ...); with the saved gate
      // and up pre-activations of this row it becomes dg = dh u s (1 + g (1 - s)) and
      // du = dh g s (s = sigmoid(g)), stored into [dg | du] (bf16 [M, 2F]), so dh never
      // reaches HBM.  The row's g / u segments were prefetched into L2 before the
      // accumulator was ready (prefetch_epilogue); here the loads of the next 32 columns
      // are in flight while the current ones are processed.
      const __nv_bfloat16* gr = a.gu + static_cast<long>(row_ok ? row : 0) * 2 * a.F;
      float u[32];
      uint4 gv[4], uv[4], gn[4], un[4];
      auto load = [&](int col, uint4 (&g4)[4], uint4 (&u4)[4]) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          g4[j] = row_ok && col < a.N ? __ldg(reinterpret_cast<const uint4*>(gr + col) + j) : make_uint4(0, 0, 0, 0);
          u4[j] = row_ok && col < a.N ? __ldg(reinterpret_cast<const uint4*>(gr + a.F + col) + j) : make_uint4(0, 0, 0, 0);
        }
      };
      load(nb * BN, gv, uv);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        const int col = nb * BN + c;
        if (col >= a.N) break;  // uniform across the warp
        if (c + 32 < BN) load(col + 32, gn, un);
        tmem_load_f32(tacc + c, v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t* gp = &gv[j].x;
          const uint32_t* up = &uv[j].x;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 g2 = unpack_bf16x2(gp[k]), u2 = unpack_bf16x2(up[k]);
            const int i = 8 * j + 2 * k;
            const float s0 = sigmoidf_(g2.x), s1 = sigmoidf_(g2.y);
            const float d0 = v[i], d1 = v[i + 1];
            v[i] = d0 * u2.x * s0 * (1.f + g2.x * (1.f - s0));
            v[i + 1] = d1 * u2.y * s1 * (1.f + g2.y * (1.f - s1));
            u[i] = d0 * g2.x * s0;
            u[i + 1] = d1 * g2.y * s1;
          }
        }
        uint8_t* s = st.acquire();
        stage_bf16(s, v, 1.f);
        issue_store(tm_out, s, col, row0, ST_STORE);
        st.release();
        s = st.acquire();
        stage_bf16(s, u, 1.f);
        issue_store(tm_out, s, a.F + col, row0, ST_STORE);
        st.release();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          gv[j] = gn[j];
          uv[j] = un[j];
        }
      }
      break;
    }
    case EPI_ROPE: {
      const int half = a.head_dim / 2;
      const int p = row_ok ? min(max(a.pos[row], 0), a.n_pos - 1) : 0;
      float w[32];
      if (half == 32) {
        // head_dim 64: this row's 32 (cos, sin) pairs serve every head of the tile
        float cs[32], sn[32];
        const float4* cr = reinterpret_cast<const float4*>(a.cos_t + static_cast<long>(p) * half);
        const float4* sr = reinterpret_cast<const float4*>(a.sin_t + static_cast<long>(p) * half);
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
          const float4 c4 = cr[i4], s4 = sr[i4];
          cs[4 * i4] = c4.x; cs[4 * i4 + 1] = c4.y; cs[4 * i4 + 2] = c4.z; cs[4 * i4 + 3] = c4.w;
          sn[4 * i4] = s4.x; sn[4 * i4 + 1] = s4.y; sn[4 * i4 + 2] = s4.z; sn[4 * i4 + 3] = s4.w;
        }
#pragma unroll 1
        for (int hb = 0; hb < BN; hb += 64) {
          const int hcol = nb * BN + hb;
          tmem_load_f32x2(tacc + hb, v, tacc + hb + 32, w);
          if (hcol >= a.N) continue;
          if (hcol < a.n_rope_cols) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float x1 = v[i], x2 = w[i];
              v[i] = x1 * cs[i] - x2 * sn[i];
              w[i] = x2 * cs[i] + x1 * sn[i];
            }
          }
          uint8_t* s = st.acquire();
          stage_bf16(s, v, 1.f);
          issue_store(tm_out, s, hcol, row0, ST_STORE);
          st.release();
          s = st.acquire();
          stage_bf16(s, w, 1.f);
          issue_store(tm_out, s, hcol + 32, row0, ST_STORE);
          st.release();
        }
        break;
      }
#pragma unroll 1
      for (int hb = 0; hb < BN; hb += a.head_dim) {
        const int hcol = nb * BN + hb;
        const bool rot = hcol < a.n_rope_cols;
#pragma unroll 1
        for (int j = 0; j < half; j += 32) {
          tmem_load_f32x2(tacc + hb + j, v, tacc + hb + half + j, w);
          if (hcol >= a.N) continue;
          if (rot) {
            const float4* cr = reinterpret_cast<const float4*>(a.cos_t + static_cast<long>(p) * half + j);
            const float4* sr = reinterpret_cast<const float4*>(a.sin_t + static_cast<long>(p) * half + j);
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) {
              const float4 c4 = cr[i4], s4 = sr[i4];
              const float cs[4] = {c4.x, c4.y, c4.z, c4.w};
              const float sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = 4 * i4 + e;
                const float x1 = v[i], x2 = w[i];
                v[i] = x1 * cs[e] - x2 * sn[e];
                w[i] = x2 * cs[e] + x1 * sn[e];
              }
            }
          }
          uint8_t* s = st.acquire();
          stage_bf16(s, v, 1.f);
          issue_store(tm_out, s, hcol + j, row0, ST_STORE);
          st.release();
          s = st.acquire();
          stage_bf16(s, w, 1.f);
          issue_store(tm_out, s, hcol + half + j, row0, ST_STORE);
          st.release();
        }
      }
      break;
    }
    case EPI_CE_FWD: {
      float mx = -INFINITY, se = 0.f;
      const int64_t tgt = row_ok ? a.targets[row] : -1;
      tmem_walk(tacc, BN, [&](int c, float (&x)[32]) {
        const int col = nb * BN + c;
        const int valid = min(32, a.N - col);
        if (valid <= 0) return;
        if (a.keep_logits) {
          // the statistics are taken from the stored (bf16-rounded) logits, so the
          // backward's softmax from them is normalised against this lse
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = bf16_round(x[i]);
          uint8_t* s = st.acquire();
          stage_bf16(s, x, 1.f);
          issue_store(tm_aux, s, col, row0, ST_STORE);
          st.release();
        }
        float cm = -INFINITY;
#pragma unroll
        for (int i = 0; i < 32; ++i) cm = fmaxf(cm, i < valid ? x[i] : -INFINITY);
        const float nm = fmaxf(mx, cm);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) s += i < valid ? __expf(x[i] - nm) : 0.f;
        se = se * __expf(mx - nm) + s;
        mx = nm;
        if (tgt >= col && tgt < col + valid) {
          float t = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) t = (tgt == col + i) ? x[i] : t;
          a.tlogit[row] = t;
        }
      });
      if (row_ok) {
        a.pmax[static_cast<long>(nb) * a.M + row] = mx;
        a.psum[static_cast<long>(nb) * a.M + row] = se;
      }
      break;
    }
    case EPI_CE_BWD: {
      float l = 0.f, scale = 0.f, zf = 1.f;
      int64_t tgt = -1;
      if (row_ok) {
        l = a.lse[row];
        scale = a.row_scale[row];
        tgt = a.targets[row];
        zf = 1.f + 2.f * a.z_coeff * l;
      }
      tmem_walk(tacc, BN, [&](int c, float (&x)[32]) {
        const int col = nb * BN + c;
        if (col >= a.N) return;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float g = __expf(x[i] - l) * zf;
          g -= (tgt == col + i) ? 1.f : 0.f;
          x[i] = g * scale;
        }
        uint8_t* s = st.acquire();
        stage_bf16(s, x, 1.f);
        issue_store(tm_out, s, col, row0, ST_STORE);
        st.release();
      });
      break;
    }
    default:
      break;
  }
}

// ------------------------------------ kernel --------------------------------------
template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(256, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ CUtensorMap tm_aux,
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
      uint32_t issued_mask = 0, issued_phase = 0;  // per stage: has a load, its phase
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int mb, nb, sp;
        tile_coords(args, tile, mb, nb, sp);
        const int kb0 = sp * args.kb_per_split;
        const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
        if (args.ag.world > 0) {
          // The B rows of this tile must have been gathered (K-major B only).
          const long K = args.K;
          if (swiglu) {
            const long r0 = static_cast<long>(nb) * (BN / 2), r1 = min(r0 + BN / 2, static_cast<long>(args.F));
            ok = ag_wait_range(args.ag, args.ag.b0 + r0 * K, args.ag.b0 + r1 * K, args.status, 107, &abort_sh) &&
                 ag_wait_range(args.ag, args.ag.b0 + (args.F + r0) * K, args.ag.b0 + (args.F + r1) * K, args.status,
                               107, &abort_sh);
          } else {
            const long r0 = static_cast<long>(nb) * BN, r1 = min(r0 + BN, static_cast<long>(args.N));
            ok = ag_wait_range(args.ag, args.ag.b0 + r0 * K, args.ag.b0 + r1 * K, args.status, 107, &abort_sh);
          }
          if (!ok) break;
        }
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
          issued_mask |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded, once more) for the copies this thread issued.
        for (int s = 0; s < C::STAGES; ++s)
          if (issued_mask & (1u << s)) mbar_wait(&full_bar[s], (issued_phase >> s) & 1u, args.status, 102, nullptr);
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
  } else if (warp >= 6) {
    if (args.ag.world > 0) ag_copy_warp(args.ag);
  } else {
    const int q = warp & 3;
    Stager st{smem + C::EPI_OFF + q * kEpiWarpBytes, 0, args.epi == EPI_F32 || args.epi == EPI_ADD_F32};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb, sp;
      tile_coords(args, tile, mb, nb, sp);
      prefetch_epilogue<BN>(args, mb * C::BM + q * 32, nb);
      if (!mbar_wait_warp(&accf_bar[acc], acc_phase, args.status, 106, &abort_sh)) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      run_epilogue<BN>(args, &tm_out, &tm_aux, st, tacc, mb * C::BM + q * 32, nb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    // Bulk stores must have read their staging slots (and be complete) before exit.
    if (lane == 0) bulk_wait_all<0>();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace pb
