// Document-masked causal GQA attention for packed sequences, sm_100a (tcgen05/TMEM/TMA).
//
// Input is the fused QKV GEMM output qkv[T, (H + 2 Hkv) * D] (bf16, RoPE applied).
// Query t attends to key k iff doc_start[t] <= k <= t.  Head dims 64 and 128.
//
// Forward (persistent; work items = (query tile of 128 rows, head), pre-sorted by
// number of key tiles, most expensive first):
//   warp 0      TMA: Q tile once per item, K/V tiles into a 2-deep ring
//   warp 1      tcgen05.mma: S_j = Q K_j^T into one of two TMEM S buffers, then
//               O += P_{j-1} V_{j-1} with P read from TMEM (A operand in tensor memory)
//   warps 2..5  softmax, thread = query row: masking from doc_start, online max/sum in
//               base 2, O rescale in TMEM when the max grows, P -> TMEM (bf16), final
//               O / l and the log-sum-exp.
// Only key tiles from the first document start of the query tile up to the tile's
// last row are visited; tiles entirely inside the causal/document window skip the
// per-element mask.
//
// Backward (persistent; items = (key tile, kv head), q tiles [kv tile, last query tile
// whose document reaches the key tile], all query heads of the GQA group):
//   S^T = K Q^T and dP^T = V dO^T in TMEM (thread = key row), P^T and
//   dS^T = P^T (dP^T - delta) written once to shared memory in the 128B-swizzled
//   layout that serves both as K-major A (dV += P^T dO, dK += dS^T Q) and as MN-major
//   A (dQ = dS K); dQ partials go to an fp32 buffer with vector atomics, dK/dV stay in
//   TMEM for the whole item and are written once.
//
// All waits are bounded (common.cuh); codes 2xx.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "host_utils.h"

namespace pb {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Write 8 bf16 (one 16-byte chunk) of row ``r``, chunk ``c`` (0..15 over 128 columns)
// of a [128 rows x 128 cols] bf16 tile stored as two 128B-swizzled column halves.
__device__ __forceinline__ void st_swz_chunk(uint8_t* tile, int r, int c, uint4 v) {
  const int half = c >> 3;
  const int cc = c & 7;
  uint8_t* p = tile + half * 16384 + (r >> 3) * 1024 + (r & 7) * 128 + ((cc ^ (r & 7)) << 4);
  *reinterpret_cast<uint4*>(p) = v;
}

struct AttnArgs {
  int T, H, Hkv, D;
  float scale_log2;  // softmax scale * log2(e)
  float scale;
  const int* doc_start;
  const int* items;  // fwd: [n, 2] (q tile, head); bwd: [n, 3] (kv tile, kv head, last q tile)
  int n_items;
  __nv_bfloat16* out;  // fwd output [T, H*D]
  float* lse;          // [H, T] natural-log LSE
  // backward
  const float* delta;  // [H, T]
  float* dq_acc;       // [T, H*D] fp32
  __nv_bfloat16* dqkv;  // [T, (H+2Hkv)*D]
  long ld_dqkv;
  int* status;
};

// =================================== forward ======================================
template <int D>
struct FwdCfg {
  static constexpr int TILE_BYTES = 128 * D * 2;  // one 128-row tile of Q, K or V
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = TILE_BYTES;             // 2 stages
  static constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;  // 2 stages
  // At least 120 KB so that a second CTA (which would block in tcgen05.alloc on
  // the fully allocated TMEM) is never co-scheduled on the same SM.
  static constexpr int SMEM_USED = V_OFF + 2 * TILE_BYTES + 1024;
  static constexpr int SMEM = SMEM_USED > 122880 ? SMEM_USED : 122880;
  static constexpr uint32_t S_COL = 0;    // two S buffers: 0, 128
  static constexpr uint32_t P_COL = 256;  // two P buffers (bf16 packed): 256, 320
  static constexpr uint32_t O_COL = 384;  // D columns
  static constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 128, false, false);
  static constexpr uint32_t IDESC_O = idesc_bf16_f32(128, D, false, true);
};

__device__ __forceinline__ void load_tile_rows(void* dst, const CUtensorMap* map, uint64_t* bar, int col0, int row0,
                                               int D) {
  for (int c = 0; c < D / 64; ++c)
    tma_load_2d(static_cast<uint8_t*>(dst) + c * 16384, map, bar, col0 + c * 64, row0);
}

template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap, const AttnArgs args) {
  using C = FwdCfg<D>;
  __shared__ __align__(8) uint64_t q_full, q_empty, kv_full[2], kv_empty[2], s_full[2], p_ready, o_done, o_free,
      drain_bar;
  __shared__ uint32_t tmem_sh;
  __shared__ volatile int abort_sh;
  extern __shared__ uint8_t dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
    }
    mbar_init(&p_ready, 4);
    mbar_init(&o_done, 1);
    mbar_init(&o_free, 4);
    mbar_init(&drain_bar, 1);
    abort_sh = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tmap);
  if (warp == 1) {
    tmem_alloc(&tmem_sh, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  const int H = args.H, Hkv = args.Hkv, T = args.T;
  const int group = H / Hkv;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t kv_it = 0, q_it = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x) {
        const int qt = args.items[2 * it], h = args.items[2 * it + 1];
        const int hk = h / group;
        const int q0 = qt * 128;
        const int kt0 = args.doc_start[q0] / 128;
        if (!mbar_wait(&q_empty, (q_it & 1) ^ 1, args.status, 201, &abort_sh)) break;
        mbar_arrive_expect_tx(&q_full, C::TILE_BYTES);
        load_tile_rows(smem + C::Q_OFF, &tmap, &q_full, h * D, q0, D);
        ++q_it;
        for (int kt = kt0; kt <= qt; ++kt, ++kv_it) {
          const int s = kv_it & 1;
          if (!mbar_wait(&kv_empty[s], ((kv_it >> 1) & 1) ^ 1, args.status, 202, &abort_sh)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[s], 2 * C::TILE_BYTES);
          load_tile_rows(smem + C::K_OFF + s * C::TILE_BYTES, &tmap, &kv_full[s], (H + hk) * D, kt * 128, D);
          load_tile_rows(smem + C::V_OFF + s * C::TILE_BYTES, &tmap, &kv_full[s], (H + Hkv + hk) * D, kt * 128, D);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t kv_it = 0, q_it = 0, p_it = 0, item_n = 0;
      bool ok = true;
      const uint32_t qa = smem_u32(smem + C::Q_OFF);
      for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x, ++item_n) {
        const int qt = args.items[2 * it];
        const int q0 = qt * 128;
        const int kt0 = args.doc_start[q0] / 128;
        const int nkv = qt - kt0 + 1;
        if (!mbar_wait(&q_full, q_it & 1, args.status, 203, &abort_sh)) break;
        ++q_it;
        // O of the previous item must have been read out before it is overwritten.
        if (!mbar_wait(&o_free, (item_n & 1) ^ 1, args.status, 204, &abort_sh)) break;
        tc_fence_after();
        for (int j = 0; j <= nkv && ok; ++j) {
          if (j < nkv) {
            const uint32_t g = kv_it + j;
            const int s = g & 1;
            if (!mbar_wait(&kv_full[s], (g >> 1) & 1, args.status, 205, &abort_sh)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t ka = smem_u32(smem + C::K_OFF + s * C::TILE_BYTES);
            const uint32_t sb = tmem + C::S_COL + (g & 1) * 128;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
              umma_ss(sb, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024), C::IDESC_S,
                      kk > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[g & 1]);
            if (j == nkv - 1) umma_commit(&q_empty);
          }
          if (j > 0) {
            const uint32_t g = kv_it + j - 1;
            if (!mbar_wait(&p_ready, p_it & 1, args.status, 206, &abort_sh)) {
              ok = false;
              break;
            }
            ++p_it;
            tc_fence_after();
            const int s = g & 1;
            const uint32_t va = smem_u32(smem + C::V_OFF + s * C::TILE_BYTES);
            const uint32_t pa = tmem + C::P_COL + (g & 1) * 64;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_ts(tmem + C::O_COL, pa + kk * 8, sdesc_sw128(va + kk * 2048, 16384, 1024), C::IDESC_O,
                      (j > 1 || kk > 0) ? 1u : 0u);
            umma_commit(&o_done);
            umma_commit(&kv_empty[s]);
          }
        }
        kv_it += nkv;
      }
      umma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, args.status, 207, nullptr);
    }
  } else {
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    uint32_t kv_it = 0, o_it = 0, p_cnt = 0;
    for (int it = blockIdx.x; it < args.n_items; it += gridDim.x) {
      const int qt = args.items[2 * it], h = args.items[2 * it + 1];
      const int q0 = qt * 128;
      const int kt0 = args.doc_start[q0] / 128;
      const int nkv = qt - kt0 + 1;
      const int q = q0 + r;
      const bool qok = q < T;
      const int lo = qok ? args.doc_start[q] : 0x7fffffff;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        const uint32_t g = kv_it + j;
        if (!mbar_wait_warp(&s_full[g & 1], (g >> 1) & 1, args.status, 208, &abort_sh)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int kv0 = (kt0 + j) * 128;
        float s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + C::S_COL + (g & 1) * 128 + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(v[i]) * args.scale_log2;
        }
        const bool full = kv0 >= lo && kv0 + 127 <= q;
        float mx = -INFINITY;
        if (full) {
#pragma unroll
          for (int i = 0; i < 128; ++i) mx = fmaxf(mx, s[i]);
        } else {
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            const int k = kv0 + i;
            if (k < lo || k > q) s[i] = -INFINITY;
            mx = fmaxf(mx, s[i]);
          }
        }
        const float m_new = fmaxf(m, mx);
        const float base = m_new == -INFINITY ? 0.f : m_new;
        const float corr = fast_exp2(m - base);  // m == -inf -> 0
        float sum = 0.f;
        uint32_t pk[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float p0 = fast_exp2(s[2 * i] - base);
          const float p1 = fast_exp2(s[2 * i + 1] - base);
          sum += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
        l = l * corr + sum;
        // PV of the previous tile must be complete before O is rescaled or its P slot
        // (two tiles back) is overwritten.
        if (j > 0) {
          if (!mbar_wait_warp(&o_done, o_it & 1, args.status, 209, &abort_sh)) {
            ok = false;
            break;
          }
          ++o_it;
          tc_fence_after();
          // Warp-uniform decision: the TMEM load/store below are .sync.aligned.
          if (__any_sync(0xffffffff, corr != 1.f)) {
#pragma unroll
            for (int c = 0; c < D; c += 16) {
              uint32_t ov[16];
              tmem_ld16(tmem + lane_off + C::O_COL + c, ov);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * corr);
              tmem_st16(tmem + lane_off + C::O_COL + c, ov);
            }
          }
        }
        m = m_new;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pv[i] = pk[c * 16 + i];
          tmem_st16(tmem + lane_off + C::P_COL + (g & 1) * 64 + c * 16, pv);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready);
        ++p_cnt;
      }
      if (!ok) break;
      // Epilogue: wait for the last PV, normalise and store.
      if (!mbar_wait_warp(&o_done, o_it & 1, args.status, 210, &abort_sh)) break;
      ++o_it;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int c = 0; c < D; c += 16) {
        uint32_t ov[16];
        tmem_ld16(tmem + lane_off + C::O_COL + c, ov);
        tmem_wait_ld();
        if (qok) {
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            pk[i] = pack_bf16x2(__uint_as_float(ov[2 * i]) * inv, __uint_as_float(ov[2 * i + 1]) * inv);
          uint4* dst = reinterpret_cast<uint4*>(args.out + static_cast<long>(q) * H * D + h * D + c);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      if (qok) args.lse[static_cast<long>(h) * T + q] = l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free);
      kv_it += nkv;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =================================== backward =====================================
template <int D>
struct BwdCfg {
  static constexpr int TILE_BYTES = 128 * D * 2;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE_BYTES;
  static constexpr int Q_OFF = 2 * TILE_BYTES;
  static constexpr int DO_OFF = 3 * TILE_BYTES;
  static constexpr int P_OFF = 4 * TILE_BYTES;      // P^T  [128 kv x 128 q] bf16, 32 KB
  static constexpr int DS_OFF = P_OFF + 32768;      // dS^T [128 kv x 128 q] bf16, 32 KB
  static constexpr int VEC_OFF = DS_OFF + 32768;    // 2 x {lse2[128], delta[128], doc_start[128]}
  static constexpr int SMEM = VEC_OFF + 2 * 3 * 512 + 1024;
  static constexpr uint32_t ST_COL = 0;    // S^T, later dQ
  static constexpr uint32_t DPT_COL = 128; // dP^T
  static constexpr uint32_t DV_COL = 256;
  static constexpr uint32_t DK_COL = 256 + D;
  static constexpr uint32_t IDESC_SQ = idesc_bf16_f32(128, 128, false, false);  // S^T, dP^T
  static constexpr uint32_t IDESC_KV = idesc_bf16_f32(128, D, false, true);     // dV, dK: A K-major, B MN-major
  static constexpr uint32_t IDESC_DQ = idesc_bf16_f32(128, D, true, true);      // dQ: A MN-major, B MN-major
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                    const AttnArgs args) {
  using C = BwdCfg<D>;
  __shared__ __align__(8) uint64_t kv_full, kv_empty, qd_full, qd_empty, st_full, ds_ready, mma2_done, dq_read,
      acc_done, acc_free, drain_bar, vec_bar;
  __shared__ uint32_t tmem_sh;
  __shared__ volatile int abort_sh;
  extern __shared__ uint8_t dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(&kv_full, 1);
    mbar_init(&kv_empty, 1);
    mbar_init(&qd_full, 1);
    mbar_init(&qd_empty, 1);
    mbar_init(&st_full, 1);
    mbar_init(&ds_ready, 4);
    mbar_init(&mma2_done, 1);
    mbar_init(&dq_read, 4);
    mbar_init(&acc_done, 1);
    mbar_init(&acc_free, 4);
    mbar_init(&drain_bar, 1);
    mbar_init(&vec_bar, 128);
    abort_sh = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_sh, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_sh;
  const int H = args.H, Hkv = args.Hkv, T = args.T;
  const int group = H / Hkv;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t item_n = 0, qd_it = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x, ++item_n) {
        const int kt = args.items[3 * it], hk = args.items[3 * it + 1], qhi = args.items[3 * it + 2];
        if (!mbar_wait(&kv_empty, (item_n & 1) ^ 1, args.status, 221, &abort_sh)) break;
        mbar_arrive_expect_tx(&kv_full, 2 * C::TILE_BYTES);
        load_tile_rows(smem + C::K_OFF, &tm_qkv, &kv_full, (H + hk) * D, kt * 128, D);
        load_tile_rows(smem + C::V_OFF, &tm_qkv, &kv_full, (H + Hkv + hk) * D, kt * 128, D);
        for (int hh = 0; hh < group && ok; ++hh) {
          const int h = hk * group + hh;
          for (int qt = kt; qt <= qhi; ++qt, ++qd_it) {
            if (!mbar_wait(&qd_empty, (qd_it & 1) ^ 1, args.status, 222, &abort_sh)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&qd_full, 2 * C::TILE_BYTES);
            load_tile_rows(smem + C::Q_OFF, &tm_qkv, &qd_full, h * D, qt * 128, D);
            load_tile_rows(smem + C::DO_OFF, &tm_do, &qd_full, h * D, qt * 128, D);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t item_n = 0, qd_it = 0;
      bool ok = true;
      const uint32_t ka = smem_u32(smem + C::K_OFF), va = smem_u32(smem + C::V_OFF);
      const uint32_t qa = smem_u32(smem + C::Q_OFF), da = smem_u32(smem + C::DO_OFF);
      const uint32_t pa = smem_u32(smem + C::P_OFF), dsa = smem_u32(smem + C::DS_OFF);
      for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x, ++item_n) {
        const int kt = args.items[3 * it], qhi = args.items[3 * it + 2];
        if (!mbar_wait(&kv_full, item_n & 1, args.status, 223, &abort_sh)) break;
        if (!mbar_wait(&acc_free, (item_n & 1) ^ 1, args.status, 224, &abort_sh)) break;
        tc_fence_after();
        bool first = true;
        const int n_inner = group * (qhi - kt + 1);
        for (int n = 0; n < n_inner; ++n, ++qd_it) {
          if (!mbar_wait(&qd_full, qd_it & 1, args.status, 225, &abort_sh)) {
            ok = false;
            break;
          }
          // S^T / dQ columns: the previous dQ must have been read out.
          if (!mbar_wait(&dq_read, (qd_it & 1) ^ 1, args.status, 226, &abort_sh)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_ss(tmem + C::ST_COL, sdesc_sw128(ka + off, 16, 1024), sdesc_sw128(qa + off, 16, 1024), C::IDESC_SQ,
                    kk > 0 ? 1u : 0u);
            umma_ss(tmem + C::DPT_COL, sdesc_sw128(va + off, 16, 1024), sdesc_sw128(da + off, 16, 1024),
                    C::IDESC_SQ, kk > 0 ? 1u : 0u);
          }
          umma_commit(&st_full);
          if (!mbar_wait(&ds_ready, qd_it & 1, args.status, 227, &abort_sh)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;  // K-major A over q (K dim)
            const uint32_t boff = kk * 2048;                          // MN-major B: 16 q rows
            const uint32_t acc = (first && kk == 0) ? 0u : 1u;
            umma_ss(tmem + C::DV_COL, sdesc_sw128(pa + aoff, 16, 1024), sdesc_sw128(da + boff, 16384, 1024),
                    C::IDESC_KV, acc);
            umma_ss(tmem + C::DK_COL, sdesc_sw128(dsa + aoff, 16, 1024), sdesc_sw128(qa + boff, 16384, 1024),
                    C::IDESC_KV, acc);
          }
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = kk * 2048;  // 16 kv rows
            umma_ss(tmem + C::ST_COL, sdesc_sw128(dsa + off, 16384, 1024), sdesc_sw128(ka + off, 16384, 1024),
                    C::IDESC_DQ, kk > 0 ? 1u : 0u);
          }
          umma_commit(&mma2_done);
          umma_commit(&qd_empty);
          first = false;
        }
        if (!ok) break;
        umma_commit(&acc_done);
        umma_commit(&kv_empty);
      }
      umma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, args.status, 228, nullptr);
    }
  } else {
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;  // key row within the tile (and query row for dQ)
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    float* vec_base = reinterpret_cast<float*>(smem + C::VEC_OFF);
    uint8_t* ptile = smem + C::P_OFF;
    uint8_t* dstile = smem + C::DS_OFF;
    uint32_t item_n = 0, qd_it = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x, ++item_n) {
      const int kt = args.items[3 * it], hk = args.items[3 * it + 1], qhi = args.items[3 * it + 2];
      const int kv = kt * 128 + r;
      for (int hh = 0; hh < group && ok; ++hh) {
        const int h = hk * group + hh;
        for (int qt = kt; qt <= qhi; ++qt, ++qd_it) {
          const int q0 = qt * 128;
          // Per-query vectors of this tile, double-buffered by iteration parity.  Every
          // thread arrives on vec_bar after writing its element; a thread can only be
          // here once all threads passed the previous iteration's vec_bar, i.e. after
          // they finished reading the buffer two iterations back.
          float* s_lse = vec_base + (qd_it & 1) * 384;
          float* s_delta = s_lse + 128;
          int* s_ds = reinterpret_cast<int*>(s_delta + 128);
          {
            const int q = q0 + r;
            const bool qok = q < T;
            s_lse[r] = qok ? args.lse[static_cast<long>(h) * T + q] * kLog2e : INFINITY;
            s_delta[r] = qok ? args.delta[static_cast<long>(h) * T + q] : 0.f;
            s_ds[r] = qok ? args.doc_start[q] : 0x7fffffff;
          }
          mbar_arrive(&vec_bar);
          if (!mbar_wait_warp(&vec_bar, qd_it & 1, args.status, 233, &abort_sh)) {
            ok = false;
            break;
          }
          if (!mbar_wait_warp(&st_full, qd_it & 1, args.status, 229, &abort_sh)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // P/dS smem of the previous iteration was consumed by its MMAs: this thread
          // waited for them (mma2_done) before reading that iteration's dQ.
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t sv[32], dv[32];
            tmem_ld32(tmem + lane_off + C::ST_COL + c * 32, sv);
            tmem_ld32(tmem + lane_off + C::DPT_COL + c * 32, dv);
            tmem_wait_ld();
            uint32_t pp[16], dd[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float p2[2], d2[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int j = c * 32 + 2 * i + e;
                const int q = q0 + j;
                const bool allowed = q >= kv && s_ds[j] <= kv;
                const float p = allowed ? fast_exp2(__uint_as_float(sv[2 * i + e]) * args.scale_log2 - s_lse[j]) : 0.f;
                p2[e] = p;
                d2[e] = p * (__uint_as_float(dv[2 * i + e]) - s_delta[j]);
              }
              pp[i] = pack_bf16x2(p2[0], p2[1]);
              dd[i] = pack_bf16x2(d2[0], d2[1]);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              st_swz_chunk(ptile, r, c * 4 + k, make_uint4(pp[4 * k], pp[4 * k + 1], pp[4 * k + 2], pp[4 * k + 3]));
              st_swz_chunk(dstile, r, c * 4 + k, make_uint4(dd[4 * k], dd[4 * k + 1], dd[4 * k + 2], dd[4 * k + 3]));
            }
          }
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ds_ready);
          // dQ rows (thread = query row) -> fp32 atomics.
          if (!mbar_wait_warp(&mma2_done, qd_it & 1, args.status, 231, &abort_sh)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int q = q0 + r;
#pragma unroll 1
          for (int c = 0; c < D; c += 32) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_off + C::ST_COL + c, v);
            tmem_wait_ld();
            if (q < T) {
              float4* dst = reinterpret_cast<float4*>(args.dq_acc + static_cast<long>(q) * H * D + h * D + c);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                atomicAdd(dst + i, make_float4(__uint_as_float(v[4 * i]) * args.scale, __uint_as_float(v[4 * i + 1]) * args.scale,
                                               __uint_as_float(v[4 * i + 2]) * args.scale,
                                               __uint_as_float(v[4 * i + 3]) * args.scale));
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dq_read);
        }
      }
      if (!ok) break;
      // dK (scaled) and dV of this key tile.
      if (!mbar_wait_warp(&acc_done, item_n & 1, args.status, 232, &abort_sh)) break;
      tc_fence_after();
      const int hcol_k = (H + hk) * D, hcol_v = (H + Hkv + hk) * D;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t kvv[32], vvv[32];
        tmem_ld32(tmem + lane_off + C::DK_COL + c, kvv);
        tmem_ld32(tmem + lane_off + C::DV_COL + c, vvv);
        tmem_wait_ld();
        if (kv < T) {
          uint32_t pk[16], pv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            pk[i] = pack_bf16x2(__uint_as_float(kvv[2 * i]) * args.scale, __uint_as_float(kvv[2 * i + 1]) * args.scale);
            pv[i] = pack_bf16x2(__uint_as_float(vvv[2 * i]), __uint_as_float(vvv[2 * i + 1]));
          }
          uint4* dk = reinterpret_cast<uint4*>(args.dqkv + static_cast<long>(kv) * args.ld_dqkv + hcol_k + c);
          uint4* dvp = reinterpret_cast<uint4*>(args.dqkv + static_cast<long>(kv) * args.ld_dqkv + hcol_v + c);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dk[i] = make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
            dvp[i] = make_uint4(pv[4 * i], pv[4 * i + 1], pv[4 * i + 2], pv[4 * i + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[h, t] = sum_d O[t, h, d] * dO[t, h, d]
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                  float* __restrict__ delta, int T, int H, int D) {
  const long idx = blockIdx.x * (long)(blockDim.x / 32) + threadIdx.x / 32;  // (t, h) pair per warp
  const int lane = threadIdx.x % 32;
  if (idx >= static_cast<long>(T) * H) return;
  const int t = static_cast<int>(idx / H), h = static_cast<int>(idx % H);
  const __nv_bfloat16* a = o + static_cast<long>(t) * H * D + h * D;
  const __nv_bfloat16* b = dout + static_cast<long>(t) * H * D + h * D;
  float s = 0.f;
  for (int d = lane * 2; d < D; d += 64) {
    const float2 x = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(a + d));
    const float2 y = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(b + d));
    s += x.x * y.x + x.y * y.y;
  }
  s = warp_sum(s);
  if (lane == 0) delta[static_cast<long>(h) * T + t] = s;
}

__global__ void dq_convert_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dqkv, long ld, int T,
                                  int HD) {
  const long n = static_cast<long>(T) * HD / 2;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long e = 2 * i;
    const int t = static_cast<int>(e / HD), c = static_cast<int>(e % HD);
    const float2 v = reinterpret_cast<const float2*>(acc)[i];
    *reinterpret_cast<uint32_t*>(dqkv + t * ld + c) = pack_bf16x2(v.x, v.y);
  }
}

// ------------------------------------ host ----------------------------------------
template <typename K>
static void set_smem(K kern, int bytes) {
  PB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

std::vector<at::Tensor> attn_fwd(at::Tensor qkv, at::Tensor doc_start, at::Tensor items, int64_t H, int64_t Hkv,
                                 int64_t D, double scale, at::Tensor out) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.is_contiguous());
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim must be 64 or 128");
  TORCH_CHECK(H % Hkv == 0 && qkv.size(1) == (H + 2 * Hkv) * D, "attention: qkv width");
  TORCH_CHECK(doc_start.scalar_type() == at::kInt && items.scalar_type() == at::kInt && items.is_contiguous());
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int T = qkv.size(0);
  auto lse = at::empty({H, T}, qkv.options().dtype(at::kFloat));
  if (T == 0) return {out, lse};
  CUtensorMap tm = make_tmap_bf16_2d(qkv.data_ptr(), qkv.size(1), T, qkv.stride(0) * 2, 64, 128);
  AttnArgs a{};
  a.T = T;
  a.H = (int)H;
  a.Hkv = (int)Hkv;
  a.D = (int)D;
  a.scale = (float)scale;
  a.scale_log2 = (float)scale * kLog2e;
  a.doc_start = doc_start.data_ptr<int>();
  a.items = items.data_ptr<int>();
  a.n_items = items.size(0);
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.lse = lse.data_ptr<float>();
  a.status = status_ptr(qkv.device().index());
  const int grid = std::min<int>(a.n_items, num_sms(qkv.device().index()));
  auto s = at::cuda::getCurrentCUDAStream();
  if (D == 64) {
    set_smem(attn_fwd_kernel<64>, FwdCfg<64>::SMEM);
    attn_fwd_kernel<64><<<grid, 192, FwdCfg<64>::SMEM, s>>>(tm, a);
  } else {
    set_smem(attn_fwd_kernel<128>, FwdCfg<128>::SMEM);
    attn_fwd_kernel<128><<<grid, 192, FwdCfg<128>::SMEM, s>>>(tm, a);
  }
  PB_CUDA_CHECK(cudaGetLastError());
  return {out, lse};
}

void attn_bwd(at::Tensor qkv, at::Tensor out, at::Tensor dout, at::Tensor lse, at::Tensor doc_start,
              at::Tensor items, int64_t H, int64_t Hkv, int64_t D, double scale, at::Tensor dqkv, at::Tensor dq_acc,
              at::Tensor delta) {
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim must be 64 or 128");
  TORCH_CHECK(dout.is_contiguous() && dout.scalar_type() == at::kBFloat16 && out.is_contiguous());
  TORCH_CHECK(dqkv.is_contiguous() && dq_acc.is_contiguous() && items.scalar_type() == at::kInt);
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int T = qkv.size(0);
  if (T == 0) return;
  auto s = at::cuda::getCurrentCUDAStream();
  const long pairs = static_cast<long>(T) * H;
  attn_delta_kernel<<<(pairs + 7) / 8, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
                                                    reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
                                                    delta.data_ptr<float>(), T, (int)H, (int)D);
  PB_CUDA_CHECK(cudaGetLastError());
  CUtensorMap tq = make_tmap_bf16_2d(qkv.data_ptr(), qkv.size(1), T, qkv.stride(0) * 2, 64, 128);
  CUtensorMap td = make_tmap_bf16_2d(dout.data_ptr(), dout.size(1), T, dout.stride(0) * 2, 64, 128);
  AttnArgs a{};
  a.T = T;
  a.H = (int)H;
  a.Hkv = (int)Hkv;
  a.D = (int)D;
  a.scale = (float)scale;
  a.scale_log2 = (float)scale * kLog2e;
  a.doc_start = doc_start.data_ptr<int>();
  a.items = items.data_ptr<int>();
  a.n_items = items.size(0);
  a.lse = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.dq_acc = dq_acc.data_ptr<float>();
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.ld_dqkv = dqkv.stride(0);
  a.status = status_ptr(qkv.device().index());
  const int grid = std::min<int>(a.n_items, num_sms(qkv.device().index()));
  if (D == 64) {
    set_smem(attn_bwd_kernel<64>, BwdCfg<64>::SMEM);
    attn_bwd_kernel<64><<<grid, 192, BwdCfg<64>::SMEM, s>>>(tq, td, a);
  } else {
    set_smem(attn_bwd_kernel<128>, BwdCfg<128>::SMEM);
    attn_bwd_kernel<128><<<grid, 192, BwdCfg<128>::SMEM, s>>>(tq, td, a);
  }
  PB_CUDA_CHECK(cudaGetLastError());
  const long n2 = static_cast<long>(T) * H * D / 2;
  dq_convert_kernel<<<std::max<long>(1, std::min<long>((n2 + 255) / 256, 4L * num_sms(qkv.device().index()))), 256,
                      0, s>>>(dq_acc.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
                              dqkv.stride(0), T, (int)(H * D));
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
