// Document-masked causal GQA attention for packed sequences, sm_100a (tcgen05/TMEM/TMA).
//
// Input is the fused QKV GEMM output qkv[T, (H + 2 Hkv) * D] (bf16, RoPE applied).
// Query t attends to key k iff doc_start[t] <= k <= t.  Head dims 64 and 128.
//
// Forward (persistent; work items = (query tile of 128 rows, head), dealt to the CTAs
// from a cost-ordered plan):
//   warp 0        TMA: Q tile once per item (two buffers), K/V tiles into a ring
//   warp 1        tcgen05.mma: S_j = Q K_j^T into TMEM, then O += P_{j-1} V_{j-1} with P
//                 read from TMEM (A operand in tensor memory), one tile stream across items
//   warps 2..9    softmax, thread = query row, two groups of four warps on the two key
//                 column halves: masking from doc_start, online max/sum in base 2, lazy O
//                 rescale in TMEM, P -> TMEM (bf16), then the row's (max, sum) to shared
//                 memory, and on to the next item
//   warps 10..13  epilogue, thread = query row: merges the groups' O accumulators,
//                 O / l -> bf16 output, the log-sum-exp; frees the O buffer (two at
//                 head_dim 64, so the next item's P V products do not wait for it).
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
  const int* doc_end;  // last token of the document containing each token (backward)
  const int* items;  // fwd: [n, 3] (q tile, head, first kv tile); bwd: [n, 3] (kv tile, head, last q tile)
  int n_items;
  __nv_bfloat16* out;  // fwd output [T, H*D]
  float* lse;          // [H, T] natural-log LSE
  // backward
  const float* delta;  // [H, T]
  int* status;
  // Optional event trace (nullptr: off): [CTA][kTraceRoles][kTraceMax] SM clock stamps.
  unsigned long long* trace;
};

// Event trace of the attention kernels, for finding where an item's time goes: each
// role's lane 0 stamps clock64() at its steps (see the roles in each kernel).  Off
// unless a buffer was set with attn_trace(); the test is one uniform branch.
constexpr int kTraceRoles = 8, kTraceMax = 128;
__device__ __forceinline__ void trace_ev(unsigned long long* tr, int role, uint32_t idx) {
  if (tr != nullptr && idx < static_cast<uint32_t>(kTraceMax))
    tr[(static_cast<size_t>(blockIdx.x) * kTraceRoles + role) * kTraceMax + idx] = clock64();
}

// =================================== forward ======================================
// Two softmax warpgroups per query tile: group g owns key columns [64g, 64g + 64) of
// every 128-wide key tile and runs its own online softmax (max, sum) with its own O
// accumulator in TMEM; the two partial results are merged once at the end.  This
// doubles the softmax warps per SM without any per-tile exchange between them.
constexpr float kLazyRescaleLog2 = 8.f;  // forward: rescale O only when the max grows > 2^8

template <int D>
struct FwdCfg {
  static constexpr int TILE_BYTES = 128 * D * 2;  // one 128-row tile of Q, K or V
  // Two Q buffers: the producer loads the next item's Q while the current item's last
  // key tiles are still in flight, so an item boundary costs no Q-load latency.
  static constexpr int Q_OFF = 0;                      // 2 buffers
  // K/V ring: four stages at head_dim 64, so the producer runs into the next item's key
  // tiles while the current item's last ones are in use; two at 128 (shared memory).
  static constexpr int KV_STAGES = D == 64 ? 4 : 2;
  static constexpr int K_OFF = 2 * TILE_BYTES;
  static constexpr int V_OFF = K_OFF + KV_STAGES * TILE_BYTES;
  // (max, sum) per row of both softmax groups for two items: [item & 1][group][128][2]
  static constexpr int STAT_OFF = V_OFF + KV_STAGES * TILE_BYTES;
  static constexpr int STAT_BYTES = 2 * 2 * 128 * 2 * 4;
  // At least 120 KB so that a second CTA (which would block in tcgen05.alloc on
  // the fully allocated TMEM) is never co-scheduled on the same SM.  The last 1024 bytes
  // are the slack of aligning the dynamic shared memory base to 1024.
  static constexpr int SMEM_USED = STAT_OFF + STAT_BYTES + 1024;
  static constexpr int SMEM = SMEM_USED > 122880 ? SMEM_USED : 122880;
  // TMEM columns: S (128), P[group][2 slots] x 32 (64 bf16 each), O[buffer][group] x D.
  // Two O buffers at head_dim 64, so the next item's P V products run while the
  // epilogue warps still read this item's O; one at 128 (512 columns in all).
  static constexpr int O_BUFS = D == 64 ? 2 : 1;
  static constexpr uint32_t S_COL = 0;
  static constexpr uint32_t P_COL = 128;
  static constexpr uint32_t O_COL = 256;
  static_assert(O_COL + O_BUFS * 2 * D <= 512, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 128, false, false);
  static constexpr uint32_t IDESC_O = idesc_bf16_f32(128, D, false, true);
};

__device__ __forceinline__ void load_tile_rows(void* dst, const CUtensorMap* map, uint64_t* bar, int col0, int row0,
                                               int D) {
  for (int c = 0; c < D / 64; ++c)
    tma_load_2d(static_cast<uint8_t*>(dst) + c * 16384, map, bar, col0 + c * 64, row0);
}

__device__ __forceinline__ int3 ld_item(const int* items, int i) {
  return make_int3(items[3 * i], items[3 * i + 1], items[3 * i + 2]);
}

// Debug builds: an item outside the token range / head count is reported (status 240)
// and replaced by an empty one on a valid tile.
__device__ __forceinline__ int3 checked_item(int3 it, int T, int H, int* status) {
  const int nt = (T + 127) / 128;
  if (!PB_BOUNDS_OK(it.x >= 0 && it.x < nt && it.y >= 0 && it.y < H && it.z >= 0 && it.z < nt, status, 240))
    return make_int3(0, 0, 0);
  return it;
}

template <int D>
__global__ void __launch_bounds__(448, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmap, const AttnArgs args) {
  using C = FwdCfg<D>;
  // p_ready / o_done [group][P slot] (tile g uses slot g & 1): one barrier per slot, so
  // with the softmax groups running up to two tiles ahead of the P V products no
  // barrier ever completes a second phase before its first has been waited for.
  // o_ready / o_free [O buffer] and stats_ready / stats_free [item & 1] hand an item's
  // result from the softmax groups and the MMA warp to the epilogue warps and back.
  __shared__ __align__(8) uint64_t q_full[2], q_empty[2], kv_full[FwdCfg<D>::KV_STAGES], kv_empty[FwdCfg<D>::KV_STAGES],
      s_full, s_free, p_ready[2][2], o_done[2][2], o_ready[2], o_free[2], stats_ready[2], stats_free[2], drain_bar;
  __shared__ uint32_t tmem_sh;
  __shared__ volatile int abort_sh;
  extern __shared__ uint8_t dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < C::KV_STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&s_free, 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_ready[i][0], 4);
      mbar_init(&p_ready[i][1], 4);
      mbar_init(&o_done[i][0], 1);
      mbar_init(&o_done[i][1], 1);
      mbar_init(&o_ready[i], 1);
      mbar_init(&o_free[i], 4);
      mbar_init(&stats_ready[i], 8);
      mbar_init(&stats_free[i], 4);
    }
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
  float* stats = reinterpret_cast<float*>(smem + C::STAT_OFF);
  // trace roles: 0 Q load issued (per item; slot 127: start), 1 K/V load issued, 2 S
  // issued, 3 P V issued (per tile), 4 S read by softmax warp 2, 5 its P ready (per
  // tile), 6 epilogue warp 10 starts an item, 7 ... ends it
  if (threadIdx.x == 0) trace_ev(args.trace, 0, kTraceMax - 1);

  if (warp == 0) {
    if (lane == 0) {
      uint32_t kv_it = 0, q_it = 0;
      bool ok = true;
      int3 nx = blockIdx.x < args.n_items ? checked_item(ld_item(args.items, blockIdx.x), args.T, args.H, args.status) : make_int3(0, 0, 0);
      for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x) {
        const int qt = nx.x, h = nx.y, kt0 = nx.z;
        if (it + (int)gridDim.x < args.n_items) nx = checked_item(ld_item(args.items, it + gridDim.x), args.T, args.H, args.status);
        const int hk = h / group;
        const int q0 = qt * 128;
        const int qb = q_it & 1;
        if (!mbar_wait(&q_empty[qb], ((q_it >> 1) & 1) ^ 1, args.status, 201, &abort_sh)) break;
        mbar_arrive_expect_tx(&q_full[qb], C::TILE_BYTES);
        load_tile_rows(smem + C::Q_OFF + qb * C::TILE_BYTES, &tmap, &q_full[qb], h * D, q0, D);
        trace_ev(args.trace, 0, q_it);
        ++q_it;
        for (int kt = kt0; kt <= qt; ++kt, ++kv_it) {
          const int s = kv_it % C::KV_STAGES;
          if (!mbar_wait(&kv_empty[s], ((kv_it / C::KV_STAGES) & 1) ^ 1, args.status, 202, &abort_sh)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[s], 2 * C::TILE_BYTES);
          load_tile_rows(smem + C::K_OFF + s * C::TILE_BYTES, &tmap, &kv_full[s], (H + hk) * D, kt * 128, D);
          load_tile_rows(smem + C::V_OFF + s * C::TILE_BYTES, &tmap, &kv_full[s], (H + Hkv + hk) * D, kt * 128, D);
          trace_ev(args.trace, 1, kv_it);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // The key tiles of all this CTA's items form one stream g = 0, 1, ...: S_g is issued
      // (once both groups have read S_{g-1}) before P_{g-1} V_{g-1}, across item
      // boundaries too, so when the softmax warps finish an item the next item's first
      // scores are already in TMEM.
      bool ok = true;
      uint32_t q_it = 0;                                    // items whose Q the S side used
      int it_s = blockIdx.x, j_s = 0;                      // S side: item, tile within it
      int3 cur_s = it_s < args.n_items ? checked_item(ld_item(args.items, it_s), args.T, args.H, args.status)
                                       : make_int3(0, 0, 0);
      int nkv_s = cur_s.x - cur_s.z + 1;
      int qb_s = 0;
      uint32_t qa_s = smem_u32(smem + C::Q_OFF);
      int it_p = blockIdx.x, j_p = 0;                      // P V side, one tile behind
      int nkv_p = nkv_s;
      uint32_t item_p = 0;                                  // items the P V side has finished
      uint32_t ob = 0;                                      // O buffer of the P V side's item
      uint32_t g = 0, gp = 0;                               // global tile index of each side
      while (ok && (it_s < args.n_items || gp < g)) {
        if (it_s < args.n_items) {
          if (j_s == 0) {
            qb_s = q_it & 1;
            qa_s = smem_u32(smem + C::Q_OFF + qb_s * C::TILE_BYTES);
            if (!mbar_wait(&q_full[qb_s], (q_it >> 1) & 1, args.status, 203, &abort_sh)) break;
            ++q_it;
          }
          const int s = g % C::KV_STAGES;
          if (!mbar_wait(&kv_full[s], (g / C::KV_STAGES) & 1, args.status, 205, &abort_sh)) break;
          // one S buffer: both groups must have read S_{g-1}
          if (g > 0 && !mbar_wait(&s_free, (g - 1) & 1, args.status, 211, &abort_sh)) break;
          tc_fence_after();
          const uint32_t ka = smem_u32(smem + C::K_OFF + s * C::TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_ss(tmem + C::S_COL, sdesc_sw128(qa_s + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024), C::IDESC_S,
                    kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full);
          trace_ev(args.trace, 2, g);
          ++g;
          if (++j_s == nkv_s) {
            umma_commit(&q_empty[qb_s]);
            j_s = 0;
            it_s += gridDim.x;
            if (it_s < args.n_items) {
              cur_s = checked_item(ld_item(args.items, it_s), args.T, args.H, args.status);
              nkv_s = cur_s.x - cur_s.z + 1;
            }
          }
        }
        // P V of the previous tile of the stream (all of them once the S side is done)
        if (gp + 1 < g || (it_s >= args.n_items && gp < g)) {
          const int s = gp % C::KV_STAGES;
          const uint32_t va = smem_u32(smem + C::V_OFF + s * C::TILE_BYTES);
          if (j_p == 0) {
            // The first P V of an item overwrites its O buffer: the epilogue must have
            // read the item that used the buffer before.
            ob = item_p % C::O_BUFS;
            if (!mbar_wait(&o_free[ob], ((item_p / C::O_BUFS) & 1) ^ 1, args.status, 204, &abort_sh)) break;
          }
#pragma unroll
          for (int grp = 0; grp < 2; ++grp) {
            if (!mbar_wait(&p_ready[grp][gp & 1], (gp >> 1) & 1, args.status, 206, &abort_sh)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t pa = tmem + C::P_COL + (grp * 2 + (gp & 1)) * 32;
            const uint32_t oc = tmem + C::O_COL + (ob * 2 + grp) * D;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_ts(oc, pa + kk * 8, sdesc_sw128(va + grp * 8192 + kk * 2048, 16384, 1024), C::IDESC_O,
                      (j_p > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&o_done[grp][gp & 1]);
          }
          if (!ok) break;
          umma_commit(&kv_empty[s]);
          trace_ev(args.trace, 3, gp);
          ++gp;
          if (++j_p == nkv_p) {
            umma_commit(&o_ready[ob]);  // every P V of the item: its O is final
            ++item_p;
            j_p = 0;
            it_p += gridDim.x;
            if (it_p < args.n_items) {
              const int3 c = checked_item(ld_item(args.items, it_p), args.T, args.H, args.status);
              nkv_p = c.x - c.z + 1;
            }
          }
        }
      }
      umma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, args.status, 207, nullptr);
    }
  } else if (warp < 10) {
    // ---------------- softmax groups (thread = query row) ----------------
    const int grp = (warp - 2) / 4;  // 0: key columns 0-63, 1: key columns 64-127
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    uint32_t kv_it = 0, item_n = 0;
    uint32_t pv_waited = 0;  // P V products (global tile index) whose completion this warp saw
    int3 nx = blockIdx.x < args.n_items ? checked_item(ld_item(args.items, blockIdx.x), args.T, args.H, args.status) : make_int3(0, 0, 0);
    int nlo = (blockIdx.x < args.n_items && nx.x * 128 + r < T) ? args.doc_start[nx.x * 128 + r] : 0x7fffffff;
    for (int it = blockIdx.x; it < args.n_items; it += gridDim.x, ++item_n) {
      const int qt = nx.x, kt0 = nx.z;
      const int lo = nlo;
      if (it + (int)gridDim.x < args.n_items) {
        nx = checked_item(ld_item(args.items, it + gridDim.x), args.T, args.H, args.status);
        nlo = nx.x * 128 + r < T ? args.doc_start[nx.x * 128 + r] : 0x7fffffff;
      }
      const uint32_t ob = item_n % C::O_BUFS;
      const int nkv = qt - kt0 + 1;
      const int q = qt * 128 + r;
      const bool qok = q < T;
      float m = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < nkv; ++j) {
        const uint32_t g = kv_it + j;
        if (!mbar_wait_warp(&s_full, g & 1, args.status, 208, &abort_sh)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int kv0 = (kt0 + j) * 128 + grp * 64;
        if (warp == 2 && lane == 0) trace_ev(args.trace, 4, g);
        // Both 32-column halves of this group's raw scores, one wait for the two loads.
        uint32_t sv[2][32];
        tmem_ld32(tmem + lane_off + C::S_COL + grp * 64, sv[0]);
        tmem_ld32(tmem + lane_off + C::S_COL + grp * 64 + 32, sv[1]);
        tmem_wait_ld_regs(sv[0]);
        reg_fence(sv[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free);  // the next S may overwrite the buffer
        // raw score i of this thread's row (masked to -inf below)
#define PB_S(i) __uint_as_float(sv[(i) >> 5][(i) & 31])
        // Tiles inside every row's window (most tiles of long documents) skip the mask;
        // the test is warp-uniform so the warp never splits over it.
        const bool inside = kv0 >= lo && kv0 + 63 <= q;
        if (!__all_sync(0xffffffff, inside)) {
          const int hi = qok ? q : -1;
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int k = kv0 + i;
            if (!(k >= lo && k <= hi)) sv[i >> 5][i & 31] = __float_as_uint(-INFINITY);
          }
        }
        // Row max of the raw scores with eight independent chains (the scale is positive,
        // so it is applied once to the max).
        float mx8[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) mx8[c] = PB_S(c);
#pragma unroll
        for (int i = 8; i < 64; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], PB_S(i));
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]))) * args.scale_log2;
        // Lazy rescaling: the exponent base only moves when the running max grows by more
        // than 2^8 (or on the first finite max), so most tiles neither touch O nor wait
        // for the previous P V product.  Exact: O and l always share the base, and
        // P <= 2^8 stays well inside bf16 / fp32 range.
        const float m_new = fmaxf(m, mx);
        const bool need = m != -INFINITY && m_new > m + kLazyRescaleLog2;
        const bool rescale = __any_sync(0xffffffff, need);  // warp-uniform: TMEM ops below
        const float base = (rescale || m == -INFINITY) ? (m_new == -INFINITY ? 0.f : m_new) : m;
        const float corr = m == -INFINITY ? 0.f : fast_exp2(m - base);  // 1 when the base stays
        // p = 2^(raw * scale - base): one FFMA and one ex2 per score; four partial sums.
        const float sl2 = args.scale_log2, nb = -base;
        float sum4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p0 = fast_exp2(fmaf(PB_S(2 * i), sl2, nb));
          const float p1 = fast_exp2(fmaf(PB_S(2 * i + 1), sl2, nb));
          sum4[i & 3] += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
        }
#undef PB_S
        const float sum = (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
        l = l * corr + sum;
        // P V products that must be complete, waited in stream order: tiles <= g - 2
        // (their P slot is reused now; across item boundaries too) and, to rescale this
        // item's O, tile g - 1.
        const bool rs = rescale && j > 0;
        const uint32_t need_done = rs ? g : (g >= 2 ? g - 1 : 0);
        while (pv_waited < need_done) {
          const uint32_t t = pv_waited;
          if (!mbar_wait_warp(&o_done[grp][t & 1], (t >> 1) & 1, args.status, 209, &abort_sh)) {
            ok = false;
            break;
          }
          ++pv_waited;
        }
        if (!ok) break;
        tc_fence_after();
        if (rs) {
          const uint32_t oc = C::O_COL + (ob * 2 + grp) * D;
#pragma unroll
          for (int c = 0; c < D; c += 16) {
            uint32_t ov[16];
            tmem_ld16(tmem + lane_off + oc + c, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * corr);
            tmem_st16(tmem + lane_off + oc + c, ov);
          }
        }
        m = m_new == -INFINITY ? m : base;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pv[i] = pk[c * 16 + i];
          tmem_st16(tmem + lane_off + C::P_COL + (grp * 2 + (g & 1)) * 32 + c * 16, pv);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready[grp][g & 1]);
        if (warp == 2 && lane == 0) trace_ev(args.trace, 5, g);
      }
      if (!ok) break;
      // Publish this row's (max, sum) for the epilogue and go on with the next item.
      const uint32_t sb = item_n & 1;
      if (!mbar_wait_warp(&stats_free[sb], ((item_n >> 1) & 1) ^ 1, args.status, 212, &abort_sh)) break;
      stats[((sb * 2 + grp) * 128 + r) * 2] = m;
      stats[((sb * 2 + grp) * 128 + r) * 2 + 1] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(&stats_ready[sb]);
      kv_it += nkv;
    }
  } else {
    // ---------------- epilogue (thread = query row) ----------------
    // Merges the two groups' partial O accumulators of an item with their (max, sum),
    // writes O / l as bf16 and the log-sum-exp, and frees the O buffer and the stats.
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    uint32_t item_n = 0;
    for (int it = blockIdx.x; it < args.n_items; it += gridDim.x, ++item_n) {
      const int3 c3 = checked_item(ld_item(args.items, it), args.T, args.H, args.status);
      const int h = c3.y;
      const int q = c3.x * 128 + r;
      const bool qok = q < T;
      const uint32_t sb = item_n & 1, ob = item_n % C::O_BUFS;
      if (!mbar_wait_warp(&stats_ready[sb], (item_n >> 1) & 1, args.status, 213, &abort_sh)) break;
      if (!mbar_wait_warp(&o_ready[ob], (item_n / C::O_BUFS) & 1, args.status, 210, &abort_sh)) break;
      if (warp == 10 && lane == 0) trace_ev(args.trace, 6, item_n);
      tc_fence_after();
      const float ma = stats[((sb * 2) * 128 + r) * 2], la = stats[((sb * 2) * 128 + r) * 2 + 1];
      const float mb = stats[((sb * 2 + 1) * 128 + r) * 2], lb = stats[((sb * 2 + 1) * 128 + r) * 2 + 1];
      const float mm = fmaxf(ma, mb);
      const float base = mm == -INFINITY ? 0.f : mm;
      const float fa = fast_exp2(ma - base), fb = fast_exp2(mb - base);
      const float lt = la * fa + lb * fb;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const float sa = fa * inv, sbb = fb * inv;
      const uint32_t oc = C::O_COL + ob * 2 * D;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        uint32_t oa[32], obv[32];
        tmem_ld32(tmem + lane_off + oc + c, oa);
        tmem_ld32(tmem + lane_off + oc + D + c, obv);
        tmem_wait_ld_regs(oa);
        reg_fence(obv);
        if (qok) {
          uint4* dst = reinterpret_cast<uint4*>(args.out + static_cast<long>(q) * H * D + h * D + c);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint32_t pk[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int e = 8 * k + 2 * i;
              pk[i] = pack_bf16x2(__uint_as_float(oa[e]) * sa + __uint_as_float(obv[e]) * sbb,
                                  __uint_as_float(oa[e + 1]) * sa + __uint_as_float(obv[e + 1]) * sbb);
            }
            dst[k] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        }
      }
      if (qok) args.lse[static_cast<long>(h) * T + q] = lt > 0.f ? (base + __log2f(lt)) * kLn2 : -INFINITY;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&o_free[ob]);
        mbar_arrive(&stats_free[sb]);
        if (warp == 10) trace_ev(args.trace, 7, item_n);
      }
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
// Items = (key tile, query head, last query tile).  Warp roles (320 threads):
//   0      TMA: K/V once per item, Q/dO per query tile (QSTAGES-deep ring)
//   1      tcgen05.mma: S^T = K Q^T, dP^T = V dO^T; then dV += P^T dO, dK += dS^T Q,
//          dQ = dS K
//   2..9   P^T / dS^T, thread = key row; warps 2-5 take query columns 0-63 and warps
//          6-9 columns 64-127 (the gradient math needs no cross-column reduction);
//          at item end dK (group 0) and dV (group 1) rows -> TMA reduce-add into the
//          fp32 dK|dV accumulator (the GQA heads of a group add up there)
//   10..13 dQ, thread = query row -> TMA reduce-add into the fp32 dQ accumulator
// so the next tile's S^T/dP^T MMAs, this tile's dQ write-out and the next tile's
// softmax-gradient math overlap.
template <int D>
struct BwdCfg {
  static constexpr int TILE_BYTES = 128 * D * 2;
  static constexpr bool SPLIT_DQ = 256 + 3 * D <= 512;  // dQ in its own TMEM columns
  static constexpr int QSTAGES = D == 64 ? 2 : 1;
  static constexpr int DQ_SLOTS = D == 64 ? 2 : 1;      // 4 KB staging slots per dQ warp
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE_BYTES;
  static constexpr int Q_OFF = 2 * TILE_BYTES;  // stage s: Q at Q_OFF + 2*s*TILE, dO right after
  static constexpr int VSTAGE_OFF = Q_OFF + QSTAGES * 2 * TILE_BYTES;  // stage s: lse[128], delta[128] fp32
  static constexpr int P_OFF = VSTAGE_OFF + 2048;                      // P^T  [128 kv x 128 q] bf16
  static constexpr int DS_OFF = P_OFF + 32768;                   // dS^T [128 kv x 128 q] bf16
  static constexpr int DQS_OFF = DS_OFF + 32768;                 // dQ staging, 4 warps
  static constexpr int SMEM = DQS_OFF + 4 * DQ_SLOTS * 4096 + 1024;
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr uint32_t ST_COL = 0;
  static constexpr uint32_t DPT_COL = 128;
  static constexpr uint32_t DQ_COL = SPLIT_DQ ? 256 : 0;
  static constexpr uint32_t DK_COL = SPLIT_DQ ? 256 + D : 256;
  static constexpr uint32_t DV_COL = DK_COL + D;
  static constexpr uint32_t IDESC_SQ = idesc_bf16_f32(128, 128, false, false);  // S^T, dP^T
  static constexpr uint32_t IDESC_KV = idesc_bf16_f32(128, D, false, true);     // dV, dK
  static constexpr uint32_t IDESC_DQ = idesc_bf16_f32(128, D, true, true);      // dQ
};

// 32 fp32 of this lane's row -> 128B-swizzled [32 x 32] fp32 staging box.
__device__ __forceinline__ void stage_row_f32(uint8_t* s, const uint32_t (&v)[32], float scale) {
  const int r = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float4 q = make_float4(__uint_as_float(v[4 * j]) * scale, __uint_as_float(v[4 * j + 1]) * scale,
                           __uint_as_float(v[4 * j + 2]) * scale, __uint_as_float(v[4 * j + 3]) * scale);
    *reinterpret_cast<float4*>(s + r * 128 + ((j ^ (r & 7)) << 4)) = q;
  }
}

__device__ __forceinline__ void reduce_box(const CUtensorMap* map, const uint8_t* s, int col, int row) {
  fence_async_smem();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    tma_reduce_add_2d(map, s, col, row);
    bulk_commit();
  }
}

template <int D>
__global__ void __launch_bounds__(448, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dkv,
                    const AttnArgs args) {
  using C = BwdCfg<D>;
  __shared__ __align__(8) uint64_t kv_full, kv_empty, qd_full[2], qd_empty[2], st_full, ds_ready, mma2_done, dq_free,
      acc_done, acc_free, drain_bar, st_free, dpt_free;
  __shared__ uint32_t tmem_sh;
  __shared__ volatile int abort_sh;
  extern __shared__ uint8_t dyn[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    mbar_init(&kv_full, 1);
    mbar_init(&kv_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(&st_full, 1);
    mbar_init(&ds_ready, 8);
    mbar_init(&mma2_done, 1);
    mbar_init(&dq_free, 4);
    mbar_init(&acc_done, 1);
    mbar_init(&acc_free, 8);
    mbar_init(&drain_bar, 1);
    mbar_init(&st_free, 8);   // the gradient warps have read S^T out of TMEM
    mbar_init(&dpt_free, 8);  // ... and dP^T
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
  // trace roles: 0 K/V load issued (per item; slot 127: start), 1 Q/dO load issued, 2
  // S^T / dP^T issued, 3 ds_ready seen by the MMA warp, 4 dV/dK/dQ issued (per tile), 5
  // S^T read by gradient warp 2, 6 its dS^T ready (per tile), 7 its dK/dV written (item)
  if (threadIdx.x == 0) trace_ev(args.trace, 0, kTraceMax - 1);

  if (warp == 0) {
    if (lane == 0) {
      uint32_t item_n = 0, g = 0;
      bool ok = true;
      int3 nx = blockIdx.x < args.n_items ? checked_item(ld_item(args.items, blockIdx.x), args.T, args.H, args.status) : make_int3(0, 0, 0);
      for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x, ++item_n) {
        const int kt = nx.x, h = nx.y, qhi = nx.z;
        if (it + (int)gridDim.x < args.n_items) nx = checked_item(ld_item(args.items, it + gridDim.x), args.T, args.H, args.status);
        const int hk = h / group;
        if (!mbar_wait(&kv_empty, (item_n & 1) ^ 1, args.status, 221, &abort_sh)) break;
        mbar_arrive_expect_tx(&kv_full, 2 * C::TILE_BYTES);
        load_tile_rows(smem + C::K_OFF, &tm_qkv, &kv_full, (H + hk) * D, kt * 128, D);
        load_tile_rows(smem + C::V_OFF, &tm_qkv, &kv_full, (H + Hkv + hk) * D, kt * 128, D);
        trace_ev(args.trace, 0, item_n);
        for (int qt = kt; qt <= qhi; ++qt, ++g) {
          const int s = g % C::QSTAGES;
          const uint32_t ph = (g / C::QSTAGES) & 1;
          if (!mbar_wait(&qd_empty[s], ph ^ 1, args.status, 222, &abort_sh)) {
            ok = false;
            break;
          }
          // Q, dO tiles and this tile's lse / delta rows (T % 4 == 0 keeps them 16B aligned).
          const uint32_t vb = static_cast<uint32_t>(min(128, T - qt * 128)) * 4u;
          mbar_arrive_expect_tx(&qd_full[s], 2 * C::TILE_BYTES + 2 * vb);
          uint8_t* qs = smem + C::Q_OFF + s * 2 * C::TILE_BYTES;
          load_tile_rows(qs, &tm_qkv, &qd_full[s], h * D, qt * 128, D);
          load_tile_rows(qs + C::TILE_BYTES, &tm_do, &qd_full[s], h * D, qt * 128, D);
          uint8_t* vs = smem + C::VSTAGE_OFF + s * 1024;
          bulk_load(vs, args.lse + static_cast<long>(h) * T + qt * 128, vb, &qd_full[s]);
          bulk_load(vs + 512, args.delta + static_cast<long>(h) * T + qt * 128, vb, &qd_full[s]);
          trace_ev(args.trace, 1, g);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t item_n = 0, g = 0;
      bool ok = true;
      const uint32_t ka = smem_u32(smem + C::K_OFF), va = smem_u32(smem + C::V_OFF);
      const uint32_t pa = smem_u32(smem + C::P_OFF), dsa = smem_u32(smem + C::DS_OFF);
      // S^T(gx) = K Q^T and dP^T(gx) = V dO^T of global tile gx: each overwrites its TMEM
      // columns once the gradient warps have read out tile gx - 1's.
      auto issue_st = [&](uint32_t gx) -> bool {
        const int sx = gx % C::QSTAGES;
        const uint32_t qa = smem_u32(smem + C::Q_OFF + sx * 2 * C::TILE_BYTES);
        const uint32_t da = qa + C::TILE_BYTES;
        if (!mbar_wait(&qd_full[sx], (gx / C::QSTAGES) & 1, args.status, 225, &abort_sh)) return false;
        // Without separate dQ columns, dQ(gx-1) lives where S^T(gx) goes.
        if (!C::SPLIT_DQ && gx > 0 && !mbar_wait(&dq_free, (gx - 1) & 1, args.status, 226, &abort_sh)) return false;
        if (gx > 0 && !mbar_wait(&st_free, (gx - 1) & 1, args.status, 234, &abort_sh)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_ss(tmem + C::ST_COL, sdesc_sw128(ka + off, 16, 1024), sdesc_sw128(qa + off, 16, 1024), C::IDESC_SQ,
                  kk > 0 ? 1u : 0u);
        }
        if (gx > 0 && !mbar_wait(&dpt_free, (gx - 1) & 1, args.status, 235, &abort_sh)) return false;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_ss(tmem + C::DPT_COL, sdesc_sw128(va + off, 16, 1024), sdesc_sw128(da + off, 16, 1024), C::IDESC_SQ,
                  kk > 0 ? 1u : 0u);
        }
        umma_commit(&st_full);
        trace_ev(args.trace, 2, gx);
        return true;
      };
      int3 nx = blockIdx.x < args.n_items ? checked_item(ld_item(args.items, blockIdx.x), args.T, args.H, args.status) : make_int3(0, 0, 0);
      for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x, ++item_n) {
        const int kt = nx.x, qhi = nx.z;
        if (it + (int)gridDim.x < args.n_items) nx = checked_item(ld_item(args.items, it + gridDim.x), args.T, args.H, args.status);
        if (!mbar_wait(&kv_full, item_n & 1, args.status, 223, &abort_sh)) break;
        // dK / dV accumulators and the staging smem of the previous item must be free
        // before this item's first S^T (whose completion lets the gradient warps write
        // the P^T / dS^T tiles that double as that staging).
        if (!mbar_wait(&acc_free, (item_n & 1) ^ 1, args.status, 224, &abort_sh)) break;
        if (!issue_st(g)) break;
        for (int qt = kt; qt <= qhi; ++qt, ++g) {
          const int s = g % C::QSTAGES;
          const uint32_t qa = smem_u32(smem + C::Q_OFF + s * 2 * C::TILE_BYTES);
          const uint32_t da = qa + C::TILE_BYTES;
          // The next tile's S^T / dP^T go to the tensor pipe now, so they run while the
          // gradient warps compute this tile's P^T / dS^T.  (With dQ in the S^T columns
          // the order must stay tile by tile.)
          if (C::SPLIT_DQ && qt < qhi && !issue_st(g + 1)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&ds_ready, g & 1, args.status, 227, &abort_sh)) {
            ok = false;
            break;
          }
          const bool first = qt == kt;
          trace_ev(args.trace, 3, g);
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
          if (C::SPLIT_DQ && g > 0 && !mbar_wait(&dq_free, (g - 1) & 1, args.status, 226, &abort_sh)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = kk * 2048;  // 16 kv rows
            umma_ss(tmem + C::DQ_COL, sdesc_sw128(dsa + off, 16384, 1024), sdesc_sw128(ka + off, 16384, 1024),
                    C::IDESC_DQ, kk > 0 ? 1u : 0u);
          }
          umma_commit(&mma2_done);
          umma_commit(&qd_empty[s]);
          trace_ev(args.trace, 4, g);
          if (!C::SPLIT_DQ && qt < qhi && !issue_st(g + 1)) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
        umma_commit(&acc_done);
        umma_commit(&kv_empty);
      }
      umma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, args.status, 228, nullptr);
    }
  } else if (warp < 10) {
    // ---------------- P^T / dS^T (thread = key row) ----------------
    const int grp = (warp - 2) / 4;  // query columns [64 grp, 64 grp + 64)
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    uint8_t* ptile = smem + C::P_OFF;
    uint8_t* dstile = smem + C::DS_OFF;
    uint32_t item_n = 0, g = 0;
    bool ok = true;
    int3 nx = blockIdx.x < args.n_items ? checked_item(ld_item(args.items, blockIdx.x), args.T, args.H, args.status) : make_int3(0, 0, 0);
    int nde = (blockIdx.x < args.n_items && nx.x * 128 + r < T) ? args.doc_end[nx.x * 128 + r] : -1;
    for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x, ++item_n) {
      const int kt = nx.x, h = nx.y, qhi = nx.z;
      // Key row kv is attended by queries q in [kv, doc_end(kv)] (none past T).
      const int de = nde;
      if (it + (int)gridDim.x < args.n_items) {
        nx = checked_item(ld_item(args.items, it + gridDim.x), args.T, args.H, args.status);
        nde = nx.x * 128 + r < T ? args.doc_end[nx.x * 128 + r] : -1;
      }
      const int hk = h / group;
      const int kv = kt * 128 + r;
      for (int qt = kt; qt <= qhi; ++qt, ++g) {
        const int q0 = qt * 128;
        const int s = g % C::QSTAGES;
        if (!mbar_wait_warp(&st_full, g & 1, args.status, 229, &abort_sh)) {
          ok = false;
          break;
        }
        // The lse / delta rows arrived with the Q/dO stage (already complete here; the
        // wait makes the bulk-copied data visible to this thread).
        if (!mbar_wait_warp(&qd_full[s], (g / C::QSTAGES) & 1, args.status, 233, &abort_sh)) {
          ok = false;
          break;
        }
        if (warp == 2 && lane == 0) trace_ev(args.trace, 5, g);
        const float* s_lse = reinterpret_cast<const float*>(smem + C::VSTAGE_OFF + s * 1024);
        const float* s_delta = s_lse + 128;
        tc_fence_after();
        // S^T -> P^T (bf16, this group's 64 query columns), then release S^T's TMEM
        // columns so the next tile's S^T MMA can run while this tile's gradient math does.
        // dS^T below uses the same bf16 P^T that the dV MMA reads (registers: 14 warps
        // leave 128 per thread).
        uint32_t pp[32];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t sv[32];
          tmem_ld32(tmem + lane_off + C::ST_COL + grp * 64 + cc * 32, sv);
          tmem_wait_ld();
          if (cc == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&st_free);
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float p2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int j = grp * 64 + cc * 32 + 2 * i + e;
              const int q = q0 + j;
              const bool allowed = q >= kv && q <= de;
              p2[e] = allowed ? fast_exp2(__uint_as_float(sv[2 * i + e]) * args.scale_log2 - s_lse[j] * kLog2e) : 0.f;
            }
            pp[cc * 16 + i] = pack_bf16x2(p2[0], p2[1]);
          }
        }
        // The previous tile's dV/dK/dQ MMAs read P/dS from shared memory.
        if (g > 0 && !mbar_wait_warp(&mma2_done, (g - 1) & 1, args.status, 230, &abort_sh)) {
          ok = false;
          break;
        }
        if (lane == 0) bulk_wait_read<0>();  // dK/dV staging of the previous item used these tiles
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          st_swz_chunk(ptile, r, grp * 8 + k, make_uint4(pp[4 * k], pp[4 * k + 1], pp[4 * k + 2], pp[4 * k + 3]));
        // dP^T -> dS^T = P^T (dP^T - delta), 32 columns at a time
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t dv[32];
          tmem_ld32(tmem + lane_off + C::DPT_COL + grp * 64 + cc * 32, dv);
          tmem_wait_ld();
          if (cc == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&dpt_free);
          }
          uint32_t dd[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 p = unpack_bf16x2(pp[cc * 16 + i]);
            const int j = grp * 64 + cc * 32 + 2 * i;
            // select (not multiply): delta past T is stale smem; masked P is exactly 0
            const float d0 = p.x != 0.f ? p.x * (__uint_as_float(dv[2 * i]) - s_delta[j]) : 0.f;
            const float d1 = p.y != 0.f ? p.y * (__uint_as_float(dv[2 * i + 1]) - s_delta[j + 1]) : 0.f;
            dd[i] = pack_bf16x2(d0, d1);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k)
            st_swz_chunk(dstile, r, grp * 8 + cc * 4 + k, make_uint4(dd[4 * k], dd[4 * k + 1], dd[4 * k + 2], dd[4 * k + 3]));
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ds_ready);
        if (warp == 2 && lane == 0) trace_ev(args.trace, 6, g);
      }
      if (!ok) break;
      // dK (scaled) and dV rows of this key tile -> fp32 accumulators (TMA reduce-add).
      if (!mbar_wait_warp(&acc_done, item_n & 1, args.status, 232, &abort_sh)) break;
      tc_fence_after();
      // Staging in this group's own halves of the P and dS tiles (free after acc_done).
      uint8_t* stg = smem + (q4 < 2 ? C::P_OFF : C::DS_OFF) + grp * 16384 + (q4 & 1) * 8192;
      int slot = 0;
#pragma unroll 1
      for (int c = grp * D; c < grp * D + D; c += 32) {
        const bool is_k = c < D;
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + (is_k ? C::DK_COL + c : C::DV_COL + c - D), v);
        tmem_wait_ld();
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
        uint8_t* sl = stg + slot * 4096;
        stage_row_f32(sl, v, is_k ? args.scale : 1.f);
        reduce_box(&tm_dkv, sl, is_k ? hk * D + c : (Hkv + hk) * D + c - D, kt * 128 + q4 * 32);
        slot ^= 1;
      }
      // The staging areas overlap other warps' P^T / dS^T rows: they may be rewritten
      // (next item) only after these stores have read them; acc_free orders that.
      if (lane == 0) bulk_wait_read<0>();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_free);
      if (warp == 2 && lane == 0) trace_ev(args.trace, 7, item_n);
    }
    if (lane == 0) bulk_wait_all<0>();
    __syncwarp();
  } else {
    // ---------------- dQ write-out (thread = query row) ----------------
    const int q4 = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(q4 * 32) << 16;
    uint8_t* stg = smem + C::DQS_OFF + q4 * C::DQ_SLOTS * 4096;
    int slot = 0;
    uint32_t g = 0;
    bool ok = true;
    int3 nx = blockIdx.x < args.n_items ? checked_item(ld_item(args.items, blockIdx.x), args.T, args.H, args.status) : make_int3(0, 0, 0);
    for (int it = blockIdx.x; it < args.n_items && ok; it += gridDim.x) {
      const int kt = nx.x, h = nx.y, qhi = nx.z;
      if (it + (int)gridDim.x < args.n_items) nx = checked_item(ld_item(args.items, it + gridDim.x), args.T, args.H, args.status);
      for (int qt = kt; qt <= qhi; ++qt, ++g) {
        if (!mbar_wait_warp(&mma2_done, g & 1, args.status, 231, &abort_sh)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t v[D];
#pragma unroll
        for (int c = 0; c < D; c += 32) tmem_ld32(tmem + lane_off + C::DQ_COL + c, *reinterpret_cast<uint32_t(*)[32]>(v + c));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&dq_free);
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          if (lane == 0) {
            if (C::DQ_SLOTS == 2) bulk_wait_read<1>();
            else bulk_wait_read<0>();
          }
          __syncwarp();
          uint8_t* sl = stg + slot * 4096;
          stage_row_f32(sl, *reinterpret_cast<uint32_t(*)[32]>(v + c), args.scale);
          reduce_box(&tm_dq, sl, h * D + c, qt * 128 + q4 * 32);
          if (C::DQ_SLOTS == 2) slot ^= 1;
        }
      }
    }
    if (lane == 0) bulk_wait_all<0>();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[h, t] = sum_d O[t, h, d] * dO[t, h, d]; one thread per (t, h), 16-byte loads.
// The kernel also zeroes the fp32 dQ and dK|dV accumulators (both receive TMA
// reduce-adds from the backward kernel), consecutive threads writing consecutive
// 16-byte words.
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                  float* __restrict__ delta, int T, int H, int D, float* __restrict__ dq_acc,
                                  float* __restrict__ dkv_acc, int Hkv) {
  const long idx = blockIdx.x * (long)blockDim.x + threadIdx.x;
  const long nthreads = static_cast<long>(gridDim.x) * blockDim.x;
  {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    const long nq = static_cast<long>(T) * H * D / 4, nk = static_cast<long>(T) * 2 * Hkv * D / 4;
    for (long i = idx; i < nq; i += nthreads) reinterpret_cast<float4*>(dq_acc)[i] = z;
    for (long i = idx; i < nk; i += nthreads) reinterpret_cast<float4*>(dkv_acc)[i] = z;
  }
  if (idx >= static_cast<long>(T) * H) return;
  const int t = static_cast<int>(idx / H), h = static_cast<int>(idx % H);
  const uint4* a = reinterpret_cast<const uint4*>(o + static_cast<long>(t) * H * D + h * D);
  const uint4* b = reinterpret_cast<const uint4*>(dout + static_cast<long>(t) * H * D + h * D);
  // all loads of the row (D <= 128: at most 16 + 16 of 16 bytes) before any use
  uint4 x[16], y[16];
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (i < D / 8) {
      x[i] = a[i];
      y[i] = b[i];
    }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (i >= D / 8) break;
    const uint32_t* xp = &x[i].x;
    const uint32_t* yp = &y[i].x;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 fx = unpack_bf16x2(xp[k]), fy = unpack_bf16x2(yp[k]);
      s += fx.x * fy.x + fx.y * fy.y;
    }
  }
  delta[static_cast<long>(h) * T + t] = s;
}

// dQ and dK (fp32 accumulators) -> bf16 into dqkv rotated back by the inverse RoPE
// (the forward applied RoPE to q and k in the QKV GEMM epilogue); dV -> bf16.
__global__ void dqkv_finalize_kernel(const float* __restrict__ dq_acc, const float* __restrict__ dkv_acc,
                                     __nv_bfloat16* __restrict__ dqkv, long ld, const int* __restrict__ pos,
                                     const float* __restrict__ cos_t, const float* __restrict__ sin_t, int n_pos,
                                     int T, int H, int Hkv, int D) {
  const int half = D / 2, g4 = half / 4;
  const int heads = H + 2 * Hkv;
  const long total = static_cast<long>(T) * heads * g4;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int t = static_cast<int>(i / (heads * g4));
    const int rem = static_cast<int>(i % (heads * g4));
    const int hs = rem / g4, j = (rem % g4) * 4;
    const float* src = hs < H ? dq_acc + static_cast<long>(t) * H * D + hs * D
                              : dkv_acc + static_cast<long>(t) * 2 * Hkv * D + (hs - H) * D;
    const float4 a = *reinterpret_cast<const float4*>(src + j);
    const float4 b = *reinterpret_cast<const float4*>(src + half + j);
    float x1[4] = {a.x, a.y, a.z, a.w}, x2[4] = {b.x, b.y, b.z, b.w};
    float y1[4], y2[4];
    if (pos != nullptr && hs < H + Hkv) {
      const int p = min(max(pos[t], 0), n_pos - 1);
      const float4 c4 = *reinterpret_cast<const float4*>(cos_t + static_cast<long>(p) * half + j);
      const float4 s4 = *reinterpret_cast<const float4*>(sin_t + static_cast<long>(p) * half + j);
      const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        y1[e] = x1[e] * cs[e] + x2[e] * sn[e];
        y2[e] = x2[e] * cs[e] - x1[e] * sn[e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        y1[e] = x1[e];
        y2[e] = x2[e];
      }
    }
    __nv_bfloat16* dst = dqkv + t * ld + hs * D;
    *reinterpret_cast<uint2*>(dst + j) = make_uint2(pack_bf16x2(y1[0], y1[1]), pack_bf16x2(y1[2], y1[3]));
    *reinterpret_cast<uint2*>(dst + half + j) = make_uint2(pack_bf16x2(y2[0], y2[1]), pack_bf16x2(y2[2], y2[3]));
  }
}

// ------------------------------------ host ----------------------------------------
template <typename K>
static void set_smem(K kern, int bytes) {
  PB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

// Event-trace buffer of the next attention launches (0: off), set by attn_trace().
static unsigned long long* g_attn_trace = nullptr;

void attn_trace(int64_t ptr) { g_attn_trace = reinterpret_cast<unsigned long long*>(ptr); }

std::vector<at::Tensor> attn_fwd(at::Tensor qkv, at::Tensor doc_start, at::Tensor items, int64_t H, int64_t Hkv,
                                 int64_t D, double scale, at::Tensor out) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 2 && qkv.is_contiguous());
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim must be 64 or 128");
  TORCH_CHECK(H % Hkv == 0 && qkv.size(1) == (H + 2 * Hkv) * D, "attention: qkv width");
  TORCH_CHECK(doc_start.scalar_type() == at::kInt && items.scalar_type() == at::kInt && items.is_contiguous());
  TORCH_CHECK(items.dim() == 2 && items.size(1) == 3, "attention: forward items are (q tile, head, first kv tile)");
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int T = qkv.size(0);
  auto lse = at::empty({H, T}, qkv.options().dtype(at::kFloat));
  if (T == 0) return {out, lse};
  CUtensorMap tm = make_tmap_bf16_2d(qkv.data_ptr(), qkv.size(1), T, qkv.stride(0) * 2, 64, 128);
  AttnArgs a{};
  a.trace = g_attn_trace;
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
    attn_fwd_kernel<64><<<pb::smem_max(attn_fwd_kernel<64>, grid), 448, FwdCfg<64>::SMEM, s>>>(tm, a);
  } else {
    set_smem(attn_fwd_kernel<128>, FwdCfg<128>::SMEM);
    attn_fwd_kernel<128><<<pb::smem_max(attn_fwd_kernel<128>, grid), 448, FwdCfg<128>::SMEM, s>>>(tm, a);
  }
  PB_CUDA_CHECK(cudaGetLastError());
  return {out, lse};
}

void attn_bwd(at::Tensor qkv, at::Tensor out, at::Tensor dout, at::Tensor lse, at::Tensor doc_start,
              at::Tensor doc_end, at::Tensor items, int64_t H, int64_t Hkv, int64_t D, double scale, at::Tensor dqkv, at::Tensor dq_acc,
              at::Tensor dkv_acc, at::Tensor delta, c10::optional<at::Tensor> pos, c10::optional<at::Tensor> cos_t,
              c10::optional<at::Tensor> sin_t) {
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim must be 64 or 128");
  TORCH_CHECK(dout.is_contiguous() && dout.scalar_type() == at::kBFloat16 && out.is_contiguous());
  TORCH_CHECK(dqkv.is_contiguous() && dq_acc.is_contiguous() && dkv_acc.is_contiguous());
  TORCH_CHECK(items.scalar_type() == at::kInt && items.dim() == 2 && items.size(1) == 3);
  TORCH_CHECK(dq_acc.size(1) == H * D && dkv_acc.size(1) == 2 * Hkv * D, "attention: accumulator widths");
  TORCH_CHECK(qkv.size(0) % 4 == 0, "attention backward: token count must be a multiple of 4");
  TORCH_CHECK(doc_end.scalar_type() == at::kInt && doc_end.numel() == qkv.size(0), "attention: doc_end");
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int T = qkv.size(0);
  TORCH_CHECK(dq_acc.size(0) == T && dkv_acc.size(0) == T && delta.numel() == static_cast<long>(T) * H,
              "attention: accumulator rows");
  if (T == 0) return;
  auto s = at::cuda::getCurrentCUDAStream();
  const long pairs = static_cast<long>(T) * H;
  attn_delta_kernel<<<(pairs + 255) / 256, 256, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
                                                      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
                                                      delta.data_ptr<float>(), T, (int)H, (int)D,
                                                      dq_acc.data_ptr<float>(), dkv_acc.data_ptr<float>(), (int)Hkv);
  PB_CUDA_CHECK(cudaGetLastError());
  CUtensorMap tq = make_tmap_bf16_2d(qkv.data_ptr(), qkv.size(1), T, qkv.stride(0) * 2, 64, 128);
  CUtensorMap td = make_tmap_bf16_2d(dout.data_ptr(), dout.size(1), T, dout.stride(0) * 2, 64, 128);
  CUtensorMap tdq = make_tmap_2d(dq_acc.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dq_acc.size(1), T,
                                 dq_acc.stride(0) * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tdkv = make_tmap_2d(dkv_acc.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, dkv_acc.size(1), T,
                                  dkv_acc.stride(0) * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  AttnArgs a{};
  a.trace = g_attn_trace;
  a.T = T;
  a.H = (int)H;
  a.Hkv = (int)Hkv;
  a.D = (int)D;
  a.scale = (float)scale;
  a.scale_log2 = (float)scale * kLog2e;
  a.doc_start = doc_start.data_ptr<int>();
  a.doc_end = doc_end.data_ptr<int>();
  a.items = items.data_ptr<int>();
  a.n_items = items.size(0);
  a.lse = lse.data_ptr<float>();
  a.delta = delta.data_ptr<float>();
  a.status = status_ptr(qkv.device().index());
  const int grid = std::min<int>(a.n_items, num_sms(qkv.device().index()));
  if (D == 64) {
    set_smem(attn_bwd_kernel<64>, BwdCfg<64>::SMEM);
    attn_bwd_kernel<64><<<pb::smem_max(attn_bwd_kernel<64>, grid), 448, BwdCfg<64>::SMEM, s>>>(tq, td, tdq, tdkv, a);
  } else {
    set_smem(attn_bwd_kernel<128>, BwdCfg<128>::SMEM);
    attn_bwd_kernel<128><<<pb::smem_max(attn_bwd_kernel<128>, grid), 448, BwdCfg<128>::SMEM, s>>>(tq, td, tdq, tdkv, a);
  }
  PB_CUDA_CHECK(cudaGetLastError());
  const long n4 = static_cast<long>(T) * (H + 2 * Hkv) * (D / 8);
  dqkv_finalize_kernel<<<std::max<long>(1, std::min<long>((n4 + 255) / 256, 8L * num_sms(qkv.device().index()))),
                         256, 0, s>>>(dq_acc.data_ptr<float>(), dkv_acc.data_ptr<float>(),
                                      reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), dqkv.stride(0),
                                      pos.has_value() ? pos->data_ptr<int>() : nullptr,
                                      cos_t.has_value() ? cos_t->data_ptr<float>() : nullptr,
                                      sin_t.has_value() ? sin_t->data_ptr<float>() : nullptr,
                                      cos_t.has_value() ? (int)cos_t->size(0) : 1, T, (int)H, (int)Hkv, (int)D);
  PB_CUDA_CHECK(cudaGetLastError());
}

}  // namespace pb
