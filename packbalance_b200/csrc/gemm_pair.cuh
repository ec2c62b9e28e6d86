// Pair (2-SM) variant of the tcgen05 GEMM: a cluster of two CTAs on neighbouring SMs
// computes one 256 x BN tile (BN = 256 or 192) with tcgen05.mma.cta_group::2.
//
// Each CTA stages its own 128 rows of A and one half (128 rows) of the tile's B; the
// MMA, issued by one thread of the even CTA, reads both CTAs' shared memory at the same
// offsets and writes each CTA's 128 x 256 fp32 accumulator into that CTA's TMEM.  Per
// 64-deep k-block a CTA therefore loads 32 KB instead of the single-CTA kernel's 48 KB
// for the same FLOPs (B is not fetched twice), and five or six pipeline stages fit in
// shared memory where the single-CTA kernel has four.  The epilogues are the single-CTA
// kernel's (run_epilogue), each CTA finishing its own 128 rows.
//
// Barriers:
//   full[s]   even CTA only; one arrive.expect_tx of both CTAs' bytes by the even CTA's
//             producer, and the TMA loads of both CTAs complete their bytes on it (the
//             odd CTA names it through its cluster address).
//   empty[s]  both CTAs; the MMA commit is multicast to both, so each producer reuses
//             its stage once the MMAs that read it (in both CTAs) are done.
//   accf[a]   both CTAs; MMA commit multicast at the end of a tile.
//   acce[a]   even CTA only; counts the 8 epilogue warps of the pair (4 local, 4 remote).
// TMEM is allocated with cta_group::2 by warp 1 of both CTAs.  A cluster barrier after
// set-up and another before TMEM release and exit keep either CTA from touching the
// other's barriers before they exist or after it has left.
//
// Abort without loads in flight: the odd CTA's loads complete on the even CTA's full
// barrier, which the odd CTA cannot wait on, and the even CTA may stop (a bounded wait ran
// out) before it has armed a stage the odd CTA already loads into.  When the odd producer
// leaves its loop, normally or not, it stores its count of issued k-blocks with a done bit
// into ``odd_done`` in the even CTA's shared memory (release, cluster scope).  An aborting
// even producer first sets the odd CTA's abort flag (so its waits end at once), waits
// (bounded) for that count, arms the stages of the k-blocks the odd CTA issued beyond its
// own arming with the odd CTA's bytes only, and then waits (bounded) for every armed
// stage.  So no load is in flight when the final cluster barrier lets either CTA exit.
// The normal path exchanges nothing per k-block.
//
// Only TMA loads from this GPU's own memory are issued (no all-gather role, no cluster
// multicast of loads); the launch that gathers B from peers uses the single-CTA kernel.
#pragma once

#include "gemm_kernel.cuh"

namespace pb {

// STAGES pipeline stages and NSLOT 2 KB store-staging slots per epilogue warp share the
// shared memory: (6, 4) or (5, 8) for BN = 256 (32 KB stages), (5, 8) for BN = 192.
template <int BN_, int STAGES_, int NSLOT_>
struct PairCfg {
  static constexpr int BM = 128;  // rows per CTA; the pair's tile has 2 * BM rows
  static constexpr int BN = BN_;  // columns of the pair's tile; each CTA stages BN / 2 rows of B
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = STAGES_;
  static constexpr int NSLOT = NSLOT_;
  using Stg = StagerT<NSLOT>;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr uint32_t TMEM_COLS = BN == 192 ? 512 : 2 * BN;  // allocations are powers of two
  static constexpr int SMEM_BYTES = EPI_OFF + 4 * Stg::kBytes + 1024;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Cluster address of the shared-memory variable at ``saddr`` in CTA ``rank`` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// All threads of both CTAs.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_release_cluster(uint32_t cluster_saddr, uint32_t v) {
  asm volatile("st.release.cluster.shared::cluster.u32 [%0], %1;" ::"r"(cluster_saddr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_cluster(const volatile uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cluster.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32((const void*)p)) : "memory");
  return v;
}
constexpr uint32_t kOddDone = 0x80000000u;
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
// Tiled 2-D load into this CTA's shared memory, completing its bytes on the barrier at
// the cluster address ``bar`` (the even CTA's full barrier).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at the same offset in both CTAs once this thread's MMAs are done.
__device__ __forceinline__ void umma_commit_both(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "h"(mask)
               : "memory");
}
__device__ __forceinline__ void umma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// BN is 256, or 192 with a K-major B.
// Launched with cluster dimension (2, 1, 1) and 192 threads: warp 0 TMA producer (both
// CTAs), warp 1 TMEM allocation (both) and MMA issuer (even CTA), warps 2-5 epilogue.
// ``args.m_tiles`` counts 256-row tiles.
template <int BN, bool A_MN, bool B_MN, int STAGES, int NSLOT>
__global__ void __launch_bounds__(192, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ CUtensorMap tm_aux,
                     const GemmArgs args) {
  using C = PairCfg<BN, STAGES, NSLOT>;
  // an MN-major B half is staged as 64-column chunks
  static_assert(!B_MN || (BN / 2) % 64 == 0, "MN-major B needs BN / 2 to be a multiple of 64");
  constexpr uint32_t IDESC = idesc_bf16_f32(2 * C::BM, C::BN, A_MN, B_MN);
  __shared__ __align__(8) uint64_t full_bar[C::STAGES];
  __shared__ __align__(8) uint64_t empty_bar[C::STAGES];
  __shared__ __align__(8) uint64_t accf_bar[2];
  __shared__ __align__(8) uint64_t acce_bar[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ volatile int abort_sh;
  __shared__ volatile uint32_t odd_done_sh;  // even CTA: the odd producer's issued k-blocks | kOddDone
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t cta = cluster_ctarank();  // 0 issues the MMAs
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    odd_done_sh = 0;
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&accf_bar[s], 1);
      mbar_init(&acce_bar[s], 8);
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
    tmem_alloc_pair(&tmem_base_sh, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;
  const int num_tiles = args.m_tiles * args.n_tiles * args.splits;
  const bool swiglu = args.epi == EPI_SWIGLU;
  const uint32_t full0 = cluster_addr(smem_u32(&full_bar[0]), 0);
  const uint32_t acce0 = cluster_addr(smem_u32(&acce_bar[0]), 0);

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_mask = 0, armed_phase = 0;  // even CTA: per stage, armed and its phase
      uint32_t n_kb = 0;                         // k-blocks armed (even) / issued (odd)
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        int mb, nb, sp;
        tile_coords(args, tile, mb, nb, sp);
        const int kb0 = sp * args.kb_per_split;
        const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
        const int row_a = (mb * 2 + static_cast<int>(cta)) * C::BM;
        // this CTA's half of the tile's B rows (SWIGLU: gate rows in CTA 0, up rows in CTA 1)
        const int row_b = swiglu ? (cta ? args.F : 0) + nb * (C::BN / 2) : nb * C::BN + static_cast<int>(cta) * (C::BN / 2);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, args.status, 121, &abort_sh)) {
            ok = false;
            break;
          }
          if (cta == 0) {
            if (args.test_arm_limit > 0 && n_kb >= static_cast<uint32_t>(args.test_arm_limit)) {
              ok = false;  // test of the abort path: stop arming as if stalled
              break;
            }
            mbar_arrive_expect_tx(&full_bar[stage], 2 * C::STAGE_BYTES);
            armed_mask |= 1u << stage;
            armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          }
          ++n_kb;
          const uint32_t bar = full0 + stage * 8;
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          const int k0 = kb * C::BK;
          if (!A_MN) {
            tma_load_2d_pair(sa, &tma_a, bar, k0, row_a);
          } else {
            tma_load_2d_pair(sa, &tma_a, bar, row_a, k0);
            tma_load_2d_pair(sa + 8192, &tma_a, bar, row_a + 64, k0);
          }
          if (!B_MN) {
            tma_load_2d_pair(sb, &tma_b, bar, k0, row_b);
          } else {
#pragma unroll
            for (int j = 0; j < C::BN / 128; ++j) tma_load_2d_pair(sb + j * 8192, &tma_b, bar, row_b + j * 64, k0);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (cta == 1) {
        // issued count for the even CTA's abort path (read only there)
        st_release_cluster(cluster_addr(smem_u32((const void*)&odd_done_sh), 0), n_kb | kOddDone);
      } else if (!ok) {
        // Stop the odd producer (its waits check this flag), except in the abort-path test,
        // where its own bounded wait has to run out.
        if (args.test_arm_limit <= 0) st_release_cluster(cluster_addr(smem_u32((const void*)&abort_sh), 1), 1u);
        // The odd CTA's count of issued k-blocks (bounded: its waits end within one
        // timeout); k-blocks it issued beyond this CTA's arming get armed with its bytes
        // only (at most STAGES of them, each on its own stage), so their phases complete.
        uint32_t done = 0;
        const uint64_t t0 = globaltimer();
        while (!((done = ld_acquire_cluster(&odd_done_sh)) & kOddDone)) {
          if (globaltimer() - t0 > 2 * PB_WAIT_TIMEOUT_NS) {
            report_error(args.status, 127);
            break;
          }
        }
        if (done & kOddDone) {
          const uint32_t n_odd = done & ~kOddDone;
          for (uint32_t kb = n_kb; kb < n_odd && kb < n_kb + C::STAGES; ++kb) {
            mbar_arrive_expect_tx(&full_bar[stage], C::STAGE_BYTES);
            armed_mask |= 1u << stage;
            armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1;
            }
          }
        }
        // Drain: wait (bounded, once more) for every armed stage; the odd CTA's loads of
        // those stages complete on the same barriers.
        for (int s = 0; s < C::STAGES; ++s)
          if (armed_mask & (1u << s)) mbar_wait(&full_bar[s], (armed_phase >> s) & 1u, args.status, 122, nullptr);
      }
    }
  } else if (warp == 1) {
    if (cta == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        int mb, nb, sp;
        tile_coords(args, tile, mb, nb, sp);
        const int kb0 = sp * args.kb_per_split;
        const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1, args.status, 123, &abort_sh)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * C::BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, args.status, 124, &abort_sh)) {
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
            umma_ss_pair(d_tmem, ad, bd, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_both(&empty_bar[stage]);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_both(&accf_bar[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // All MMAs issued by this thread must finish before either CTA releases TMEM.
      umma_commit_pair_local(&drain_bar);
      mbar_wait(&drain_bar, 0, args.status, 125, nullptr);
    }
  } else {
    const int q = warp & 3;
    typename C::Stg st{smem + C::EPI_OFF + q * C::Stg::kBytes, 0, args.epi == EPI_F32 || args.epi == EPI_ADD_F32};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs) {
      int mb, nb, sp;
      tile_coords(args, tile, mb, nb, sp);
      prefetch_epilogue<C::BN>(args, (mb * 2 + static_cast<int>(cta)) * C::BM + q * 32, nb);
      if (!mbar_wait_warp(&accf_bar[acc], acc_phase, args.status, 126, &abort_sh)) break;
      tc_fence_after();
      const uint32_t tacc = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * C::BN;
      run_epilogue<C::BN>(args, &tm_out, &tm_aux, st, tacc, (mb * 2 + static_cast<int>(cta)) * C::BM + q * 32, nb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce0 + acc * 8);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (lane == 0) bulk_wait_all<0>();
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace pb
