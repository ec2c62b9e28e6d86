// Host launcher of the tcgen05 GEMM (kernel and epilogues in gemm_kernel.cuh).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "gemm_kernel.cuh"
#include "gemm_pair.cuh"
#include "host_utils.h"

namespace pb {

// BN=256 launches (and, in mode 2, BN=192 launches with a K-major B) without a fused
// gather and with more than 128 rows run on CTA pairs (gemm_pair.cuh): mode 1 with 6 pipeline stages and 4 store-staging slots per
// epilogue warp, mode 2 (the default: measured faster with the store-heavy epilogues)
// with 5 stages and 8 slots; mode 0: always the single-CTA kernel.
static int g_pair_mode = 2;

// Tests of the pair kernel's abort path only: GemmArgs::test_arm_limit of the next
// launches (0 = off).
static int g_pair_test_arm_limit = 0;

int64_t gemm_pair_test_arm_limit(int64_t n) {
  const int prev = g_pair_test_arm_limit;
  g_pair_test_arm_limit = static_cast<int>(std::max<int64_t>(0, n));
  return prev;
}

int64_t gemm_pair_mode(int64_t mode) {
  const int prev = g_pair_mode;
  if (mode >= 0) {
    TORCH_CHECK(mode <= 2, "gemm_pair_mode: 0, 1 or 2");
    g_pair_mode = (int)mode;
  }
  return prev;
}

// ------------------------------------ host ----------------------------------------
template <int BN, bool A_MN, bool B_MN>
static void launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const CUtensorMap& tx,
                        const GemmArgs& args, int grid, cudaStream_t stream) {
  const int threads = args.ag.world > 0 ? 256 : 192;
  using C = GemmCfg<BN>;
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN>;
  static bool configured[64] = {false};
  int dev = 0;
  PB_CUDA_CHECK(cudaGetDevice(&dev));
  if (!configured[dev]) {
    PB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
    configured[dev] = true;
  }
  kern<<<pb::smem_max(kern, grid), threads, C::SMEM_BYTES, stream>>>(ta, tb, to, tx, args);
  PB_CUDA_CHECK(cudaGetLastError());
}

template <int BN, bool A_MN, bool B_MN, int STAGES, int NSLOT>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const CUtensorMap& tx,
                        const GemmArgs& args, int max_ctas, cudaStream_t stream) {
  using PC = PairCfg<BN, STAGES, NSLOT>;
  auto kern = gemm_pair_kernel<BN, A_MN, B_MN, STAGES, NSLOT>;
  static int max_clusters[64] = {0};
  int dev = 0;
  PB_CUDA_CHECK(cudaGetDevice(&dev));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = PC::SMEM_BYTES;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (max_clusters[dev] == 0) {
    PB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PC::SMEM_BYTES));
    cfg.gridDim = dim3(2 * (num_sms(dev) / 2), 1, 1);
    int n = 0;
    PB_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
    max_clusters[dev] = std::max(1, n);
  }
  const int tiles = args.m_tiles * args.n_tiles * args.splits;
  int clusters = std::min(tiles, max_clusters[dev]);
  if (max_ctas > 0) clusters = std::min(clusters, std::max(1, max_ctas / 2));
  cfg.gridDim = pb::smem_max(kern, dim3(2 * std::max(clusters, 1), 1, 1));
  PB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, to, tx, args));
}

template <int STAGES, int NSLOT>
static void dispatch_pair_cfg(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                              const CUtensorMap& to, const CUtensorMap& tx, const GemmArgs& args, int max_ctas,
                              cudaStream_t s) {
  if (!a_mn && !b_mn) launch_pair<256, false, false, STAGES, NSLOT>(ta, tb, to, tx, args, max_ctas, s);
  else if (!a_mn && b_mn) launch_pair<256, false, true, STAGES, NSLOT>(ta, tb, to, tx, args, max_ctas, s);
  else if (a_mn && b_mn) launch_pair<256, true, true, STAGES, NSLOT>(ta, tb, to, tx, args, max_ctas, s);
  else launch_pair<256, true, false, STAGES, NSLOT>(ta, tb, to, tx, args, max_ctas, s);
}

static void dispatch_pair(int mode, int bn, bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                          const CUtensorMap& to, const CUtensorMap& tx, const GemmArgs& args, int max_ctas,
                          cudaStream_t s) {
  if (bn == 192) {  // K-major B only (pair_ok)
    if (!a_mn) launch_pair<192, false, false, 5, 8>(ta, tb, to, tx, args, max_ctas, s);
    else launch_pair<192, true, false, 5, 8>(ta, tb, to, tx, args, max_ctas, s);
  } else if (mode == 2) {
    dispatch_pair_cfg<5, 8>(a_mn, b_mn, ta, tb, to, tx, args, max_ctas, s);
  } else {
    dispatch_pair_cfg<6, 4>(a_mn, b_mn, ta, tb, to, tx, args, max_ctas, s);
  }
}

template <int BN>
static void dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                           const CUtensorMap& tx, const GemmArgs& args, int grid, cudaStream_t s) {
  if (!a_mn && !b_mn) launch_gemm<BN, false, false>(ta, tb, to, tx, args, grid, s);
  else if (!a_mn && b_mn) launch_gemm<BN, false, true>(ta, tb, to, tx, args, grid, s);
  else if (a_mn && b_mn) launch_gemm<BN, true, true>(ta, tb, to, tx, args, grid, s);
  else launch_gemm<BN, true, false>(ta, tb, to, tx, args, grid, s);
}

// All-gather spec shared by gemm_tc and fsdp_all_gather (ag_copy.cuh): 13 fields, and an
// optional 14th, copy_own.
void parse_ag_spec(const std::vector<int64_t>& ag, AgSpec& s) {
  TORCH_CHECK(ag.size() == 13 || ag.size() == 14, "ag spec: 13 or 14 fields");
  s.src = reinterpret_cast<const __nv_bfloat16* const*>(ag[0]);
  s.dst = reinterpret_cast<__nv_bfloat16*>(ag[1]);
  s.lo = ag[2];
  s.hi = ag[3];
  s.unit0 = ag[4];
  s.cs = ag[5];
  s.b0 = ag[6];
  s.split = ag[7];
  s.rank = (int)ag[8];
  s.world = (int)ag[9];
  s.piece_shift = (int)ag[10];
  s.block_shift = (int)ag[11];
  s.counters = reinterpret_cast<uint32_t*>(ag[12]);
  s.copy_own = ag.size() > 13 ? (int)(ag[13] != 0) : 0;
  s.rot = 0;
  TORCH_CHECK(s.world >= 2 && s.world <= 8 && s.rank >= 0 && s.rank < s.world, "ag: rank/world");
  TORCH_CHECK(s.lo % 8 == 0 && s.hi % 8 == 0 && s.unit0 % 8 == 0 && s.cs % 8 == 0 && s.cs > 0 && s.split % 8 == 0,
              "ag: ranges must be 16-byte aligned");
  TORCH_CHECK(s.piece_shift >= 3 && s.piece_shift <= s.block_shift && s.block_shift <= 30, "ag: piece/block size");
  TORCH_CHECK(s.lo >= s.unit0 && s.hi <= s.unit0 + s.world * s.cs && s.lo + 2 * s.split <= s.hi,
              "ag: range outside its unit");
}

static const void* opt_ptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

// Epilogue box over a 2-D output view: 32 x 32 elements, 128B (fp32) or 64B (bf16) swizzle.
static CUtensorMap epi_map(const at::Tensor& t) {
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "gemm_tc: epilogue tensors must be 2-D row-major");
  TORCH_CHECK((t.stride(0) * t.element_size()) % 16 == 0 && reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0,
              "gemm_tc: epilogue tensor rows must be 16B aligned");
  const bool f32 = t.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || t.scalar_type() == at::kBFloat16, "gemm_tc: epilogue tensors are fp32 or bf16");
  return make_tmap_2d(t.data_ptr(), f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                      t.size(1), t.size(0), t.stride(0) * t.element_size(), 32, 32,
                      f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

// Python-facing entry.  ``a``/``b`` are 2-D bf16 views with unit inner stride; M, N, K
// are the logical GEMM sizes (for SWIGLU N = 2F and ``b`` is the [2F, K] gate|up matrix).
void gemm_tc(at::Tensor a, at::Tensor b, at::Tensor out, int64_t M, int64_t N, int64_t K, bool a_mn, bool b_mn,
             int64_t epi, int64_t bn, int64_t splits, int64_t max_ctas, double alpha,
             c10::optional<at::Tensor> aux, c10::optional<at::Tensor> pos, c10::optional<at::Tensor> cos_t,
             c10::optional<at::Tensor> sin_t, int64_t head_dim, int64_t n_rope_cols,
             c10::optional<at::Tensor> targets, c10::optional<at::Tensor> pmax, c10::optional<at::Tensor> psum,
             c10::optional<at::Tensor> tlogit, c10::optional<at::Tensor> lse, c10::optional<at::Tensor> row_scale,
             double z_coeff, std::vector<int64_t> ag) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda(), "gemm_tc: CUDA tensors required");
  TORCH_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_tc: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1, "gemm_tc: 2-D row-major");
  TORCH_CHECK(bn == 64 || bn == 128 || bn == 192 || bn == 256, "gemm_tc: bn must be 64/128/192/256");
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
  const bool swiglu_bwd = epi == EPI_SWIGLU_BWD;

  GemmArgs g{};
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.F = swiglu ? (int)(N / 2) : (swiglu_bwd ? (int)N : 0);
  const bool pair = g_pair_mode && M > 128 && ag.empty() && (bn == 256 || (bn == 192 && !b_mn && g_pair_mode == 2));
  g.m_tiles = pair ? (int)((M + 255) / 256) : (int)((M + 127) / 128);
  g.n_tiles = swiglu ? (int)((N / 2 + bn / 2 - 1) / (bn / 2)) : (int)((N + bn - 1) / bn);
  g.k_blocks = (int)((K + 63) / 64);
  g.splits = (int)std::max<int64_t>(1, std::min<int64_t>(splits, g.k_blocks));
  g.kb_per_split = (g.k_blocks + g.splits - 1) / g.splits;
  g.splits = (g.k_blocks + g.kb_per_split - 1) / g.kb_per_split;
  g.epi = (int)epi;
  g.alpha = (float)alpha;
  g.test_arm_limit = pair ? g_pair_test_arm_limit : 0;
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
    TORCH_CHECK(cos_t.has_value() && sin_t.has_value() && pos.has_value(), "gemm_tc: RoPE tables");
  }
  if (swiglu) {
    TORCH_CHECK((N / 2) % 32 == 0, "gemm_tc: SWIGLU F must be a multiple of 32");
    TORCH_CHECK(aux.has_value() && aux->size(1) == N && aux->size(0) == M, "gemm_tc: SWIGLU saves g|u in aux [M, 2F]");
  }
  if (swiglu_bwd) {
    TORCH_CHECK(N % 32 == 0, "gemm_tc: SWIGLU_BWD F must be a multiple of 32");
    TORCH_CHECK(aux.has_value() && aux->is_contiguous() && aux->scalar_type() == at::kBFloat16 &&
                    aux->size(0) == M && aux->size(1) == 2 * N,
                "gemm_tc: SWIGLU_BWD reads the saved g|u from aux (bf16 [M, 2F], contiguous)");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(aux->data_ptr()) % 16 == 0, "gemm_tc: aux must be 16B aligned");
    g.gu = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr());
  }
  if (g.splits > 1) TORCH_CHECK(epi == EPI_ADD_F32, "gemm_tc: split-K needs the ADD_F32 epilogue");
  const bool has_out = epi != EPI_CE_FWD;
  CUtensorMap to{}, tx{};
  if (has_out) {
    TORCH_CHECK(out.dim() == 2 && out.size(0) == M, "gemm_tc: out rows");
    TORCH_CHECK(out.size(1) == (swiglu ? N / 2 : (swiglu_bwd ? 2 * N : N)), "gemm_tc: out columns");
    TORCH_CHECK((epi == EPI_F32 || epi == EPI_ADD_F32) == (out.scalar_type() == at::kFloat),
                "gemm_tc: fp32 output for F32/ADD_F32 epilogues, bf16 otherwise");
    to = epi_map(out);
  }
  if (swiglu) tx = epi_map(*aux);
  if (epi == EPI_CE_FWD && aux.has_value()) {
    TORCH_CHECK(aux->scalar_type() == at::kBFloat16 && aux->size(0) == M && aux->size(1) == N,
                "gemm_tc: CE_FWD keeps the logits in aux (bf16 [M, N])");
    tx = epi_map(*aux);
    g.keep_logits = 1;
  }

  // Operand TMA descriptors: 128-byte swizzle, 64-element (128 B) inner box.
  CUtensorMap ta = a_mn ? make_tmap_bf16_2d(a.data_ptr(), M, K, a.stride(0) * 2, 64, 64)
                        : make_tmap_bf16_2d(a.data_ptr(), K, M, a.stride(0) * 2, 64, 128);
  CUtensorMap tb;
  if (b_mn) tb = make_tmap_bf16_2d(b.data_ptr(), N, K, b.stride(0) * 2, 64, 64);
  else tb = make_tmap_bf16_2d(b.data_ptr(), K, N, b.stride(0) * 2, 64, (swiglu || pair) ? bn / 2 : bn);

  cudaStream_t stream0 = at::cuda::getCurrentCUDAStream();
  if (!ag.empty()) {
    // Fused all-gather of B: {src_ptrs_dev, dst, lo, hi, unit0, cs, b0, split, rank, world,
    //                         piece_shift, block_shift, counters[, copy_own]}
    TORCH_CHECK(!b_mn, "gemm_tc: the fused all-gather feeds a K-major B");
    AgSpec& s = g.ag;
    parse_ag_spec(ag, s);
    TORCH_CHECK(reinterpret_cast<const char*>(b.data_ptr()) == reinterpret_cast<const char*>(s.dst) + 2 * s.b0,
                "gemm_tc: B must be the gathered buffer at element b0");
    if (s.split > 0) {
      // gate|up interleaved copies: tiles in plain order
      TORCH_CHECK(swiglu && s.b0 == s.lo && s.split == (N / 2) * K, "gemm_tc: split gather is for the gate|up GEMM");
      g.n_rot = 0;
    } else {
      // Copies start right after this rank's own range (or at lo when the range holds
      // none of it); tiles start with this rank's own rows (no wait), else with the
      // rows of the first piece copied, so the MMAs follow the copies.  When the own
      // chunk is copied too (from local memory, the fastest pieces), copies start at it.
      const long own0 = s.unit0 + s.rank * s.cs, own1 = own0 + s.cs;
      const bool mine = own0 < s.hi && own1 > s.lo;
      const long np = (s.hi - s.lo + (1L << s.piece_shift) - 1) >> s.piece_shift;
      if (s.copy_own) s.rot = mine ? (int)((std::max(own0, s.lo) - s.lo) >> s.piece_shift) : 0;
      else s.rot = (mine && own1 < s.hi) ? (int)((own1 - s.lo) >> s.piece_shift) : 0;
      if (s.rot >= np) s.rot = 0;
      const long first = mine ? std::max(own0, s.lo) : s.lo;
      const long row = std::max<long>(0, (first - s.b0) / K);
      const long rows_per_tile = swiglu ? bn / 2 : bn;
      const long brow = swiglu ? row % (N / 2) : row;
      g.n_rot = brow < (swiglu ? N / 2 : N) ? (int)((brow / rows_per_tile) % g.n_tiles) : 0;
    }
    const long nblocks = (s.hi - s.lo + (1L << s.block_shift) - 1) >> s.block_shift;
    PB_CUDA_CHECK(cudaMemsetAsync(s.counters, 0, sizeof(uint32_t) * (1 + nblocks), stream0));
  }
  if (pair) {
    dispatch_pair(g_pair_mode, (int)bn, a_mn, b_mn, ta, tb, to, tx, g, (int)max_ctas, at::cuda::getCurrentCUDAStream());
    return;
  }
  const int tiles = g.m_tiles * g.n_tiles * g.splits;
  int grid = std::min<int>(tiles, num_sms(a.device().index()));
  if (max_ctas > 0) grid = std::min<int>(grid, (int)max_ctas);
  grid = std::max(grid, 1);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  if (bn == 256) dispatch_major<256>(a_mn, b_mn, ta, tb, to, tx, g, grid, stream);
  else if (bn == 192) dispatch_major<192>(a_mn, b_mn, ta, tb, to, tx, g, grid, stream);
  else if (bn == 128) dispatch_major<128>(a_mn, b_mn, ta, tb, to, tx, g, grid, stream);
  else dispatch_major<64>(a_mn, b_mn, ta, tb, to, tx, g, grid, stream);
}

}  // namespace pb
