// Allocation-free C entry point: fused LM-head cross-entropy forward.
//
// This entry point has no counterpart in the reference implementation.  Its interface,
// the callers it is for, its scratch limit and its sharing rules are declared in
// noalloc.h, which this file includes so that the compiler checks the definitions
// against those declarations.
//
// Who it is for.  Some callers of this library are not allowed to allocate device
// memory at the time they run a step: code that lives inside another runtime which
// owns the whole device heap through its own pool and forbids cudaMalloc outside it,
// processes that reserve their memory once at start-up and must stay within that
// budget for their lifetime, and latency-critical loops where cudaMalloc / cudaFree
// (which can synchronize the device) are not acceptable.  The regular extension op
// (``gemm_tc`` + ``ce_finalize`` from Python) gets its partial-sum buffers from
// PyTorch's allocator; this variant keeps them in a fixed static array instead.
//
// Scratch.  One file-scope __device__ array of kScratchFloats fp32 (16 MiB) holds the
// per-tile row partials (2 * ceil(V / 256) * T floats) and the target logits (T floats).
// Every GPU that loads this library holds that array until the process exits.  Calls
// whose (2 * ceil(V / 256) + 1) * T exceeds kScratchFloats are rejected (return code 2,
// message from pb_noalloc_last_error()); pb_noalloc_scratch_floats() reports the limit.
// The array keeps the previous call's contents; this function clears the parts that
// must start at zero (the target-logit slots and *loss_out) on ``stream`` itself.
// All calls share the one array, so calls whose GPU work overlaps (different streams
// without ordering between them, or different host threads) race on it.
//
// Set-up.  The first call on a device (with that device current) looks up the
// device addresses of the static arrays with cudaGetSymbolAddress and caches them;
// host code must never pass the array's host-side symbol to a kernel.  That first call
// should come before any stream capture.
//
// Return codes: 0 ok, 1 CUDA error, 2 size beyond the scratch limit, 3 bad argument
// (including a device ordinal at or above PB_NOALLOC_MAX_DEVICES).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstring>
#include <cstdio>
#include <mutex>

#include "ce_kernels.cuh"
#include "gemm_kernel.cuh"
#include "noalloc.h"

namespace pb {
namespace noalloc {

constexpr long kScratchFloats = PB_NOALLOC_SCRATCH_FLOATS;  // 16 MiB
constexpr int kTile = 256;                         // logits columns per CE tile

__device__ __align__(256) float g_scratch[kScratchFloats];
__device__ __align__(256) int g_status;

struct DeviceState {
  bool ready = false;
  float* scratch = nullptr;
  int* status = nullptr;
  int sms = 0;
};

DeviceState g_state[PB_NOALLOC_MAX_DEVICES];
std::mutex g_mu;
thread_local char g_msg[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool bf16_map(CUtensorMap* m, const void* ptr, int64_t inner, int64_t outer, uint32_t box_outer) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(inner * 2)};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return encoder()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Once per device, with the device current: device addresses of the static arrays.
int setup(int dev, DeviceState** out) {
  if (dev < 0 || dev >= PB_NOALLOC_MAX_DEVICES)
    return fail(3, "device ordinal %d is outside the supported range [0, %d)", dev, PB_NOALLOC_MAX_DEVICES);
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceState& s = g_state[dev];
  if (!s.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return fail(1, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    s.scratch = static_cast<float*>(p);
    e = cudaGetSymbolAddress(&p, g_status);
    if (e != cudaSuccess) return fail(1, "cudaGetSymbolAddress(status): %s", cudaGetErrorString(e));
    s.status = static_cast<int*>(p);
    e = cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(1, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    e = cudaFuncSetAttribute(gemm_tc_kernel<kTile, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             GemmCfg<kTile>::SMEM_BYTES);
    if (e != cudaSuccess) return fail(1, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    s.ready = true;
  }
  *out = &s;
  return 0;
}

}  // namespace noalloc
}  // namespace pb

using namespace pb;
using namespace pb::noalloc;

extern "C" const char* pb_noalloc_last_error() { return g_msg; }

extern "C" long pb_noalloc_scratch_floats() { return kScratchFloats; }

// First error code a kernel of this entry point recorded (bounded-wait timeouts);
// optionally clears it.  Synchronous, allocation-free.
extern "C" int pb_noalloc_status(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_status, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
  }
  return v;
}

extern "C" int pb_lmhead_ce_forward_noalloc(const void* x, const void* w, const int64_t* targets, int T, int d, int V,
                                            int64_t ignore_index, float z_coeff, float* loss_out, float* lse_out,
                                            cudaStream_t stream) {
  g_msg[0] = '\0';
  if (T <= 0 || d <= 0 || V <= 0) return fail(3, "T, d and V must be positive (got %d, %d, %d)", T, d, V);
  const long ntiles = (static_cast<long>(V) + kTile - 1) / kTile;
  const long need = (2 * ntiles + 1) * static_cast<long>(T);
  if (need > kScratchFloats)
    return fail(2,
                "scratch limit: (2 * ceil(V / %d) + 1) * T = %ld floats exceeds the static scratch of %ld floats "
                "(T = %d, V = %d); split the rows into smaller calls",
                kTile, need, kScratchFloats, T, V);
  if (d % 8 != 0) return fail(3, "d must be a multiple of 8 (16-byte rows), got %d", d);
  if (x == nullptr || w == nullptr || targets == nullptr || loss_out == nullptr || lse_out == nullptr)
    return fail(3, "null pointer argument");
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(w) % 16)
    return fail(3, "x and w must be 16-byte aligned");
  if (encoder() == nullptr) return fail(1, "cuTensorMapEncodeTiled is unavailable");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(1, "cudaGetDevice: %s", cudaGetErrorString(e));
  DeviceState* st = nullptr;
  if (int rc = setup(dev, &st)) return rc;

  CUtensorMap ta, tb, unused;
  memset(&unused, 0, sizeof(unused));
  if (!bf16_map(&ta, x, d, T, 128) || !bf16_map(&tb, w, d, V, kTile)) return fail(1, "tensor map encoding failed");

  float* pmax = st->scratch;
  float* psum = pmax + ntiles * T;
  float* tlogit = psum + ntiles * T;
  if ((e = cudaMemsetAsync(tlogit, 0, sizeof(float) * T, stream)) != cudaSuccess ||
      (e = cudaMemsetAsync(loss_out, 0, sizeof(float), stream)) != cudaSuccess)
    return fail(1, "cudaMemsetAsync: %s", cudaGetErrorString(e));
  GemmArgs g{};
  g.M = T;
  g.N = V;
  g.K = d;
  g.m_tiles = (T + 127) / 128;
  g.n_tiles = static_cast<int>(ntiles);
  g.k_blocks = (d + 63) / 64;
  g.splits = 1;
  g.kb_per_split = g.k_blocks;
  g.epi = EPI_CE_FWD;
  g.alpha = 1.f;
  g.targets = targets;
  g.pmax = pmax;
  g.psum = psum;
  g.tlogit = tlogit;
  g.status = st->status;
  const long tiles = static_cast<long>(g.m_tiles) * g.n_tiles;
  const int grid = static_cast<int>(tiles < st->sms ? tiles : st->sms);
  gemm_tc_kernel<kTile, false, false><<<grid, 192, GemmCfg<kTile>::SMEM_BYTES, stream>>>(ta, tb, unused, unused, g);
  ce_finalize_kernel<<<ce_finalize_blocks(T), kCeRows * kCeGroups, 0, stream>>>(pmax, psum, static_cast<int>(ntiles), T, tlogit, targets,
                                                          ignore_index, z_coeff, lse_out, loss_out);
  if ((e = cudaGetLastError()) != cudaSuccess) return fail(1, "kernel launch: %s", cudaGetErrorString(e));
  return 0;
}
