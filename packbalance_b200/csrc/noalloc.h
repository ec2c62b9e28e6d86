// Allocation-free C entry point of the fused LM-head cross-entropy forward.
//
// This interface has no counterpart in the reference implementation.
//
// It is for callers that may not allocate device memory while they run: code hosted
// inside another runtime that owns the whole device heap through its own pool, a
// process whose memory budget is fixed at start-up, or a loop where cudaMalloc /
// cudaFree (which can synchronise the device) are not acceptable.  The regular
// extension op gets its scratch from PyTorch's allocator; this entry point keeps it in
// one static device array of PB_NOALLOC_SCRATCH_FLOATS floats (16 MiB) that every GPU
// which loads the library holds until the process exits.
//
// Limits and sharing:
//   * a call needs (2 * ceil(V / 256) + 1) * T floats of scratch; larger calls are
//     rejected with PB_NOALLOC_TOO_LARGE before any memory is touched (for V = 32000
//     that allows T <= 16711 rows);
//   * every call shares the one array, so calls whose GPU work overlaps (streams with
//     no ordering between them, or several host threads) race on it;
//   * the first call on a device, with that device current, looks up the array's
//     device address (cudaGetSymbolAddress) and caches it; make that first call before
//     any stream capture;
//   * at most PB_NOALLOC_MAX_DEVICES device ordinals are supported.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define PB_NOALLOC_SCRATCH_FLOATS (4L * 1024 * 1024)
#define PB_NOALLOC_MAX_DEVICES 64

// Return codes of pb_lmhead_ce_forward_noalloc.
#define PB_NOALLOC_OK 0
#define PB_NOALLOC_CUDA_ERROR 1  // a CUDA call failed; pb_noalloc_last_error() names it
#define PB_NOALLOC_TOO_LARGE 2   // the call needs more than PB_NOALLOC_SCRATCH_FLOATS floats
#define PB_NOALLOC_BAD_ARG 3     // bad size, null or misaligned pointer, or device ordinal

#ifdef __cplusplus
extern "C" {
#endif

// For x [T, d] bf16 and w [V, d] bf16 (row-major, 16-byte aligned, d a multiple of 8)
// and int64 targets [T] on the current device, enqueue on `stream`:
//   lse_out[t]  = logsumexp_v(x_t . w_v)                                  (fp32 [T])
//   loss_out[0] = sum over t with targets[t] != ignore_index of
//                 lse_out[t] - x_t . w_{targets[t]} + z_coeff * lse_out[t]^2
// Allocates nothing.  After return codes PB_NOALLOC_TOO_LARGE and PB_NOALLOC_BAD_ARG
// nothing was enqueued and the outputs are untouched.
int pb_lmhead_ce_forward_noalloc(const void* x, const void* w, const int64_t* targets, int T, int d, int V,
                                 int64_t ignore_index, float z_coeff, float* loss_out, float* lse_out,
                                 cudaStream_t stream);

// Message of the calling thread's last failed call ("" after a successful one).
const char* pb_noalloc_last_error(void);

// Size of the static scratch array in floats (PB_NOALLOC_SCRATCH_FLOATS).
long pb_noalloc_scratch_floats(void);

// First error code that a kernel of this entry point recorded on the current device
// (a bounded wait that ran out), 0 if none, -1 if it could not be read.  Synchronous;
// a non-zero `clear` resets it.
int pb_noalloc_status(int clear);

#ifdef __cplusplus
}
#endif
