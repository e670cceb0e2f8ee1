// Allocation-free entry point of the fused limb GEMM.
//
// This entry point has no counterpart in the reference (FerrumVir/arc-chain);
// it exists for callers of this library that cannot allocate device memory
// themselves.  Examples: a host runtime that owns its GPU memory budget and
// forbids allocation after start-up, code running inside a custom allocator
// or memory-pool callback (where calling cudaMalloc would re-enter the
// allocator), and embedding hosts that only hand out pointers to buffers they
// manage.  Such callers still pass their inputs and outputs; the partial-sum
// buffer and tile counters that arcb_fgemm() normally receives from the
// caller live instead in one fixed device array inside this library.
//
// Limits: the scratch array is ARCB_NOALLOC_SCRATCH_BYTES (4 MiB) per GPU,
// held by every GPU that loads the library until the process exits.  It holds
//   * one counter per 128-row tile of M, at most ARCB_NOALLOC_MAX_TILES tiles
//     (M <= 523,904 rows), and
//   * the int32 partial sums, 8 * B * M values, at most
//     ARCB_NOALLOC_MAX_PARTIALS of them (e.g. M = 32,000 rows at B = 4).
// Larger problems are rejected with a negative return code (see below) and
// nothing is launched.
//
// Behaviour:
//   * The first call on each device looks up the device address of the
//     scratch array with cudaGetSymbolAddress (with that device current) and
//     remembers it; make that first call before any stream capture begins.
//   * Every call clears the scratch it uses (cudaMemsetAsync on `stream`,
//     which allocates nothing) and then launches the fused GEMM; it never
//     calls cudaMalloc, cudaFree or any allocating library routine.
//   * All calls on a device share the one array, and it keeps the last call's
//     contents.  Calls whose work overlaps on the GPU (different streams, or
//     different host threads without ordering) race on it and give wrong
//     results: order them on one stream.
//   * Only the finalizing epilogue modes are accepted (store, residual,
//     RoPE/KV, SwiGLU); the partial-only mode is rejected, because it leaves
//     its result in the scratch array where the caller cannot read it.  The
//     descriptor must also leave the tensor-parallel push mode and every
//     peer target (peer outputs, peer arrival counters) unset: those work on
//     peer-mapped buffers that the caller allocates, so they are not for
//     callers of this entry point, and are rejected the same way.
#pragma once
#include <stdint.h>

#define ARCB_NOALLOC_SCRATCH_BYTES (4u << 20)
#define ARCB_NOALLOC_MAX_TILES 4093
#define ARCB_NOALLOC_MAX_PARTIALS (((4u << 20) / 4u) - 4096u)

// Return codes besides 0 (success) and positive CUDA error numbers.
#define ARCB_NOALLOC_ERR_TOO_MANY_TILES (-20)   // M needs more than MAX_TILES tiles
#define ARCB_NOALLOC_ERR_PARTIALS (-21)         // 8 * B * M > MAX_PARTIALS
#define ARCB_NOALLOC_ERR_MODE (-22)             // partial-only, push or peer-target mode requested
#define ARCB_NOALLOC_ERR_SYMBOL (-23)           // cudaGetSymbolAddress failed
#define ARCB_NOALLOC_ERR_ARGS (-24)             // non-positive sizes or null descriptors

#ifdef __cplusplus
extern "C" {
#endif

// Same arguments as arcb_fgemm() minus the partial-sum buffer, the tile
// counters and the PDL flag.  `epi` points to the epilogue descriptor in
// host memory; it must not request the push mode.
int arcb_fgemm_noalloc(const void* tmA, const void* tmB, int M, int K, int B, int bn, const int* lmax,
                       const void* epi, void* stream);

#ifdef __cplusplus
}
#endif
