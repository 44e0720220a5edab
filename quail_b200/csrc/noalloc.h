// C entry point of the fp8 block-scaled GEMM that allocates no memory.
//
// This entry point has no counterpart in the reference: the reference only
// calls its GEMMs from PyTorch, which allocates freely.
//
// Who it is for: host code that must not allocate device memory while it
// runs. An inference server that reserves the whole GPU for its own memory
// pool at start-up has no free bytes for a library to cudaMalloc later; a
// latency-critical loop cannot afford cudaMalloc/cudaFree, which may
// synchronize the device; a plain C program that links only the CUDA
// runtime has no PyTorch caching allocator to draw scratch from. Such a
// caller passes its inputs and outputs, and the scratch the GEMM needs
// lives in a fixed-size device array inside this library instead.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Scratch held in a file-scope device array, per GPU that loads the
// library, until the process exits: one status word plus the activation
// scales re-laid out for the kernel, 4 MiB in all. A call needs
// 4 * M * (K / 128) bytes of it for the scales, so M * (K / 128) may be at
// most QB_NOALLOC_MAX_SCALES.
#define QB_NOALLOC_SCRATCH_BYTES (4u << 20)
#define QB_NOALLOC_MAX_SCALES ((QB_NOALLOC_SCRATCH_BYTES - 256u) / 4u)

// Return codes
#define QB_NOALLOC_OK 0
#define QB_NOALLOC_BAD_ARGUMENT (-1)    // a null pointer, an unaligned pointer or stride, or a bad shape
#define QB_NOALLOC_TOO_LARGE (-2)       // M * (K / 128) is above QB_NOALLOC_MAX_SCALES
#define QB_NOALLOC_SETUP_FAILED (-3)    // cudaGetSymbolAddress or a driver entry point failed
#define QB_NOALLOC_LAUNCH_FAILED (-4)   // a kernel launch or an async memset returned an error
#define QB_NOALLOC_KERNEL_TIMEOUT (-5)  // status_out requested and a bounded wait in the kernel ran out

// D[M, N] (bf16, row stride ldd elements) = dequant(A) . dequant(B)^T on the
// current device, enqueued on `stream`.
//
//   a        [M, K] e4m3, row stride lda bytes (a multiple of 16)
//   a_scale  [M, K/128] fp32, row-major: one scale per token and 128-wide K
//            group (the layout most quantizers write)
//   b        [N, K] e4m3, row stride ldb bytes (a multiple of 16)
//   b_scale  [ceil(N/128), K/128] fp32: one scale per 128x128 weight block
//            (the `weight_scale_inv` of fp8 checkpoints)
//   K is a multiple of 128, N a multiple of 16, ldd a multiple of 8.
//
// The first call on a device looks up the scratch array's device address
// (cudaGetSymbolAddress) with that device current and sets the kernel's
// shared-memory limit; make that first call before any stream capture. If
// that set-up fails (QB_NOALLOC_SETUP_FAILED), nothing is remembered and
// the next call on the device tries it again.
// Every call reuses the same scratch array: it clears the status word,
// then overwrites the scales, so two calls whose work overlaps on the GPU
// (different streams, or different host threads on one device) race on
// the scratch and must not be issued that way.
//
// status_out: NULL to return right after enqueueing; otherwise the call
// synchronizes `stream`, stores the kernel's status word there (0 = ok) and
// returns QB_NOALLOC_KERNEL_TIMEOUT if it is not zero. With M == 0 nothing
// is launched and *status_out is set to 0.
int qb_gemm_fp8_noalloc(const void* a, int64_t lda, const float* a_scale, const void* b, int64_t ldb,
                        const float* b_scale, void* d, int64_t ldd, int M, int N, int K, cudaStream_t stream,
                        int* status_out);

#ifdef __cplusplus
}
#endif
