// qb_gemm_fp8_noalloc: the fp8 block-scaled tcgen05 GEMM with its scratch in
// a static device array (see noalloc.h for who needs this and its limits).
//
// The scratch: word 0 is the status word the kernel's bounded waits write
// on timeout (the entry point PyTorch calls keeps it in a cudaMalloc'd
// word); from byte 256 on, the caller's row-major activation scales
// re-laid out as [K/128, M], the layout the kernel reads.
//
// This file calls no cudaMalloc, cudaFree or allocating library routine:
// only cudaGetSymbolAddress, cudaFuncSetAttribute, cudaDeviceGetAttribute,
// cudaMemsetAsync, kernel launches and (when asked for the status) a
// stream synchronize plus a device-to-host copy into the caller's int.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm_sm100_kernel.cuh"
#include "noalloc.h"

namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[QB_NOALLOC_SCRATCH_BYTES];

constexpr int kBN = 256;
constexpr int kStages = 4;
constexpr int kSmem = kStages * (128 * 128 + kBN * 128) + 1024 + 256 + 4096;

struct DeviceSetup {
  bool ok = false;
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch on this device
  int sms = 0;
};

std::mutex g_mu;
DeviceSetup g_setup[64];

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn g_encode = nullptr;

// [M, G] row-major -> [G, M]
__global__ void transpose_scales_kernel(const float* __restrict__ src, float* __restrict__ dst, int M, int G) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * G) return;
  const int g = i / M, m = i % M;
  dst[i] = src[(size_t)m * G + g];
}

// once per device, with that device current
DeviceSetup* setup_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceSetup& s = g_setup[dev];
  if (s.ok) return &s;
  // a failed set-up is not remembered: the next call on this device tries again
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return nullptr;
  s.scratch = static_cast<uint8_t*>(p);
  if (cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return nullptr;
  if (cudaFuncSetAttribute(qb::gemm_sm100_kernel<kBN, true, qb::kEpiBf16, kStages>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return nullptr;
  if (!g_encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        fn == nullptr || q != cudaDriverEntryPointSuccess)
      return nullptr;
    g_encode = reinterpret_cast<EncodeFn>(fn);
  }
  s.ok = true;
  return &s;
}

bool encode_fp8_kmajor(CUtensorMap* map, const void* ptr, int64_t rows, int64_t K, int64_t ld_bytes, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
  cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int qb_gemm_fp8_noalloc(const void* a, int64_t lda, const float* a_scale, const void* b, int64_t ldb,
                                   const float* b_scale, void* d, int64_t ldd, int M, int N, int K,
                                   cudaStream_t stream, int* status_out) {
  if (!a || !a_scale || !b || !b_scale || !d) return QB_NOALLOC_BAD_ARGUMENT;
  if (M < 0 || N <= 0 || K <= 0 || K % 128 != 0 || N % 16 != 0) return QB_NOALLOC_BAD_ARGUMENT;
  if (lda < K || ldb < K || lda % 16 != 0 || ldb % 16 != 0 || ldd < N || ldd % 8 != 0)
    return QB_NOALLOC_BAD_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) & 15) return QB_NOALLOC_BAD_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(d) & 15) return QB_NOALLOC_BAD_ARGUMENT;
  const int G = K / 128;
  if ((int64_t)M * G > (int64_t)QB_NOALLOC_MAX_SCALES) return QB_NOALLOC_TOO_LARGE;

  DeviceSetup* s = setup_current_device();
  if (!s) return QB_NOALLOC_SETUP_FAILED;
  int* status = reinterpret_cast<int*>(s->scratch);
  float* sa = reinterpret_cast<float*>(s->scratch + 256);

  // the status word must start at zero on every call
  if (cudaMemsetAsync(status, 0, sizeof(int), stream) != cudaSuccess) return QB_NOALLOC_LAUNCH_FAILED;
  if (M == 0) {
    // nothing to compute; the caller still gets the status word it asked for
    if (status_out) *status_out = 0;
    return QB_NOALLOC_OK;
  }

  const int n = M * G;
  transpose_scales_kernel<<<(n + 255) / 256, 256, 0, stream>>>(a_scale, sa, M, G);
  if (cudaGetLastError() != cudaSuccess) return QB_NOALLOC_LAUNCH_FAILED;

  CUtensorMap ta, tb;
  if (!encode_fp8_kmajor(&ta, a, M, K, lda, 128) || !encode_fp8_kmajor(&tb, b, N, K, ldb, kBN))
    return QB_NOALLOC_BAD_ARGUMENT;

  qb::GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.D = static_cast<__nv_bfloat16*>(d);
  p.ldd = (int)ldd;
  p.sa = sa;
  p.lds = M;
  p.sb = b_scale;
  p.sb_gran = 128;
  p.err = status;
  p.num_m_tiles = (M + 127) / 128;
  p.num_n_tiles = (N + kBN - 1) / kBN;
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  const int grid = std::min(tiles, s->sms);
  qb::gemm_sm100_kernel<kBN, true, qb::kEpiBf16, kStages><<<grid, 64 + kBN, kSmem, stream>>>(ta, tb, p);
  if (cudaGetLastError() != cudaSuccess) return QB_NOALLOC_LAUNCH_FAILED;

  if (status_out) {
    if (cudaStreamSynchronize(stream) != cudaSuccess) return QB_NOALLOC_LAUNCH_FAILED;
    if (cudaMemcpy(status_out, status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
      return QB_NOALLOC_LAUNCH_FAILED;
    if (*status_out != 0) return QB_NOALLOC_KERNEL_TIMEOUT;
  }
  return QB_NOALLOC_OK;
}
