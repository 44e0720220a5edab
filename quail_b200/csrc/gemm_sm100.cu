// K1 / K2: persistent tcgen05 GEMMs for sm_100a.
//
//   D[M, N] = A[M, K] . B[N, K]^T
//
// bf16 (kind::f16): the accumulator lives in TMEM for the whole K loop.
// fp8 block-scaled (kind::f8f6f4): A is e4m3 with one fp32 scale per token
// and 128-wide K group (stored transposed, [K/128, lds]); B is e4m3 with one
// fp32 scale per (gran rows, 128 K) block, gran = 128 for HF
// `weight_scale_inv` or 64 for the gate/up-interleaved weight. Each 128-wide
// K block is accumulated by the tensor core into one of two TMEM buffers and
// the epilogue warps promote it into fp32 registers with the product of the
// two scales while the tensor core fills the other buffer.
//
// This replaces the reference's DeepGEMM `fp8_gemm_nt` call site
// (quail/backends/quail/executor/attention.py:479-499) and its F.linear
// bf16 projections (attention.py:480-481).
//
// Warp roles (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (one elected thread; each CTA loads its own tiles)
//   warp 1      TMEM allocator + UMMA issuer (one elected thread)
//   warps 2..   epilogue: BN/32 warps; warp w reads TMEM lanes 32*(w%4)..+31
//               and half (w-2)/4 of the tile's columns.
//
// Epilogues: bf16 store; bf16 store plus a residual add; SwiGLU of a
// gate/up-interleaved tile ([g 64 | u 64 | g 64 | u 64] per 256 columns) to
// bf16, or to e4m3 with one fp32 scale per token and 128 outputs.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "gemm_sm100_kernel.cuh"

namespace qb {

// ------------------------------------------------------------------ host side

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && ptr != nullptr && q == cudaDriverEntryPointSuccess,
                "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

CUtensorMap make_tmap_2d(const void* ptr, CUtensorMapDataType dtype, int elem_bytes, int64_t inner,
                         int64_t outer, int64_t row_stride_elems, int box_inner, int box_outer,
                         CUtensorMapSwizzle swizzle) {
  CUtensorMap m;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((row_stride_elems * elem_bytes) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(row_stride_elems * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

// 3-D bf16 tensor map, 128-byte swizzle: dims {d0, d1, d2} (d0 contiguous),
// byte strides of dims 1 and 2, box {box0, box1, box2} (box0 * 2 bytes = 128).
CUtensorMap make_tmap_3d_bf16(const void* ptr, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_bytes,
                              int64_t stride2_bytes, int box0, int box1, int box2) {
  CUtensorMap m;
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(stride1_bytes % 16 == 0 && stride2_bytes % 16 == 0, "TMA strides must be multiples of 16 bytes");
  TORCH_CHECK(box0 * 2 == 128, "128-byte swizzle: the inner box is 64 bf16");
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)stride1_bytes, (cuuint64_t)stride2_bytes};
  cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, (cuuint32_t)box2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (3-D) failed: ", (int)r);
  return m;
}

int num_sms(int dev) {
  static int cached[64] = {0};
  if (!cached[dev]) cudaDeviceGetAttribute(&cached[dev], cudaDevAttrMultiProcessorCount, dev);
  return cached[dev];
}

int* device_error_word(int dev);

template <int BN, bool FP8, int EPI, int STAGES>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams& p, cudaStream_t st,
                   int dev) {
  auto kern = gemm_sm100_kernel<BN, FP8, EPI, STAGES>;
  constexpr int smem = STAGES * (128 * 128 + BN * 128) + 1024 /*align*/ + 256 /*bars*/ + 4096 /*xchg*/;
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev] = true;
  }
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  const int grid = std::min(tiles, num_sms(dev));
  kern<<<grid, 64 + BN, smem, st>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// a: [M, K] (bf16 or e4m3), b: [N, K]; returns/writes per the epilogue.
void gemm_sm100(const torch::Tensor& a, const torch::Tensor& b, const c10::optional<torch::Tensor>& sa,
                const c10::optional<torch::Tensor>& sb, int64_t sb_gran, int64_t epi, torch::Tensor& out,
                const c10::optional<torch::Tensor>& out_scale, const c10::optional<torch::Tensor>& residual,
                int64_t bn) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda(), "gemm_sm100: CUDA tensors expected");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "gemm_sm100: shape mismatch");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm_sm100: K must be contiguous");
  const bool fp8 = a.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(fp8 == (b.scalar_type() == at::kFloat8_e4m3fn), "gemm_sm100: A and B must share a type");
  TORCH_CHECK(fp8 || (a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16),
              "gemm_sm100: bf16 or e4m3 operands");
  const int M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(K % 128 == 0, "gemm_sm100: K must be a multiple of 128");
  TORCH_CHECK(N % 16 == 0, "gemm_sm100: N must be a multiple of 16");
  const int dev = a.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  if (M == 0) return;

  GemmParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.err = device_error_word(dev);
  const int BN = (int)bn;
  TORCH_CHECK(BN == 128 || BN == 256, "gemm_sm100: BN is 128 or 256");
  p.num_m_tiles = (M + 127) / 128;
  p.num_n_tiles = (N + BN - 1) / BN;
  p.n_fast = M > N ? 1 : 0;
  if (epi == kEpiSwigluFp8 || epi == kEpiSwigluBf16 || epi == kEpiGegluBf16)
    TORCH_CHECK(N % BN == 0, "SwiGLU / GeGLU: N must be a multiple of BN");

  if (epi == kEpiSwigluFp8) {
    TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn && out.size(0) == M && out.size(1) == N / 2,
                "SwiGLU fp8 output shape");
    TORCH_CHECK(out_scale.has_value(), "SwiGLU fp8 needs an output scale tensor");
    p.Y = reinterpret_cast<uint8_t*>(out.data_ptr());
    p.ldy = out.stride(0);
    p.Ys = out_scale->data_ptr<float>();
    p.ldys = out_scale->stride(0);
    TORCH_CHECK(out_scale->size(0) == N / 256 && out_scale->size(1) >= M, "SwiGLU fp8 scale shape");
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1, "bf16 output expected");
    const int want_n = (epi == kEpiSwigluBf16 || epi == kEpiGegluBf16) ? N / 2 : N;
    TORCH_CHECK(out.size(0) == M && out.size(1) == want_n, "gemm_sm100: output shape");
    TORCH_CHECK(out.stride(0) % 8 == 0, "gemm_sm100: output row stride must be a multiple of 8");
    p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    p.ldd = out.stride(0);
  }
  if (epi == kEpiResidual) {
    TORCH_CHECK(residual.has_value() && residual->scalar_type() == at::kBFloat16, "residual epilogue");
    p.R = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
  }
  CUtensorMap ta, tb;
  if (fp8) {
    TORCH_CHECK(sa.has_value() && sb.has_value(), "fp8 GEMM needs scales");
    TORCH_CHECK(sa->scalar_type() == at::kFloat && sb->scalar_type() == at::kFloat, "fp32 scales");
    TORCH_CHECK(sa->size(0) == K / 128 && sa->size(1) >= M && sa->stride(1) == 1, "A scales: [K/128, >=M]");
    TORCH_CHECK(sb->is_contiguous() && sb->size(1) == K / 128 &&
                    sb->size(0) == (N + sb_gran - 1) / sb_gran,
                "B scales: [ceil(N/gran), K/128]");
    TORCH_CHECK(sb_gran == 128 || sb_gran == 64, "B scale granularity is 64 or 128 rows");
    p.sa = sa->data_ptr<float>();
    p.lds = sa->stride(0);
    p.sb = sb->data_ptr<float>();
    p.sb_gran = sb_gran;
    ta = make_tmap_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, a.stride(0), 128, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    tb = make_tmap_2d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, b.stride(0), 128, BN,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  } else {
    ta = make_tmap_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, M, a.stride(0), 64, 128,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    tb = make_tmap_2d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, N, b.stride(0), 64, BN,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  }

#define QB_GEMM_CASE(BN_, FP8_, EPI_, ST_)                                  \
  if (BN == BN_ && fp8 == FP8_ && epi == EPI_) {                           \
    launch<BN_, FP8_, EPI_, ST_>(ta, tb, p, st, dev);                       \
    return;                                                                \
  }
  QB_GEMM_CASE(256, true, kEpiBf16, 4)
  QB_GEMM_CASE(256, true, kEpiResidual, 4)
  QB_GEMM_CASE(256, true, kEpiSwigluFp8, 4)
  QB_GEMM_CASE(256, true, kEpiSwigluBf16, 4)
  QB_GEMM_CASE(128, true, kEpiBf16, 6)
  QB_GEMM_CASE(128, true, kEpiResidual, 6)
  QB_GEMM_CASE(256, false, kEpiBf16, 4)
  QB_GEMM_CASE(256, false, kEpiResidual, 4)
  QB_GEMM_CASE(256, false, kEpiSwigluBf16, 4)
  QB_GEMM_CASE(256, false, kEpiGegluBf16, 4)
  QB_GEMM_CASE(128, false, kEpiBf16, 6)
  QB_GEMM_CASE(128, false, kEpiResidual, 6)
#undef QB_GEMM_CASE
  TORCH_CHECK(false, "gemm_sm100: unsupported combination BN=", BN, " fp8=", fp8, " epi=", epi);
}

}  // namespace qb
