// K15: NVFP4 GEMM on tcgen05 (kind::mxf4nvf4, 16-element blocks).
//
//   D[M, N] = alpha * sum_k (A[m, k] * sa[m, k/16]) * (B[n, k] * sb[n, k/16])   (+ residual)
//
// A and B are E2M1 (4-bit floats, two per byte, element 2i in the low
// nibble), K-major. The block scales are UE4M3 bytes (e4m3 with the sign bit
// clear), one per row and 16-wide K block, in the same atom layout as the MX
// GEMM's UE8M0 bytes: a 128-row x 64-K chunk is 512 bytes, row r and 16-wide
// block j at byte (r % 32) * 16 + ((r % 128) / 32) * 4 + j, chunks ordered
// [row / 128][K / 64]. alpha carries the two tensors' global fp32 scales
// (the NVFP4 checkpoint format: values x block scale x tensor scale).
//
// Structure of the MX fp8 kernel (gemm_mx_sm100.cu), with a 256-wide K stage
// (128 bytes of packed E2M1 per row, the same 128B-swizzled TMA tiles): per
// stage the producer TMA-loads A and B and bulk-copies 4 A scale chunks and
// 4 per 128 B rows; the MMA thread copies them into TMEM (one 4-column
// region per 64-wide K step) and issues four kind::mxf4nvf4.block_scale.block16
// MMAs (K = 64 each, all four scale bytes of the step's region). The
// epilogue scales by alpha while draining TMEM.
//
// Instruction-descriptor fields (A/B format E2M1 = 1, scale format UE4M3 = 0,
// K = 64) follow the CUTLASS sm100 UMMA descriptor definition.
//
// Reference: the reference's NVFP4 MLP for qwen3.8-27b-nvfp4 runs
// scaled_fp4_quant + cutlass_scaled_fp4_mm / flashinfer mm_fp4
// (quail/backends/quail/executor/models/qwen3_5_kernels.py:276-355).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "mx_common.cuh"
#include "tile_order.cuh"

#include <cuda_fp8.h>

namespace qb {

namespace {

constexpr int kF4BN = 256;
constexpr int kF4Stages = 4;
constexpr int kF4ABytes = 128 * 128;               // 128 rows x 256 fp4
constexpr int kF4BBytes = kF4BN * 128;
constexpr int kF4SfaBytes = 4 * 512;               // 4 chunks (K = 4 x 64) of 128 rows
constexpr int kF4SfbBytes = 4 * 512 * (kF4BN / 128);
constexpr int kF4Smem = kF4Stages * (kF4ABytes + kF4BBytes + kF4SfaBytes + kF4SfbBytes) + 1024 + 256;
constexpr int kF4SfaCol = kF4BN;                   // 4 steps x 4 columns
constexpr int kF4SfbCol = kF4BN + 16;              // 4 steps x 8 columns

struct F4Params {
  int M, N, K;
  float alpha;
  const float* row_scale;   // optional per-row scale of A (dynamic activation quantization)
  __nv_bfloat16* D;
  int ldd;
  const __nv_bfloat16* R;
  int ldr;
  const uint8_t* sfa;   // [ceil(M/128)][K/64][512]
  const uint8_t* sfb;   // [ceil(N/128)][K/64][512]
  int* err;
  int num_m_tiles, num_n_tiles;
  int n_fast;   // tile order (gemm_sm100_kernel.cuh: tile_coords)
};

__device__ __forceinline__ void umma_nvfp4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

// E2M1 x E2M1 -> f32, UE4M3 scales, K = 64, both K-major
__host__ __device__ constexpr uint32_t make_idesc_nvfp4(int M, int N) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (0u << 23) | ((uint32_t)(M >> 4) << 24);
}

template <int EPI>
__global__ void __launch_bounds__(64 + kF4BN, 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const F4Params p) {
  constexpr int BM = 128, BN = kF4BN, STAGES = kF4Stages;
  constexpr int EPI_THREADS = BN;
  constexpr int TMEM_COLS = 512;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * kF4ABytes;
  uint8_t* sSFA = sB + STAGES * kF4BBytes;
  uint8_t* sSFB = sSFA + STAGES * kF4SfaBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + STAGES * kF4SfbBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* done_bar = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_k = p.K / 256;
  const int num_tiles = p.num_m_tiles * p.num_n_tiles;
  const int sfb_chunks = (p.N + 127) / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, EPI_THREADS);
    mbar_init(done_bar, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      int last_par[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, p.num_m_tiles, p.num_n_tiles, p.n_fast, tm, tn);
        const int nchunks = min(BN / 128, sfb_chunks - tn * (BN / 128));
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kF4ABytes + kF4BBytes + kF4SfaBytes + nchunks * 2048);
          // x coordinates are bytes: 128 bytes (256 values) per stage
          tma_load_2d(&tmA, &full[stage], sA + stage * kF4ABytes, kb * 128, tm * BM);
          tma_load_2d(&tmB, &full[stage], sB + stage * kF4BBytes, kb * 128, tn * BN);
          // 4 consecutive 64-wide K chunks per 128-row block: 2048 contiguous bytes
          bulk_load(sSFA + stage * kF4SfaBytes, p.sfa + ((size_t)tm * (num_k * 4) + kb * 4) * 512, 2048,
                    &full[stage]);
          for (int c = 0; c < nchunks; ++c)
            bulk_load(sSFB + stage * kF4SfbBytes + c * 2048,
                      p.sfb + ((size_t)(tn * (BN / 128) + c) * (num_k * 4) + kb * 4) * 512, 2048, &full[stage]);
          last_par[stage] = (int)phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
#pragma unroll
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_wait(&full[s], (uint32_t)last_par[s], p.err, kErrTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0, aphase = 0;
      bool ok = true;
      const uint32_t t_sfa = tmem_base + kF4SfaCol;
      const uint32_t t_sfb = tmem_base + kF4SfbCol;
      constexpr uint32_t idesc = make_idesc_nvfp4(BM, BN);
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(acc_empty, aphase ^ 1, p.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // the stage's scale chunks into TMEM (in order with the MMAs below):
          // step k's A chunk at columns 4k.., its B chunks at 8k.. and 8k + 4..
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            tmem_cp_sf(t_sfa + k * 4, sf_chunk_desc(smem_u32(sSFA + stage * kF4SfaBytes + k * 512)));
#pragma unroll
            for (int c = 0; c < BN / 128; ++c)
              tmem_cp_sf(t_sfb + k * 8 + c * 4,
                         sf_chunk_desc(smem_u32(sSFB + stage * kF4SfbBytes + c * 2048 + k * 512)));
          }
          const uint32_t a0 = smem_u32(sA + stage * kF4ABytes);
          const uint32_t b0 = smem_u32(sB + stage * kF4BBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_nvfp4(tmem_base, sw128_kmajor_desc(a0 + k * 32), sw128_kmajor_desc(b0 + k * 32), idesc,
                       t_sfa + k * 4, t_sfb + k * 8, (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) {
          tc_commit(acc_full);
          aphase ^= 1;
        }
      }
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err, kErrTimeoutMma);
    }
  } else {
    const int ew = warp - 2;
    const int q = warp & 3;
    const int h = ew >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t aphase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int tm, tn;
        tile_coords(t, p.num_m_tiles, p.num_n_tiles, p.n_fast, tm, tn);
      const int m = tm * BM + row;
      const int n0 = tn * BN + h * 128;
      if (!mbar_wait(acc_full, aphase, p.err, kErrTimeoutEpilogue)) break;
      aphase ^= 1;
      tc_fence_after();
      float acc[128];
      const uint32_t taddr = tmem_base + lane_base + (uint32_t)(h * 128);
      const float scale = p.alpha * ((p.row_scale != nullptr && m < p.M) ? p.row_scale[m] : 1.f);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        QB_TMEM_LD32(taddr + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[c * 32 + i] = __uint_as_float(r[i]) * scale;
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
      if (m >= p.M) continue;
      __nv_bfloat16* dst = p.D + (size_t)m * p.ldd + n0;
#pragma unroll
      for (int j = 0; j < 128; j += 8) {
        if (n0 + j < p.N) {
          float v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = acc[j + i];
          if constexpr (EPI == kEpiResidual) {
            float rv[8];
            ld_bf16x8f(p.R + (size_t)m * p.ldr + n0 + j, rv);
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] += rv[i];
          }
          st_bf16x8(dst + j, v);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc<TMEM_COLS>(tmem_base);
  }
}

// ------------------------------------------------------------------ activation quantization
// One CTA per row: x (bf16 [T, K]; with swiglu, [T, 2K] = gate | up and the
// value is silu(gate) * up) -> packed E2M1 [T, K/2], UE4M3 block-scale atoms
// and the row's scale g = amax / (448 * 6): block scale = e4m3(amax_block / 6 / g),
// code = E2M1(x / (block scale * g)), both by the hardware's round-to-nearest
// conversions. The GEMM's epilogue multiplies by g (row_scale).
__device__ __forceinline__ float f4_in(const __nv_bfloat16* row, int K, int j, bool swiglu) {
  const float a = __bfloat162float(row[j]);
  if (!swiglu) return a;
  const float u = __bfloat162float(row[K + j]);
  return a / (1.f + __expf(-a)) * u;
}

__device__ __forceinline__ uint8_t f4_pack2(float lo, float hi) {
  // cvt packs its first source into the upper nibble
  uint16_t r;
  asm("{\n\t.reg .b8 b;\n\tcvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n\tcvt.u16.u8 %0, b;\n\t}"
      : "=h"(r)
      : "f"(hi), "f"(lo));
  return (uint8_t)r;
}

__global__ void __launch_bounds__(256) nvfp4_quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int K,
                                                               int swiglu, uint8_t* __restrict__ q, int ldq,
                                                               uint8_t* __restrict__ sf, float* __restrict__ row_scale) {
  __shared__ float red[8];
  const int t = blockIdx.x, tid = threadIdx.x;
  const __nv_bfloat16* row = x + (size_t)t * ldx;
  const int nb = K / 16;
  float amax = 0.f;
  for (int b = tid; b < nb; b += 256)
#pragma unroll
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(f4_in(row, K, b * 16 + i, swiglu)));
  amax = warp_max(amax);
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  __syncthreads();
  amax = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) amax = fmaxf(amax, red[w]);
  const float g = fmaxf(amax, 1e-30f) / (448.f * 6.f);
  if (tid == 0) row_scale[t] = g;
  const float ig = 1.f / g;
  for (int b = tid; b < nb; b += 256) {
    float v[16], bmax = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[i] = f4_in(row, K, b * 16 + i, swiglu);
      bmax = fmaxf(bmax, fabsf(v[i]));
    }
    const __nv_fp8_e4m3 bs(bmax * (1.f / 6.f) * ig);
    const float bsf = float(bs);
    const float inv = bsf > 0.f ? 1.f / (bsf * g) : 0.f;
    __align__(8) uint8_t out[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) out[i] = f4_pack2(v[2 * i] * inv, v[2 * i + 1] * inv);
    *reinterpret_cast<uint2*>(q + (size_t)t * ldq + b * 8) = *reinterpret_cast<const uint2*>(out);
    sf[((size_t)(t / 128) * (K / 64) + b / 4) * 512 + (t % 32) * 16 + ((t % 128) / 32) * 4 + (b % 4)] =
        *reinterpret_cast<const uint8_t*>(&bs);
  }
}

template <int EPI>
void launch_f4(const CUtensorMap& ta, const CUtensorMap& tb, F4Params& p, cudaStream_t st, int dev) {
  auto kern = gemm_nvfp4_kernel<EPI>;
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kF4Smem));
    configured[dev] = true;
  }
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  kern<<<std::min(tiles, num_sms(dev)), 64 + kF4BN, kF4Smem, st>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

// a: [M, K/2] packed E2M1 (uint8), sfa: its UE4M3 block-scale atoms; b: [N, K/2], sfb;
// out bf16 [M, N] = alpha * a . b^T (+ residual with EPI_RESIDUAL).
void gemm_nvfp4(const torch::Tensor& a, const torch::Tensor& sfa, const torch::Tensor& b, const torch::Tensor& sfb,
                double alpha, int64_t epi, torch::Tensor& out, const c10::optional<torch::Tensor>& residual,
                const c10::optional<torch::Tensor>& row_scale) {
  TORCH_CHECK(a.scalar_type() == at::kByte && b.scalar_type() == at::kByte, "gemm_nvfp4: packed E2M1 as uint8");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.stride(1) == 1 && b.stride(1) == 1,
              "gemm_nvfp4: shapes");
  const int M = a.size(0), K = 2 * a.size(1), N = b.size(0);
  TORCH_CHECK(K % 256 == 0 && N % 16 == 0, "gemm_nvfp4: K % 256 == 0 and N % 16 == 0");
  TORCH_CHECK(a.stride(0) % 16 == 0 && b.stride(0) % 16 == 0, "gemm_nvfp4: row strides of 16-byte multiples");
  TORCH_CHECK(sfa.scalar_type() == at::kByte && sfb.scalar_type() == at::kByte && sfa.is_contiguous() &&
                  sfb.is_contiguous(),
              "gemm_nvfp4: uint8 scale bytes");
  TORCH_CHECK(sfa.numel() >= (int64_t)((M + 127) / 128) * (K / 64) * 512, "gemm_nvfp4: A scale bytes too small");
  TORCH_CHECK(sfb.numel() >= (int64_t)((N + 127) / 128) * (K / 64) * 512, "gemm_nvfp4: B scale bytes too small");
  TORCH_CHECK(epi == kEpiBf16 || epi == kEpiResidual, "gemm_nvfp4: bf16 or residual epilogue");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.stride(0) % 8 == 0 &&
                  out.size(0) == M && out.size(1) == N,
              "gemm_nvfp4: bf16 out [M, N]");
  const int dev = a.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  if (M == 0) return;
  F4Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.alpha = (float)alpha;
  p.sfa = sfa.data_ptr<uint8_t>();
  p.sfb = sfb.data_ptr<uint8_t>();
  p.err = device_error_word(dev);
  p.num_m_tiles = (M + 127) / 128;
  p.n_fast = M > N ? 1 : 0;
  p.num_n_tiles = (N + kF4BN - 1) / kF4BN;
  p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldd = out.stride(0);
  if (row_scale.has_value()) {
    TORCH_CHECK(row_scale->scalar_type() == at::kFloat && row_scale->numel() >= M, "gemm_nvfp4: fp32 row scales");
    p.row_scale = row_scale->data_ptr<float>();
  }
  if (epi == kEpiResidual) {
    TORCH_CHECK(residual.has_value() && residual->scalar_type() == at::kBFloat16, "residual");
    p.R = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
  }
  // byte-addressed tensor maps: K/2 bytes per row, 128-byte (256-value) boxes
  CUtensorMap ta = make_tmap_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, M, a.stride(0), 128, 128,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K / 2, N, b.stride(0), 128, kF4BN,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (epi == kEpiBf16)
    launch_f4<kEpiBf16>(ta, tb, p, st, dev);
  else
    launch_f4<kEpiResidual>(ta, tb, p, st, dev);
}

// x bf16 [T, K] (swiglu: [T, 2K] gate | up) -> q uint8 [T, K/2], sf atoms, row_scale fp32 [T]
void nvfp4_quant_rows(const torch::Tensor& x, bool swiglu, torch::Tensor& q, torch::Tensor& sf,
                      torch::Tensor& row_scale) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "nvfp4_quant_rows: bf16 rows");
  const int T = x.size(0), K = swiglu ? x.size(1) / 2 : x.size(1);
  TORCH_CHECK(K % 64 == 0, "nvfp4_quant_rows: K % 64 == 0");
  TORCH_CHECK(q.scalar_type() == at::kByte && q.size(0) >= T && q.size(1) == K / 2 && q.stride(0) % 8 == 0,
              "nvfp4_quant_rows: q [T, K/2]");
  TORCH_CHECK(sf.scalar_type() == at::kByte && sf.numel() >= (int64_t)((T + 127) / 128) * (K / 64) * 512,
              "nvfp4_quant_rows: scale atoms");
  TORCH_CHECK(row_scale.scalar_type() == at::kFloat && row_scale.numel() >= T, "nvfp4_quant_rows: row scales");
  if (T == 0) return;
  const int dev = x.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  if (T % 128) {
    // rows past T in the last 128-row atom block read as zero scales
    const int64_t tail = (int64_t)(T / 128) * (K / 64) * 512;
    C10_CUDA_CHECK(cudaMemsetAsync(sf.data_ptr<uint8_t>() + tail, 0, (size_t)(K / 64) * 512, st));
  }
  nvfp4_quant_rows_kernel<<<T, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), K,
                                             swiglu ? 1 : 0, q.data_ptr<uint8_t>(), q.stride(0),
                                             sf.data_ptr<uint8_t>(), row_scale.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
