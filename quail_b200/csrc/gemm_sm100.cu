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
//   warp 0      TMA producer (one elected thread; no cluster multicast)
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

namespace qb {

struct GemmParams {
  int M, N, K;
  __nv_bfloat16* D;
  int ldd;
  const __nv_bfloat16* R;  // residual for kEpiResidual (may alias D)
  int ldr;
  uint8_t* Y;  // e4m3 output of kEpiSwigluFp8
  int ldy;
  float* Ys;  // [N/256, ldys] scales of Y
  int ldys;
  const float* sa;  // [K/128, lds]
  int lds;
  const float* sb;  // [ceil(N/gran), K/128]
  int sb_gran;
  int* err;
  int num_m_tiles, num_n_tiles;
};

__device__ __forceinline__ void tile_coords(int t, int num_m_tiles, int& tm, int& tn) {
  // column-major raster: consecutive CTAs share one B tile, A stays in L2
  tm = t % num_m_tiles;
  tn = t / num_m_tiles;
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void store_bf16x8(__nv_bfloat16* dst, const float* v) {
  __align__(16) __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
}

__device__ __forceinline__ void load_bf16x8(const __nv_bfloat16* src, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(src);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <int BN, bool FP8, int EPI, int STAGES>
__global__ void __launch_bounds__(64 + BN, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
  constexpr int BM = 128;
  constexpr int A_BYTES = BM * 128;
  constexpr int B_BYTES = BN * 128;
  constexpr int EPI_THREADS = BN;
  constexpr int TMEM_COLS = 2 * BN;
  constexpr int BK = FP8 ? 128 : 64;  // elements per 128-byte K stage
  constexpr uint32_t IDESC = make_idesc(BM, BN, FP8 ? 0 : 1, FP8 ? 0 : 1);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  // [2 tile parity][2 half][128 rows] amax values, then as many flags
  float* xchg = reinterpret_cast<float*>(tmem_slot + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_k = p.K / BK;
  const int num_tiles = p.num_m_tiles * p.num_n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_THREADS);
    }
    mbar_init(done_bar, 1);
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < 1024; i += blockDim.x) reinterpret_cast<int*>(xchg)[i] = 0;
  if (threadIdx.x == 0) {
    fence_proxy_async_smem();
  }
  if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
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
        tile_coords(t, p.num_m_tiles, tm, tn);
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          tma_load_2d(&tmA, &full[stage], sA + stage * A_BYTES, kb * BK, tm * BM);
          tma_load_2d(&tmB, &full[stage], sB + stage * B_BYTES, kb * BK, tn * BN);
          last_par[stage] = (int)phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // let the copies already issued land before the CTA exits
#pragma unroll
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_wait(&full[s], (uint32_t)last_par[s], p.err, kErrTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int abuf = 0;
      uint32_t aphase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!FP8) {
          if (!mbar_wait(&acc_empty[abuf], aphase ^ 1, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        for (int kb = 0; kb < num_k; ++kb) {
          if (FP8) {
            if (!mbar_wait(&acc_empty[abuf], aphase ^ 1, p.err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          if (!mbar_wait(&full[stage], phase, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(abuf * BN);
          const uint32_t a0 = smem_u32(sA + stage * A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = sw128_kmajor_desc(a0 + k * 32);
            const uint64_t bd = sw128_kmajor_desc(b0 + k * 32);
            if (FP8)
              umma_f8(d, ad, bd, IDESC, k > 0 ? 1u : 0u);
            else
              umma_f16(d, ad, bd, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (FP8) {
            tc_commit(&acc_full[abuf]);
            abuf ^= 1;
            if (abuf == 0) aphase ^= 1;
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!FP8 && ok) {
          tc_commit(&acc_full[abuf]);
          abuf ^= 1;
          if (abuf == 0) aphase ^= 1;
        }
      }
      // every MMA issued above has completed once this barrier flips
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err, kErrTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int q = warp & 3;
    const int h = ew >> 2;  // column half (BN = 256) or 0 (BN = 128)
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int abuf = 0;
    uint32_t aphase = 0;
    const int KB = p.K / 128;
    int tile_count = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++tile_count) {
      int tm, tn;
      tile_coords(t, p.num_m_tiles, tm, tn);
      const int m = tm * BM + row;
      const int n0 = tn * BN + h * 128;  // first of this thread's 128 columns
      bool ok = true;
      if constexpr (FP8) {
        float acc[128];
#pragma unroll
        for (int i = 0; i < 128; ++i) acc[i] = 0.f;
        const int nb_max = (p.N + p.sb_gran - 1) / p.sb_gran - 1;
        const int nb0 = min(n0 / p.sb_gran, nb_max);
        const int nb1 = min((n0 + 64) / p.sb_gran, nb_max);
        for (int kb = 0; kb < num_k; ++kb) {
          const float sa_v = (m < p.M) ? __ldg(&p.sa[(size_t)kb * p.lds + m]) : 0.f;
          const float s0 = sa_v * __ldg(&p.sb[(size_t)nb0 * KB + kb]);
          const float s1 = sa_v * __ldg(&p.sb[(size_t)nb1 * KB + kb]);
          if (!mbar_wait(&acc_full[abuf], aphase, p.err, kErrTimeoutEpilogue)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t taddr = tmem_base + lane_base + (uint32_t)(abuf * BN + h * 128);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t r[16];
            QB_TMEM_LD16(taddr + c * 16, r);
            tmem_ld_wait();
            const float s = (c < 4) ? s0 : s1;
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[c * 16 + i] = fmaf(s, __uint_as_float(r[i]), acc[c * 16 + i]);
          }
          tc_fence_before();
          mbar_arrive(&acc_empty[abuf]);
          abuf ^= 1;
          if (abuf == 0) aphase ^= 1;
        }
        if (!ok) break;
        if constexpr (EPI == kEpiBf16 || EPI == kEpiResidual) {
          if (m < p.M) {
            __nv_bfloat16* dst = p.D + (size_t)m * p.ldd + n0;
#pragma unroll
            for (int j = 0; j < 128; j += 8) {
              if (n0 + j < p.N) {
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = acc[j + i];
                if constexpr (EPI == kEpiResidual) {
                  float rv[8];
                  load_bf16x8(p.R + (size_t)m * p.ldr + n0 + j, rv);
#pragma unroll
                  for (int i = 0; i < 8; ++i) v[i] += rv[i];
                }
                store_bf16x8(dst + j, v);
              }
            }
          }
        } else if constexpr (EPI == kEpiSwigluBf16 || EPI == kEpiSwigluFp8) {
          // this thread holds gate (acc[0..63]) and up (acc[64..127]) of
          // outputs 64h .. 64h+63 of output tile tn (128 outputs per tile)
          float amax = 0.f;
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            acc[i] = silu(acc[i]) * acc[64 + i];
            amax = fmaxf(amax, fabsf(acc[i]));
          }
          const int out0 = tn * (BN / 2) + h * 64;
          if constexpr (EPI == kEpiSwigluBf16) {
            if (m < p.M && out0 < p.N / 2) {
              __nv_bfloat16* dst = p.D + (size_t)m * p.ldd + out0;
#pragma unroll
              for (int j = 0; j < 64; j += 8) store_bf16x8(dst + j, &acc[j]);
            }
          } else {
            static_assert(BN == 256 || EPI != kEpiSwigluFp8, "fp8 SwiGLU needs 128 outputs per tile");
            // exchange the half-group amax with the thread that holds the
            // other 64 outputs of this row (same TMEM lane quarter, other
            // half): a flag per (tile parity, half, row) carries the tile
            // counter, waited on with a bounded spin
            const int par = tile_count & 1;
            volatile float* xv = xchg;
            volatile int* xf = reinterpret_cast<volatile int*>(xchg + 512);
            xv[(par * 2 + h) * 128 + row] = amax;
            __threadfence_block();
            xf[(par * 2 + h) * 128 + row] = tile_count + 1;
            const long long t0 = clock64();
            while (xf[(par * 2 + (h ^ 1)) * 128 + row] != tile_count + 1) {
              if (clock64() - t0 > kWaitBudgetCycles) {
                atomicCAS(p.err, 0, kErrTimeoutEpilogue);
                break;
              }
            }
            __threadfence_block();
            amax = fmaxf(amax, xv[(par * 2 + (h ^ 1)) * 128 + row]);
            const float scale = fmaxf(amax, 1e-12f) / kFp8Max;
            const float inv = 1.0f / scale;
            if (m < p.M && out0 < p.N / 2) {
              uint8_t* dst = p.Y + (size_t)m * p.ldy + out0;
#pragma unroll
              for (int j = 0; j < 64; j += 16) {
                __align__(16) __nv_fp8x4_e4m3 pk[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  pk[i] = __nv_fp8x4_e4m3(make_float4(acc[j + 4 * i] * inv, acc[j + 4 * i + 1] * inv,
                                                      acc[j + 4 * i + 2] * inv, acc[j + 4 * i + 3] * inv));
                *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(pk);
              }
              if (h == 0) p.Ys[(size_t)tn * p.ldys + m] = scale;
            }
          }
        }
      } else {
        // bf16: the full-K accumulator is in TMEM buffer abuf
        if (!mbar_wait(&acc_full[abuf], aphase, p.err, kErrTimeoutEpilogue)) break;
        tc_fence_after();
        const uint32_t taddr = tmem_base + lane_base + (uint32_t)(abuf * BN + h * 128);
        if constexpr (EPI == kEpiBf16 || EPI == kEpiResidual) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            QB_TMEM_LD32(taddr + c * 32, r);
            tmem_ld_wait();
            if (m < p.M) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                const int n = n0 + c * 32 + j;
                if (n < p.N) {
                  float v[8];
#pragma unroll
                  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[j + i]);
                  if constexpr (EPI == kEpiResidual) {
                    float rv[8];
                    load_bf16x8(p.R + (size_t)m * p.ldr + n, rv);
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[i] += rv[i];
                  }
                  store_bf16x8(p.D + (size_t)m * p.ldd + n, v);
                }
              }
            }
          }
        } else {
          // SwiGLU to bf16 (bf16 models): gate chunk c, up chunk c + 2
          const int out0 = tn * (BN / 2) + h * 64;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t g[32], u[32];
            QB_TMEM_LD32(taddr + c * 32, g);
            QB_TMEM_LD32(taddr + 64 + c * 32, u);
            tmem_ld_wait();
            if (m < p.M && out0 < p.N / 2) {
              float v[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = silu(__uint_as_float(g[i])) * __uint_as_float(u[i]);
              __nv_bfloat16* dst = p.D + (size_t)m * p.ldd + out0 + c * 32;
#pragma unroll
              for (int j = 0; j < 32; j += 8) store_bf16x8(dst + j, &v[j]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[abuf]);
        abuf ^= 1;
        if (abuf == 0) aphase ^= 1;
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
  if (epi == kEpiSwigluFp8 || epi == kEpiSwigluBf16) TORCH_CHECK(N % BN == 0, "SwiGLU: N must be a multiple of BN");

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
    const int want_n = (epi == kEpiSwigluBf16) ? N / 2 : N;
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
  QB_GEMM_CASE(128, false, kEpiBf16, 6)
  QB_GEMM_CASE(128, false, kEpiResidual, 6)
#undef QB_GEMM_CASE
  TORCH_CHECK(false, "gemm_sm100: unsupported combination BN=", BN, " fp8=", fp8, " epi=", epi);
}

}  // namespace qb
