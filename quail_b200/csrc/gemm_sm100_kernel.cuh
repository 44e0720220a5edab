// Device code of the persistent tcgen05 GEMM (K1 / K2): parameters, tile
// raster, epilogue helpers and the kernel template. Included by the
// translation units that launch it.
#pragma once

#include "common.cuh"
#include "gemm_epi.h"

#include "tile_order.cuh"

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
  int n_fast;   // tile order: 0 = m fastest (consecutive CTAs share a B tile), 1 = n fastest
};

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }
// GELU, tanh form (Hendrycks and Gimpel 2016): 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3)))
__device__ __forceinline__ float gelu_tanh(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

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
        tile_coords(t, p.num_m_tiles, p.num_n_tiles, p.n_fast, tm, tn);
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
      tile_coords(t, p.num_m_tiles, p.num_n_tiles, p.n_fast, tm, tn);
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
        } else if constexpr (EPI == kEpiSwigluBf16 || EPI == kEpiSwigluFp8 || EPI == kEpiGegluBf16) {
          // this thread holds gate (acc[0..63]) and up (acc[64..127]) of
          // outputs 64h .. 64h+63 of output tile tn (128 outputs per tile)
          float amax = 0.f;
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            if constexpr (EPI == kEpiGegluBf16) {
              acc[i] = gelu_tanh(acc[i]) * acc[64 + i];
            } else {
              acc[i] = silu(acc[i]) * acc[64 + i];
            }
            amax = fmaxf(amax, fabsf(acc[i]));
          }
          const int out0 = tn * (BN / 2) + h * 64;
          if constexpr (EPI == kEpiSwigluBf16 || EPI == kEpiGegluBf16) {
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
            const long long budget = wait_budget(p.err);
            while (xf[(par * 2 + (h ^ 1)) * 128 + row] != tile_count + 1) {
              if (clock64() - t0 > budget) {
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
          // SwiGLU / GeGLU to bf16 (bf16 models): gate chunk c, up chunk c + 2
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
              for (int i = 0; i < 32; ++i) {
                const float gv = __uint_as_float(g[i]);
                if constexpr (EPI == kEpiGegluBf16) {
                  v[i] = gelu_tanh(gv) * __uint_as_float(u[i]);
                } else {
                  v[i] = silu(gv) * __uint_as_float(u[i]);
                }
              }
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

}  // namespace qb
