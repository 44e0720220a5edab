// K1 (MX): fp8 GEMM with hardware block scaling on tcgen05.
//
//   D[M, N] = sum_k (A[m, k] * 2^(ea[m, k/32] - 127)) * (B[n, k] * 2^(eb[n, k/32] - 127))
//
// A and B are e4m3, K-major. The scales are UE8M0 (power-of-two) bytes, one
// per row and 32-wide K block, stored in the tcgen05 scale-factor atom
// layout: for a 128-row x 128-K chunk, 512 bytes where row r, K block j sits
// at byte (r % 32) * 16 + ((r % 128) / 32) * 4 + j; chunks ordered
// [row / 128][K / 128]. Weights quantized with 128x128 blocks repeat one
// byte over their 4 K blocks; activations get one byte per 32 values.
//
// Mainloop per 128-wide K stage: the producer TMA-loads the A and B tiles
// (128B swizzle, one CTA each) and bulk-copies the stage's scale chunks
// into shared memory; the MMA thread copies the scale chunks into TMEM
// (tcgen05.cp 32x128b.warpx4: 32 rows x 16 bytes broadcast to the 4 lane
// quarters) and issues four kind::mxf8f6f4.block_scale MMAs (K = 32 each,
// scale byte selected by sf_id). The accumulator stays in TMEM for the
// whole K loop: no promotion work in registers. The epilogue drains it to
// registers, hands the TMEM buffer back, then converts and stores.
//
// This is the reference's DeepGEMM-on-Blackwell path (vLLM fp8_gemm_nt with
// UE8M0 scales, quail/backends/quail/executor/attention.py:483-492), written
// here as our own kernel.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "mx_common.cuh"
#include "tile_order.cuh"

namespace qb {

struct MxParams {
  int M, N, K;
  __nv_bfloat16* D;
  int ldd;
  const __nv_bfloat16* R;
  int ldr;
  uint8_t* Y;       // e4m3 SwiGLU output [M, N/2]
  int ldy;
  uint8_t* Ysf;     // its UE8M0 scales in the atom layout, K = N/2
  const uint8_t* sfa;  // [ceil(M/128)][K/128][512]
  const uint8_t* sfb;  // [ceil(N/128)][K/128][512]
  int* err;
  int num_m_tiles, num_n_tiles;
  int n_fast;                    // tile order (gemm_sm100_kernel.cuh: tile_coords)
  // kEpiQkvRope: the columns are QH q heads, KH k heads, KH v heads of 128
  int QH, KH, norm_qk;
  float eps;
  const int* positions;          // [M] rotary position of each token
  const int* slots;              // [M] arena row of each token (< 0: not stored)
  const __nv_bfloat16* qn;       // [128] q RMSNorm weight
  const __nv_bfloat16* kn;       // [128] k RMSNorm weight
  const float* cos_sin;          // [max_pos, 128]: cos[64] | sin[64]
  __nv_bfloat16* q_out;          // [M, QH, 128]
  __nv_bfloat16* k_cache;        // [slots, KH, 128]
  __nv_bfloat16* v_cache;
  // kEpiResidualMx: the new residual rows (as stored, bf16) also go out as e4m3
  // with UE8M0 scales per 32 columns (xq [M, N], xq_sf atoms with K = N), and
  // each thread's 128-column partial sum of squares goes to ss_out[m, n / 128]
  // (no atomics: a fixed order of summation, so reruns are bitwise equal): the
  // next GEMM's input without a normalization pass
  uint8_t* xq;
  uint8_t* xq_sf;
  float* ss_out;
  // any epilogue: with row_ss ([M, ss_parts] partial sums), rows are first scaled
  // by 1 / rms = rsqrt(sum(row_ss[m, :]) * inv_k + ss_eps): the RMSNorm of the A
  // rows, whose weight is folded into B
  const float* row_ss;
  int ss_parts;
  float inv_k, ss_eps;
};

template <int EPI>
__global__ void __launch_bounds__(64 + kMxBN, 1)
    gemm_mx_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const MxParams p) {
  constexpr int BM = 128, BN = kMxBN, STAGES = kMxStages;
  constexpr int EPI_THREADS = BN;
  constexpr int TMEM_COLS = 512;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * kMxABytes;
  uint8_t* sSFA = sB + STAGES * kMxBBytes;
  uint8_t* sSFB = sSFA + STAGES * kMxSfaBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + STAGES * kMxSfbBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* done_bar = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_k = p.K / 128;
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
          mbar_arrive_expect_tx(&full[stage], kMxABytes + kMxBBytes + kMxSfaBytes + nchunks * 512);
          tma_load_2d(&tmA, &full[stage], sA + stage * kMxABytes, kb * 128, tm * BM);
          tma_load_2d(&tmB, &full[stage], sB + stage * kMxBBytes, kb * 128, tn * BN);
          bulk_load(sSFA + stage * kMxSfaBytes, p.sfa + ((size_t)tm * num_k + kb) * 512, 512, &full[stage]);
          for (int c = 0; c < nchunks; ++c)
            bulk_load(sSFB + stage * kMxSfbBytes + c * 512,
                      p.sfb + ((size_t)(tn * (BN / 128) + c) * num_k + kb) * 512, 512, &full[stage]);
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
      const uint32_t t_sfa = tmem_base + kMxSfaCol;
      const uint32_t t_sfb = tmem_base + kMxSfbCol;
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
          // scale factors of this stage into TMEM (in order with the MMAs below)
          tmem_cp_sf(t_sfa, sf_chunk_desc(smem_u32(sSFA + stage * kMxSfaBytes)));
#pragma unroll
          for (int c = 0; c < BN / 128; ++c)
            tmem_cp_sf(t_sfb + c * 4, sf_chunk_desc(smem_u32(sSFB + stage * kMxSfbBytes + c * 512)));
          const uint32_t a0 = smem_u32(sA + stage * kMxABytes);
          const uint32_t b0 = smem_u32(sB + stage * kMxBBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            umma_mx(tmem_base, sw128_kmajor_desc(a0 + k * 32), sw128_kmajor_desc(b0 + k * 32),
                    make_idesc_mx(BM, BN, k, k), t_sfa | ((uint32_t)k << 30), t_sfb | ((uint32_t)k << 30),
                    (kb > 0 || k > 0) ? 1u : 0u);
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
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        QB_TMEM_LD32(taddr + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[c * 32 + i] = __uint_as_float(r[i]);
      }
      // the accumulator is in registers: the next tile's MMAs may start
      tc_fence_before();
      mbar_arrive(acc_empty);
      if (m >= p.M) continue;
      if constexpr (EPI != kEpiResidual && EPI != kEpiResidualMx) {
        if (p.row_ss != nullptr) {
          // ss_parts == 0: row_ss already holds 1 / rms per row (row_rinv below)
          float rinv;
          if (p.ss_parts == 0) {
            rinv = p.row_ss[m];
          } else {
            float ss = 0.f;
            for (int j = 0; j < p.ss_parts; ++j) ss += p.row_ss[(size_t)m * p.ss_parts + j];
            rinv = rsqrtf(ss * p.inv_k + p.ss_eps);
          }
#pragma unroll
          for (int i = 0; i < 128; ++i) acc[i] *= rinv;
        }
      }
      if constexpr (EPI == kEpiResidualMx) {
        // residual add, bf16 store, then the stored row as MX e4m3 and its sum of squares
        if (n0 >= p.N) continue;
        __nv_bfloat16* dst = p.D + (size_t)m * p.ldd + n0;
        uint32_t word = 0;
        float ss = 0.f;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float rv[8];
            ld_bf16x8f(p.R + (size_t)m * p.ldr + n0 + g * 32 + j, rv);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              v[j + i] = __bfloat162float(__float2bfloat16(acc[g * 32 + j + i] + rv[i]));
            st_bf16x8(dst + g * 32 + j, &v[j]);
          }
          float amax = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            amax = fmaxf(amax, fabsf(v[i]));
            ss = fmaf(v[i], v[i], ss);
          }
          const uint8_t e = ue8m0_of(amax);
          const float inv = ue8m0_inv(e);
          word |= (uint32_t)e << (8 * g);
          uint8_t* xd = p.xq + (size_t)m * p.N + n0 + g * 32;
#pragma unroll
          for (int j = 0; j < 32; j += 16) {
            __align__(16) __nv_fp8x4_e4m3 pk[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              pk[i] = __nv_fp8x4_e4m3(make_float4(v[j + 4 * i] * inv, v[j + 4 * i + 1] * inv, v[j + 4 * i + 2] * inv,
                                                  v[j + 4 * i + 3] * inv));
            *reinterpret_cast<uint4*>(xd + j) = *reinterpret_cast<const uint4*>(pk);
          }
        }
        *reinterpret_cast<uint32_t*>(p.xq_sf + ((size_t)(m / 128) * (p.N / 128) + n0 / 128) * 512 + (m % 32) * 16 +
                                     ((m % 128) / 32) * 4) = word;
        p.ss_out[(size_t)m * (p.N / 128) + n0 / 128] = ss;
      } else if constexpr (EPI == kEpiQkvRope) {
        // this thread's row of one head: per-head RMSNorm and NeoX RoPE of q and k in
        // fp32, then q to q_out and k / v straight into the token's arena row
        if (n0 >= p.N) continue;
        const int hd = n0 >> 7;
        if (hd < p.QH + p.KH) {
          if (p.norm_qk) {
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < 128; ++i) ss = fmaf(acc[i], acc[i], ss);
            const float rinv = rsqrtf(ss * (1.f / 128.f) + p.eps);
            const __nv_bfloat16* wn = hd < p.QH ? p.qn : p.kn;
#pragma unroll
            for (int j = 0; j < 128; j += 8) {
              float w8[8];
              ld_bf16x8f(wn + j, w8);
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[j + i] = acc[j + i] * rinv * w8[i];
            }
          }
          const float* cs = p.cos_sin + (size_t)p.positions[m] * 128;
#pragma unroll
          for (int i = 0; i < 64; i += 4) {
            const float4 c = __ldg(reinterpret_cast<const float4*>(cs + i));
            const float4 sn = __ldg(reinterpret_cast<const float4*>(cs + 64 + i));
            const float cc[4] = {c.x, c.y, c.z, c.w}, ss4[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float x = acc[i + k], y = acc[i + 64 + k];
              acc[i + k] = x * cc[k] - y * ss4[k];
              acc[i + 64 + k] = y * cc[k] + x * ss4[k];
            }
          }
        }
        __nv_bfloat16* dst;
        if (hd < p.QH) {
          dst = p.q_out + ((size_t)m * p.QH + hd) * 128;
        } else {
          const int slot = p.slots[m];
          if (slot < 0) continue;
          const bool is_k = hd < p.QH + p.KH;
          const int kvh = is_k ? hd - p.QH : hd - p.QH - p.KH;
          dst = (is_k ? p.k_cache : p.v_cache) + ((size_t)slot * p.KH + kvh) * 128;
        }
#pragma unroll
        for (int j = 0; j < 128; j += 8) st_bf16x8(dst + j, &acc[j]);
      } else if constexpr (EPI == kEpiBf16 || EPI == kEpiResidual) {
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
      } else {
        // gate = acc[0..63], up = acc[64..127] of outputs out0 .. out0+63
        const int out0 = tn * (BN / 2) + h * 64;
        if (out0 >= p.N / 2) continue;
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          if constexpr (EPI == kEpiGegluFp8) {
            acc[i] = gelu_tanh_f(acc[i]) * acc[64 + i];
          } else {
            acc[i] = silu_f(acc[i]) * acc[64 + i];
          }
        }
        if constexpr (EPI == kEpiSwigluBf16) {
          __nv_bfloat16* dst = p.D + (size_t)m * p.ldd + out0;
#pragma unroll
          for (int j = 0; j < 64; j += 8) st_bf16x8(dst + j, &acc[j]);
        } else {
          // two 32-wide groups, one UE8M0 scale each, in the next GEMM's A-scale layout
          uint8_t e[2];
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            float amax = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(acc[g * 32 + i]));
            e[g] = ue8m0_of(amax);
            const float inv = ue8m0_inv(e[g]);
            uint8_t* dst = p.Y + (size_t)m * p.ldy + out0 + g * 32;
#pragma unroll
            for (int j = 0; j < 32; j += 16) {
              __align__(16) __nv_fp8x4_e4m3 pk[4];
#pragma unroll
              for (int i = 0; i < 4; ++i)
                pk[i] = __nv_fp8x4_e4m3(make_float4(acc[g * 32 + j + 4 * i] * inv, acc[g * 32 + j + 4 * i + 1] * inv,
                                                    acc[g * 32 + j + 4 * i + 2] * inv,
                                                    acc[g * 32 + j + 4 * i + 3] * inv));
              *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(pk);
            }
          }
          const int kst = out0 / 128, kblk = (out0 % 128) / 32;
          const int ko = p.N / 2 / 128;
          uint8_t* sf = p.Ysf + ((size_t)(m / 128) * ko + kst) * 512 + (m % 32) * 16 + ((m % 128) / 32) * 4 + kblk;
          *reinterpret_cast<uint16_t*>(sf) = (uint16_t)e[0] | ((uint16_t)e[1] << 8);
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

// ------------------------------------------------------------------ host side

template <int EPI>
static void launch_mx(const CUtensorMap& ta, const CUtensorMap& tb, MxParams& p, cudaStream_t st, int dev) {
  auto kern = gemm_mx_kernel<EPI>;
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMxSmem));
    configured[dev] = true;
  }
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  kern<<<std::min(tiles, num_sms(dev)), 64 + kMxBN, kMxSmem, st>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// a: [M, K] e4m3, sfa: MX scale bytes of a; b: [N, K] e4m3, sfb: of b.
void gemm_mx(const torch::Tensor& a, const torch::Tensor& sfa, const torch::Tensor& b, const torch::Tensor& sfb,
             int64_t epi, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf,
             const c10::optional<torch::Tensor>& residual, const c10::optional<torch::Tensor>& row_ss,
             double ss_eps, const c10::optional<torch::Tensor>& xq, const c10::optional<torch::Tensor>& xq_sf,
             const c10::optional<torch::Tensor>& ss_out) {
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && b.scalar_type() == at::kFloat8_e4m3fn, "gemm_mx: e4m3");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.stride(1) == 1 && b.stride(1) == 1,
              "gemm_mx: shapes");
  const int M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(K % 128 == 0 && N % 16 == 0, "gemm_mx: K % 128 == 0 and N % 16 == 0");
  TORCH_CHECK(sfa.scalar_type() == at::kByte && sfb.scalar_type() == at::kByte && sfa.is_contiguous() &&
                  sfb.is_contiguous(),
              "gemm_mx: uint8 scale bytes");
  TORCH_CHECK(sfa.numel() >= (int64_t)((M + 127) / 128) * (K / 128) * 512, "gemm_mx: A scale bytes too small");
  TORCH_CHECK(sfb.numel() >= (int64_t)((N + 127) / 128) * (K / 128) * 512, "gemm_mx: B scale bytes too small");
  const int dev = a.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  if (M == 0) return;
  MxParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.sfa = sfa.data_ptr<uint8_t>();
  p.sfb = sfb.data_ptr<uint8_t>();
  p.err = device_error_word(dev);
  p.num_m_tiles = (M + 127) / 128;
  p.n_fast = M > N ? 1 : 0;
  p.num_n_tiles = (N + kMxBN - 1) / kMxBN;
  if (epi == kEpiSwigluFp8 || epi == kEpiGegluFp8) {
    TORCH_CHECK(N % kMxBN == 0, "SwiGLU / GeGLU: N must be a multiple of 256");
    TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn && out.size(0) == M && out.size(1) == N / 2 &&
                    out.stride(1) == 1 && out.stride(0) % 16 == 0,
                "SwiGLU fp8 output");
    TORCH_CHECK(out_sf.has_value() && out_sf->numel() >= (int64_t)((M + 127) / 128) * (N / 2 / 128) * 512,
                "SwiGLU fp8 output scale bytes");
    p.Y = reinterpret_cast<uint8_t*>(out.data_ptr());
    p.ldy = out.stride(0);
    p.Ysf = out_sf->data_ptr<uint8_t>();
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(1) == 1 && out.stride(0) % 8 == 0, "bf16 out");
    TORCH_CHECK(out.size(0) == M && out.size(1) == (epi == kEpiSwigluBf16 ? N / 2 : N), "gemm_mx: out shape");
    p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    p.ldd = out.stride(0);
  }
  if (epi == kEpiResidual || epi == kEpiResidualMx) {
    TORCH_CHECK(residual.has_value() && residual->scalar_type() == at::kBFloat16, "residual");
    p.R = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    p.ldr = residual->stride(0);
  }
  if (epi == kEpiResidualMx) {
    TORCH_CHECK(N % 128 == 0, "kEpiResidualMx: N must be a multiple of 128");
    TORCH_CHECK(xq.has_value() && xq->scalar_type() == at::kFloat8_e4m3fn && xq->is_contiguous() &&
                    xq->size(0) >= M && xq->size(1) == N,
                "kEpiResidualMx: xq [M, N] e4m3");
    TORCH_CHECK(xq_sf.has_value() && xq_sf->numel() >= (int64_t)((M + 127) / 128) * (N / 128) * 512,
                "kEpiResidualMx: xq scale bytes");
    TORCH_CHECK(ss_out.has_value() && ss_out->scalar_type() == at::kFloat && ss_out->numel() >= (int64_t)M * (N / 128),
                "kEpiResidualMx: ss_out [M, N / 128] fp32 partial sums of squares");
    p.xq = reinterpret_cast<uint8_t*>(xq->data_ptr());
    p.xq_sf = xq_sf->data_ptr<uint8_t>();
    p.ss_out = ss_out->data_ptr<float>();
  }
  if (row_ss.has_value()) {
    TORCH_CHECK(row_ss->scalar_type() == at::kFloat && row_ss->size(0) >= M && row_ss->is_contiguous() &&
                    row_ss->dim() <= 2,
                "row_ss: [M, parts] partial sums of squares, or [M] 1 / rms");
    p.row_ss = row_ss->data_ptr<float>();
    p.ss_parts = row_ss->dim() == 2 ? (int)row_ss->size(1) : 0;
    p.inv_k = 1.f / (float)K;
    p.ss_eps = (float)ss_eps;
  }
  CUtensorMap ta = make_tmap_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, a.stride(0), 128, 128,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, b.stride(0), 128, kMxBN,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  switch (epi) {
    case kEpiQkvRope: TORCH_CHECK(false, "gemm_mx: the QKV epilogue is gemm_mx_qkv_rope"); break;
    case kEpiBf16: launch_mx<kEpiBf16>(ta, tb, p, st, dev); break;
    case kEpiResidual: launch_mx<kEpiResidual>(ta, tb, p, st, dev); break;
    case kEpiResidualMx: launch_mx<kEpiResidualMx>(ta, tb, p, st, dev); break;
    case kEpiSwigluFp8: launch_mx<kEpiSwigluFp8>(ta, tb, p, st, dev); break;
    case kEpiSwigluBf16: launch_mx<kEpiSwigluBf16>(ta, tb, p, st, dev); break;
    case kEpiGegluFp8: launch_mx<kEpiGegluFp8>(ta, tb, p, st, dev); break;
    default: TORCH_CHECK(false, "gemm_mx: unknown epilogue ", epi);
  }
}

// The QKV projection with K4 fused into its epilogue: x [M, K] e4m3 times
// wqkv [(QH + 2 KH) * 128, K] e4m3; per head of 128 columns the epilogue
// applies q / k RMSNorm (norm_qk) and NeoX RoPE at positions[m], writes q to
// q_out [M, QH, 128] and k / v to row slots[m] of the paged caches
// [*, KH, 128] (slots < 0 are not stored). Replaces a bf16 qkv round trip
// through memory and the separate qk_norm_rope_kv launch.
void gemm_mx_qkv_rope(const torch::Tensor& a, const torch::Tensor& sfa, const torch::Tensor& b,
                      const torch::Tensor& sfb, const torch::Tensor& positions, const torch::Tensor& slots,
                      const torch::Tensor& qn, const torch::Tensor& kn, const torch::Tensor& cos_sin,
                      torch::Tensor& q_out, torch::Tensor& k_cache, torch::Tensor& v_cache, int64_t QH, int64_t KH,
                      double eps, bool norm_qk, const c10::optional<torch::Tensor>& row_ss) {
  TORCH_CHECK(a.scalar_type() == at::kFloat8_e4m3fn && b.scalar_type() == at::kFloat8_e4m3fn, "qkv_rope: e4m3");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1) && a.stride(1) == 1 && b.stride(1) == 1,
              "qkv_rope: shapes");
  const int M = a.size(0), K = a.size(1), N = b.size(0);
  TORCH_CHECK(K % 128 == 0 && N == (QH + 2 * KH) * 128 && N % kMxBN == 0, "qkv_rope: N = (QH + 2 KH) * 128");
  TORCH_CHECK(sfa.numel() >= (int64_t)((M + 127) / 128) * (K / 128) * 512 &&
                  sfb.numel() >= (int64_t)((N + 127) / 128) * (K / 128) * 512,
              "qkv_rope: scale bytes");
  TORCH_CHECK(positions.scalar_type() == at::kInt && slots.scalar_type() == at::kInt && positions.numel() >= M &&
                  slots.numel() >= M,
              "qkv_rope: int32 positions / slots per row");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == 128 && cos_sin.is_contiguous(),
              "qkv_rope: cos_sin [max_pos, 128] fp32");
  TORCH_CHECK(q_out.is_contiguous() && q_out.numel() >= (int64_t)M * QH * 128 &&
                  q_out.scalar_type() == at::kBFloat16,
              "qkv_rope: q_out [M, QH, 128] bf16");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(-1) == 128 &&
                  k_cache.size(-2) == KH && k_cache.scalar_type() == at::kBFloat16,
              "qkv_rope: caches [*, KH, 128] bf16");
  TORCH_CHECK(qn.scalar_type() == at::kBFloat16 && kn.scalar_type() == at::kBFloat16 && qn.numel() == 128 &&
                  kn.numel() == 128,
              "qkv_rope: bf16 norm weights of 128");
  const int dev = a.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  if (M == 0) return;
  MxParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.sfa = sfa.data_ptr<uint8_t>();
  p.sfb = sfb.data_ptr<uint8_t>();
  p.err = device_error_word(dev);
  p.num_m_tiles = (M + 127) / 128;
  p.n_fast = M > N ? 1 : 0;
  p.num_n_tiles = N / kMxBN;
  p.QH = (int)QH;
  p.KH = (int)KH;
  p.norm_qk = norm_qk ? 1 : 0;
  p.eps = (float)eps;
  p.positions = positions.data_ptr<int>();
  p.slots = slots.data_ptr<int>();
  p.qn = reinterpret_cast<const __nv_bfloat16*>(qn.data_ptr());
  p.kn = reinterpret_cast<const __nv_bfloat16*>(kn.data_ptr());
  p.cos_sin = cos_sin.data_ptr<float>();
  p.q_out = reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr());
  p.k_cache = reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr());
  p.v_cache = reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr());
  if (row_ss.has_value()) {
    TORCH_CHECK(row_ss->scalar_type() == at::kFloat && row_ss->size(0) >= M && row_ss->is_contiguous() &&
                    row_ss->dim() <= 2,
                "row_ss: [M, parts] partial sums of squares, or [M] 1 / rms");
    p.row_ss = row_ss->data_ptr<float>();
    p.ss_parts = row_ss->dim() == 2 ? (int)row_ss->size(1) : 0;
    p.inv_k = 1.f / (float)K;
    p.ss_eps = (float)eps;
  }
  CUtensorMap ta = make_tmap_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, a.stride(0), 128, 128,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, b.stride(0), 128, kMxBN,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  launch_mx<kEpiQkvRope>(ta, tb, p, st, dev);
}

// 1 / rms per row from the partial sums of squares a kEpiResidualMx epilogue
// wrote ([M, parts], summed in a fixed order): one float per row for the
// epilogues of the GEMMs that read those rows.
__global__ void row_rinv_kernel(const float* __restrict__ parts, int n_parts, int M, float inv_k, float eps,
                                float* __restrict__ out) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float ss = 0.f;
  for (int j = 0; j < n_parts; ++j) ss += parts[(size_t)m * n_parts + j];
  out[m] = rsqrtf(ss * inv_k + eps);
}

void row_rinv(const torch::Tensor& parts, int64_t K, double eps, torch::Tensor& out) {
  TORCH_CHECK(parts.scalar_type() == at::kFloat && parts.dim() == 2 && parts.is_contiguous(), "parts [M, n] fp32");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.numel() >= parts.size(0), "out [M] fp32");
  const int M = parts.size(0);
  if (M == 0) return;
  const int dev = parts.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  row_rinv_kernel<<<(M + 255) / 256, 256, 0, st>>>(parts.data_ptr<float>(), (int)parts.size(1), M, 1.f / (float)K,
                                                   (float)eps, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
