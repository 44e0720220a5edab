// K13: Gated DeltaNet layers of hybrid decoders (Qwen3.5), over packed chunks.
//
//   gdn_conv       one CTA per (sequence, 128-channel block): causal depthwise
//                  conv (width W) over the sequence's own tokens, continuing the
//                  conv window of its source state slot; SiLU; q and k heads
//                  L2-normalized (q also scaled by d_k^-1/2); the new window
//                  (last W-1 inputs) written to the sequence's destination slot.
//   gdn_recurrent  per (sequence, value head, column block): a few adjacent
//                  threads own one column j of the d_k x d_v state S in registers
//                  (the columns evolve independently; row partial sums combine by
//                  shuffles): per token
//                    S = exp(g) S;  S += k (beta (v - S^T k))^T;  o = S^T q
//                  with g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b);
//                  the reductions run over i inside a thread pair, so a token
//                  costs one barrier. S is read from the source slot and written
//                  to the destination slot.
//                  (passes of one-token sequences and d_k < 128; the chunked
//                  tensor-core form of the same recurrence is gdn_chunk.cu)
//   gdn_gated_norm one warp per (token, value head): RMSNorm(o) * w * silu(z) -> bf16.
//   short_conv     LFM2's gated short convolution: y = C * conv(B * x), one thread
//                  per channel over a sequence's tokens, window in a state slot.
//
// The state slots are fp32: conv [slots, G, W-1, C], ssm [slots, G, Hv, d_k, d_v]
// (G = Gated DeltaNet layers). Source slot -1 means a zero state.
//
// Reference: the reference runs these phases through vLLM / FLA kernels with
// checkpoint slots (quail/backends/quail/executor/gdn.py:27-1088); the math is
// the chunk-free recurrent form of the gated delta rule.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace qb {

constexpr int kGdnSeqInts = 12;

// ------------------------------------------------------------------ conv
// mixed: bf16 [T, ldm], channels [0, C) = q (Hk*dk) | k (Hk*dk) | v (Hv*dv).
// out: fp32 [T, C]. head_dim: channels per q/k head (dk), a multiple of 32.
template <int W>
__global__ void __launch_bounds__(128) gdn_conv_kernel(const __nv_bfloat16* __restrict__ mixed, int ldm, int C,
                                                       int qk_channels, int head_dim,
                                                       const float* __restrict__ wconv,  // [C, W]
                                                       const int* __restrict__ seqs, const int* __restrict__ sio,
                                                       float* __restrict__ conv_state, int gi, int G,
                                                       float q_scale, float* __restrict__ out) {
  __shared__ float red[4];
  const int s = blockIdx.x;
  const int c = blockIdx.y * 128 + threadIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q0 = seqs[s * kGdnSeqInts], n = seqs[s * kGdnSeqInts + 1];
  const int src = sio[2 * s], dst = sio[2 * s + 1];
  const bool live = c < C;
  float win[W - 1];
  float w[W];
#pragma unroll
  for (int j = 0; j < W; ++j) w[j] = live ? wconv[(size_t)c * W + j] : 0.f;
#pragma unroll
  for (int j = 0; j < W - 1; ++j)
    win[j] = (live && src >= 0) ? conv_state[(((size_t)src * G + gi) * (W - 1) + j) * C + c] : 0.f;
  // the block's channels are one or more whole heads; q/k heads get normalized
  const bool is_qk = blockIdx.y * 128 < qk_channels;
  const int group_warps = head_dim >= 32 ? head_dim / 32 : 1;
  for (int t = 0; t < n; ++t) {
    const float x = live ? __bfloat162float(mixed[(size_t)(q0 + t) * ldm + c]) : 0.f;
    float acc = w[W - 1] * x;
#pragma unroll
    for (int j = 0; j < W - 1; ++j) acc += w[j] * win[j];
#pragma unroll
    for (int j = 0; j < W - 2; ++j) win[j] = win[j + 1];
    win[W - 2] = x;
    float y = acc / (1.f + __expf(-acc));  // SiLU
    if (is_qk) {
      float ss = warp_sum(y * y);
      if (group_warps > 1) {
        __syncthreads();
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        const int g0 = (warp / group_warps) * group_warps;
        ss = 0.f;
        for (int k = 0; k < group_warps; ++k) ss += red[g0 + k];
      }
      y *= rsqrtf(fmaxf(ss, 1e-12f));
      if (c < qk_channels / 2) y *= q_scale;
    }
    if (live) out[(size_t)(q0 + t) * C + c] = y;
  }
  if (live && dst >= 0)   // dst < 0: the state is not kept (a padding row of a replayed decode pass)
#pragma unroll
    for (int j = 0; j < W - 1; ++j) conv_state[(((size_t)dst * G + gi) * (W - 1) + j) * C + c] = win[j];
}

// ------------------------------------------------------------------ recurrent
// conv_out fp32 [T, C]: q at head hk*DK, k at qk/2 + hk*DK, v at qk + h*DV.
// ab: bf16 [T, ldab] with b at column b_col + h, a at column a_col + h.
// out: fp32 [T, Hv*DV].
template <int DK, int PARTS>
__global__ void __launch_bounds__(128 * PARTS) gdn_recurrent_kernel(
    const float* __restrict__ conv_out, int C, int qk_channels, const __nv_bfloat16* __restrict__ ab, int ldab,
    int b_col, int a_col, const float* __restrict__ A_log, const float* __restrict__ dt_bias, int Hv, int Hk, int DV,
    const int* __restrict__ seqs, const int* __restrict__ sio, float* __restrict__ ssm_state, int gi, int G,
    float* __restrict__ out) {
  // PARTS adjacent threads own one column j of S (ROWS rows each; partial sums
  // combined by shuffles); one CTA owns all (up to 128) columns of the head, so
  // the per-token staging and barrier are shared by the whole state
  constexpr int ROWS = DK / PARTS;
  constexpr int CPC = 128;
  __shared__ float sq[2][DK], sk[2][DK], sgb[2][2];
  const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int j = blockIdx.z * CPC + tid / PARTS, part = tid % PARTS, r0 = part * ROWS;
  const int hk = h / (Hv / Hk);
  const int q0 = seqs[s * kGdnSeqInts], n = seqs[s * kGdnSeqInts + 1];
  const int src = sio[2 * s], dst = sio[2 * s + 1];
  const bool live = j < DV;
  float S[ROWS];
  const size_t slot_stride = (size_t)G * Hv * DK * DV;
  const size_t head_off = ((size_t)gi * Hv + h) * DK * DV;
#pragma unroll
  for (int i = 0; i < ROWS; ++i)
    S[i] = (live && src >= 0) ? ssm_state[(size_t)src * slot_stride + head_off + (size_t)(r0 + i) * DV + j] : 0.f;
  const float A = -__expf(A_log[h]);
  const float dtb = dt_bias[h];
  auto stage = [&](int t, int buf) {
    const float* row = conv_out + (size_t)(q0 + t) * C;
    for (int i = tid; i < DK; i += blockDim.x) {
      sq[buf][i] = row[hk * DK + i];
      sk[buf][i] = row[qk_channels / 2 + hk * DK + i];
    }
    if (tid == 0) {
      const float a = __bfloat162float(ab[(size_t)(q0 + t) * ldab + a_col + h]) + dtb;
      const float sp = a > 20.f ? a : log1pf(__expf(a));  // softplus
      sgb[buf][0] = __expf(A * sp);                        // decay exp(g)
      const float b = __bfloat162float(ab[(size_t)(q0 + t) * ldab + b_col + h]);
      sgb[buf][1] = 1.f / (1.f + __expf(-b));              // beta
    }
  };
  auto part_sum = [&](float x) {
#pragma unroll
    for (int o = 1; o < PARTS; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
  };
  if (n > 0) stage(0, 0);
  __syncthreads();
  for (int t = 0; t < n; ++t) {
    const int buf = t & 1;
    const float v = live ? conv_out[(size_t)(q0 + t) * C + qk_channels + h * DV + j] : 0.f;
    if (t + 1 < n) stage(t + 1, buf ^ 1);  // the other buffer: read last iteration, freed by its barrier
    const float decay = sgb[buf][0], beta = sgb[buf][1];
    const float* kk = sk[buf] + r0;
    const float* qq = sq[buf] + r0;
    float kv0 = 0.f, kv1 = 0.f;
#pragma unroll
    for (int i = 0; i < ROWS; i += 2) {
      kv0 += S[i] * kk[i];
      kv1 += S[i + 1] * kk[i + 1];
    }
    const float kv = part_sum(kv0 + kv1);
    const float delta = beta * (v - decay * kv);
    float o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int i = 0; i < ROWS; i += 2) {
      S[i] = decay * S[i] + kk[i] * delta;
      S[i + 1] = decay * S[i + 1] + kk[i + 1] * delta;
      o0 += S[i] * qq[i];
      o1 += S[i + 1] * qq[i + 1];
    }
    const float o = part_sum(o0 + o1);
    if (live && part == 0) out[(size_t)(q0 + t) * Hv * DV + h * DV + j] = o;
    __syncthreads();
  }
  if (live && dst >= 0)
#pragma unroll
    for (int i = 0; i < ROWS; ++i)
      ssm_state[(size_t)dst * slot_stride + head_off + (size_t)(r0 + i) * DV + j] = S[i];
}

// ------------------------------------------------------------------ gated norm
// o fp32 [T, Hv*DV]; z bf16 at z[t * ldz + z_col + h*DV + d]; w [DV] (plain weight).
__global__ void gdn_gated_norm_kernel(const float* __restrict__ o, const __nv_bfloat16* __restrict__ z, int ldz,
                                      int z_col, const __nv_bfloat16* __restrict__ w, int T, int Hv, int DV,
                                      float eps, __nv_bfloat16* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int idx = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (idx >= T * Hv) return;
  const int t = idx / Hv, h = idx % Hv;
  const float* row = o + (size_t)t * Hv * DV + h * DV;
  const __nv_bfloat16* zr = z + (size_t)t * ldz + z_col + h * DV;
  __nv_bfloat16* yr = y + (size_t)t * Hv * DV + h * DV;
  if (DV == 128 && ((ldz | z_col) & 3) == 0) {
    // 4 values per lane: one float4 of o, 8 bytes of z and of y
    const float4 v = *reinterpret_cast<const float4*>(row + lane * 4);
    const float r = rsqrtf(warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w) / DV + eps);
    const uint2 zraw = *reinterpret_cast<const uint2*>(zr + lane * 4);
    const uint2 wraw = *reinterpret_cast<const uint2*>(w + lane * 4);
    const float2 z01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zraw.x));
    const float2 z23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&zraw.y));
    const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wraw.x));
    const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wraw.y));
    auto g = [](float zz) { return zz / (1.f + __expf(-zz)); };
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x * r * w01.x * g(z01.x), v.y * r * w01.y * g(z01.y));
    const __nv_bfloat162 b = __floats2bfloat162_rn(v.z * r * w23.x * g(z23.x), v.w * r * w23.y * g(z23.y));
    uint2 out;
    out.x = *reinterpret_cast<const uint32_t*>(&a);
    out.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(yr + lane * 4) = out;
    return;
  }
  float ss = 0.f;
  for (int d = lane; d < DV; d += 32) ss += row[d] * row[d];
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / DV + eps);
  for (int d = lane; d < DV; d += 32) {
    const float zz = __bfloat162float(zr[d]);
    yr[d] = __float2bfloat16(row[d] * r * __bfloat162float(w[d]) * (zz / (1.f + __expf(-zz))));
  }
}

// ------------------------------------------------------------------ short conv (LFM2)
// bcx bf16 [T, ld] = [B (H) | C (H) | x (H)]; y = C * causal_conv(B * x), no activation,
// continuing the window (last W-1 values of B * x) of the source slot.
template <int W>
__global__ void __launch_bounds__(128) short_conv_kernel(const __nv_bfloat16* __restrict__ bcx, int ld, int H,
                                                         const float* __restrict__ wconv, const int* __restrict__ seqs,
                                                         const int* __restrict__ sio, float* __restrict__ state,
                                                         int li, int NL, __nv_bfloat16* __restrict__ y) {
  const int s = blockIdx.x;
  const int c = blockIdx.y * 128 + threadIdx.x;
  if (c >= H) return;
  const int q0 = seqs[s * kGdnSeqInts], n = seqs[s * kGdnSeqInts + 1];
  const int src = sio[2 * s], dst = sio[2 * s + 1];
  float w[W], win[W - 1];
#pragma unroll
  for (int j = 0; j < W; ++j) w[j] = wconv[(size_t)c * W + j];
#pragma unroll
  for (int j = 0; j < W - 1; ++j) win[j] = src >= 0 ? state[(((size_t)src * NL + li) * (W - 1) + j) * H + c] : 0.f;
  for (int t = 0; t < n; ++t) {
    const __nv_bfloat16* row = bcx + (size_t)(q0 + t) * ld;
    const float bx = __bfloat162float(row[c]) * __bfloat162float(row[2 * H + c]);
    float acc = w[W - 1] * bx;
#pragma unroll
    for (int j = 0; j < W - 1; ++j) acc += w[j] * win[j];
#pragma unroll
    for (int j = 0; j < W - 2; ++j) win[j] = win[j + 1];
    win[W - 2] = bx;
    y[(size_t)(q0 + t) * H + c] = __float2bfloat16(__bfloat162float(row[H + c]) * acc);
  }
  if (dst < 0) return;   // no state kept (whole-sequence passes)
#pragma unroll
  for (int j = 0; j < W - 1; ++j) state[(((size_t)dst * NL + li) * (W - 1) + j) * H + c] = win[j];
}

void short_conv(const torch::Tensor& bcx, const torch::Tensor& wconv, const torch::Tensor& seqs,
                const torch::Tensor& state_io, torch::Tensor& state, int64_t li, torch::Tensor& y) {
  TORCH_CHECK(bcx.scalar_type() == at::kBFloat16 && bcx.stride(1) == 1, "short_conv: bf16 [T, 3H]");
  const int H = y.size(1), W = wconv.size(1);
  TORCH_CHECK(wconv.scalar_type() == at::kFloat && wconv.size(0) == H && state.size(3) == H && state.size(2) == W - 1,
              "short_conv: fp32 weight [H, W], state [slots, L, W-1, H]");
  const int S = seqs.size(0);
  if (S == 0 || bcx.size(0) == 0) return;
  const int dev = bcx.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  dim3 grid(S, (H + 127) / 128);
  TORCH_CHECK(W == 3 || W == 4 || W == 7, "short_conv: width 3, 4 or 7");
#define QB_SHORT_CONV(WW)                                                                                    \
  short_conv_kernel<WW><<<grid, 128, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(bcx.data_ptr()),       \
                                              (int)bcx.stride(0), H, wconv.data_ptr<float>(), seqs.data_ptr<int>(), \
                                              state_io.data_ptr<int>(), state.data_ptr<float>(), (int)li,   \
                                              (int)state.size(1), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()))
  if (W == 3)
    QB_SHORT_CONV(3);
  else if (W == 4)
    QB_SHORT_CONV(4);
  else
    QB_SHORT_CONV(7);
#undef QB_SHORT_CONV
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------ host side
void launch_gdn_chunk(const float* conv_out, int C, int qk_channels, const __nv_bfloat16* ab, int ldab, int b_col,
                      int a_col, const float* A_log, const float* dt_bias, int Hv, int Hk, const int* seqs,
                      const int* sio, int S, float* ssm_state, int gi, int G, float* out, int dev,
                      cudaStream_t st);
int64_t gdn_chunk_ws_bytes(int64_t T, int64_t S, int64_t Hv, int64_t C);
void launch_gdn_chunk_split(const __nv_bfloat16* mixed, const float* wconv, float* conv_state, float q_scale,
                            float* conv_out, int C, int qk_channels, const __nv_bfloat16* ab, int ldab,
                            int b_col, int a_col, const float* A_log, const float* dt_bias, int Hv, int Hk,
                            const int* seqs, const int* sio, int T, int S, float* ssm_state, int gi, int G,
                            float* out, uint8_t* ws, int dev, cudaStream_t st);

// proj: bf16 [T, ld] = [qkv (C) | z (Hv*DV) | b (Hv) | a (Hv)] (the fused in-projection);
// returns bf16 [T, Hv*DV] gated-norm output (the out_proj input).
void gdn_layer(const torch::Tensor& proj, const torch::Tensor& wconv, const torch::Tensor& A_log,
               const torch::Tensor& dt_bias, const torch::Tensor& norm_w, const torch::Tensor& seqs,
               const torch::Tensor& state_io, torch::Tensor& conv_state, torch::Tensor& ssm_state, int64_t gi,
               int64_t Hk, int64_t Hv, int64_t DK, int64_t DV, double eps, torch::Tensor& conv_out,
               torch::Tensor& o, torch::Tensor& y, int64_t mode) {
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && proj.stride(1) == 1, "gdn: bf16 in-projection");
  const int T = proj.size(0), ld = proj.stride(0);
  const int C = 2 * Hk * DK + Hv * DV;
  const int W = wconv.size(1);
  TORCH_CHECK(wconv.scalar_type() == at::kFloat && wconv.size(0) == C, "gdn: fp32 conv weight [C, W]");
  TORCH_CHECK(proj.size(1) >= C + Hv * DV + 2 * Hv, "gdn: projection width");
  TORCH_CHECK(DK % 32 == 0 && DK <= 128 && DV <= 128 && Hv % Hk == 0 && (2 * Hk * DK) % 128 == 0,
              "gdn: head sizes (d_k a multiple of 32, at most 128; q+k channels a multiple of 128)");
  TORCH_CHECK(conv_state.size(2) == W - 1 && conv_state.size(3) == C, "gdn: conv state [slots, G, W-1, C]");
  const int G = conv_state.size(1);
  const int S = seqs.size(0);
  if (T == 0 || S == 0) return;
  const int dev = proj.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  const int* sq = seqs.data_ptr<int>();
  const int* sio = state_io.data_ptr<int>();
  const int b_col = C + Hv * DV, a_col = b_col + Hv;
  TORCH_CHECK(DV <= 128, "gdn: d_v <= 128");
  // mode 0: the split chunked form when some sequence has several new tokens
  // (T > S) and d_k = d_v = 128, else the per-token form; 1: per-token;
  // 2: chunked, one kernel; 3: chunked, split (index + prep + scan)
  const bool chunked = DK == 128 && DV == 128 && ld % 4 == 0 && (mode == 2 || mode == 3 || (mode == 0 && T > S));
  TORCH_CHECK(mode < 2 || chunked, "gdn: the chunked form needs d_k = d_v = 128");
  const float q_scale = (float)(1.0 / std::sqrt((double)DK));
  TORCH_CHECK(W == 4, "gdn: conv width 4");
  if (chunked && mode != 2) {
    // the workspace comes from PyTorch's caching allocator on the current stream;
    // the conv runs token-parallel over the same chunk list
    auto ws = at::empty({gdn_chunk_ws_bytes(T, S, Hv, C)}, proj.options().dtype(at::kByte));
    launch_gdn_chunk_split(reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), wconv.data_ptr<float>(),
                           conv_state.data_ptr<float>(), q_scale, conv_out.data_ptr<float>(), C, (int)(2 * Hk * DK),
                           reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), ld, b_col, a_col,
                           A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), (int)Hv, (int)Hk, sq, sio, T, S,
                           ssm_state.data_ptr<float>(), (int)gi, G, o.data_ptr<float>(), ws.data_ptr<uint8_t>(), dev,
                           st);
  } else {
    dim3 g1(S, (C + 127) / 128);
    gdn_conv_kernel<4><<<g1, 128, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), ld, C,
                                           (int)(2 * Hk * DK), (int)DK, wconv.data_ptr<float>(), sq, sio,
                                           conv_state.data_ptr<float>(), (int)gi, G, q_scale,
                                           conv_out.data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  if (chunked && mode == 2) {
    launch_gdn_chunk(conv_out.data_ptr<float>(), C, (int)(2 * Hk * DK),
                     reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), ld, b_col, a_col,
                     A_log.data_ptr<float>(), dt_bias.data_ptr<float>(), (int)Hv, (int)Hk, sq, sio, S,
                     ssm_state.data_ptr<float>(), (int)gi, G, o.data_ptr<float>(), dev, st);
  }
#define QB_GDN_REC(DKK, PP)                                                                                     \
  if (!chunked && DK == DKK) {                                                                                  \
    dim3 g2(S, Hv, 1);                                                                                           \
    gdn_recurrent_kernel<DKK, PP><<<g2, 128 * PP, 0, st>>>(conv_out.data_ptr<float>(), C, (int)(2 * Hk * DK),        \
                                                      reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), \
                                                      ld, b_col, a_col, A_log.data_ptr<float>(),               \
                                                      dt_bias.data_ptr<float>(), (int)Hv, (int)Hk, (int)DV, sq, \
                                                      sio, ssm_state.data_ptr<float>(), (int)gi, G,            \
                                                      o.data_ptr<float>());                                    \
  }
  QB_GDN_REC(32, 1)
  QB_GDN_REC(64, 2)
  QB_GDN_REC(128, 2)
#undef QB_GDN_REC
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int warps = T * (int)Hv;
  gdn_gated_norm_kernel<<<(warps + 7) / 8, 256, 0, st>>>(
      o.data_ptr<float>(), reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), ld, C,
      reinterpret_cast<const __nv_bfloat16*>(norm_w.data_ptr()), T, (int)Hv, (int)DV, (float)eps,
      reinterpret_cast<__nv_bfloat16*>(y.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
