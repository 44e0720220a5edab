// Memory-bound per-token kernels of the decoder layer, one pass each:
//
//   K10 embed_gather           token ids -> bf16 rows
//   K3  rmsnorm_quant          RMSNorm of the residual stream -> e4m3 + one fp32
//                              scale per 128 columns (transposed [H/128, lds],
//                              the A-scale layout of the fp8 GEMM), or -> bf16
//   K4  qk_norm_rope_kv        per-head RMSNorm of q and k, NeoX RoPE, q out,
//                              k/v written into the paged KV arena by slot
//       quant_rows             bf16 -> e4m3 + 1x128 scales
//       silu_mul_quant         standalone SwiGLU (+ e4m3 quant) for shapes the
//                              fused GEMM epilogue does not take
//   K9  final_norm_readout     gather the last row of each question, final
//                              RMSNorm, dot with the retained answer rows of
//                              the LM head (yes/no or label-token rows)
//
// They replace the reference's Triton kernels add_rms_norm_quant,
// qk_norm_rope, kv_row_scatter, silu_mul_quant
// (quail/backends/quail/executor/attention.py:772-903) and the readout's
// F.linear over retained rows (quail/backends/quail/executor/readout.py:22-92).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_sm100.h"

namespace qb {

__device__ __forceinline__ void ld_bf16x8(const __nv_bfloat16* p, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ void st_bf16x8(__nv_bfloat16* p, const float* v) {
  __align__(16) __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(h);
}

__device__ __forceinline__ uint2 pack_fp8x8(const float* v, float inv) {
  __nv_fp8x4_e4m3 a(make_float4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv));
  __nv_fp8x4_e4m3 b(make_float4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv));
  uint2 r;
  r.x = *reinterpret_cast<uint32_t*>(&a);
  r.y = *reinterpret_cast<uint32_t*>(&b);
  return r;
}

// ---------------------------------------------------------------- K10 embed
__global__ void embed_gather_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                    __nv_bfloat16* __restrict__ out, int T, int H, int vocab) {
  const int t = blockIdx.x;
  if (t >= T) return;
  int id = ids[t];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// ---------------------------------------------------------------- K3 norm
// One warp per row; each lane owns 8 contiguous columns of every 256-column
// slab, so a 128-column quant group is 16 lanes (half a warp).
__device__ __forceinline__ uint8_t ue8m0_of_amax(float amax) {
  const float sc = fmaxf(amax, 1e-30f) / kFp8Max;
  uint32_t bits = __float_as_uint(sc);
  uint32_t e = (bits >> 23) & 0xff;
  if (bits & 0x7fffff) e += 1;
  return (uint8_t)min(max(e, 1u), 253u);
}
__device__ __forceinline__ float ue8m0_inverse(uint8_t e) { return __uint_as_float((uint32_t)(254 - e) << 23); }

// byte offset of (row m, 32-wide K block j) in the MX scale atom layout of a
// matrix with kst = K/128 K stages
__device__ __forceinline__ size_t sf_atom_offset(int m, int j, int kst) {
  return ((size_t)(m >> 7) * kst + (j >> 2)) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 + (j & 3);
}

// RAW (with MX): no normalization; the row is quantized as it is and its sum
// of squares goes to ss_out[row] (the GEMM that consumes it applies 1/rms).
template <int H, bool FP8, bool MX = false, bool RAW = false>
__global__ void rmsnorm_quant_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                     const __nv_bfloat16* __restrict__ w, float eps,
                                     uint8_t* __restrict__ y8, float* __restrict__ ys, int ldys,
                                     __nv_bfloat16* __restrict__ ybf, int ldy, int T,
                                     float* __restrict__ ss_out = nullptr) {
  constexpr int SLABS = H / 256;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const __nv_bfloat16* row = x + (size_t)warp * ldx;
  float v[SLABS][8];
  float ss = 0.f;
#pragma unroll
  for (int s = 0; s < SLABS; ++s) {
    ld_bf16x8(row + s * 256 + lane * 8, v[s]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[s][i] * v[s][i];
  }
  ss = warp_sum(ss);
  if constexpr (RAW) {
    if (lane == 0) ss_out[warp] = ss;
  }
  const float rinv = rsqrtf(ss / H + eps);
#pragma unroll
  for (int s = 0; s < SLABS; ++s) {
    if constexpr (!RAW) {
      float wv[8];
      ld_bf16x8(w + s * 256 + lane * 8, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[s][i] = v[s][i] * rinv * wv[i];
    }
    if constexpr (FP8 && MX) {
      // one UE8M0 scale per 32 columns (4 lanes)
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[s][i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const uint8_t e = ue8m0_of_amax(amax);
      *reinterpret_cast<uint2*>(y8 + (size_t)warp * H + s * 256 + lane * 8) = pack_fp8x8(v[s], ue8m0_inverse(e));
      if ((lane & 3) == 0) reinterpret_cast<uint8_t*>(ys)[sf_atom_offset(warp, s * 8 + (lane >> 2), H / 128)] = e;
    } else if constexpr (FP8) {
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[s][i]));
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float scale = fmaxf(amax, 1e-12f) / kFp8Max;
      *reinterpret_cast<uint2*>(y8 + (size_t)warp * H + s * 256 + lane * 8) = pack_fp8x8(v[s], 1.0f / scale);
      if ((lane & 15) == 0) ys[(size_t)(s * 2 + (lane >> 4)) * ldys + warp] = scale;
    } else {
      st_bf16x8(ybf + (size_t)warp * ldy + s * 256 + lane * 8, v[s]);
    }
  }
}

// ---------------------------------------------------------------- quant rows
template <bool SWIGLU, bool MX = false>
__global__ void quant_rows_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int K,
                                  uint8_t* __restrict__ y8, int ldy, float* __restrict__ ys, int ldys,
                                  __nv_bfloat16* __restrict__ ybf, int T) {
  // one warp per (row, 256-column slab); SWIGLU reads [gate | up] halves of
  // a 2K-wide row
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int slabs = K / 256;
  const int t = gw / slabs, s = gw % slabs;
  if (t >= T) return;
  float v[8];
  const int col = s * 256 + lane * 8;
  if (SWIGLU) {
    float u[8];
    ld_bf16x8(x + (size_t)t * ldx + col, v);
    ld_bf16x8(x + (size_t)t * ldx + K + col, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] / (1.0f + __expf(-v[i])) * u[i];
  } else {
    ld_bf16x8(x + (size_t)t * ldx + col, v);
  }
  if (MX) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const uint8_t e = ue8m0_of_amax(amax);
    *reinterpret_cast<uint2*>(y8 + (size_t)t * ldy + col) = pack_fp8x8(v, ue8m0_inverse(e));
    if ((lane & 3) == 0) reinterpret_cast<uint8_t*>(ys)[sf_atom_offset(t, col / 32, K / 128)] = e;
  } else if (y8) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = fmaxf(amax, 1e-12f) / kFp8Max;
    *reinterpret_cast<uint2*>(y8 + (size_t)t * ldy + col) = pack_fp8x8(v, 1.0f / scale);
    if ((lane & 15) == 0) ys[(size_t)(s * 2 + (lane >> 4)) * ldys + t] = scale;
  } else {
    st_bf16x8(ybf + (size_t)t * ldy + col, v);
  }
}

// ---------------------------------------------------------------- K4 qk norm + rope + kv write
// One warp per (token, head) over the QH + 2*KH heads of a qkv row. D = 128:
// lane l owns elements 4l..4l+3; NeoX rotation pairs i with i +- 64, which is
// lane l ^ 16.
__global__ void qk_norm_rope_kv_kernel(const __nv_bfloat16* __restrict__ qkv, int ldqkv,
                                       const int* __restrict__ positions,
                                       const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
                                       const float* __restrict__ cos_sin,  // [max_pos, 128]: cos[64] | sin[64]
                                       const int* __restrict__ slots, __nv_bfloat16* __restrict__ q_out,
                                       __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                                       int T, int QH, int KH, float eps, int norm_qk) {
  constexpr int D = 128;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = QH + 2 * KH;
  const int t = gw / heads, hd = gw % heads;
  if (t >= T) return;
  const __nv_bfloat16* src = qkv + (size_t)t * ldqkv + hd * D + lane * 4;
  float v[4];
  {
    uint2 u = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
    float2 a = __bfloat1622float2(h2[0]), b = __bfloat1622float2(h2[1]);
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
  const bool is_v = hd >= QH + KH;
  if (!is_v) {
    if (norm_qk) {
      float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
      ss = warp_sum(ss);
      const float rinv = rsqrtf(ss / D + eps);
      const __nv_bfloat16* w = (hd < QH ? qw : kw) + lane * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = v[i] * rinv * __bfloat162float(w[i]);
    }
    const int pos = positions[t];
    const int base = (lane & 15) * 4;  // index into the 64 frequencies
    const float* cs = cos_sin + (size_t)pos * D;
    float o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float c = cs[base + i], s = cs[64 + base + i];
      const float partner = __shfl_xor_sync(0xffffffffu, v[i], 16);
      o[i] = (lane < 16) ? (v[i] * c - partner * s) : (v[i] * c + partner * s);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = o[i];
  }
  __align__(8) __nv_bfloat162 outp[2] = {__floats2bfloat162_rn(v[0], v[1]), __floats2bfloat162_rn(v[2], v[3])};
  const uint2 packed = *reinterpret_cast<const uint2*>(outp);
  if (hd < QH) {
    *reinterpret_cast<uint2*>(q_out + ((size_t)t * QH + hd) * D + lane * 4) = packed;
  } else {
    const int slot = slots[t];
    if (slot < 0) return;
    const int kvh = is_v ? hd - QH - KH : hd - QH;
    __nv_bfloat16* dst = (is_v ? v_cache : k_cache) + ((size_t)slot * KH + kvh) * D + lane * 4;
    *reinterpret_cast<uint2*>(dst) = packed;
  }
}

// ---------------------------------------------------------------- K9 readout
// One CTA per question row: gather the row, final RMSNorm in fp32, then one
// warp per retained head row computes the dot product.
template <int H>
__global__ void final_norm_readout_kernel(const __nv_bfloat16* __restrict__ x, int ldx,
                                          const int* __restrict__ rows, const __nv_bfloat16* __restrict__ w,
                                          float eps, const __nv_bfloat16* __restrict__ head, int nhead,
                                          float* __restrict__ logits, __nv_bfloat16* __restrict__ normed_out, int R) {
  constexpr int PER = H / 256;  // 8-element chunks per thread with 32 threads... use block of 256
  __shared__ float sx[H];
  __shared__ float red[32];
  const int r = blockIdx.x;
  if (r >= R) return;
  const __nv_bfloat16* src = x + (size_t)rows[r] * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    float v[8];
    ld_bf16x8(src + i, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sx[i + j] = v[j];
      ss += v[j] * v[j];
    }
  }
  ss = warp_sum(ss);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.f;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const float rinv = rsqrtf(red[0] / H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    // round to bf16 like the reference's normed rows before the head GEMM
    const float nv = __bfloat162float(__float2bfloat16(sx[i] * rinv * __bfloat162float(w[i])));
    sx[i] = nv;
    if (normed_out) normed_out[(size_t)r * H + i] = __float2bfloat16(nv);
  }
  __syncthreads();
  const int nwarps = blockDim.x >> 5;
  for (int j = warp; j < nhead; j += nwarps) {
    const __nv_bfloat16* hr = head + (size_t)j * H;
    float acc = 0.f;
    for (int i = lane * 8; i < H; i += 256) {
      float hv[8];
      ld_bf16x8(hr + i, hv);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc += hv[k] * sx[i + k];
    }
    acc = warp_sum(acc);
    if (lane == 0) logits[(size_t)r * nhead + j] = acc;
  }
  (void)PER;
}


// ---------------------------------------------------------------- full-vocab readout
// One CTA per row of bf16 logits [R, V]: argmax and log-sum-exp over the
// vocabulary (greedy decoding for AI.MAP / AI.EXTRACT, normalized label
// log-probabilities for AI.CLASSIFY). Online max/sum per thread, then a
// block reduction.
__global__ void row_argmax_lse_kernel(const __nv_bfloat16* __restrict__ logits, int ld, int V,
                                      int* __restrict__ arg, float* __restrict__ lse) {
  const int r = blockIdx.x;
  const __nv_bfloat16* row = logits + (size_t)r * ld;
  float m = -INFINITY, s = 0.f;
  int am = 0;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float x = __bfloat162float(row[i]);
    if (x > m) {
      s = s * __expf(m - x) + 1.f;
      m = x;
      am = i;
    } else {
      s += __expf(x - m);
    }
  }
  __shared__ float sm[32], ss[32];
  __shared__ int sa[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const int a2 = __shfl_xor_sync(0xffffffffu, am, o);
    const float mn = fmaxf(m, m2);
    const float sn = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mn));
    if (m2 > m || (m2 == m && a2 < am)) am = a2;
    m = mn;
    s = sn;
  }
  if (lane == 0) {
    sm[warp] = m;
    ss[warp] = s;
    sa[warp] = am;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
    am = lane < nw ? sa[lane] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const int a2 = __shfl_xor_sync(0xffffffffu, am, o);
      const float mn = fmaxf(m, m2);
      const float sn = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mn));
      if (m2 > m || (m2 == m && a2 < am)) am = a2;
      m = mn;
      s = sn;
    }
    if (lane == 0) {
      arg[r] = am;
      lse[r] = m + __logf(s);
    }
  }
}

// ------------------------------------------------------------------ host side

static cudaStream_t cur_stream(const torch::Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.get_device());
}

void embed_gather(const torch::Tensor& ids, const torch::Tensor& table, torch::Tensor& out) {
  TORCH_CHECK(ids.scalar_type() == at::kInt && table.scalar_type() == at::kBFloat16, "embed_gather types");
  const int T = ids.numel(), H = table.size(1);
  TORCH_CHECK(H % 8 == 0 && out.size(0) >= T && out.size(1) == H && out.is_contiguous(), "embed_gather shapes");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(ids.get_device());
  embed_gather_kernel<<<T, 128, 0, cur_stream(ids)>>>(ids.data_ptr<int>(),
                                                      reinterpret_cast<const __nv_bfloat16*>(table.data_ptr()),
                                                      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), T, H,
                                                      table.size(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// x: [T, H] bf16 (row stride ldx). fp8 mode: y8 [T, H] e4m3 contiguous,
// ys [H/128, >=T]. bf16 mode: ybf [T, H].
void rmsnorm_quant(const torch::Tensor& x, const torch::Tensor& w, double eps, const c10::optional<torch::Tensor>& y8,
                   const c10::optional<torch::Tensor>& ys, const c10::optional<torch::Tensor>& ybf, int64_t T) {
  const int H = x.size(1);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && w.numel() == H, "rmsnorm_quant inputs");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(x.get_device());
  const int threads = 256, blocks = (int)((T * 32 + threads - 1) / threads);
  const bool fp8 = y8.has_value();
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  uint8_t* y8p = fp8 ? reinterpret_cast<uint8_t*>(y8->data_ptr()) : nullptr;
  float* ysp = fp8 ? ys->data_ptr<float>() : nullptr;
  const int ldys = fp8 ? ys->stride(0) : 0;
  __nv_bfloat16* ybp = fp8 ? nullptr : reinterpret_cast<__nv_bfloat16*>(ybf->data_ptr());
  const int ldy = fp8 ? H : ybf->stride(0);
  if (fp8) TORCH_CHECK(y8->is_contiguous() && y8->size(1) == H && ys->size(0) == H / 128 && ys->size(1) >= T, "fp8 out");
#define QB_NORM_CASE(HH)                                                                                \
  if (H == HH) {                                                                                        \
    if (fp8)                                                                                            \
      rmsnorm_quant_kernel<HH, true><<<blocks, threads, 0, cur_stream(x)>>>(xp, x.stride(0), wp, eps, y8p, \
                                                                            ysp, ldys, ybp, ldy, T);    \
    else                                                                                                \
      rmsnorm_quant_kernel<HH, false><<<blocks, threads, 0, cur_stream(x)>>>(xp, x.stride(0), wp, eps, y8p, \
                                                                             ysp, ldys, ybp, ldy, T);   \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                     \
    return;                                                                                             \
  }
  QB_NORM_CASE(256)
  QB_NORM_CASE(512)
  QB_NORM_CASE(1024)
  QB_NORM_CASE(2048)
  QB_NORM_CASE(2560)
  QB_NORM_CASE(2816)
  QB_NORM_CASE(4096)
  QB_NORM_CASE(5120)
#undef QB_NORM_CASE
  TORCH_CHECK(false, "rmsnorm_quant: unsupported hidden size ", H);
}

// x: [T, H] bf16 -> e4m3 [T, H] + UE8M0 scale bytes of x itself (no normalization) and
// ss [T, 1] fp32, the sum of squares of each row: the input of a GEMM that applies the
// row's 1/rms in its epilogue (the norm weight folded into its B operand).
void quant_mx_ss(const torch::Tensor& x, torch::Tensor& y8, torch::Tensor& sf, torch::Tensor& ss, int64_t T) {
  const int H = x.size(1);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1, "quant_mx_ss: bf16 rows");
  TORCH_CHECK(y8.is_contiguous() && y8.size(1) == H && y8.size(0) >= T, "quant_mx_ss output");
  TORCH_CHECK(sf.scalar_type() == at::kByte && sf.numel() >= (T + 127) / 128 * (H / 128) * 512, "scale bytes");
  TORCH_CHECK(ss.scalar_type() == at::kFloat && ss.numel() >= T, "ss: fp32 per row");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(x.get_device());
  const int threads = 256, blocks = (int)((T * 32 + threads - 1) / threads);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto yp = reinterpret_cast<uint8_t*>(y8.data_ptr());
  auto sp = reinterpret_cast<float*>(sf.data_ptr());
#define QB_QSS_CASE(HH)                                                                                        \
  if (H == HH) {                                                                                               \
    rmsnorm_quant_kernel<HH, true, true, true><<<blocks, threads, 0, cur_stream(x)>>>(                         \
        xp, x.stride(0), nullptr, 0.f, yp, sp, 0, nullptr, 0, (int)T, ss.data_ptr<float>());                   \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                            \
    return;                                                                                                    \
  }
  QB_QSS_CASE(1024)
  QB_QSS_CASE(2048)
  QB_QSS_CASE(2560)
  QB_QSS_CASE(2816)
  QB_QSS_CASE(4096)
  QB_QSS_CASE(5120)
#undef QB_QSS_CASE
  TORCH_CHECK(false, "quant_mx_ss: unsupported hidden size ", H);
}

// x: [T, H] bf16 -> e4m3 [T, H] + UE8M0 scale bytes (MX atom layout, one per 32 columns)
void rmsnorm_quant_mx(const torch::Tensor& x, const torch::Tensor& w, double eps, torch::Tensor& y8,
                      torch::Tensor& sf, int64_t T) {
  const int H = x.size(1);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.stride(1) == 1 && w.numel() == H, "rmsnorm_quant_mx inputs");
  TORCH_CHECK(y8.is_contiguous() && y8.size(1) == H && y8.size(0) >= T, "rmsnorm_quant_mx output");
  TORCH_CHECK(sf.scalar_type() == at::kByte && sf.numel() >= (T + 127) / 128 * (H / 128) * 512, "scale bytes");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(x.get_device());
  const int threads = 256, blocks = (int)((T * 32 + threads - 1) / threads);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr());
  auto yp = reinterpret_cast<uint8_t*>(y8.data_ptr());
  auto sp = reinterpret_cast<float*>(sf.data_ptr());
#define QB_NORM_MX(HH)                                                                                   \
  if (H == HH) {                                                                                         \
    rmsnorm_quant_kernel<HH, true, true><<<blocks, threads, 0, cur_stream(x)>>>(xp, x.stride(0), wp, eps, yp, \
                                                                                sp, 0, nullptr, 0, T);   \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                      \
    return;                                                                                              \
  }
  QB_NORM_MX(256)
  QB_NORM_MX(512)
  QB_NORM_MX(1024)
  QB_NORM_MX(2048)
  QB_NORM_MX(2560)
  QB_NORM_MX(2816)
  QB_NORM_MX(4096)
  QB_NORM_MX(5120)
#undef QB_NORM_MX
  TORCH_CHECK(false, "rmsnorm_quant_mx: unsupported hidden size ", H);
}

// x: [T, K] (or [T, 2K] with swiglu) bf16 -> e4m3 [T, K] + scales [K/128, >=T], or bf16 [T, K]
void quant_rows(const torch::Tensor& x, bool swiglu, const c10::optional<torch::Tensor>& y8,
                const c10::optional<torch::Tensor>& ys, const c10::optional<torch::Tensor>& ybf, int64_t T) {
  const int K = swiglu ? x.size(1) / 2 : x.size(1);
  TORCH_CHECK(K % 256 == 0 && x.stride(1) == 1 && x.scalar_type() == at::kBFloat16, "quant_rows: K % 256");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(x.get_device());
  const int warps = (int)T * (K / 256);
  const int threads = 256, blocks = (warps * 32 + threads - 1) / threads;
  uint8_t* y8p = y8.has_value() ? reinterpret_cast<uint8_t*>(y8->data_ptr()) : nullptr;
  float* ysp = ys.has_value() ? ys->data_ptr<float>() : nullptr;
  const int ldys = ys.has_value() ? ys->stride(0) : 0;
  __nv_bfloat16* ybp = ybf.has_value() ? reinterpret_cast<__nv_bfloat16*>(ybf->data_ptr()) : nullptr;
  const int ldy = y8.has_value() ? y8->stride(0) : ybf->stride(0);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  if (swiglu)
    quant_rows_kernel<true><<<blocks, threads, 0, cur_stream(x)>>>(xp, x.stride(0), K, y8p, ldy, ysp, ldys, ybp, T);
  else
    quant_rows_kernel<false><<<blocks, threads, 0, cur_stream(x)>>>(xp, x.stride(0), K, y8p, ldy, ysp, ldys, ybp, T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void quant_rows_mx(const torch::Tensor& x, bool swiglu, torch::Tensor& y8, torch::Tensor& sf, int64_t T) {
  const int K = swiglu ? x.size(1) / 2 : x.size(1);
  TORCH_CHECK(K % 256 == 0 && x.stride(1) == 1 && x.scalar_type() == at::kBFloat16, "quant_rows_mx: K % 256");
  TORCH_CHECK(y8.stride(1) == 1 && y8.size(1) == K && sf.numel() >= (T + 127) / 128 * (K / 128) * 512,
              "quant_rows_mx outputs");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(x.get_device());
  const int warps = (int)T * (K / 256);
  const int threads = 256, blocks = (warps * 32 + threads - 1) / threads;
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  auto yp = reinterpret_cast<uint8_t*>(y8.data_ptr());
  auto sp = reinterpret_cast<float*>(sf.data_ptr());
  if (swiglu)
    quant_rows_kernel<true, true><<<blocks, threads, 0, cur_stream(x)>>>(xp, x.stride(0), K, yp, y8.stride(0), sp, 0,
                                                                         nullptr, T);
  else
    quant_rows_kernel<false, true><<<blocks, threads, 0, cur_stream(x)>>>(xp, x.stride(0), K, yp, y8.stride(0), sp,
                                                                          0, nullptr, T);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void qk_norm_rope_kv(const torch::Tensor& qkv, const torch::Tensor& positions, const torch::Tensor& qw,
                     const torch::Tensor& kw, const torch::Tensor& cos_sin, const torch::Tensor& slots,
                     torch::Tensor& q_out, torch::Tensor& k_cache, torch::Tensor& v_cache, int64_t QH, int64_t KH,
                     double eps, bool norm_qk, int64_t T) {
  TORCH_CHECK(qkv.size(1) >= (QH + 2 * KH) * 128 && qkv.stride(1) == 1, "qk_norm_rope_kv: D must be 128");
  TORCH_CHECK(cos_sin.scalar_type() == at::kFloat && cos_sin.size(1) == 128, "cos_sin [max_pos, 128]");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && q_out.is_contiguous(), "contiguous caches");
  if (T == 0) return;
  c10::cuda::CUDAGuard g(qkv.get_device());
  const long warps = T * (QH + 2 * KH);
  const int threads = 256;
  const int blocks = (int)((warps * 32 + threads - 1) / threads);
  qk_norm_rope_kv_kernel<<<blocks, threads, 0, cur_stream(qkv)>>>(
      reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr()), qkv.stride(0), positions.data_ptr<int>(),
      reinterpret_cast<const __nv_bfloat16*>(qw.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(kw.data_ptr()),
      cos_sin.data_ptr<float>(), slots.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()),
      (int)T, (int)QH, (int)KH, (float)eps, norm_qk ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void final_norm_readout(const torch::Tensor& x, const torch::Tensor& rows, const torch::Tensor& w, double eps,
                        const torch::Tensor& head, torch::Tensor& logits, const c10::optional<torch::Tensor>& normed) {
  const int H = x.size(1), R = rows.numel(), NH = head.size(0);
  TORCH_CHECK(head.size(1) == H && head.is_contiguous() && logits.is_contiguous() && logits.size(0) >= R &&
                  logits.size(1) == NH,
              "final_norm_readout shapes");
  if (R == 0) return;
  c10::cuda::CUDAGuard g(x.get_device());
  __nv_bfloat16* np = normed.has_value() ? reinterpret_cast<__nv_bfloat16*>(normed->data_ptr()) : nullptr;
#define QB_RO_CASE(HH)                                                                                   \
  if (H == HH) {                                                                                         \
    final_norm_readout_kernel<HH><<<R, 256, 0, cur_stream(x)>>>(                                         \
        reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), x.stride(0), rows.data_ptr<int>(),         \
        reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (float)eps,                                \
        reinterpret_cast<const __nv_bfloat16*>(head.data_ptr()), NH, logits.data_ptr<float>(), np, R);   \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                      \
    return;                                                                                              \
  }
  QB_RO_CASE(256)
  QB_RO_CASE(512)
  QB_RO_CASE(1024)
  QB_RO_CASE(2048)
  QB_RO_CASE(2560)
  QB_RO_CASE(2816)
  QB_RO_CASE(4096)
  QB_RO_CASE(5120)
#undef QB_RO_CASE
  TORCH_CHECK(false, "final_norm_readout: unsupported hidden size ", H);
}

void row_argmax_lse(const torch::Tensor& logits, torch::Tensor& arg, torch::Tensor& lse) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1, "row_argmax_lse: bf16 rows");
  TORCH_CHECK(arg.scalar_type() == at::kInt && lse.scalar_type() == at::kFloat, "row_argmax_lse outputs");
  const int R = logits.size(0), V = logits.size(1);
  if (R == 0) return;
  c10::cuda::CUDAGuard g(logits.get_device());
  row_argmax_lse_kernel<<<R, 512, 0, cur_stream(logits)>>>(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()),
                                                           logits.stride(0), V, arg.data_ptr<int>(),
                                                           lse.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
