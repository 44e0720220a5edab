// K7: merge two attention reads of the same query rows over disjoint key sets.
//
//   out[t] = (o_a[t] * e^{lse_a[t]} + o_b[s] * e^{lse_b[s]}) / (e^{lse_a[t]} + e^{lse_b[s]}),  s = source[t]
//
// per (row, head); rows with source -1 keep o_a. The tree attention path reads each
// row's own keys in one call (o_a) and the keys of a shared resident prefix in a
// second call over the stacked rows of all its readers (o_b); this kernel joins them
// and writes the next GEMM's input: bf16, or e4m3 with one UE8M0 scale byte per 32
// columns in the MX scale-factor atom layout (128 rows x 128 columns per 512 bytes).
// One thread per (row, 32-column group): 64 bytes of each input, read once.
//
// Reference: the online-softmax merge of quail/backends/quail/executor/attention.py
// (merge_partial, the fused merge_attn_quant Triton kernel), written here for sm_100a.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "mx_common.cuh"

namespace qb {
namespace {

template <bool FP8>
__global__ void __launch_bounds__(256) attention_merge_kernel(
    const __nv_bfloat16* __restrict__ oa, const float* __restrict__ la, const __nv_bfloat16* __restrict__ ob,
    const float* __restrict__ lb, const int* __restrict__ source, int T, int QH, int D, int W, int rows_b,
    __nv_bfloat16* __restrict__ out, uint8_t* __restrict__ o8, uint8_t* __restrict__ osf) {
  const int groups = W / 32;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)T * groups) return;
  const int t = (int)(idx / groups), g = (int)(idx % groups);
  const int head = (g * 32) / D;
  const int s = source[t];
  const bool has_b = s >= 0 && s < rows_b;          // host-staged index, checked
  float wa = 1.f, wb = 0.f;
  if (has_b) {
    const float a = la[(size_t)t * QH + head], b = lb[(size_t)s * QH + head];
    const float m = fmaxf(a, b);
    if (m == -INFINITY) {
      wa = 0.f;
    } else {
      wa = a == -INFINITY ? 0.f : __expf(a - m);
      wb = b == -INFINITY ? 0.f : __expf(b - m);
      const float z = 1.f / (wa + wb);
      wa *= z;
      wb *= z;
    }
  }
  float v[32];
  const uint4* pa = reinterpret_cast<const uint4*>(oa + (size_t)t * W + g * 32);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4 u = pa[k];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      v[k * 8 + 2 * e] = f.x * wa;
      v[k * 8 + 2 * e + 1] = f.y * wa;
    }
  }
  if (has_b && wb != 0.f) {
    const uint4* pb = reinterpret_cast<const uint4*>(ob + (size_t)s * W + g * 32);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 u = pb[k];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        v[k * 8 + 2 * e] += f.x * wb;
        v[k * 8 + 2 * e + 1] += f.y * wb;
      }
    }
  }
  if constexpr (!FP8) {
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * W + g * 32);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      __align__(16) __nv_bfloat162 h[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[k * 8 + 2 * e], v[k * 8 + 2 * e + 1]);
      dst[k] = *reinterpret_cast<const uint4*>(h);
    }
  } else {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const uint8_t e8 = ue8m0_of(amax);
    const float sc = ue8m0_inv(e8);
    uint4* dst = reinterpret_cast<uint4*>(o8 + (size_t)t * W + g * 32);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      __align__(16) __nv_fp8x4_e4m3 pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = k * 16 + 4 * e;
        pk[e] = __nv_fp8x4_e4m3(make_float4(v[i] * sc, v[i + 1] * sc, v[i + 2] * sc, v[i + 3] * sc));
      }
      dst[k] = *reinterpret_cast<const uint4*>(pk);
    }
    // scale byte of (row t, 32-column block g): chunk [t / 128][g / 4] of 512 bytes
    const size_t chunk = (size_t)(t >> 7) * (W / 128) + (g >> 2);
    osf[chunk * 512 + (t & 31) * 16 + ((t & 127) >> 5) * 4 + (g & 3)] = e8;
  }
}

}  // namespace

void attention_merge(const torch::Tensor& o_a, const torch::Tensor& lse_a, const torch::Tensor& o_b,
                     const torch::Tensor& lse_b, const torch::Tensor& source, int64_t QH, torch::Tensor& out,
                     const c10::optional<torch::Tensor>& out_sf) {
  TORCH_CHECK(o_a.scalar_type() == at::kBFloat16 && o_b.scalar_type() == at::kBFloat16 && o_a.is_contiguous() &&
                  o_b.is_contiguous() && o_a.dim() == 2 && o_b.dim() == 2 && o_b.size(1) == o_a.size(1),
              "attention_merge: contiguous bf16 o_a [T, W], o_b [R, W]");
  TORCH_CHECK(lse_a.scalar_type() == at::kFloat && lse_b.scalar_type() == at::kFloat && lse_a.is_contiguous() &&
                  lse_b.is_contiguous() && lse_a.numel() == o_a.size(0) * QH && lse_b.numel() == o_b.size(0) * QH,
              "attention_merge: fp32 lse [rows, QH]");
  TORCH_CHECK(source.scalar_type() == at::kInt && source.numel() == o_a.size(0), "attention_merge: int32 source [T]");
  const int T = o_a.size(0), W = o_a.size(1);
  TORCH_CHECK(W % 128 == 0 && W % QH == 0 && (W / QH) % 32 == 0, "attention_merge: W = QH * D, D a multiple of 32");
  if (T == 0) return;
  const int dev = o_a.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  const long long n = (long long)T * (W / 32);
  const int grid = (int)((n + 255) / 256);
  const int D = W / (int)QH, R = o_b.size(0);
  if (out.scalar_type() == at::kFloat8_e4m3fn) {
    TORCH_CHECK(out_sf.has_value() && out_sf->scalar_type() == at::kByte &&
                    out_sf->numel() >= (int64_t)((T + 127) / 128) * (W / 128) * 512,
                "attention_merge: e4m3 output needs its MX scale bytes");
    attention_merge_kernel<true><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(o_a.data_ptr()), lse_a.data_ptr<float>(),
        reinterpret_cast<const __nv_bfloat16*>(o_b.data_ptr()), lse_b.data_ptr<float>(), source.data_ptr<int>(), T,
        (int)QH, D, W, R, nullptr, reinterpret_cast<uint8_t*>(out.data_ptr()), out_sf->data_ptr<uint8_t>());
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "attention_merge: bf16 or e4m3 output");
    attention_merge_kernel<false><<<grid, 256, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(o_a.data_ptr()), lse_a.data_ptr<float>(),
        reinterpret_cast<const __nv_bfloat16*>(o_b.data_ptr()), lse_b.data_ptr<float>(), source.data_ptr<int>(), T,
        (int)QH, D, W, R, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), nullptr, nullptr);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
