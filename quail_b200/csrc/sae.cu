// K14: sparse-autoencoder features of residual-stream rows: per row, the
// `keep` largest of (x . W_enc^T + b_enc), clamped at zero, strongest first.
//
// The encode GEMM runs on the bf16 tcgen05 GEMM (pre-activations bf16
// [R, F]); this kernel adds the fp32 bias and selects. One CTA of 1024
// threads per row: an exact radix select over the positive values' float
// bits (4 passes of 8-bit digits with a shared-memory histogram) finds the
// keep-th largest value; the values above it, and as many equal to it as
// still fit, are gathered, bitonic-sorted in shared memory and written as
// one packed fp32 row: `keep` feature indices (exact in fp32 below 2^24), then
// their strengths (0 past the row's positive features).
//
// Reference: quail/backends/quail/executor/sae/encoder.py:58-83 (bf16 GEMM,
// fp32 bias, torch.topk, clamp at zero, packed indices + strengths).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace qb {

constexpr int kSaeThreads = 1024;
constexpr int kSaeMaxKeep = 1024;

__global__ void __launch_bounds__(kSaeThreads) sae_topk_kernel(const __nv_bfloat16* __restrict__ pre, int ld,
                                                               const float* __restrict__ bias, int F, int keep,
                                                               float* __restrict__ out) {
  __shared__ unsigned hist[256];
  __shared__ unsigned s_prefix, s_need;
  __shared__ int s_count, s_eq;
  __shared__ float sv[kSaeMaxKeep];
  __shared__ int si[kSaeMaxKeep];
  const int r = blockIdx.x, t = threadIdx.x;
  const __nv_bfloat16* row = pre + (size_t)r * ld;
  auto key_of = [&](int j) -> unsigned {
    const float v = __bfloat162float(row[j]) + bias[j];
    return v > 0.f ? __float_as_uint(v) : 0u;  // 0 = not a candidate
  };
  // count the positives; if at most `keep`, every positive is selected
  if (t == 0) {
    s_count = 0;
    s_eq = 0;
  }
  __syncthreads();
  int mine = 0;
  for (int j = t; j < F; j += kSaeThreads) mine += key_of(j) != 0u;
  atomicAdd(&s_count, mine);
  __syncthreads();
  const int positives = s_count;
  __syncthreads();  // every thread has read the count before it is reused below
  unsigned thresh = 1u, need_eq = 0x7fffffffu;  // select key >= thresh (all positives)
  if (positives > keep) {
    if (t == 0) {
      s_prefix = 0u;
      s_need = (unsigned)keep;
    }
    for (int d = 3; d >= 0; --d) {
      for (int i = t; i < 256; i += kSaeThreads) hist[i] = 0u;
      __syncthreads();
      const unsigned prefix = s_prefix;
      for (int j = t; j < F; j += kSaeThreads) {
        const unsigned k = key_of(j);
        if (k == 0u) continue;
        if (d < 3 && (k >> (8 * (d + 1))) != prefix) continue;
        atomicAdd(&hist[(k >> (8 * d)) & 255u], 1u);
      }
      __syncthreads();
      if (t == 0) {
        unsigned need = s_need, acc = 0u;
        int b = 255;
        for (; b > 0; --b) {
          if (acc + hist[b] >= need) break;
          acc += hist[b];
        }
        s_need = need - acc;              // still needed from bin b downwards: taken inside bin b
        s_prefix = (prefix << 8) | (unsigned)b;
      }
      __syncthreads();
    }
    thresh = s_prefix;   // the keep-th largest key; take every key above it and s_need equal to it
    need_eq = s_need;
  }
  if (t == 0) s_count = 0;
  __syncthreads();
  for (int j = t; j < F; j += kSaeThreads) {
    const unsigned k = key_of(j);
    if (k == 0u || k < thresh) continue;
    bool take = k > thresh || positives <= keep;
    if (!take) take = (unsigned)atomicAdd(&s_eq, 1) < need_eq;
    if (take) {
      const int slot = atomicAdd(&s_count, 1);
      if (slot < keep) {
        sv[slot] = __uint_as_float(k);
        si[slot] = j;
      }
    }
  }
  __syncthreads();
  const int n = min(s_count, keep);
  int np2 = 1;
  while (np2 < keep) np2 <<= 1;
  for (int i = n + t; i < np2; i += kSaeThreads) {
    sv[i] = -1.f;
    si[i] = 0x7fffffff;
  }
  __syncthreads();
  // bitonic sort, descending by value, ascending index on ties
  for (int size = 2; size <= np2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = t; i < np2; i += kSaeThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float a = sv[i], b = sv[j];
          const bool a_first = a > b || (a == b && si[i] < si[j]);
          if (a_first != desc) {
            sv[i] = b;
            sv[j] = a;
            const int ti = si[i];
            si[i] = si[j];
            si[j] = ti;
          }
        }
      }
      __syncthreads();
    }
  }
  float* o = out + (size_t)r * 2 * keep;
  for (int i = t; i < keep; i += kSaeThreads) {
    const bool ok = i < n;
    o[i] = ok ? (float)si[i] : 0.f;
    o[keep + i] = ok ? sv[i] : 0.f;
  }
}

// pre [R, F] bf16 (x . W_enc^T), bias [F] fp32 -> out [R, 2 * keep] fp32
void sae_topk(const torch::Tensor& pre, const torch::Tensor& bias, int64_t keep, torch::Tensor& out) {
  TORCH_CHECK(pre.scalar_type() == at::kBFloat16 && pre.dim() == 2 && pre.stride(1) == 1, "sae_topk: bf16 [R, F]");
  TORCH_CHECK(bias.scalar_type() == at::kFloat && bias.numel() == pre.size(1), "sae_topk: fp32 bias [F]");
  TORCH_CHECK(keep >= 1 && keep <= kSaeMaxKeep && pre.size(1) < (1 << 24), "sae_topk: 1 <= keep <= 1024, F < 2^24");
  const int R = pre.size(0);
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.size(0) == R && out.size(1) == 2 * keep && out.is_contiguous(),
              "sae_topk: out [R, 2 keep] fp32");
  if (R == 0) return;
  const int dev = pre.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  sae_topk_kernel<<<R, kSaeThreads, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(pre.data_ptr()),
                                              (int)pre.stride(0), bias.data_ptr<float>(), (int)pre.size(1),
                                              (int)keep, out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
