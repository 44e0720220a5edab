// Kernels around the matrix multiplies of LFM3 (d1) layers.
//
//   post_norm_add_norm  the sandwich norm of a block: h += RMSNorm(y) * w_post (in place,
//                       bf16), then x = RMSNorm(h) * w_next for the next block (bf16), one
//                       CTA per row, one read of y and h, one write of h and x.
//   kv_copy_rows        copies K and V rows between arena slots (a set-attention question's
//                       keys, written once in its pass's rows, also go to the question's own
//                       pages, so the question reads only its state and itself).
//
// Reference: quail/backends/quail/executor/models/lfm3_kernels.py (the Triton kernels of the
// same steps: post_norm_add_norm; the set-attention merge is replaced here by the row copy).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>

namespace qb {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) t += red[w];
  return t;
}

__global__ void __launch_bounds__(kNormThreads) post_norm_add_norm_kernel(
    const __nv_bfloat16* __restrict__ y, int ldy, __nv_bfloat16* __restrict__ h, int ldh,
    const __nv_bfloat16* __restrict__ wpost, const __nv_bfloat16* __restrict__ wnext, __nv_bfloat16* __restrict__ x,
    int ldx, int H, float eps) {
  __shared__ float red[kNormThreads / 32];
  const size_t row = blockIdx.x;
  const __nv_bfloat16* yr = y + row * ldy;
  __nv_bfloat16* hr = h + row * ldh;
  float ss = 0.f;
  for (int c = threadIdx.x; c < H; c += kNormThreads) {
    const float v = __bfloat162float(yr[c]);
    ss += v * v;
  }
  const float r1 = rsqrtf(block_sum(ss, red) / H + eps);
  float ss2 = 0.f;
  for (int c = threadIdx.x; c < H; c += kNormThreads) {
    const float n = __bfloat162float(__float2bfloat16(__bfloat162float(yr[c]) * r1)) * __bfloat162float(wpost[c]);
    const __nv_bfloat16 nh = __float2bfloat16(__bfloat162float(hr[c]) + __bfloat162float(__float2bfloat16(n)));
    hr[c] = nh;
    const float v = __bfloat162float(nh);
    ss2 += v * v;
  }
  if (wnext == nullptr) return;
  const float r2 = rsqrtf(block_sum(ss2, red) / H + eps);
  __nv_bfloat16* xr = x + row * ldx;
  // each thread reads back only the h values it wrote itself
  for (int c = threadIdx.x; c < H; c += kNormThreads)
    xr[c] = __float2bfloat16(__bfloat162float(__float2bfloat16(__bfloat162float(hr[c]) * r2)) *
                             __bfloat162float(wnext[c]));
}

__global__ void __launch_bounds__(128) kv_copy_rows_kernel(__nv_bfloat16* __restrict__ kc,
                                                           __nv_bfloat16* __restrict__ vc,
                                                           const int* __restrict__ src, const int* __restrict__ dst,
                                                           int row_elems, long long slots) {
  const int s = src[blockIdx.x], d = dst[blockIdx.x];
  if (s < 0 || d < 0 || s >= slots || d >= slots) return;   // host-staged indices, checked
  const uint4* ks = reinterpret_cast<const uint4*>(kc + (size_t)s * row_elems);
  const uint4* vs = reinterpret_cast<const uint4*>(vc + (size_t)s * row_elems);
  uint4* kd = reinterpret_cast<uint4*>(kc + (size_t)d * row_elems);
  uint4* vd = reinterpret_cast<uint4*>(vc + (size_t)d * row_elems);
  for (int i = threadIdx.x; i < row_elems / 8; i += blockDim.x) {
    kd[i] = ks[i];
    vd[i] = vs[i];
  }
}

}  // namespace

void post_norm_add_norm(const torch::Tensor& y, torch::Tensor& h, const torch::Tensor& wpost,
                        const c10::optional<torch::Tensor>& wnext, const c10::optional<torch::Tensor>& x, double eps) {
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && h.scalar_type() == at::kBFloat16 && y.stride(1) == 1 &&
                  h.stride(1) == 1 && y.size(0) == h.size(0) && y.size(1) == h.size(1),
              "post_norm_add_norm: bf16 y, h [T, H]");
  TORCH_CHECK(wnext.has_value() == x.has_value(), "post_norm_add_norm: the next norm's weight and output go together");
  const int T = y.size(0), H = y.size(1);
  if (T == 0) return;
  const int dev = y.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  post_norm_add_norm_kernel<<<T, kNormThreads, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), (int)y.stride(0),
      reinterpret_cast<__nv_bfloat16*>(h.data_ptr()), (int)h.stride(0),
      reinterpret_cast<const __nv_bfloat16*>(wpost.data_ptr()),
      wnext.has_value() ? reinterpret_cast<const __nv_bfloat16*>(wnext->data_ptr()) : nullptr,
      x.has_value() ? reinterpret_cast<__nv_bfloat16*>(x->data_ptr()) : nullptr, x.has_value() ? (int)x->stride(0) : 0,
      H, (float)eps);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void kv_copy_rows(torch::Tensor& k_cache, torch::Tensor& v_cache, const torch::Tensor& src, const torch::Tensor& dst) {
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.scalar_type() == at::kBFloat16,
              "kv_copy_rows: contiguous bf16 caches [pages, P, KH, D]");
  TORCH_CHECK(src.numel() == dst.numel() && src.scalar_type() == at::kInt && dst.scalar_type() == at::kInt,
              "kv_copy_rows: int32 src / dst of one length");
  const int n = src.numel();
  if (n == 0) return;
  const int row = k_cache.size(2) * k_cache.size(3);
  TORCH_CHECK(row % 8 == 0, "kv_copy_rows: KH * D a multiple of 8");
  const long long slots = (long long)k_cache.size(0) * k_cache.size(1);
  const int dev = k_cache.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  kv_copy_rows_kernel<<<n, 128, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()),
                                         reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), src.data_ptr<int>(),
                                         dst.data_ptr<int>(), row, slots);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
