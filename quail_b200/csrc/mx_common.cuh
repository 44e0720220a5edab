// Device helpers of the MX (UE8M0 block-scaled) tcgen05 GEMMs: bulk copies of
// scale chunks, scale-factor copies into TMEM, the block-scaled MMA and its
// instruction descriptor, UE8M0 conversion, tile constants.
#pragma once

#include "common.cuh"

namespace qb {

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// tcgen05.cp 32 rows x 128 bits from shared memory to TMEM lanes 0..31,
// replicated to the four lane quarters.
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// K-major, no-swizzle descriptor of a 32-row x 16-byte chunk (8-row core
// matrices 128 bytes apart)
__device__ __forceinline__ uint64_t sf_chunk_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)(128 >> 4) << 32;  // stride byte offset
  d |= (uint64_t)1 << 46;           // sm_100 descriptor version
  return d;                          // layout type 0: no swizzle
}

__device__ __forceinline__ void umma_mx(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t sfa, uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa), "r"(sfb)
      : "memory");
}

// block-scaled instruction descriptor: e4m3 x e4m3 -> f32, UE8M0 scales
__host__ __device__ constexpr uint32_t make_idesc_mx(int M, int N, int a_sf_id, int b_sf_id) {
  return ((uint32_t)b_sf_id << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(M >> 4) << 24) | ((uint32_t)a_sf_id << 29);
}

__device__ __forceinline__ uint8_t ue8m0_of(float amax) {
  // smallest power of two >= amax / 448, as a biased exponent
  const float s = fmaxf(amax, 1e-30f) / kFp8Max;
  uint32_t bits = __float_as_uint(s);
  uint32_t e = (bits >> 23) & 0xff;
  if (bits & 0x7fffff) e += 1;
  return (uint8_t)min(max(e, 1u), 253u);
}
__device__ __forceinline__ float ue8m0_inv(uint8_t e) { return __uint_as_float((uint32_t)(254 - e) << 23); }

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }
// GELU, tanh form (Hendrycks and Gimpel, "Gaussian Error Linear Units", 2016, eq. for the
// tanh approximation): 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3)))
__device__ __forceinline__ float gelu_tanh_f(float x) {
  return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
}

__device__ __forceinline__ void st_bf16x8(__nv_bfloat16* dst, const float* v) {
  __align__(16) __nv_bfloat162 h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
}
__device__ __forceinline__ void ld_bf16x8f(const __nv_bfloat16* src, float* v) {
  uint4 u = *reinterpret_cast<const uint4*>(src);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = __bfloat1622float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

constexpr int kMxBN = 256;
constexpr int kMxStages = 4;
constexpr int kMxABytes = 128 * 128;
constexpr int kMxBBytes = kMxBN * 128;
constexpr int kMxSfaBytes = 512;
constexpr int kMxSfbBytes = 512 * (kMxBN / 128);
constexpr int kMxSmem = kMxStages * (kMxABytes + kMxBBytes) + kMxStages * (kMxSfaBytes + kMxSfbBytes) + 1024 + 256;
constexpr int kMxSfaCol = kMxBN;       // TMEM columns after the accumulator
constexpr int kMxSfbCol = kMxBN + 4;


// Bytes of shared memory that a pipeline of `stages` MX stages needs (tiles,
// scale chunks, 1024 alignment slack, barriers).
__host__ __device__ constexpr int mx_pipeline_smem(int stages) {
  return stages * (kMxABytes + kMxBBytes + kMxSfaBytes + kMxSfbBytes) + 1024 + 256;
}

// Store a warp's 32 accumulator rows (row = lane, 128 fp32 columns in acc) as
// bf16 to per-row destinations, through an 8 KB shared buffer, so that each
// store instruction writes two rows' contiguous 256 bytes instead of 32 rows'
// 16 bytes: peer stores then cross NVLink in large packets. dst_of(r) gives
// row r's first column, or nullptr to skip the row. The 16-byte chunks of a
// row are XOR-swizzled by the row index against bank conflicts.
template <class DstOf>
__device__ __forceinline__ void warp_push_rows(const float* acc, uint8_t* wbuf, int lane, DstOf dst_of) {
  uint4* mine = reinterpret_cast<uint4*>(wbuf + lane * 256);
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    __align__(16) __nv_bfloat162 h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(acc[c * 8 + 2 * i], acc[c * 8 + 2 * i + 1]);
    mine[c ^ (lane & 15)] = *reinterpret_cast<const uint4*>(h);
  }
  __syncwarp();
  const int c = lane & 15;
#pragma unroll 4
  for (int k = 0; k < 16; ++k) {
    const int r = 2 * k + (lane >> 4);
    const uint4 v = reinterpret_cast<const uint4*>(wbuf + r * 256)[c ^ (r & 15)];
    __nv_bfloat16* dst = dst_of(r);
    if (dst != nullptr) reinterpret_cast<uint4*>(dst)[c] = v;
  }
  __syncwarp();
}

}  // namespace qb
