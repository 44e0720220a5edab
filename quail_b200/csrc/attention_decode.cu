// K8: decode attention over the paged KV arena, for sequences with one new
// query token (AI.MAP / AI.EXTRACT decode steps, one-token continuations).
//
// One CTA per (sequence, KV head) computes all G = QH / KH query heads of that
// KV head together: the G heads are the rows of one 16-row tensor-core tile,
// so every K/V row read from the arena serves all G heads. The sequence's KV
// (up to four segments: shared prefix, document, own tokens) is cut into
// 16-token blocks; warp w takes blocks w, w + 4, ... with its own online
// softmax and a double-buffered cp.async pipeline (page lookups per token
// row), and the four partial results are merged in shared memory at the end.
// Decode attention is bound by the KV bytes read, so the math is mma.sync
// m16n8k16 (bf16 in, fp32 accumulate) on rows that are mostly the G heads.
//
// Output: bf16 [T, QH * 128], or e4m3 + UE8M0 scale atoms (one per 32
// columns) ready to be the o_proj GEMM's A operand.
//
// Reference: the reference's split-KV decode for short queries
// (quail/backends/quail/executor/attention.py:97-375, Triton kernels).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include "common.cuh"
#include "mx_common.cuh"

namespace qb {

namespace {

constexpr int kDecD = 128;
constexpr int kDecBk = 16;               // KV tokens per block
constexpr int kDecWarps = 4;
constexpr int kDecRowBytes = 272;        // 256 + 16 padding: conflict-free ldmatrix rows
constexpr int kDecBufBytes = kDecBk * kDecRowBytes;         // one K or V block
constexpr int kDecWarpBytes = 2 * 2 * kDecBufBytes;         // K, V x two stages
constexpr int kDecSmem = kDecWarps * kDecWarpBytes;         // 69,632 bytes
constexpr int kDecSeqInts = 12;
constexpr int kDecMaxSeg = 4;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace

// MODE 0: bf16 out; MODE 2: e4m3 + scale atoms. G: query heads per KV head (<= 16).
template <int MODE, int G>
__global__ void __launch_bounds__(128, 3)
    decode_attn_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
                       const __nv_bfloat16* __restrict__ vc, const int* __restrict__ seqs,
                       const int* __restrict__ dseqs, const int* __restrict__ page_list, int page_tokens, int QH,
                       int KH, float scale_log2, __nv_bfloat16* __restrict__ o, int ldo, uint8_t* __restrict__ o8,
                       uint8_t* __restrict__ osf) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int seq = dseqs[blockIdx.x];
  const int kvh = blockIdx.y;
  const int h0 = kvh * G;
  const int* sd = seqs + seq * kDecSeqInts;
  const int q_row = sd[0] + sd[1] - 1;  // the sequence's last (only) query token
  const int nseg = sd[2];
  int seg_len[kDecMaxSeg], seg_off[kDecMaxSeg], seg_blocks[kDecMaxSeg];
  int total = 0;
#pragma unroll
  for (int i = 0; i < kDecMaxSeg; ++i) {
    seg_len[i] = i < nseg ? sd[4 + i] : 0;
    seg_off[i] = i < nseg ? sd[8 + i] : 0;
    seg_blocks[i] = (seg_len[i] + kDecBk - 1) / kDecBk;
    total += seg_blocks[i];
  }
  const size_t row_stride = (size_t)KH * kDecD;
  const int pshift = __ffs(page_tokens) - 1;
  const int pmask = page_tokens - 1;

  // Q fragments (A operand, rows = heads h0 .. h0 + G - 1), unscaled bf16
  uint32_t qa[8][4];
  {
    const int r0 = g, r1 = g + 8;
    const __nv_bfloat16* q0p = q + ((size_t)q_row * QH + h0 + r0) * kDecD;
    const __nv_bfloat16* q1p = q + ((size_t)q_row * QH + h0 + r1) * kDecD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = kk * 16 + t4 * 2;
      qa[kk][0] = r0 < G ? *reinterpret_cast<const uint32_t*>(q0p + c) : 0u;
      qa[kk][1] = r1 < G ? *reinterpret_cast<const uint32_t*>(q1p + c) : 0u;
      qa[kk][2] = r0 < G ? *reinterpret_cast<const uint32_t*>(q0p + c + 8) : 0u;
      qa[kk][3] = r1 < G ? *reinterpret_cast<const uint32_t*>(q1p + c + 8) : 0u;
    }
  }

  uint8_t* wbase = smem + warp * kDecWarpBytes;
  const uint32_t wbase_s = smem_u32(wbase);
  // block b -> (segment, block within segment)
  auto locate = [&](int b, int& s, int& bb) {
    s = 0;
    bb = b;
#pragma unroll
    for (int i = 0; i < kDecMaxSeg - 1; ++i)
      if (s == i && bb >= seg_blocks[i]) {
        bb -= seg_blocks[i];
        s = i + 1;
      }
  };
  // 16 rows x 16 chunks of 16 bytes for K and V of block b into stage st
  auto load_block = [&](int b, int st) {
    int s, bb;
    locate(b, s, bb);
    int slen = seg_len[0], soff = seg_off[0];
#pragma unroll
    for (int i = 1; i < kDecMaxSeg; ++i)
      if (s == i) {
        slen = seg_len[i];
        soff = seg_off[i];
      }
    const uint32_t kdst = wbase_s + (st * 2 + 0) * kDecBufBytes;
    const uint32_t vdst = wbase_s + (st * 2 + 1) * kDecBufBytes;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int idx = it * 32 + lane, r = idx >> 4, c = idx & 15;
      const int jj = bb * kDecBk + r;
      const bool valid = jj < slen;
      size_t off = 0;
      if (valid) {
        const int page = page_list[soff + (jj >> pshift)];
        off = (size_t)((page << pshift) + (jj & pmask)) * row_stride + (size_t)kvh * kDecD + c * 8;
      }
      cp_async16(kdst + r * kDecRowBytes + c * 16, kc + off, valid);
      cp_async16(vdst + r * kDecRowBytes + c * 16, vc + off, valid);
    }
  };
  auto valid_rows = [&](int b) {
    int s, bb;
    locate(b, s, bb);
    int slen = seg_len[0];
#pragma unroll
    for (int i = 1; i < kDecMaxSeg; ++i)
      if (s == i) slen = seg_len[i];
    return min(kDecBk, slen - bb * kDecBk);
  };

  float oacc[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) oacc[n][i] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  int b = warp;
  if (b < total) load_block(b, 0);
  cp_commit();
  for (int it = 0; b < total; ++it, b += kDecWarps) {
    const int st = it & 1;
    const int nb = b + kDecWarps;
    if (nb < total) load_block(nb, st ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncwarp();
    const uint32_t ks = wbase_s + (st * 2 + 0) * kDecBufBytes;
    const uint32_t vs = wbase_s + (st * 2 + 1) * kDecBufBytes;
    // S[16 x 16] = Q K^T: two n-tiles of 8 tokens, 8 k-steps of 16 dims
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < 8; kk += 2) {
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        // matrices: tokens n*8..+7 x dims (kk*16 + 0/8/16/24 .. +7)
        const int mrow = n * 8 + (lane & 7);
        const int mcol = kk * 16 + (lane >> 3) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(ks + mrow * kDecRowBytes + mcol * 2, b0, b1, b2, b3);
        mma16816(s[n], qa[kk], b0, b1);
        mma16816(s[n], qa[kk + 1], b2, b3);
      }
    }
    // online softmax (base 2) over this block; rows g (c0, c1) and g + 8 (c2, c3)
    const int nvalid = valid_rows(b);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int col = n * 8 + t4 * 2 + (i & 1);
        s[n][i] = col < nvalid ? s[n][i] * scale_log2 : -INFINITY;
        mx[i >> 1] = fmaxf(mx[i >> 1], s[n][i]);
      }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(m_run[r], mx[r]);
      corr[r] = m_run[r] == -INFINITY ? 0.f : ex2(m_run[r] - mnew);
      m_run[r] = mnew;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float mr = m_run[i >> 1];
        s[n][i] = mr == -INFINITY ? 0.f : ex2(s[n][i] - mr);
        rs[i >> 1] += s[n][i];
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_run[r] = l_run[r] * corr[r] + rs[r];
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      oacc[n][0] *= corr[0];
      oacc[n][1] *= corr[0];
      oacc[n][2] *= corr[1];
      oacc[n][3] *= corr[1];
    }
    // O += P V: P (16 x 16 tokens) as the A operand, V rows via transposed ldmatrix
    uint32_t pa[4] = {pack_bf16(s[0][0], s[0][1]), pack_bf16(s[0][2], s[0][3]), pack_bf16(s[1][0], s[1][1]),
                      pack_bf16(s[1][2], s[1][3])};
#pragma unroll
    for (int n = 0; n < 16; n += 2) {
      // matrices: tokens 0..7 / 8..15 x dims n*8 .. +7 and (n+1)*8 .. +7
      const int mrow = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int mcol = (n + (lane >> 4)) * 8;
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vs + mrow * kDecRowBytes + mcol * 2, b0, b1, b2, b3);
      mma16816(oacc[n], pa, b0, b1);
      mma16816(oacc[n + 1], pa, b2, b3);
    }
    __syncwarp();
  }
  cp_wait<0>();
  __syncthreads();

  // merge the four warps: each writes (m, l, O) of its rows into shared memory
  float* mbuf = reinterpret_cast<float*>(smem);                 // [4][16]
  float* lbuf = mbuf + kDecWarps * 16;                          // [4][16]
  float* obuf = lbuf + kDecWarps * 16;                          // [4][16][128]
  if (t4 == 0) {
    mbuf[warp * 16 + g] = m_run[0];
    mbuf[warp * 16 + g + 8] = m_run[1];
    lbuf[warp * 16 + g] = l_run[0];
    lbuf[warp * 16 + g + 8] = l_run[1];
  }
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int col = n * 8 + t4 * 2;
    float* r0 = obuf + ((size_t)warp * 16 + g) * kDecD + col;
    float* r1 = obuf + ((size_t)warp * 16 + g + 8) * kDecD + col;
    r0[0] = oacc[n][0];
    r0[1] = oacc[n][1];
    r1[0] = oacc[n][2];
    r1[1] = oacc[n][3];
  }
  __syncthreads();
  // thread per (head row, 32-column group)
  const int tid = threadIdx.x;
  if (tid < G * 4) {
    const int r = tid >> 2, c4 = tid & 3;
    float mt = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) mt = fmaxf(mt, mbuf[w * 16 + r]);
    float wgt[kDecWarps], lt = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      const float mw = mbuf[w * 16 + r];
      wgt[w] = mw == -INFINITY ? 0.f : ex2(mw - mt);
      lt += lbuf[w * 16 + r] * wgt[w];
    }
    const float inv_l = lt > 0.f ? 1.f / lt : 0.f;
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) acc += obuf[((size_t)w * 16 + r) * kDecD + c4 * 32 + i] * wgt[w];
      v[i] = acc * inv_l;
    }
    const int head = h0 + r;
    if constexpr (MODE == 0) {
      __nv_bfloat16* dst = o + (size_t)q_row * ldo + head * kDecD + c4 * 32;
#pragma unroll
      for (int i = 0; i < 32; i += 8) st_bf16x8(dst + i, &v[i]);
    } else {
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
      const uint8_t e = ue8m0_of(amax);
      const float inv = ue8m0_inv(e);
      uint8_t* dst = o8 + (size_t)q_row * (QH * kDecD) + head * kDecD + c4 * 32;
#pragma unroll
      for (int i = 0; i < 32; i += 16) {
        __align__(16) __nv_fp8x4_e4m3 pk[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          pk[u] = __nv_fp8x4_e4m3(make_float4(v[i + 4 * u] * inv, v[i + 4 * u + 1] * inv, v[i + 4 * u + 2] * inv,
                                              v[i + 4 * u + 3] * inv));
        *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(pk);
      }
      const int kchunks = QH;  // K = QH * 128: one 128-column chunk per head
      osf[((size_t)(q_row >> 7) * kchunks + head) * 512 + (q_row & 31) * 16 + ((q_row & 127) >> 5) * 4 + c4] = e;
    }
  }
}

template <int MODE, int G>
static void launch_dec(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& vc,
                       const torch::Tensor& seqs, const torch::Tensor& dseqs, const torch::Tensor& page_list,
                       int P, int QH, int KH, float sl2, __nv_bfloat16* o, int ldo, uint8_t* o8, uint8_t* osf,
                       cudaStream_t st, int dev) {
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(decode_attn_kernel<MODE, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kDecSmem));
    configured[dev] = true;
  }
  dim3 grid(dseqs.numel(), KH);
  decode_attn_kernel<MODE, G><<<grid, 128, kDecSmem, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr()), seqs.data_ptr<int>(), dseqs.data_ptr<int>(),
      page_list.data_ptr<int>(), P, QH, KH, sl2, o, ldo, o8, osf);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// q [T, QH, 128] bf16; k/v cache [pages, P, KH, 128] bf16; seqs [S, 12];
// dseqs [n] int32: the sequences (one query token each) this kernel serves.
// out: bf16 [T, QH*128], or e4m3 [T, QH*128] with out_sf scale atoms.
void decode_attention(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                      const torch::Tensor& seqs, const torch::Tensor& dseqs, const torch::Tensor& page_list,
                      double softmax_scale, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf) {
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && q.is_contiguous() && q.scalar_type() == at::kBFloat16,
              "q: [T, QH, 128] bf16");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == 128 && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "kv cache: [pages, P, KH, 128]");
  TORCH_CHECK(seqs.dim() == 2 && seqs.size(1) == kDecSeqInts && dseqs.scalar_type() == at::kInt, "seqs / dseqs");
  const int QH = q.size(1), KH = k_cache.size(2), P = k_cache.size(1);
  TORCH_CHECK(QH % KH == 0, "QH % KH");
  TORCH_CHECK((P & (P - 1)) == 0, "page_tokens must be a power of two");
  const int G = QH / KH;
  if (dseqs.numel() == 0) return;
  const int dev = q.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  const float sl2 = (float)(softmax_scale * 1.4426950408889634);
  const bool fp8 = out.scalar_type() == at::kFloat8_e4m3fn;
  TORCH_CHECK(out.size(0) == q.size(0) && out.size(1) == QH * 128 && out.is_contiguous(), "out: [T, QH*128]");
  __nv_bfloat16* o = fp8 ? nullptr : reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  uint8_t* o8 = fp8 ? reinterpret_cast<uint8_t*>(out.data_ptr()) : nullptr;
  uint8_t* osf = nullptr;
  if (fp8) {
    TORCH_CHECK(out_sf.has_value() && out_sf->scalar_type() == at::kByte, "e4m3 output needs scale atoms");
    osf = out_sf->data_ptr<uint8_t>();
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "bf16 or e4m3 output");
  }
#define QB_DEC(GG)                                                                                          \
  if (G == GG) {                                                                                            \
    if (fp8)                                                                                                \
      launch_dec<2, GG>(q, k_cache, v_cache, seqs, dseqs, page_list, P, QH, KH, sl2, o, QH * 128, o8, osf,  \
                        st, dev);                                                                           \
    else                                                                                                    \
      launch_dec<0, GG>(q, k_cache, v_cache, seqs, dseqs, page_list, P, QH, KH, sl2, o, QH * 128, o8, osf,  \
                        st, dev);                                                                           \
    return;                                                                                                 \
  }
  QB_DEC(1)
  QB_DEC(2)
  QB_DEC(4)
  QB_DEC(8)
  QB_DEC(16)
#undef QB_DEC
  TORCH_CHECK(false, "decode_attention: q heads per KV head must be 1, 2, 4, 8 or 16");
}

}  // namespace qb
