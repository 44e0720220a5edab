// K6: packed-prompt prefill attention over the paged KV arena.
//
// Every query row is one sequence of the chunk (a question over one
// document). A sequence reads up to four KV segments in order; each segment
// is a run of pages listed in `page_list` (its own page table) and holds
// `len` tokens starting at the first page's slot 0:
//
//   seg 0: the shared instruction prefix   (one copy in the arena for every row)
//   seg 1: the document                     (shared by all questions on it)
//   ...
//   last : the sequence's own tokens        (the chunk's new rows live at its end)
//
// Earlier segments are fully visible; the last one is causal. This is the
// block-diagonal-per-row attention with the shared prefix computed once and
// reused: the prefix's KV is written once and every row reads it through its
// segment table, with no copy and no second attention call to merge.
// It covers the reference's "tree" (varlen call over packed rows + paged
// call over the parent's pages + LSE merge) and "unified" paths
// (quail/backends/quail/executor/attention.py:1395-1573) in one kernel.
//
// Tiles: one CTA = 32 query tokens of one sequence x up to 4 q heads of one
// GQA group (two warps of 16 rows per head); KV tiles of 64 rows double-buffered with cp.async; QK^T and PV on
// mma.sync m16n8k16 bf16 with fp32 accumulators and an online softmax in
// registers. Output is bf16 or e4m3 + one fp32 scale per (token, head) = the
// 1x128 A-scale layout [QH, lds] that the fp8 o_proj GEMM reads.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_sm100.h"

namespace qb {

constexpr int kMaxSeg = 4;
// per-sequence descriptor: q_start, q_len, nseg, pad, len[4], off[4]
constexpr int kSeqDescInts = 12;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint8_t ue8m0_amax(float amax) {
  const float sc = fmaxf(amax, 1e-30f) / kFp8Max;
  uint32_t bits = __float_as_uint(sc);
  uint32_t e = (bits >> 23) & 0xff;
  if (bits & 0x7fffff) e += 1;
  return (uint8_t)min(max(e, 1u), 253u);
}
__device__ __forceinline__ float ue8m0_inv_f(uint8_t e) { return __uint_as_float((uint32_t)(254 - e) << 23); }

// smem tile: 64 rows x 128 bf16 (256 B), 16-byte chunk c of row r stored at
// chunk c ^ (r & 7)
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int chunk) {
  return base + row * 256 + ((chunk ^ (row & 7)) << 4);
}

// MODE: 0 bf16 out; 1 e4m3 + fp32 scale per (token, head) [QH, ldos];
// 2 e4m3 + UE8M0 bytes per 32 values in the MX scale atom layout (K = QH*128)
//
// One CTA = 32 query tokens of one sequence x HPB q heads of one GQA group
// (HPB * 32 rows, two warps of 16 rows per head): the group's K/V tiles are
// loaded once into shared memory and read by every head of the group.
template <int MODE, int HPB>
__global__ void __launch_bounds__(HPB * 64)
    prefill_attn_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
                        const __nv_bfloat16* __restrict__ vc, const int* __restrict__ seqs,
                        const int* __restrict__ tiles, const int* __restrict__ page_list, int page_tokens,
                        int QH, int KH, float scale_log2, __nv_bfloat16* __restrict__ o, int ldo,
                        uint8_t* __restrict__ o8, float* __restrict__ os, int ldos) {
  constexpr int D = 128, TPB = 32, ROWS = HPB * TPB, BKV = 64, NT = HPB * 64;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + ROWS * 256;
  const uint32_t sV0 = sK0 + 2 * BKV * 256;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int seq = tiles[blockIdx.x * 2], q0 = tiles[blockIdx.x * 2 + 1];
  const int head0 = blockIdx.y * HPB;
  const int head = head0 + (warp >> 1);
  const int kvh = head0 / (QH / KH);
  const int* sd = seqs + seq * kSeqDescInts;
  const int q_start = sd[0], q_len = sd[1], nseg = sd[2];
  const bool bidir = (sd[3] & 1) != 0;   // own segment read both ways (document-isolated block)
  int seg_len[kMaxSeg], seg_off[kMaxSeg];
#pragma unroll
  for (int i = 0; i < kMaxSeg; ++i) {
    seg_len[i] = i < nseg ? sd[4 + i] : 0;
    seg_off[i] = i < nseg ? sd[8 + i] : 0;
  }
  const int own_len = seg_len[nseg - 1];
  const int rows_here = min(TPB, q_len - q0);
  // own-segment position of this tile's last query token
  const int max_pos = own_len - q_len + q0 + rows_here - 1;
  int seg_tiles[kMaxSeg];
#pragma unroll
  for (int i = 0; i < kMaxSeg; ++i) {
    int visible = seg_len[i];
    if (i == nseg - 1 && !bidir) visible = min(visible, max_pos + 1);
    seg_tiles[i] = i < nseg ? (visible + BKV - 1) / BKV : 0;
  }
  int total_tiles = 0;
#pragma unroll
  for (int i = 0; i < kMaxSeg; ++i) total_tiles += seg_tiles[i];

  const size_t row_stride = (size_t)KH * D;  // elements between consecutive token slots

  // ---- Q tile: smem row r = head offset (r / 32) x token (r % 32)
#pragma unroll
  for (int it = 0; it < ROWS * 16 / NT; ++it) {
    const int idx = it * NT + tid, r = idx >> 4, c = idx & 15;
    const int tok = r & (TPB - 1), hh = r / TPB;
    const bool valid = tok < rows_here;
    const __nv_bfloat16* src = q + ((size_t)(q_start + q0 + (valid ? tok : 0)) * QH + head0 + hh) * D + c * 8;
    cp_async16(swz(sQ, r, c), src, valid);
  }
  cp_async_commit();

  auto load_kv = [&](int tile, int buf) {
    int s = 0, tt = tile;
#pragma unroll
    for (int i = 0; i < kMaxSeg - 1; ++i)
      if (s == i && tt >= seg_tiles[i]) {
        tt -= seg_tiles[i];
        s = i + 1;
      }
    int slen = seg_len[0], soff = seg_off[0];
#pragma unroll
    for (int i = 1; i < kMaxSeg; ++i)
      if (s == i) {
        slen = seg_len[i];
        soff = seg_off[i];
      }
    const uint32_t kb = sK0 + buf * BKV * 256, vb = sV0 + buf * BKV * 256;
#pragma unroll
    for (int it = 0; it < BKV * 16 / NT; ++it) {
      const int idx = it * NT + tid, r = idx >> 4, c = idx & 15;
      const int j = tt * BKV + r;
      const bool valid = j < slen;
      size_t off = 0;
      if (valid) {
        const int page = page_list[soff + j / page_tokens];
        off = ((size_t)page * page_tokens + (j % page_tokens)) * row_stride + (size_t)kvh * D + c * 8;
      }
      cp_async16(swz(kb, r, c), kc + off, valid);
      cp_async16(swz(vb, r, c), vc + off, valid);
    }
  };

  float oacc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  // token offsets (within the 32-token tile) of this thread's two rows
  const int rbase = (warp & 1) * 16 + g;
  const int pos0 = own_len - q_len + q0 + rbase, pos1 = pos0 + 8;

  if (total_tiles > 0) load_kv(0, 0);
  cp_async_commit();

  uint32_t qf[8][4];
  bool q_loaded = false;

  for (int tile = 0; tile < total_tiles; ++tile) {
    const int buf = tile & 1;
    if (tile + 1 < total_tiles) load_kv(tile + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (!q_loaded) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int mi = lane >> 3, ri = lane & 7;
        ldmatrix_x4(swz(sQ, warp * 16 + (mi & 1) * 8 + ri, kk * 2 + (mi >> 1)), qf[kk][0], qf[kk][1], qf[kk][2],
                    qf[kk][3]);
      }
      q_loaded = true;
    }
    // which segment / tile is this
    int s = 0, tt = tile;
#pragma unroll
    for (int i = 0; i < kMaxSeg - 1; ++i)
      if (s == i && tt >= seg_tiles[i]) {
        tt -= seg_tiles[i];
        s = i + 1;
      }
    int slen = seg_len[0];
#pragma unroll
    for (int i = 1; i < kMaxSeg; ++i)
      if (s == i) slen = seg_len[i];
    const bool causal = (s == nseg - 1) && !bidir;

    const uint32_t kb = sK0 + buf * BKV * 256, vb = sV0 + buf * BKV * 256;
    float sacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {
        const int mi = lane >> 3, ri = lane & 7;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(swz(kb, nb * 8 + (mi >> 1) * 8 + ri, kk * 2 + (mi & 1)), b0, b1, b2, b3);
        mma_bf16(sacc[nb], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma_bf16(sacc[nb + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    // mask + online softmax
    const int j0 = tt * BKV;
    float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = j0 + nb * 8 + 2 * t4 + (c & 1);
        const int pos = (c < 2) ? pos0 : pos1;
        bool vis = j < slen;
        if (causal) vis = vis && (j <= pos);
        const float v = vis ? sacc[nb][c] * scale_log2 : -INFINITY;
        sacc[nb][c] = v;
        tmax[c >> 1] = fmaxf(tmax[c >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
      tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
      const float mnew = fmaxf(mrow[r], tmax[r]);
      corr[r] = (mnew == -INFINITY) ? 1.f : exp2f(mrow[r] - mnew);
      mrow[r] = mnew;
    }
    float tsum[2] = {0.f, 0.f};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float m = mrow[c >> 1];
        const float p = (m == -INFINITY) ? 0.f : exp2f(sacc[nb][c] - m);
        sacc[nb][c] = p;
        tsum[c >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) lrow[r] = lrow[r] * corr[r] + tsum[r];
#pragma unroll
    for (int db = 0; db < 16; ++db) {
      oacc[db][0] *= corr[0];
      oacc[db][1] *= corr[0];
      oacc[db][2] *= corr[1];
      oacc[db][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a0 = pack_bf16(sacc[2 * kk][0], sacc[2 * kk][1]);
      const uint32_t a1 = pack_bf16(sacc[2 * kk][2], sacc[2 * kk][3]);
      const uint32_t a2 = pack_bf16(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
#pragma unroll
      for (int db = 0; db < 16; db += 2) {
        const int mi = lane >> 3, ri = lane & 7;
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_t(swz(vb, kk * 16 + (mi & 1) * 8 + ri, db + (mi >> 1)), b0, b1, b2, b3);
        mma_bf16(oacc[db], a0, a1, a2, a3, b0, b1);
        mma_bf16(oacc[db + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // finalize
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  const float inv0 = lrow[0] > 0.f ? 1.f / lrow[0] : 0.f;
  const float inv1 = lrow[1] > 0.f ? 1.f / lrow[1] : 0.f;
  const int r0 = rbase, r1 = rbase + 8;
  const size_t tok0 = (size_t)q_start + q0 + r0, tok1 = tok0 + 8;
  if constexpr (MODE == 0) {
#pragma unroll
    for (int db = 0; db < 16; ++db) {
      const int col = head * D + db * 8 + 2 * t4;
      if (r0 < rows_here)
        *reinterpret_cast<uint32_t*>(o + tok0 * ldo + col) = pack_bf16(oacc[db][0] * inv0, oacc[db][1] * inv0);
      if (r1 < rows_here)
        *reinterpret_cast<uint32_t*>(o + tok1 * ldo + col) = pack_bf16(oacc[db][2] * inv1, oacc[db][3] * inv1);
    }
  } else if constexpr (MODE == 1) {
    float am0 = 0.f, am1 = 0.f;
#pragma unroll
    for (int db = 0; db < 16; ++db) {
      oacc[db][0] *= inv0;
      oacc[db][1] *= inv0;
      oacc[db][2] *= inv1;
      oacc[db][3] *= inv1;
      am0 = fmaxf(am0, fmaxf(fabsf(oacc[db][0]), fabsf(oacc[db][1])));
      am1 = fmaxf(am1, fmaxf(fabsf(oacc[db][2]), fabsf(oacc[db][3])));
    }
    am0 = fmaxf(am0, __shfl_xor_sync(0xffffffffu, am0, 1));
    am0 = fmaxf(am0, __shfl_xor_sync(0xffffffffu, am0, 2));
    am1 = fmaxf(am1, __shfl_xor_sync(0xffffffffu, am1, 1));
    am1 = fmaxf(am1, __shfl_xor_sync(0xffffffffu, am1, 2));
    const float s0 = fmaxf(am0, 1e-12f) / kFp8Max, s1 = fmaxf(am1, 1e-12f) / kFp8Max;
    const float i0 = 1.f / s0, i1 = 1.f / s1;
#pragma unroll
    for (int db = 0; db < 16; ++db) {
      const int col = head * D + db * 8 + 2 * t4;
      if (r0 < rows_here) {
        __nv_fp8x2_e4m3 v(make_float2(oacc[db][0] * i0, oacc[db][1] * i0));
        *reinterpret_cast<__nv_fp8x2_e4m3*>(o8 + tok0 * ldo + col) = v;
      }
      if (r1 < rows_here) {
        __nv_fp8x2_e4m3 v(make_float2(oacc[db][2] * i1, oacc[db][3] * i1));
        *reinterpret_cast<__nv_fp8x2_e4m3*>(o8 + tok1 * ldo + col) = v;
      }
    }
    if (t4 == 0) {
      if (r0 < rows_here) os[(size_t)head * ldos + tok0] = s0;
      if (r1 < rows_here) os[(size_t)head * ldos + tok1] = s1;
    }
  } else {
    // four 32-wide groups per head: group j = d-blocks 4j..4j+3, spread over the quad
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float am0 = 0.f, am1 = 0.f;
#pragma unroll
      for (int db = 4 * j; db < 4 * j + 4; ++db) {
        oacc[db][0] *= inv0;
        oacc[db][1] *= inv0;
        oacc[db][2] *= inv1;
        oacc[db][3] *= inv1;
        am0 = fmaxf(am0, fmaxf(fabsf(oacc[db][0]), fabsf(oacc[db][1])));
        am1 = fmaxf(am1, fmaxf(fabsf(oacc[db][2]), fabsf(oacc[db][3])));
      }
      am0 = fmaxf(am0, __shfl_xor_sync(0xffffffffu, am0, 1));
      am0 = fmaxf(am0, __shfl_xor_sync(0xffffffffu, am0, 2));
      am1 = fmaxf(am1, __shfl_xor_sync(0xffffffffu, am1, 1));
      am1 = fmaxf(am1, __shfl_xor_sync(0xffffffffu, am1, 2));
      const uint8_t e0 = ue8m0_amax(am0), e1 = ue8m0_amax(am1);
      w0 |= (uint32_t)e0 << (8 * j);
      w1 |= (uint32_t)e1 << (8 * j);
      const float i0 = ue8m0_inv_f(e0), i1 = ue8m0_inv_f(e1);
#pragma unroll
      for (int db = 4 * j; db < 4 * j + 4; ++db) {
        const int col = head * D + db * 8 + 2 * t4;
        if (r0 < rows_here) {
          __nv_fp8x2_e4m3 v(make_float2(oacc[db][0] * i0, oacc[db][1] * i0));
          *reinterpret_cast<__nv_fp8x2_e4m3*>(o8 + tok0 * ldo + col) = v;
        }
        if (r1 < rows_here) {
          __nv_fp8x2_e4m3 v(make_float2(oacc[db][2] * i1, oacc[db][3] * i1));
          *reinterpret_cast<__nv_fp8x2_e4m3*>(o8 + tok1 * ldo + col) = v;
        }
      }
    }
    if (t4 == 0) {
      // K stage = head (head_dim 128): the 4 bytes of one atom word
      uint8_t* sfb = reinterpret_cast<uint8_t*>(os);
      auto word = [&](size_t tok) {
        return reinterpret_cast<uint32_t*>(sfb + ((tok >> 7) * QH + head) * 512 + (tok & 31) * 16 +
                                           ((tok & 127) >> 5) * 4);
      };
      if (r0 < rows_here) *word(tok0) = w0;
      if (r1 < rows_here) *word(tok1) = w1;
    }
  }
}

template <int MODE, int HPB>
static void launch_attn(dim3 grid, cudaStream_t st, const __nv_bfloat16* qp, const __nv_bfloat16* kp,
                        const __nv_bfloat16* vp, const int* seqs, const int* tiles, const int* pl, int P, int QH,
                        int KH, float sl2, __nv_bfloat16* o, int ldo, uint8_t* o8, float* os, int ldos) {
  constexpr int smem = HPB * 32 * 256 + 2 * 2 * 64 * 256;
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(prefill_attn_kernel<MODE, HPB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        smem));
    configured = true;
  }
  prefill_attn_kernel<MODE, HPB><<<grid, HPB * 64, smem, st>>>(qp, kp, vp, seqs, tiles, pl, P, QH, KH, sl2, o, ldo, o8,
                                                               os, ldos);
}

template <int MODE>
static void launch_attn_hpb(int hpb, int n_tiles, int QH, cudaStream_t st, const __nv_bfloat16* qp,
                            const __nv_bfloat16* kp, const __nv_bfloat16* vp, const int* seqs, const int* tiles,
                            const int* pl, int P, int KH, float sl2, __nv_bfloat16* o, int ldo, uint8_t* o8,
                            float* os, int ldos) {
  dim3 grid(n_tiles, QH / hpb);
  if (hpb == 4)
    launch_attn<MODE, 4>(grid, st, qp, kp, vp, seqs, tiles, pl, P, QH, KH, sl2, o, ldo, o8, os, ldos);
  else if (hpb == 2)
    launch_attn<MODE, 2>(grid, st, qp, kp, vp, seqs, tiles, pl, P, QH, KH, sl2, o, ldo, o8, os, ldos);
  else
    launch_attn<MODE, 1>(grid, st, qp, kp, vp, seqs, tiles, pl, P, QH, KH, sl2, o, ldo, o8, os, ldos);
}

// q: [T, QH, 128] bf16; caches: [pages, P, KH, 128] bf16; seqs: [S, 12] int32;
// tiles: [n_tiles, 2] int32 (sequence, first query token; 32-token tiles);
// page_list: int32.
void prefill_attention(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                       const torch::Tensor& seqs, const torch::Tensor& tiles, const torch::Tensor& page_list,
                       double softmax_scale, torch::Tensor& out, const c10::optional<torch::Tensor>& out_scale) {
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && q.is_contiguous(), "q: [T, QH, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == 128 && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "caches: [pages, P, KH, 128]");
  TORCH_CHECK(seqs.size(1) == kSeqDescInts && seqs.scalar_type() == at::kInt, "seqs: [S, 12] int32");
  const int QH = q.size(1), KH = k_cache.size(2), P = k_cache.size(1);
  TORCH_CHECK(QH % KH == 0, "QH must be a multiple of KH");
  const int group = QH / KH;
  // heads per CTA (QB_ATTN_HPB caps it): 4 shares each K/V tile across a whole
  // GQA group of 4 q heads; measured fastest on Qwen3-4B (88.3 vs 90.3 ms/step at 2)
  static const int max_hpb = [] {
    const char* e = getenv("QB_ATTN_HPB");
    return e ? atoi(e) : 4;
  }();
  int hpb = group % 4 == 0 ? 4 : (group % 2 == 0 ? 2 : 1);
  hpb = std::min(hpb, std::max(max_hpb, 1));
  const int n_tiles = tiles.size(0);
  if (n_tiles == 0) return;
  c10::cuda::CUDAGuard guard(q.get_device());
  cudaStream_t st = at::cuda::getCurrentCUDAStream(q.get_device());
  const float sl2 = (float)(softmax_scale * 1.4426950408889634);
  auto qp = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  auto kp = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  auto vp = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  const int* sq = seqs.data_ptr<int>();
  const int* tl = tiles.data_ptr<int>();
  const int* pl = page_list.data_ptr<int>();
  if (out.scalar_type() == at::kFloat8_e4m3fn && out_scale.has_value() && out_scale->scalar_type() == at::kByte) {
    TORCH_CHECK(out_scale->numel() >= (q.size(0) + 127) / 128 * QH * 512, "MX attention output scale bytes");
    launch_attn_hpb<2>(hpb, n_tiles, QH, st, qp, kp, vp, sq, tl, pl, P, KH, sl2, nullptr, out.stride(0),
                       reinterpret_cast<uint8_t*>(out.data_ptr()), reinterpret_cast<float*>(out_scale->data_ptr()),
                       0);
  } else if (out.scalar_type() == at::kFloat8_e4m3fn) {
    TORCH_CHECK(out_scale.has_value() && out_scale->size(0) == QH, "fp8 attention output needs [QH, >=T] scales");
    launch_attn_hpb<1>(hpb, n_tiles, QH, st, qp, kp, vp, sq, tl, pl, P, KH, sl2, nullptr, out.stride(0),
                       reinterpret_cast<uint8_t*>(out.data_ptr()), out_scale->data_ptr<float>(),
                       out_scale->stride(0));
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "attention output bf16 or e4m3");
    launch_attn_hpb<0>(hpb, n_tiles, QH, st, qp, kp, vp, sq, tl, pl, P, KH, sl2,
                       reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), nullptr, nullptr, 0);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
