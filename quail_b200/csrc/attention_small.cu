// Paged segmented attention for head_dim 64 to 512 (hybrid models' gated attention: head_dim
// 256, partial RoPE, sigmoid output gate; Gemma 4's global layers: head_dim 512).
//
// One CTA per (16 query rows, KV head): the rows are TOK = 16 / G tokens x the
// G = QH / KH query heads of the KV head (rows past TOK x G idle when G does not
// divide 16), so every K/V row read from the arena
// serves all G heads. The sequence's visible KV (up to four segments; causal in
// the own segment) streams through shared memory in 16-token blocks
// (cp.async, double-buffered, page lookups per row). Each of the four warps
// computes the whole 16 x 16 score block over all D dims (the scores are cheap)
// and its own quarter of the output dims, so no warp holds more than D/4 output
// columns in registers; softmax statistics are identical across warps. With a
// gate tensor, the output is multiplied by sigmoid(gate) before the bf16 store.
//
// Grids: prefill tiles (sequence, first of 32 tokens) x KV heads x 32/TOK
// sub-tiles, or one-token sequences (decode steps) x KV heads.
//
// Reference: the reference runs Qwen3.5's attention layers through vLLM's
// attention backends (quail/backends/quail/executor/models/qwen3_5.py:36-391).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace qb {

namespace {

constexpr int kSmBk = 16;          // KV tokens per block
constexpr int kSmSeqInts = 12;
constexpr int kSmMaxSeg = 4;

__device__ __forceinline__ void sm_cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void sm_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void sm_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void sm_ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void sm_ldsm_x4_t(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void sm_mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t sm_pack(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ float sm_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace

template <int D>
struct SmallAttnSmem {
  static constexpr int kRowBytes = D * 2 + 16;               // padded: conflict-free ldmatrix rows
  static constexpr int kBuf = kSmBk * kRowBytes;             // one K or V block
  static constexpr int kBytes = 2 * 2 * kBuf;                // K, V x two stages
};

template <int D, int G>
__global__ void __launch_bounds__(128) small_attn_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc, const __nv_bfloat16* __restrict__ vc,
    const int* __restrict__ seqs, const int* __restrict__ tiles, int tiles_are_seqs, const int* __restrict__ page_list,
    int page_tokens, int QH, int KH, float scale_log2, __nv_bfloat16* __restrict__ out, int ldo,
    const __nv_bfloat16* __restrict__ gate, int ld_gate, int gate_hstride) {
  constexpr int TOK = 16 / G, KS = D / 16, DW = D / 4, NW = DW / 8;
  using SM = SmallAttnSmem<D>;
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
  int seq, q0;
  if (tiles_are_seqs) {
    seq = tiles[blockIdx.x];
    q0 = 0;
  } else {
    seq = tiles[2 * blockIdx.x];
    q0 = tiles[2 * blockIdx.x + 1] + blockIdx.z * TOK;
  }
  const int* sd = seqs + seq * kSmSeqInts;
  const int q_start = sd[0], q_len = sd[1], nseg = sd[2];
  const bool bidir = (sd[3] & 1) != 0;   // own segment read both ways (document-isolated block)
  // bits 8..23: a sliding window over the own segment (a row at own position p reads own keys
  // p - win + 1 .. p); 0 = none. Earlier segments are read whole unless bit 24 is set: then the
  // window spans the whole sequence (its segments hold consecutive positions), and with the
  // own segment read both ways it bounds only the earlier segments (a diffusion canvas)
  const bool win_all = ((sd[3] >> 24) & 1) != 0;
  const int win = (bidir && !win_all) ? 0 : ((sd[3] >> 8) & 0xffff);
  if (q0 >= q_len) return;
  const int kvh = blockIdx.y, h0 = kvh * G;
  int seg_len[kSmMaxSeg], seg_off[kSmMaxSeg], seg_blocks[kSmMaxSeg], seg_start[kSmMaxSeg];
  int own_start = 0;
#pragma unroll
  for (int i = 0; i < kSmMaxSeg; ++i) {
    seg_len[i] = i < nseg ? sd[4 + i] : 0;
    seg_off[i] = i < nseg ? sd[8 + i] : 0;
    seg_start[i] = own_start;                        // position of the segment's first key
    if (i < nseg - 1) own_start += seg_len[i];
  }
  const int own_len = seg_len[nseg - 1];
  const int rows_tok = min(TOK, q_len - q0);
  const int first_pos = own_len - q_len + q0;       // own-segment position of the tile's first token
  // own-segment key blocks wholly below the first row's window are skipped
  const int own_skip = (win > 0 && !bidir) ? max(0, first_pos - win + 1) / kSmBk : 0;
  int total = 0;
#pragma unroll
  for (int i = 0; i < kSmMaxSeg; ++i) {
    int vis = seg_len[i];
    if (i == nseg - 1 && !bidir) vis = min(vis, first_pos + rows_tok);
    seg_blocks[i] = i < nseg ? (vis + kSmBk - 1) / kSmBk : 0;
    if (i == nseg - 1) seg_blocks[i] = max(0, seg_blocks[i] - own_skip);
    total += seg_blocks[i];
  }
  const size_t row_stride = (size_t)KH * D;
  const int pshift = __ffs(page_tokens) - 1, pmask = page_tokens - 1;

  // Q fragments of rows g and g + 8 (token r / G, head r % G)
  const int tr0 = g / G, hr0 = g % G, tr1 = (g + 8) / G, hr1 = (g + 8) % G;
  const bool ok0 = tr0 < rows_tok, ok1 = tr1 < rows_tok;
  uint32_t qa[KS][4];
  {
    const __nv_bfloat16* p0 = q + ((size_t)(q_start + q0 + (ok0 ? tr0 : 0)) * QH + h0 + hr0) * D;
    const __nv_bfloat16* p1 = q + ((size_t)(q_start + q0 + (ok1 ? tr1 : 0)) * QH + h0 + hr1) * D;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      const int c = kk * 16 + t4 * 2;
      qa[kk][0] = ok0 ? *reinterpret_cast<const uint32_t*>(p0 + c) : 0u;
      qa[kk][1] = ok1 ? *reinterpret_cast<const uint32_t*>(p1 + c) : 0u;
      qa[kk][2] = ok0 ? *reinterpret_cast<const uint32_t*>(p0 + c + 8) : 0u;
      qa[kk][3] = ok1 ? *reinterpret_cast<const uint32_t*>(p1 + c + 8) : 0u;
    }
  }
  const int lim0 = first_pos + tr0, lim1 = first_pos + tr1;   // causal limits in the own segment

  auto locate = [&](int b, int& s, int& bb) {
    s = 0;
    bb = b;
#pragma unroll
    for (int i = 0; i < kSmMaxSeg - 1; ++i)
      if (s == i && bb >= seg_blocks[i]) {
        bb -= seg_blocks[i];
        s = i + 1;
      }
    if (s == nseg - 1) bb += own_skip;
  };
  auto load_block = [&](int b, int st) {
    int s, bb;
    locate(b, s, bb);
    int slen = seg_len[0], soff = seg_off[0];
#pragma unroll
    for (int i = 1; i < kSmMaxSeg; ++i)
      if (s == i) {
        slen = seg_len[i];
        soff = seg_off[i];
      }
    const uint32_t kd = sbase + (st * 2 + 0) * SM::kBuf, vd = sbase + (st * 2 + 1) * SM::kBuf;
    for (int idx = tid; idx < kSmBk * (D / 8); idx += 128) {
      const int r = idx / (D / 8), c = idx % (D / 8);
      const int jj = bb * kSmBk + r;
      const bool valid = jj < slen;
      size_t off = 0;
      if (valid) {
        const int page = page_list[soff + (jj >> pshift)];
        off = (size_t)((page << pshift) + (jj & pmask)) * row_stride + (size_t)kvh * D + c * 8;
      }
      sm_cp_async16(kd + r * SM::kRowBytes + c * 16, kc + off, valid);
      sm_cp_async16(vd + r * SM::kRowBytes + c * 16, vc + off, valid);
    }
  };

  float oacc[NW][4];
#pragma unroll
  for (int n = 0; n < NW; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) oacc[n][i] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  if (total > 0) load_block(0, 0);
  sm_commit();
  for (int b = 0; b < total; ++b) {
    const int st = b & 1;
    if (b + 1 < total) load_block(b + 1, st ^ 1);
    sm_commit();
    sm_wait<1>();
    __syncthreads();
    int s_idx, bb;
    locate(b, s_idx, bb);
    int slen = seg_len[0], kstart = 0;
#pragma unroll
    for (int i = 1; i < kSmMaxSeg; ++i)
      if (s_idx == i) {
        slen = seg_len[i];
        kstart = seg_start[i];
      }
    const bool own = s_idx == nseg - 1 && !bidir;
    // an earlier segment under a whole-sequence window: keys at or below row position - win drop
    const bool far = win_all && win > 0 && s_idx != nseg - 1;
    const uint32_t ks = sbase + (st * 2 + 0) * SM::kBuf, vs = sbase + (st * 2 + 1) * SM::kBuf;
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < KS; kk += 2) {
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const int mrow = n * 8 + (lane & 7);
        const int mcol = kk * 16 + (lane >> 3) * 8;
        uint32_t b0, b1, b2, b3;
        sm_ldsm_x4(ks + mrow * SM::kRowBytes + mcol * 2, b0, b1, b2, b3);
        sm_mma(s[n], qa[kk], b0, b1);
        sm_mma(s[n], qa[kk + 1], b2, b3);
      }
    }
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int jj = bb * kSmBk + n * 8 + t4 * 2 + (i & 1);
        const int lim = (i >> 1) ? lim1 : lim0;
        const bool vis = jj < slen && (!own || (jj <= lim && (win == 0 || jj > lim - win))) &&
                         (!far || kstart + jj > own_start + lim - win);
        s[n][i] = vis ? s[n][i] * scale_log2 : -INFINITY;
        mx[i >> 1] = fmaxf(mx[i >> 1], s[n][i]);
      }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(m_run[r], mx[r]);
      corr[r] = (m_run[r] == -INFINITY) ? 0.f : sm_ex2(m_run[r] - mnew);
      m_run[r] = mnew;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float mr = m_run[i >> 1];
        s[n][i] = (mr == -INFINITY || s[n][i] == -INFINITY) ? 0.f : sm_ex2(s[n][i] - mr);
        rs[i >> 1] += s[n][i];
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_run[r] = l_run[r] * corr[r] + rs[r];
    }
#pragma unroll
    for (int n = 0; n < NW; ++n) {
      oacc[n][0] *= corr[0];
      oacc[n][1] *= corr[0];
      oacc[n][2] *= corr[1];
      oacc[n][3] *= corr[1];
    }
    uint32_t pa[4] = {sm_pack(s[0][0], s[0][1]), sm_pack(s[0][2], s[0][3]), sm_pack(s[1][0], s[1][1]),
                      sm_pack(s[1][2], s[1][3])};
#pragma unroll
    for (int n = 0; n < NW; n += 2) {
      const int mrow = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int mcol = warp * DW + (n + (lane >> 4)) * 8;
      uint32_t b0, b1, b2, b3;
      sm_ldsm_x4_t(vs + mrow * SM::kRowBytes + mcol * 2, b0, b1, b2, b3);
      sm_mma(oacc[n], pa, b0, b1);
      sm_mma(oacc[n + 1], pa, b2, b3);
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
  }
  sm_wait<0>();

  const float il0 = l_run[0] > 0.f ? 1.f / l_run[0] : 0.f, il1 = l_run[1] > 0.f ? 1.f / l_run[1] : 0.f;
#pragma unroll
  for (int n = 0; n < NW; ++n) {
    const int col = warp * DW + n * 8 + t4 * 2;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const bool ok = half ? ok1 : ok0;
      if (!ok) continue;
      const int tr = half ? tr1 : tr0, hr = half ? hr1 : hr0;
      const size_t row = (size_t)q_start + q0 + tr;
      const float il = half ? il1 : il0;
      float v0 = oacc[n][half * 2] * il, v1 = oacc[n][half * 2 + 1] * il;
      if (gate != nullptr && gate_hstride < 0) {
        // one gate value per (row, head)
        const float gs = 1.f / (1.f + __expf(-__bfloat162float(gate[row * ld_gate + h0 + hr])));
        v0 *= gs;
        v1 *= gs;
      } else if (gate != nullptr) {
        const __nv_bfloat16* gp = gate + row * ld_gate + (size_t)(h0 + hr) * gate_hstride + col;
        v0 *= 1.f / (1.f + __expf(-__bfloat162float(gp[0])));
        v1 *= 1.f / (1.f + __expf(-__bfloat162float(gp[1])));
      }
      *reinterpret_cast<__nv_bfloat162*>(out + row * ldo + (size_t)(h0 + hr) * D + col) =
          __floats2bfloat162_rn(v0, v1);
    }
  }
}

template <int D, int G>
static void launch_small(dim3 grid, cudaStream_t st, const torch::Tensor& q, const torch::Tensor& kc,
                         const torch::Tensor& vc, const torch::Tensor& seqs, const int* tiles, int are_seqs,
                         const torch::Tensor& pl, int P, int QH, int KH, float sl2, torch::Tensor& out,
                         const __nv_bfloat16* gate, int ld_gate, int gate_hs, int dev) {
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(small_attn_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SmallAttnSmem<D>::kBytes));
    configured[dev] = true;
  }
  small_attn_kernel<D, G><<<grid, 128, SmallAttnSmem<D>::kBytes, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(kc.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(vc.data_ptr()), seqs.data_ptr<int>(), tiles, are_seqs,
      pl.data_ptr<int>(), P, QH, KH, sl2, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), (int)out.stride(0), gate,
      ld_gate, gate_hs);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// q [T, QH, D] bf16 (normed, rotated); caches [pages, P, KH, D]; tiles [n, 2] (32-token
// prefill tiles) and dseqs [d] (one-token sequences); out bf16 [T, QH*D]. gate: optional
// bf16 tensor whose element (token t, head h, dim d) sits at t * gate.stride(0) + h * gate_hstride + d.
void small_attention(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                     const torch::Tensor& seqs, const torch::Tensor& tiles, const torch::Tensor& dseqs,
                     const torch::Tensor& page_list, double softmax_scale, torch::Tensor& out,
                     const c10::optional<torch::Tensor>& gate, int64_t gate_hstride) {
  TORCH_CHECK(q.dim() == 3 && q.is_contiguous() && q.scalar_type() == at::kBFloat16, "q: [T, QH, D] bf16");
  const int QH = q.size(1), D = q.size(2), KH = k_cache.size(2), P = k_cache.size(1);
  TORCH_CHECK(k_cache.size(3) == D && k_cache.is_contiguous() && v_cache.is_contiguous(), "caches [pages, P, KH, D]");
  TORCH_CHECK(QH % KH == 0 && (P & (P - 1)) == 0, "QH % KH, power-of-two pages");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(1) == QH * D && out.stride(1) == 1, "out bf16 [T, QH*D]");
  const int G = QH / KH;
  const int dev = q.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  const float sl2 = (float)(softmax_scale * 1.4426950408889634);
  const __nv_bfloat16* gp = gate.has_value() ? reinterpret_cast<const __nv_bfloat16*>(gate->data_ptr()) : nullptr;
  const int ldg = gate.has_value() ? (int)gate->stride(0) : 0;
  const int nt = tiles.size(0), nd = dseqs.numel();
#define QB_SMALL(DD, GG)                                                                                          \
  if (D == DD && G == GG) {                                                                                       \
    if (nt > 0)                                                                                                   \
      launch_small<DD, GG>(dim3(nt, KH, 32 / (16 / GG) > 0 ? 32 / (16 / GG) : 1), st, q, k_cache, v_cache, seqs,   \
                           tiles.data_ptr<int>(), 0, page_list, P, QH, KH, sl2, out, gp, ldg, (int)gate_hstride, dev); \
    if (nd > 0)                                                                                                   \
      launch_small<DD, GG>(dim3(nd, KH, 1), st, q, k_cache, v_cache, seqs, dseqs.data_ptr<int>(), 1, page_list, P, \
                           QH, KH, sl2, out, gp, ldg, (int)gate_hstride, dev);                                    \
    return;                                                                                                       \
  }
  QB_SMALL(64, 1)
  QB_SMALL(64, 2)
  QB_SMALL(64, 4)
  QB_SMALL(128, 1)
  QB_SMALL(128, 4)
  QB_SMALL(256, 2)
  QB_SMALL(256, 4)
  QB_SMALL(256, 6)
  QB_SMALL(256, 8)
  QB_SMALL(512, 8)
#undef QB_SMALL
  TORCH_CHECK(false, "small_attention: unsupported head_dim / group ", D, " / ", G);
}

// ------------------------------------------------------------------ q/k norm + partial RoPE + KV write
// proj bf16 [T, ldp]: per token [q_0 | gate_0 | q_1 | gate_1 | ... (or q only) | k (KH*D) | v (KH*D)].
// One warp per (token, head) over QH q heads, KH k heads, KH v heads. q and k get
// RMSNorm (weights scaled by 1 + w when `offset`), then NeoX RoPE on their first
// `rd` dims (the partner of dim i < rd/2 is i + rd/2, one lane shuffle away);
// q goes to q_out [T, QH, D], k and v to the caches at the token's KV slot.
template <int D>
__global__ void hybrid_qk_rope_kv_kernel(const __nv_bfloat16* __restrict__ proj, int ldp, int QH, int KH, int gated,
                                         const int* __restrict__ positions, const __nv_bfloat16* __restrict__ qw,
                                         const __nv_bfloat16* __restrict__ kw, int offset,
                                         const float* __restrict__ cos_sin, int rd, const int* __restrict__ slots,
                                         __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                                         __nv_bfloat16* __restrict__ q_out, int T, float eps, int sec_h, int sec_w,
                                         int vmode) {
  constexpr int E = D / 32;
  const int lane = threadIdx.x & 31;
  const int widx = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int heads = QH + 2 * KH;
  if (widx >= T * heads) return;
  const int t = widx / heads, h = widx % heads;
  const int qstride = gated ? 2 * D : D;
  const __nv_bfloat16* src;
  const __nv_bfloat16* w = nullptr;
  if (h < QH) {
    src = proj + (size_t)t * ldp + (size_t)h * qstride;
    w = qw;
  } else if (h < QH + KH) {
    src = proj + (size_t)t * ldp + (size_t)QH * qstride + (size_t)(h - QH) * D;
    w = kw;
  } else if (vmode == 2) {
    // the values are the key projection (Gemma 4's global layers)
    src = proj + (size_t)t * ldp + (size_t)QH * qstride + (size_t)(h - QH - KH) * D;
  } else {
    src = proj + (size_t)t * ldp + (size_t)QH * qstride + (size_t)KH * D + (size_t)(h - QH - KH) * D;
  }
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = __bfloat162float(src[lane * E + e]);
  if (w == nullptr && vmode != 0) {
    // vmode 1 / 2: the values are RMS-normalized per head, with no weight
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss += x[e] * x[e];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + eps);
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] *= r;
  }
  if (w != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss += x[e] * x[e];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / D + eps);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float wv = __bfloat162float(w[lane * E + e]) + (offset ? 1.f : 0.f);
      x[e] = x[e] * r * wv;
    }
    const int half = rd / 2;
    const int xorl = half / E;  // lanes between a dim and its partner
    // sec_h / sec_w > 0: interleaved multimodal RoPE, positions [T, 3] (time, height, width);
    // frequency pair p follows height when p % 3 == 1 and p < 3 sec_h, width when p % 3 == 2
    // and p < 3 sec_w, else time
    const bool mrope = sec_h > 0 || sec_w > 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[e], xorl);
      const int i = lane * E + e;
      const int pr = i < half ? i : i - half;
      int stream = 0;
      if (mrope) stream = (pr % 3 == 1 && pr < 3 * sec_h) ? 1 : ((pr % 3 == 2 && pr < 3 * sec_w) ? 2 : 0);
      const int pos = mrope ? positions[(size_t)t * 3 + stream] : positions[t];
      if (i < half) {
        const float c = cos_sin[(size_t)pos * rd + i], sn = cos_sin[(size_t)pos * rd + half + i];
        x[e] = x[e] * c - partner * sn;
      } else if (i < rd) {
        const int j = i - half;
        const float c = cos_sin[(size_t)pos * rd + j], sn = cos_sin[(size_t)pos * rd + half + j];
        x[e] = x[e] * c + partner * sn;
      }
    }
  }
  __nv_bfloat16* dst;
  if (h < QH) {
    dst = q_out + ((size_t)t * QH + h) * D;
  } else {
    const int slot = slots[t];
    if (slot < 0) return;
    const int kh = h < QH + KH ? h - QH : h - QH - KH;
    dst = (h < QH + KH ? kc : vc) + ((size_t)slot * KH + kh) * D;
  }
#pragma unroll
  for (int e = 0; e < E; ++e) dst[lane * E + e] = __float2bfloat16(x[e]);
}

static void qk_rope_kv_impl(const torch::Tensor& proj, int64_t QH, int64_t KH, bool gated,
                            const torch::Tensor& positions, const torch::Tensor& qw, const torch::Tensor& kw,
                            bool offset, const torch::Tensor& cos_sin, const torch::Tensor& slots,
                            torch::Tensor& k_cache, torch::Tensor& v_cache, torch::Tensor& q_out, double eps,
                            int64_t sec_h, int64_t sec_w, int vmode) {
  const int T = proj.size(0), D = k_cache.size(3), rd = cos_sin.size(1);
  TORCH_CHECK(proj.scalar_type() == at::kBFloat16 && proj.stride(1) == 1, "proj bf16");
  TORCH_CHECK(q_out.is_contiguous() && q_out.size(2) == D, "q_out [T, QH, D]");
  TORCH_CHECK(rd <= D && rd % 2 == 0 && ((rd / 2) % (D / 32)) == 0, "rotary dims");
  TORCH_CHECK((sec_h == 0 && sec_w == 0) ? positions.dim() == 1 : (positions.dim() == 2 && positions.size(1) == 3),
              "positions: [T], or [T, 3] (time, height, width) with multimodal RoPE sections");
  if (T == 0) return;
  const int dev = proj.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  const int warps = T * (int)(QH + 2 * KH);
#define QB_HQR(DD)                                                                                              \
  if (D == DD) {                                                                                                \
    hybrid_qk_rope_kv_kernel<DD><<<(warps + 7) / 8, 256, 0, st>>>(                                              \
        reinterpret_cast<const __nv_bfloat16*>(proj.data_ptr()), (int)proj.stride(0), (int)QH, (int)KH,        \
        gated ? 1 : 0, positions.data_ptr<int>(), reinterpret_cast<const __nv_bfloat16*>(qw.data_ptr()),       \
        reinterpret_cast<const __nv_bfloat16*>(kw.data_ptr()), offset ? 1 : 0, cos_sin.data_ptr<float>(), rd,  \
        slots.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()),                          \
        reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(q_out.data_ptr()), \
        T, (float)eps, (int)sec_h, (int)sec_w, vmode);                                                          \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                             \
    return;                                                                                                     \
  }
  QB_HQR(64)
  QB_HQR(128)
  QB_HQR(256)
  QB_HQR(512)
#undef QB_HQR
  TORCH_CHECK(false, "hybrid_qk_rope_kv: head_dim 64, 128, 256 or 512");
}

void hybrid_qk_rope_kv(const torch::Tensor& proj, int64_t QH, int64_t KH, bool gated, const torch::Tensor& positions,
                       const torch::Tensor& qw, const torch::Tensor& kw, bool offset, const torch::Tensor& cos_sin,
                       const torch::Tensor& slots, torch::Tensor& k_cache, torch::Tensor& v_cache,
                       torch::Tensor& q_out, double eps, int64_t sec_h, int64_t sec_w) {
  qk_rope_kv_impl(proj, QH, KH, gated, positions, qw, kw, offset, cos_sin, slots, k_cache, v_cache, q_out, eps,
                  sec_h, sec_w, 0);
}

// Gemma 4: q/k per-head RMSNorm (weights) + RoPE over the whole head (a table whose unrotated
// pairs hold cos 1, sin 0), values RMS-normalized without a weight; vmode 1: proj is
// [q | k | v], vmode 2: [q | k] and the values are the key projection.
void qkv_norm_rope_kv(const torch::Tensor& proj, int64_t QH, int64_t KH, const torch::Tensor& positions,
                      const torch::Tensor& qw, const torch::Tensor& kw, const torch::Tensor& cos_sin,
                      const torch::Tensor& slots, torch::Tensor& k_cache, torch::Tensor& v_cache,
                      torch::Tensor& q_out, double eps, int64_t vmode) {
  TORCH_CHECK(vmode == 1 || vmode == 2, "qkv_norm_rope_kv: vmode 1 (own values) or 2 (values = keys)");
  qk_rope_kv_impl(proj, QH, KH, false, positions, qw, kw, false, cos_sin, slots, k_cache, v_cache, q_out, eps, 0, 0,
                  (int)vmode);
}

}  // namespace qb
