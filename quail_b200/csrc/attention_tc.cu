// K6 (tcgen05): packed-prompt prefill attention on the 5th-generation tensor
// cores, over the same segmented paged KV as csrc/attention.cu.
//
// One CTA = 128 query rows = 32 tokens of one sequence x 4 q heads of one
// GQA group (row r: head r / 32, token r % 32; TMEM lane r). Per 64-row KV
// tile j of the sequence's segments:
//
//   MMA thread   S = Q K_j^T          tcgen05.mma kind::f16, M 128, N 64, K 128 -> TMEM (64 cols)
//   128 threads  row softmax of S     tcgen05.ld, mask, online max with lazy rescaling
//                                     (O and l rescaled only when the row max grows by
//                                     more than 2^8), P = exp2(S - m) -> bf16 -> smem
//   MMA thread   O += P V_j           tcgen05.mma, M 128, N 128, K 64, V MN-major -> TMEM
//
// Q, K, V and P sit in shared memory in the 128-byte-swizzled K-major (V:
// MN-major) layouts the UMMA descriptors name; the 128 threads fill them with
// cp.async (K, V rows come through the page table). K is double-buffered
// (tile j+1 loads during tile j); two CTAs share an SM (96 KB smem and 256
// TMEM columns each), so one CTA's softmax overlaps the other's MMAs. The
// epilogue reads O from TMEM, divides by l and writes bf16 or e4m3 with one
// UE8M0 scale per 32 values (the o_proj GEMM's A operand). Every wait is
// bounded; a timeout records an error code and the CTA exits.
//
// Replaces the reference's FA4 CuTe-DSL varlen/paged calls
// (quail/backends/quail/executor/attention.py:1280-1306, 1395-1573).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_sm100.h"

namespace qb {

namespace {

constexpr int kTcRows = 128, kTcTok = 32, kTcHeads = 4, kTcBkv = 64, kTcD = 128;
constexpr int kMaxSegTc = 4;
constexpr int kSeqInts = 12;
constexpr int kQBytes = kTcRows * 256;          // 2 atoms x 128 rows x 128 B
constexpr int kKBytes = kTcBkv * 256;           // 2 atoms x 64 rows x 128 B
constexpr int kVBytes = kTcBkv * 256;
constexpr int kPBytes = kTcRows * 128;          // 1 atom x 128 rows x 128 B
constexpr int kTcSmem = kQBytes + 2 * kKBytes + kVBytes + kPBytes + 1024 + 256;
constexpr int kTmemCols = 256;                  // S: cols [0, 64), O: cols [128, 256)

__device__ __forceinline__ void cp_async16_tc(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// byte offset of 16-byte chunk c (0..15 over 128 elements) of row r in a
// K-major SW128 tile of `rows` rows split in two 64-element atoms
__device__ __forceinline__ uint32_t sw_off(int rows, int r, int c) {
  return (uint32_t)((c >> 3) * rows * 128 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// MN-major SW128 descriptor (V as the B operand of P V: d contiguous):
// 64-element MN atoms `lbo` bytes apart, 8-row K groups 1024 bytes apart
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int b_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_major << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

#define QB_TMEM_ST32(taddr, r)                                                                  \
  asm volatile(                                                                                 \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "                                           \
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"                                \
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),         \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),   \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),         \
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),       \
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),       \
      "r"(r[29]), "r"(r[30]), "r"(r[31])                                                        \
      : "memory")

// 2^x with the hardware approximation (MUFU.EX2), flushing subnormals; 2^-inf = 0
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint8_t ue8m0_tc(float amax) {
  const float sc = fmaxf(amax, 1e-30f) / kFp8Max;
  uint32_t bits = __float_as_uint(sc);
  uint32_t e = (bits >> 23) & 0xff;
  if (bits & 0x7fffff) e += 1;
  return (uint8_t)min(max(e, 1u), 253u);
}

}  // namespace

// MODE: 0 bf16 out [T, QH*128]; 2 e4m3 + UE8M0 scale atoms (K = QH*128)
template <int MODE>
__global__ void __launch_bounds__(160, 2)
    prefill_attn_tc_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
                           const __nv_bfloat16* __restrict__ vc, const int* __restrict__ seqs,
                           const int* __restrict__ tiles, const int* __restrict__ page_list, int page_tokens,
                           int QH, int KH, float scale_log2, __nv_bfloat16* __restrict__ o, int ldo,
                           uint8_t* __restrict__ o8, uint8_t* __restrict__ osf, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + kQBytes;                 // two buffers
  const uint32_t sV = sK + 2 * kKBytes;
  const uint32_t sP = sV + kVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kQBytes + 2 * kKBytes + kVBytes + kPBytes);
  uint64_t* k_ready = bars + 0;    // count 128: K_j landed
  uint64_t* s_full = bars + 1;     // commit: S_j in TMEM
  uint64_t* pv_ready = bars + 2;   // count 128: P_j written, V_j landed, O rescaled
  uint64_t* o_done = bars + 3;     // commit: P_j V_j accumulated into O
  uint64_t* mma_idle = bars + 4;   // commit: every MMA this CTA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int seq = tiles[blockIdx.x * 2], q0 = tiles[blockIdx.x * 2 + 1];
  const int head0 = blockIdx.y * kTcHeads;
  const int kvh = head0 / (QH / KH);
  const int* sd = seqs + seq * kSeqInts;
  const int q_start = sd[0], q_len = sd[1], nseg = sd[2];
  const bool bidir = (sd[3] & 1) != 0;   // own segment read both ways (document-isolated block)
  int seg_len[kMaxSegTc], seg_off[kMaxSegTc], seg_tiles[kMaxSegTc];
#pragma unroll
  for (int i = 0; i < kMaxSegTc; ++i) {
    seg_len[i] = i < nseg ? sd[4 + i] : 0;
    seg_off[i] = i < nseg ? sd[8 + i] : 0;
  }
  const int own_len = seg_len[nseg - 1];
  const int rows_here = min(kTcTok, q_len - q0);
  const int max_pos = own_len - q_len + q0 + rows_here - 1;
  int total = 0;
#pragma unroll
  for (int i = 0; i < kMaxSegTc; ++i) {
    int visible = seg_len[i];
    if (i == nseg - 1 && !bidir) visible = min(visible, max_pos + 1);
    seg_tiles[i] = i < nseg ? (visible + kTcBkv - 1) / kTcBkv : 0;
    total += seg_tiles[i];
  }
  const size_t row_stride = (size_t)KH * kTcD;
  const int pshift = __ffs(page_tokens) - 1;  // page_tokens is a power of two
  const int pmask = page_tokens - 1;

  if (tid == 0) {
    mbar_init(k_ready, 128);
    mbar_init(s_full, 1);
    mbar_init(pv_ready, 128);
    mbar_init(o_done, 1);
    mbar_init(mma_idle, 1);
    fence_barrier_init();
  }
  if (warp == 4) tmem_alloc<kTmemCols>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tO = tmem + 128;

  // which segment / tile-in-segment is tile j
  auto locate = [&](int j, int& s, int& tt) {
    s = 0;
    tt = j;
#pragma unroll
    for (int i = 0; i < kMaxSegTc - 1; ++i)
      if (s == i && tt >= seg_tiles[i]) {
        tt -= seg_tiles[i];
        s = i + 1;
      }
  };
  // the 128 softmax threads load 64 rows x 16 chunks of K or V for tile j
  auto load_rows = [&](int j, uint32_t dst, const __nv_bfloat16* base) {
    int s, tt;
    locate(j, s, tt);
    int slen = seg_len[0], soff = seg_off[0];
#pragma unroll
    for (int i = 1; i < kMaxSegTc; ++i)
      if (s == i) {
        slen = seg_len[i];
        soff = seg_off[i];
      }
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int idx = it * 128 + tid, r = idx >> 4, c = idx & 15;
      const int jj = tt * kTcBkv + r;
      const bool valid = jj < slen;
      size_t off = 0;
      if (valid) {
        const int page = page_list[soff + (jj >> pshift)];
        off = (size_t)((page << pshift) + (jj & pmask)) * row_stride + (size_t)kvh * kTcD + c * 8;
      }
      cp_async16_tc(dst + sw_off(kTcBkv, r, c), base + off, valid);
    }
  };

  if (warp < 4) {
    // ------------------------------------------------------------ softmax / load threads
    const int row = tid;  // TMEM lane, smem row
    const int tok = row & 31;
    const int pos = own_len - q_len + q0 + tok;  // own-segment position of this row's token
    // Q tile: row r = head offset (r / 32) x token (r % 32)
#pragma unroll
    for (int it = 0; it < 16; ++it) {
      const int idx = it * 128 + tid, r = idx >> 4, c = idx & 15;
      const int t = r & 31, hh = r >> 5;
      const bool valid = t < rows_here;
      const __nv_bfloat16* src = q + ((size_t)(q_start + q0 + (valid ? t : 0)) * QH + head0 + hh) * kTcD + c * 8;
      cp_async16_tc(sQ + sw_off(kTcRows, r, c), src, valid);
    }
    // groups in flight are kept in issue order: [Q + K_0], [V_0], then per tile
    // j: [K_{j+1}] issued at its start and [V_{j+1}] issued after P_j V_j
    if (total > 0) load_rows(0, sK, kc);
    cp_commit();
    if (total > 0) load_rows(0, sV, vc);
    cp_commit();
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    fence_proxy_async_smem();
    mbar_arrive(k_ready);

    const uint32_t lane_base = (uint32_t)((warp * 32) << 16);
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < total && ok; ++j) {
      const uint32_t ph = (uint32_t)(j & 1);
      const bool more = j + 1 < total;
      if (more) {
        load_rows(j + 1, sK + ((j + 1) & 1) * kKBytes, kc);
        cp_commit();
      }
      int s, tt;
      locate(j, s, tt);
      int slen = seg_len[0];
#pragma unroll
      for (int i = 1; i < kMaxSegTc; ++i)
        if (s == i) slen = seg_len[i];
      const bool causal = (s == nseg - 1) && !bidir;
      if (!mbar_wait(s_full, ph, err, kErrTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // visible columns of this tile for this row: [0, lim)
      const int j0 = tt * kTcBkv;
      int lim = slen - j0;
      if (causal) lim = min(lim, pos - j0 + 1);
      if (tok >= rows_here) lim = 0;
      // pass 1: the tile's row max (scores in the log2 domain)
      float tmax = -INFINITY;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sv[32];
        QB_TMEM_LD32(tS + lane_base + h * 32, sv);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (h * 32 + i < lim) tmax = fmaxf(tmax, __uint_as_float(sv[i]));
      }
      tmax *= scale_log2;
      // lazy rescaling: move the reference max only when it grows by more than 2^8
      float corr = 1.f;
      if (tmax > m_ref + 8.f) {
        corr = (m_ref == -INFINITY) ? 0.f : ex2_approx(m_ref - tmax);
        m_ref = tmax;
      }
      const bool need = corr != 1.f && j > 0;
      if (__any_sync(0xffffffffu, need)) {
        // O (accumulated by the previous tiles, complete after o_done) scaled in TMEM
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          QB_TMEM_LD32(tO + lane_base + c * 32, ov);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * corr);
          QB_TMEM_ST32(tO + lane_base + c * 32, ov);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      }
      l *= corr;
      // pass 2: P = exp2(s * scale - m) in bf16 into row `row` of the P tile
      const float mref = (m_ref == -INFINITY) ? 0.f : m_ref;
      float psum = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t sv[32];
        QB_TMEM_LD32(tS + lane_base + h * 32, sv);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int e0 = c * 8 + 2 * i;
            const float p0 = (h * 32 + e0 < lim) ? ex2_approx(fmaf(__uint_as_float(sv[e0]), scale_log2, -mref)) : 0.f;
            const float p1 = (h * 32 + e0 + 1 < lim) ? ex2_approx(fmaf(__uint_as_float(sv[e0 + 1]), scale_log2, -mref))
                                                      : 0.f;
            const __nv_bfloat162 hh = __floats2bfloat162_rn(p0, p1);
            const float2 back = __bfloat1622float2(hh);
            psum += back.x + back.y;
            w[i] = *reinterpret_cast<const uint32_t*>(&hh);
          }
          const int chunk = h * 4 + c;
          const uint32_t dst = sP + row * 128 + ((chunk ^ (row & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                       "r"(w[3])
                       : "memory");
        }
      }
      l += psum;
      // V_j must have landed before P_j V_j: everything but K_{j+1}
      if (more)
        asm volatile("cp.async.wait_group 1;" ::: "memory");
      else
        cp_wait_all();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(pv_ready);
      if (more) {
        // K_{j+1} (issued at the top of this tile) lets S_{j+1} start right after P_j V_j
        cp_wait_all();
        fence_proxy_async_smem();
        mbar_arrive(k_ready);
      }
      if (!mbar_wait(o_done, ph, err, kErrTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (more) {
        // V and P buffers are free again: fetch V_{j+1} while S_{j+1} is computed
        load_rows(j + 1, sV, vc);
        cp_commit();
      }
    }
    cp_wait_all();
    if (ok) {
      // ---- epilogue: O / l from TMEM
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int head = head0 + warp;
      const size_t t_out = (size_t)q_start + q0 + tok;
      const bool store = tok < rows_here;
      uint32_t word = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t ov[32];
        QB_TMEM_LD32(tO + lane_base + c * 32, ov);
        tmem_ld_wait();
        float v[32];
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = __uint_as_float(ov[i]) * inv;
          amax = fmaxf(amax, fabsf(v[i]));
        }
        if (store) {
          if constexpr (MODE == 0) {
            __nv_bfloat16* dst = o + t_out * ldo + head * kTcD + c * 32;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              __align__(16) __nv_bfloat162 h[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[i + 2 * k], v[i + 2 * k + 1]);
              *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(h);
            }
          } else {
            const uint8_t e = ue8m0_tc(amax);
            const float sc = __uint_as_float((uint32_t)(254 - e) << 23);
            word |= (uint32_t)e << (8 * c);
            uint8_t* dst = o8 + t_out * ldo + head * kTcD + c * 32;
#pragma unroll
            for (int i = 0; i < 32; i += 16) {
              __align__(16) __nv_fp8x4_e4m3 pk[4];
#pragma unroll
              for (int k = 0; k < 4; ++k)
                pk[k] = __nv_fp8x4_e4m3(make_float4(v[i + 4 * k] * sc, v[i + 4 * k + 1] * sc, v[i + 4 * k + 2] * sc,
                                                    v[i + 4 * k + 3] * sc));
              *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(pk);
            }
          }
        }
      }
      if constexpr (MODE == 2) {
        if (store)
          *reinterpret_cast<uint32_t*>(osf + ((t_out >> 7) * QH + head) * 512 + (t_out & 31) * 16 +
                                       ((t_out & 127) >> 5) * 4) = word;
      }
    }
  } else {
    // ------------------------------------------------------------ MMA issuer (warp 4)
    if (elect_one()) {
      constexpr uint32_t IS = idesc_bf16(128, kTcBkv, 0);
      constexpr uint32_t IO = idesc_bf16(128, kTcD, 1);
      bool ok = true;
      for (int j = 0; j < total && ok; ++j) {
        const uint32_t ph = (uint32_t)(j & 1);
        if (!mbar_wait(k_ready, ph, err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t kb = sK + (j & 1) * kKBytes;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t a = sQ + (ks >> 2) * (kTcRows * 128) + (ks & 3) * 32;
          const uint32_t b = kb + (ks >> 2) * (kTcBkv * 128) + (ks & 3) * 32;
          umma_f16(tS, sw128_kmajor_desc(a), sw128_kmajor_desc(b), IS, ks > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        if (!mbar_wait(pv_ready, ph, err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t a = sP + ks * 32;
          const uint32_t b = sV + ks * 16 * 128;
          umma_f16(tO, sw128_kmajor_desc(a), sw128_mnmajor_desc(b, kTcBkv * 128), IO,
                   (j > 0 || ks > 0) ? 1u : 0u);
        }
        tc_commit(o_done);
      }
      tc_commit(mma_idle);
      mbar_wait(mma_idle, 0, err, kErrTimeoutMma);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc<kTmemCols>(tmem);
  }
}

template <int MODE>
static void launch_tc(dim3 grid, cudaStream_t st, const __nv_bfloat16* qp, const __nv_bfloat16* kp,
                      const __nv_bfloat16* vp, const int* seqs, const int* tiles, const int* pl, int P, int QH,
                      int KH, float sl2, __nv_bfloat16* o, int ldo, uint8_t* o8, uint8_t* osf, int* err) {
  static bool configured = false;
  if (!configured) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(prefill_attn_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kTcSmem));
    configured = true;
  }
  prefill_attn_tc_kernel<MODE><<<grid, 160, kTcSmem, st>>>(qp, kp, vp, seqs, tiles, pl, P, QH, KH, sl2, o, ldo, o8,
                                                           osf, err);
}

// Same arguments as prefill_attention (32-token tiles); needs QH / KH a multiple of 4.
void prefill_attention_tc(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                          const torch::Tensor& seqs, const torch::Tensor& tiles, const torch::Tensor& page_list,
                          double softmax_scale, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf) {
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && q.is_contiguous(), "q: [T, QH, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == 128 && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "caches: [pages, P, KH, 128]");
  TORCH_CHECK(seqs.size(1) == kSeqInts && seqs.scalar_type() == at::kInt, "seqs: [S, 12] int32");
  const int QH = q.size(1), KH = k_cache.size(2), P = k_cache.size(1);
  TORCH_CHECK(QH % KH == 0 && (QH / KH) % kTcHeads == 0, "tcgen05 attention packs 4 q heads of one KV head");
  const int n_tiles = tiles.size(0);
  if (n_tiles == 0) return;
  const int dev = q.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  dim3 grid(n_tiles, QH / kTcHeads);
  const float sl2 = (float)(softmax_scale * 1.4426950408889634);
  auto qp = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  auto kp = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  auto vp = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  int* err = device_error_word(dev);
  if (out.scalar_type() == at::kFloat8_e4m3fn) {
    TORCH_CHECK(out_sf.has_value() && out_sf->scalar_type() == at::kByte &&
                    out_sf->numel() >= (q.size(0) + 127) / 128 * QH * 512,
                "e4m3 output needs its MX scale bytes");
    launch_tc<2>(grid, st, qp, kp, vp, seqs.data_ptr<int>(), tiles.data_ptr<int>(), page_list.data_ptr<int>(), P,
                 QH, KH, sl2, nullptr, out.stride(0), reinterpret_cast<uint8_t*>(out.data_ptr()),
                 out_sf->data_ptr<uint8_t>(), err);
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "bf16 or e4m3 output");
    launch_tc<0>(grid, st, qp, kp, vp, seqs.data_ptr<int>(), tiles.data_ptr<int>(), page_list.data_ptr<int>(), P,
                 QH, KH, sl2, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), out.stride(0), nullptr, nullptr,
                 err);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
