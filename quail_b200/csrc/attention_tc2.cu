// K6 (persistent tcgen05): packed-prompt prefill attention over the paged KV
// arena, one CTA per SM walking a list of work items.
//
// Work item = (sequence, 64-token query block, GQA group of 4 q heads). Its
// 64 tokens x 4 heads form two 128-row query tiles, A (tokens 0..31 of the
// block) and B (32..63); row r of a tile is token r / 4, head r % 4 (the
// order a 3-D TMA box {64 dims, 4 heads, 32 tokens} lands in). Both tiles
// read the same K/V tiles (the sequence's segments, 64 keys each, in
// order), so every K/V tile is loaded once for 256 query rows.
//
// Warp roles (320 threads):
//   warp 0      loader: TMA loads of Q (per item) and of K/V tiles into a
//               3-stage ring; the page of each 64-key tile comes from the
//               page list (a 64-key tile never crosses a page: pages hold a
//               multiple of 64 tokens), one lane per tile, shuffled to lane 0
//   warp 1      MMA issuer (one thread): S_t = Q_t K_j^T into TMEM, then
//               O_t += P_t V_j, ping-ponging between the tiles so the tensor
//               core computes one tile's products while the other tile's
//               softmax runs
//   warps 2-5   softmax + epilogue of tile A, one thread per row (TMEM lane)
//   warps 6-9   the same for tile B
//
// TMEM: S_A cols [0, 64), S_B [64, 128), O_A [128, 256), O_B [256, 384).
// Softmax is online in the log2 domain with lazy rescaling (O and l are
// rescaled only when a row's max grows by more than 2^8). The epilogue
// divides O by l and writes bf16, or e4m3 with one UE8M0 scale per 32
// values in the o_proj GEMM's A-scale atom layout.
//
// Masking: segments other than the sequence's own are read in full; the
// own segment causally (a key at own position p is visible to a query at
// own position >= p). Keys past a segment's end inside a loaded tile are
// other tokens' rows or zeros of the (zero-initialized) arena: finite, and
// masked to probability 0.
//
// Every wait is bounded (common.cuh); on expiry the role records an error
// code, stops, and the kernel drains its own async copies and MMAs before
// releasing TMEM.
//
// Replaces the reference's FA4 CuTe-DSL varlen / paged calls
// (quail/backends/quail/executor/attention.py:1280-1306).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_sm100.h"

namespace qb {

namespace {

constexpr int kRows = 128, kBkv = 64, kD = 128, kStages = 3;
constexpr int kMaxSeg = 4, kSeqInts = 12;
constexpr int kQBytes = kRows * 256;       // one tile: two 64-dim SW128 atoms of 128 rows
constexpr int kKVBytes = kBkv * 256;       // two atoms of 64 rows
constexpr int kPBytes = kRows * 128;       // 128 rows x 64 bf16
constexpr int kBarBytes = 256;
constexpr int kSmem = 2 * kQBytes + 2 * kStages * kKVBytes + 2 * kPBytes + kBarBytes + 1024;
constexpr int kThreads = 320;

__device__ __forceinline__ uint64_t mn_desc(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint8_t ue8m0_att(float amax) {
  const float sc = fmaxf(amax, 1e-30f) / kFp8Max;
  uint32_t bits = __float_as_uint(sc);
  uint32_t e = (bits >> 23) & 0xff;
  if (bits & 0x7fffff) e += 1;
  return (uint8_t)min(max(e, 1u), 253u);
}

#define QB_TMEM_ST32_A(taddr, r)                                                                \
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

// The geometry of one work item, computed alike by every role.
struct Item {
  int q_start, q_len, nseg, own_len, q0, head0, kvh;
  bool bidir;       // own segment read both ways (a document-isolated block)
  int seg_len[kMaxSeg], seg_off[kMaxSeg];
  int rows[2];      // valid query tokens of tiles A and B (0..32)
  int n[2];         // K/V tiles each tile reads
  int nmax;
};

__device__ __forceinline__ void load_item(Item& it, int item, const int* __restrict__ seqs,
                                          const int* __restrict__ blocks, int groups, int QH, int KH) {
  const int blk = item / groups, g = item % groups;
  const int seq = blocks[blk * 2];
  it.q0 = blocks[blk * 2 + 1];
  it.head0 = g * 4;
  it.kvh = it.head0 / (QH / KH);
  const int* sd = seqs + seq * kSeqInts;
  it.q_start = sd[0];
  it.q_len = sd[1];
  it.nseg = sd[2];
  it.bidir = (sd[3] & 1) != 0;
#pragma unroll
  for (int i = 0; i < kMaxSeg; ++i) {
    it.seg_len[i] = i < it.nseg ? sd[4 + i] : 0;
    it.seg_off[i] = i < it.nseg ? sd[8 + i] : 0;
  }
  it.own_len = 0;
#pragma unroll
  for (int i = 0; i < kMaxSeg; ++i)
    if (i == it.nseg - 1) it.own_len = it.seg_len[i];
  int before = 0;
#pragma unroll
  for (int i = 0; i < kMaxSeg - 1; ++i)
    if (i < it.nseg - 1) before += (it.seg_len[i] + kBkv - 1) / kBkv;
  it.nmax = 0;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int first = it.q0 + 32 * t;
    it.rows[t] = max(0, min(32, it.q_len - first));
    if (it.rows[t] == 0) {
      it.n[t] = 0;
    } else {
      const int max_pos = it.own_len - it.q_len + first + it.rows[t] - 1;  // own-segment position
      const int visible = it.bidir ? it.own_len : min(it.own_len, max_pos + 1);
      it.n[t] = before + (visible + kBkv - 1) / kBkv;
    }
    it.nmax = max(it.nmax, it.n[t]);
  }
}

// segment and tile-in-segment of the item's j-th K/V tile
__device__ __forceinline__ void locate(const Item& it, int j, int& s, int& tt) {
  s = 0;
  tt = j;
#pragma unroll
  for (int i = 0; i < kMaxSeg - 1; ++i) {
    const int nt = (it.seg_len[i] + kBkv - 1) / kBkv;
    if (s == i && i < it.nseg - 1 && tt >= nt) {
      tt -= nt;
      s = i + 1;
    }
  }
}

}  // namespace

template <int MODE>  // 0: bf16 out [T, QH*128]; 2: e4m3 + UE8M0 scale atoms
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_tc2_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const int* __restrict__ seqs,
                            const int* __restrict__ blocks, int n_items, const int* __restrict__ page_list,
                            int page_tokens, int QH, int KH, float scale_log2, __nv_bfloat16* __restrict__ o,
                            int ldo, uint8_t* __restrict__ o8, uint8_t* __restrict__ osf, float* __restrict__ lse,
                            int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sQ = smem;                                   // [2][kQBytes]
  uint8_t* sK = sQ + 2 * kQBytes;                       // [kStages][kKVBytes]
  uint8_t* sV = sK + kStages * kKVBytes;                // [kStages][kKVBytes]
  uint8_t* sP = sV + kStages * kKVBytes;                // [2][kPBytes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kPBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;                          // [kStages]
  uint64_t* v_full = k_full + kStages;                  // [kStages]
  uint64_t* kv_empty = v_full + kStages;                // [kStages]
  uint64_t* s_full = kv_empty + kStages;                // [2]
  uint64_t* p_full = s_full + 2;                        // [2] count 128
  uint64_t* o_done = p_full + 2;                        // [2]
  uint64_t* o_free = o_done + 2;                        // [2] count 128
  uint64_t* mma_idle = o_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_idle + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int groups = QH / 4;
  const int pshift = __ffs(page_tokens) - 1;
  const int pmask = page_tokens - 1;

  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 128);
      mbar_init(&o_done[t], 1);
      mbar_init(&o_free[t], 128);
    }
    mbar_init(mma_idle, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc<512>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ loader
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
    }
    int kv_it = 0, q_it = 0;
    int kv_par[kStages];
#pragma unroll
    for (int s = 0; s < kStages; ++s) kv_par[s] = -1;
    int q_par = -1;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      Item it;
      load_item(it, item, seqs, blocks, groups, QH, KH);
      if (lane == 0) {
        ok = mbar_wait(q_empty, (uint32_t)((q_it & 1) ^ 1), err, kErrTimeoutProducer);
        if (ok) {
          mbar_arrive_expect_tx(q_full, 2 * kQBytes);
          const int tok = it.q_start + it.q0;
          tma_load_3d(&tmQ, q_full, sQ, 0, it.head0, tok);
          tma_load_3d(&tmQ, q_full, sQ + kQBytes / 2, 64, it.head0, tok);
          tma_load_3d(&tmQ, q_full, sQ + kQBytes, 0, it.head0, tok + 32);
          tma_load_3d(&tmQ, q_full, sQ + kQBytes + kQBytes / 2, 64, it.head0, tok + 32);
          q_par = q_it & 1;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      ++q_it;
      for (int jb = 0; jb < it.nmax && ok; jb += 32) {
        // each lane looks up the arena row of one tile's first key
        int z = 0;
        const int jl = jb + lane;
        if (jl < it.nmax) {
          int s, tt;
          locate(it, jl, s, tt);
          const int j0 = tt * kBkv;
          int soff = it.seg_off[0];
#pragma unroll
          for (int i = 1; i < kMaxSeg; ++i)
            if (s == i) soff = it.seg_off[i];
          z = (page_list[soff + (j0 >> pshift)] << pshift) + (j0 & pmask);
        }
        const int cnt = min(32, it.nmax - jb);
        for (int k = 0; k < cnt; ++k) {
          const int zk = __shfl_sync(0xffffffffu, z, k);
          if (lane == 0) {
            const int st = kv_it % kStages;
            const uint32_t ph = (uint32_t)((kv_it / kStages) & 1);
            ok = mbar_wait(&kv_empty[st], ph ^ 1, err, kErrTimeoutProducer);
            if (ok) {
              mbar_arrive_expect_tx(&k_full[st], kKVBytes);
              tma_load_3d(&tmK, &k_full[st], sK + st * kKVBytes, 0, it.kvh, zk);
              tma_load_3d(&tmK, &k_full[st], sK + st * kKVBytes + kKVBytes / 2, 64, it.kvh, zk);
              mbar_arrive_expect_tx(&v_full[st], kKVBytes);
              tma_load_3d(&tmV, &v_full[st], sV + st * kKVBytes, 0, it.kvh, zk);
              tma_load_3d(&tmV, &v_full[st], sV + st * kKVBytes + kKVBytes / 2, 64, it.kvh, zk);
              kv_par[st] = (int)ph;
            }
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          ++kv_it;
        }
      }
    }
    if (!ok && lane == 0) {
      // stopped early: wait (bounded) for the copies already issued into shared memory
      if (q_par >= 0) mbar_wait(q_full, (uint32_t)q_par, err, kErrTimeoutProducer);
      for (int s = 0; s < kStages; ++s)
        if (kv_par[s] >= 0) {
          mbar_wait(&k_full[s], (uint32_t)kv_par[s], err, kErrTimeoutProducer);
          mbar_wait(&v_full[s], (uint32_t)kv_par[s], err, kErrTimeoutProducer);
        }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t IS = idesc_bf16_f32(128, kBkv, 0);
      constexpr uint32_t IO = idesc_bf16_f32(128, kD, 1);
      int kv_base = 0, q_it = 0;
      int p_cnt[2] = {0, 0}, free_cnt[2] = {0, 0};
      bool had[2] = {false, false};
      bool ok = true;
      auto issue_s = [&](int t, int j) -> bool {
        const int st = (kv_base + j) % kStages;
        if (!mbar_wait(&k_full[st], (uint32_t)(((kv_base + j) / kStages) & 1), err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ + t * kQBytes), kb = smem_u32(sK + st * kKVBytes);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t a = qa + (ks >> 2) * (kRows * 128) + (ks & 3) * 32;
          const uint32_t b = kb + (ks >> 2) * (kBkv * 128) + (ks & 3) * 32;
          umma_f16(tmem + (uint32_t)(t * 64), sw128_kmajor_desc(a), sw128_kmajor_desc(b), IS, ks > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[t]);
        return true;
      };
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        Item it;
        load_item(it, item, seqs, blocks, groups, QH, KH);
        if (!mbar_wait(q_full, (uint32_t)(q_it & 1), err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        ++q_it;
        tc_fence_after();
        for (int t = 0; t < 2 && ok; ++t)
          if (it.n[t] > 0) ok = issue_s(t, 0);
        for (int j = 0; j < it.nmax && ok; ++j) {
          const int st = (kv_base + j) % kStages;
          const uint32_t ph = (uint32_t)(((kv_base + j) / kStages) & 1);
          for (int t = 0; t < 2 && ok; ++t) {
            if (j >= it.n[t]) continue;
            if (!mbar_wait(&p_full[t], (uint32_t)(p_cnt[t] & 1), err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            ++p_cnt[t];
            if (j == 0 && had[t]) {
              // the previous item's epilogue has read O_t out of TMEM
              if (!mbar_wait(&o_free[t], (uint32_t)(free_cnt[t] & 1), err, kErrTimeoutMma)) {
                ok = false;
                break;
              }
              ++free_cnt[t];
            }
            if (!mbar_wait(&v_full[st], ph, err, kErrTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t pa = smem_u32(sP + t * kPBytes), vb = smem_u32(sV + st * kKVBytes);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_f16(tmem + 128u + (uint32_t)(t * 128), sw128_kmajor_desc(pa + ks * 32),
                       mn_desc(vb + ks * 16 * 128, kBkv * 128), IO, (j > 0 || ks > 0) ? 1u : 0u);
            tc_commit(&o_done[t]);
            if (j + 1 < it.n[t]) ok = issue_s(t, j + 1);
          }
          if (ok) tc_commit(&kv_empty[st]);
        }
        if (!ok) break;
        had[0] = had[0] || it.n[0] > 0;
        had[1] = had[1] || it.n[1] > 0;
        tc_commit(q_empty);
        kv_base += it.nmax;
      }
      tc_commit(mma_idle);
      mbar_wait(mma_idle, 0, err, kErrTimeoutMma);
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int t = (warp - 2) >> 2;                     // tile A (warps 2-5) or B (warps 6-9)
    const int quarter = warp & 3;                       // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    const int tok = row >> 2, hh = row & 3;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_base + (uint32_t)(t * 64);
    const uint32_t tO = tmem + lane_base + 128u + (uint32_t)(t * 128);
    uint8_t* myP = sP + t * kPBytes;
    const uint32_t p_row = smem_u32(myP) + row * 128;
    int s_cnt = 0, o_cnt = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      Item it;
      load_item(it, item, seqs, blocks, groups, QH, KH);
      const int n = it.n[t];
      if (n == 0) continue;
      const bool valid = tok < it.rows[t];
      const int pos = it.own_len - it.q_len + it.q0 + 32 * t + tok;  // own-segment position
      float m_ref = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        if (!mbar_wait(&s_full[t], (uint32_t)(s_cnt & 1), err, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        ++s_cnt;
        tc_fence_after();
        uint32_t sv[64];
        QB_TMEM_LD32(tS, sv);
        QB_TMEM_LD32(tS + 32, (sv + 32));
        tmem_ld_wait();
        int s, tt;
        locate(it, j, s, tt);
        int slen = it.seg_len[0];
#pragma unroll
        for (int i = 1; i < kMaxSeg; ++i)
          if (s == i) slen = it.seg_len[i];
        const int j0 = tt * kBkv;
        int lim = slen - j0;
        if (s == it.nseg - 1 && !it.bidir) lim = min(lim, pos - j0 + 1);
        if (!valid) lim = 0;
        float tmax = -INFINITY;
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i < lim) tmax = fmaxf(tmax, __uint_as_float(sv[i]));
        tmax *= scale_log2;
        float corr = 1.f;
        if (tmax > m_ref + 8.f) {
          corr = (m_ref == -INFINITY) ? 0.f : ex2f(m_ref - tmax);
          m_ref = tmax;
        }
        if (j > 0) {
          // P_{j-1} V_{j-1} is done: the P buffer is free and O is stable
          if (!mbar_wait(&o_done[t], (uint32_t)(o_cnt & 1), err, kErrTimeoutEpilogue)) {
            ok = false;
            break;
          }
          ++o_cnt;
          tc_fence_after();
          if (__any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t ov[32];
              QB_TMEM_LD32(tO + c * 32, ov);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * corr);
              QB_TMEM_ST32_A(tO + c * 32, ov);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
          }
        }
        l *= corr;
        const float mref = (m_ref == -INFINITY) ? 0.f : m_ref;
        float psum = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int e0 = c * 8 + 2 * i;
            const float p0 = e0 < lim ? ex2f(fmaf(__uint_as_float(sv[e0]), scale_log2, -mref)) : 0.f;
            const float p1 = e0 + 1 < lim ? ex2f(fmaf(__uint_as_float(sv[e0 + 1]), scale_log2, -mref)) : 0.f;
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
            const float2 back = __bfloat1622float2(h2);
            psum += back.x + back.y;
            w[i] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          const uint32_t dst = p_row + ((c ^ (row & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                       "r"(w[3])
                       : "memory");
        }
        l += psum;
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      if (!mbar_wait(&o_done[t], (uint32_t)(o_cnt & 1), err, kErrTimeoutEpilogue)) {
        ok = false;
        break;
      }
      ++o_cnt;
      tc_fence_after();
      // ---- epilogue: O / l
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int head = it.head0 + hh;
      const size_t t_out = (size_t)it.q_start + it.q0 + 32 * t + tok;
      uint32_t word = 0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t ov[32];
        QB_TMEM_LD32(tO + c * 32, ov);
        tmem_ld_wait();
        float v[32];
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          v[i] = __uint_as_float(ov[i]) * inv;
          amax = fmaxf(amax, fabsf(v[i]));
        }
        if (valid) {
          if constexpr (MODE == 0) {
            __nv_bfloat16* dst = o + t_out * ldo + head * kD + c * 32;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              __align__(16) __nv_bfloat162 h[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(v[i + 2 * k], v[i + 2 * k + 1]);
              *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(h);
            }
          } else {
            const uint8_t e = ue8m0_att(amax);
            const float sc = __uint_as_float((uint32_t)(254 - e) << 23);
            word |= (uint32_t)e << (8 * c);
            uint8_t* dst = o8 + t_out * ldo + head * kD + c * 32;
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
        if (valid)
          *reinterpret_cast<uint32_t*>(osf + ((t_out >> 7) * QH + head) * 512 + (t_out & 31) * 16 +
                                       ((t_out & 127) >> 5) * 4) = word;
      }
      // the row's log-sum-exp (natural log) for a merge with another read of the same rows
      if (lse != nullptr && valid)
        lse[t_out * QH + head] = l > 0.f ? (m_ref + __log2f(l)) * 0.69314718055994531f : -INFINITY;
      tc_fence_before();
      mbar_arrive(&o_free[t]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc<512>(tmem);
  }
}

// ------------------------------------------------------------------ host side

CUtensorMap make_tmap_3d_bf16(const void* ptr, int64_t d0, int64_t d1, int64_t d2, int64_t stride1_bytes,
                              int64_t stride2_bytes, int box0, int box1, int box2);
int num_sms(int dev);
int* device_error_word(int dev);

template <int MODE>
static void launch_tc2(int grid, cudaStream_t st, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv,
                       const int* seqs, const int* blocks, int n_items, const int* pl, int P, int QH, int KH, float sl2,
                       __nv_bfloat16* o, int ldo, uint8_t* o8, uint8_t* osf, float* lse, int* err, int dev) {
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(prefill_attn_tc2_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kSmem));
    configured[dev] = true;
  }
  prefill_attn_tc2_kernel<MODE><<<grid, kThreads, kSmem, st>>>(tq, tk, tv, seqs, blocks, n_items, pl, P, QH, KH, sl2,
                                                                o, ldo, o8, osf, lse, err);
}

// q [T, QH, 128] bf16; caches [pages, P, KH, 128] bf16 (P a multiple of 64, a
// power of two); seqs [S, 12]; blocks [n, 2] int32 (sequence, first token of a
// 64-token block); out bf16 [T, QH*128] or e4m3 with out_sf scale bytes; with a bf16 out,
// `lse` [T, QH] fp32 receives each row's log-sum-exp (rows no block covers are not written).
void prefill_attention_tc2(const torch::Tensor& q, const torch::Tensor& k_cache, const torch::Tensor& v_cache,
                           const torch::Tensor& seqs, const torch::Tensor& blocks, const torch::Tensor& page_list,
                           double softmax_scale, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf,
                           const c10::optional<torch::Tensor>& lse) {
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && q.is_contiguous() && q.scalar_type() == at::kBFloat16,
              "q: [T, QH, 128] bf16");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == 128 && k_cache.is_contiguous() && v_cache.is_contiguous() &&
                  k_cache.sizes() == v_cache.sizes() && k_cache.scalar_type() == at::kBFloat16,
              "caches: [pages, P, KH, 128] bf16");
  TORCH_CHECK(seqs.dim() == 2 && seqs.size(1) == kSeqInts && seqs.scalar_type() == at::kInt, "seqs: [S, 12] int32");
  TORCH_CHECK(blocks.dim() == 2 && blocks.size(1) == 2 && blocks.scalar_type() == at::kInt, "blocks: [n, 2] int32");
  const int T = q.size(0), QH = q.size(1), KH = k_cache.size(2), P = k_cache.size(1);
  TORCH_CHECK(QH % KH == 0 && (QH / KH) % 4 == 0, "the persistent attention packs 4 q heads of one KV head");
  TORCH_CHECK(P % kBkv == 0 && (P & (P - 1)) == 0, "page tokens: a power of two and a multiple of 64");
  const int n_blocks = blocks.size(0);
  if (n_blocks == 0 || T == 0) return;
  const int dev = q.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  const int64_t slots = k_cache.size(0) * (int64_t)P;
  // Q: dims {128, QH, T}, box {64, 4, 32}; K / V: dims {128, KH, slots}, box {64, 1, 64}
  CUtensorMap tq = make_tmap_3d_bf16(q.data_ptr(), 128, QH, T, 256, (int64_t)QH * 256, 64, 4, 32);
  CUtensorMap tk = make_tmap_3d_bf16(k_cache.data_ptr(), 128, KH, slots, 256, (int64_t)KH * 256, 64, 1, 64);
  CUtensorMap tv = make_tmap_3d_bf16(v_cache.data_ptr(), 128, KH, slots, 256, (int64_t)KH * 256, 64, 1, 64);
  const int n_items = n_blocks * (QH / 4);
  const int grid = std::min(n_items, num_sms(dev));
  const float sl2 = (float)(softmax_scale * 1.4426950408889634);
  int* err = device_error_word(dev);
  float* lse_p = nullptr;
  if (lse.has_value()) {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "a log-sum-exp output goes with a bf16 out");
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->is_contiguous() && lse->numel() >= (int64_t)T * QH,
                "lse: fp32 [T, QH]");
    lse_p = lse->data_ptr<float>();
  }
  if (out.scalar_type() == at::kFloat8_e4m3fn) {
    TORCH_CHECK(out_sf.has_value() && out_sf->scalar_type() == at::kByte &&
                    out_sf->numel() >= (int64_t)((T + 127) / 128) * QH * 512,
                "e4m3 output needs its MX scale bytes");
    launch_tc2<2>(grid, st, tq, tk, tv, seqs.data_ptr<int>(), blocks.data_ptr<int>(), n_items,
                  page_list.data_ptr<int>(), P, QH, KH, sl2, nullptr, out.stride(0),
                  reinterpret_cast<uint8_t*>(out.data_ptr()), out_sf->data_ptr<uint8_t>(), nullptr, err, dev);
  } else {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "bf16 or e4m3 output");
    launch_tc2<0>(grid, st, tq, tk, tv, seqs.data_ptr<int>(), blocks.data_ptr<int>(), n_items,
                  page_list.data_ptr<int>(), P, QH, KH, sl2, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                  out.stride(0), nullptr, nullptr, lse_p, err, dev);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
