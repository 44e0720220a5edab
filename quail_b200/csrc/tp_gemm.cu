// K12: tensor-parallel projections with the collective fused into the GEMM,
// over NVLink peer memory (no NCCL on these paths).
//
// Layout: the residual stream is sharded by tokens (rank r owns rows
// [r * rpr, (r + 1) * rpr), rpr a multiple of 128); weights are sharded by
// output columns (QKV, gate_up) or by input columns (o_proj, down).
//
//   AG -> GEMM (QKV, gate_up): every rank's normalized e4m3 shard and its MX
//     scale atoms sit at their own rows of a symmetric buffer. In each GEMM
//     CTA one elected thread of the gather warps copies peer shards, one
//     128-row m-tile at a time, into the same rows of the local buffer: a
//     non-multicast cp.async.bulk load brings an 8 KB piece from the peer's
//     memory into shared memory (two pieces in flight), a cp.async.bulk store
//     writes it to local memory (each remote tile crosses NVLink once), and
//     after the last store of the m-tile lands it releases a per-m-tile
//     ready word. The TMA producer starts with the local shard's
//     m-tiles and waits (bounded) on the ready word of each remote m-tile
//     before its first TMA load. Peers announce their shard with a ready flag
//     (written by the norm kernel that produced it).
//   GEMM -> RS (o_proj, down): the epilogue writes each bf16 output tile
//     straight into the owning rank's receive slot for this source (P2P
//     stores), fences, and adds the tile count to that rank's counter.
//   rs_reduce_norm: each rank waits (bounded) for every source's tiles, sums
//     the slots into its residual rows, applies RMSNorm and writes the e4m3 +
//     MX scales of its shard for the next AG -> GEMM, then raises its flag.
//
// TMA tensor loads here read only this GPU's memory, each CTA its own tiles;
// peer memory is read by the gather thread's bulk copies (never with
// .multicast::cluster) and written by st.global in the RS epilogue. Every wait on a peer has a clock budget and sets an error
// code instead of hanging.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "mx_common.cuh"
#include "peer_sync.cuh"

namespace qb {

constexpr int kTpMax = 8;

enum TpMode : int { kTpAgBf16 = 0, kTpAgSwiglu = 1, kTpRs = 2 };

struct TpParams {
  int M, N, K;            // M = tokens over all ranks, N = this rank's output columns
  int rank, tp, rpr;      // rows per rank (multiple of 128)
  uint32_t epoch;
  // AG
  const uint8_t* a_peer[kTpMax];     // each rank's symmetric A buffer [M, K] e4m3
  const uint8_t* sfa_peer[kTpMax];   // each rank's symmetric A scale atoms
  const uint32_t* flag_peer[kTpMax]; // each rank's shard-ready flag
  uint8_t* a_local;                  // == a_peer[rank]
  uint8_t* sfa_local;
  uint32_t* tile_ready;              // local, one word per m-tile
  // RS
  __nv_bfloat16* rs_slot[kTpMax];    // on rank d: receive slot of this source, [rpr, ldr] bf16
  int ld_slot;
  uint32_t* rs_counter[kTpMax];      // on rank d: tile counter of this source
  // outputs (AG modes, all M rows)
  __nv_bfloat16* D;
  int ldd;
  uint8_t* Y;
  int ldy;
  uint8_t* Ysf;
  const uint8_t* sfa;  // A scale atoms read by the producer (a_local's)
  const uint8_t* sfb;
  int* err;
  int num_m_tiles, num_n_tiles;
};

constexpr int kTpWarps = 12;  // producer, MMA, 8 epilogue, 2 gather (one elected thread copies)
constexpr int kTpGatherPiece = 8192;  // bytes per bulk copy; two in flight per CTA
constexpr int kTpGatherSmem = 2 * kTpGatherPiece + 256;

__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(smem_src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
constexpr int kTpThreads = kTpWarps * 32;

template <int MODE>
__global__ void __launch_bounds__(kTpThreads, 1)
    tp_gemm_mx_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const TpParams p) {
  // GEMM -> RS stages its output rows in shared memory for coalesced peer
  // stores (64 KB), so it keeps three pipeline stages instead of four
  constexpr int BM = 128, BN = kMxBN, STAGES = MODE == kTpRs ? 3 : kMxStages;
  constexpr int EPI_THREADS = BN;
  constexpr int TMEM_COLS = 512;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * kMxABytes;
  uint8_t* sSFA = sB + STAGES * kMxBBytes;
  uint8_t* sSFB = sSFA + STAGES * kMxSfaBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sSFB + STAGES * kMxSfbBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* done_bar = acc_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  int* push_count = reinterpret_cast<int*>(tmem_slot + 4);  // [kTpMax] tiles this CTA sent to each rank
  uint64_t* gbar = reinterpret_cast<uint64_t*>(push_count + kTpMax + 2);  // 8-byte aligned: 2 gather barriers
  uint8_t* gstage = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(gbar + 2) + 127) & ~static_cast<uintptr_t>(127));  // 2 x kTpGatherPiece

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_k = p.K / 128;
  const int num_tiles = p.num_m_tiles * p.num_n_tiles;
  const int sfb_chunks = (p.N + 127) / 128;
  const int tpr = p.rpr / BM;  // m-tiles per rank

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, EPI_THREADS);
    mbar_init(done_bar, 1);
    mbar_init(&gbar[0], 1);
    mbar_init(&gbar[1], 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (threadIdx.x < kTpMax) push_count[threadIdx.x] = 0;
  if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // m-tile of tile t: the local shard's tiles first, then the ring of peers
  auto tile_of = [&](int t, int& tm, int& tn) {
    const int tr = t % p.num_m_tiles;
    tn = t / p.num_m_tiles;
    tm = (MODE == kTpRs) ? tr : (tr + p.rank * tpr) % p.num_m_tiles;
  };

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      int last_par[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_par[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_of(t, tm, tn);
        if (MODE != kTpRs && tm / tpr != p.rank) {
          // a peer's m-tile: wait until the gather warps of some CTA copied it here
          if (!wait_word<false>(&p.tile_ready[tm], p.epoch, p.err)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
        }
        const int nchunks = min(BN / 128, sfb_chunks - tn * (BN / 128));
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kMxABytes + kMxBBytes + kMxSfaBytes + nchunks * 512);
          tma_load_2d(&tmA, &full[stage], sA + stage * kMxABytes, kb * 128, tm * BM);
          tma_load_2d(&tmB, &full[stage], sB + stage * kMxBBytes, kb * 128, tn * BN);
          bulk_load(sSFA + stage * kMxSfaBytes, p.sfa + ((size_t)tm * num_k + kb) * 512, 512, &full[stage]);
          for (int c = 0; c < nchunks; ++c)
            bulk_load(sSFB + stage * kMxSfbBytes + c * 512,
                      p.sfb + ((size_t)(tn * (BN / 128) + c) * num_k + kb) * 512, 512, &full[stage]);
          last_par[stage] = (int)phase;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
#pragma unroll
        for (int s = 0; s < STAGES; ++s)
          if (last_par[s] >= 0) mbar_wait(&full[s], (uint32_t)last_par[s], p.err, kErrTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0, aphase = 0;
      bool ok = true;
      const uint32_t t_sfa = tmem_base + kMxSfaCol;
      const uint32_t t_sfb = tmem_base + kMxSfbCol;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(acc_empty, aphase ^ 1, p.err, kErrTimeoutMma)) break;
        tc_fence_after();
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          tmem_cp_sf(t_sfa, sf_chunk_desc(smem_u32(sSFA + stage * kMxSfaBytes)));
#pragma unroll
          for (int c = 0; c < BN / 128; ++c)
            tmem_cp_sf(t_sfb + c * 4, sf_chunk_desc(smem_u32(sSFB + stage * kMxSfbBytes + c * 512)));
          const uint32_t a0 = smem_u32(sA + stage * kMxABytes);
          const uint32_t b0 = smem_u32(sB + stage * kMxBBytes);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_mx(tmem_base, sw128_kmajor_desc(a0 + k * 32), sw128_kmajor_desc(b0 + k * 32),
                    make_idesc_mx(BM, BN, k, k), t_sfa | ((uint32_t)k << 30), t_sfb | ((uint32_t)k << 30),
                    (kb > 0 || k > 0) ? 1u : 0u);
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) {
          tc_commit(acc_full);
          aphase ^= 1;
        }
      }
      tc_commit(done_bar);
      mbar_wait(done_bar, 0, p.err, kErrTimeoutMma);
    }
  } else if (warp < 10) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 2;
    const int q = warp & 3;
    const int h = ew >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint32_t aphase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int tm, tn;
      tile_of(t, tm, tn);
      const int m = tm * BM + row;
      const int n0 = tn * BN + h * 128;
      if (!mbar_wait(acc_full, aphase, p.err, kErrTimeoutEpilogue)) break;
      aphase ^= 1;
      tc_fence_after();
      float acc[128];
      const uint32_t taddr = tmem_base + lane_base + (uint32_t)(h * 128);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        QB_TMEM_LD32(taddr + c * 32, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[c * 32 + i] = __uint_as_float(r[i]);
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
      if (MODE != kTpRs && m >= p.M) continue;
      if constexpr (MODE == kTpAgBf16) {
        __nv_bfloat16* dst = p.D + (size_t)m * p.ldd + n0;
#pragma unroll
        for (int j = 0; j < 128; j += 8)
          if (n0 + j < p.N) st_bf16x8(dst + j, &acc[j]);
      } else if constexpr (MODE == kTpRs) {
        // the tile's rows all belong to rank d's shard: d's receive slot for this source
        const int m0 = tm * BM + q * 32;  // this warp's first row
        const int d = m0 / p.rpr;
        __nv_bfloat16* base = p.rs_slot[d] + (size_t)(m0 - d * p.rpr) * p.ld_slot + n0;
        warp_push_rows(acc, gstage + ew * 8192, lane, [&](int r) -> __nv_bfloat16* {
          return m0 + r < p.M ? base + (size_t)r * p.ld_slot : nullptr;
        });
        if (row == 0 && h == 0) push_count[d] += 1;  // one count per tile (rows of a tile share d)
      } else {
        const int out0 = tn * (BN / 2) + h * 64;
        if (out0 >= p.N / 2) continue;
#pragma unroll
        for (int i = 0; i < 64; ++i) acc[i] = silu_f(acc[i]) * acc[64 + i];
        uint8_t e[2];
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          float amax = 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(acc[g * 32 + i]));
          e[g] = ue8m0_of(amax);
          const float inv = ue8m0_inv(e[g]);
          uint8_t* dst = p.Y + (size_t)m * p.ldy + out0 + g * 32;
#pragma unroll
          for (int j = 0; j < 32; j += 16) {
            __align__(16) __nv_fp8x4_e4m3 pk[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              pk[i] = __nv_fp8x4_e4m3(make_float4(acc[g * 32 + j + 4 * i] * inv, acc[g * 32 + j + 4 * i + 1] * inv,
                                                  acc[g * 32 + j + 4 * i + 2] * inv,
                                                  acc[g * 32 + j + 4 * i + 3] * inv));
            *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(pk);
          }
        }
        const int kst = out0 / 128, kblk = (out0 % 128) / 32;
        const int ko = p.N / 2 / 128;
        uint8_t* sf = p.Ysf + ((size_t)(m / 128) * ko + kst) * 512 + (m % 32) * 16 + ((m % 128) / 32) * 4 + kblk;
        *reinterpret_cast<uint16_t*>(sf) = (uint16_t)e[0] | ((uint16_t)e[1] << 8);
      }
    }
    if constexpr (MODE == kTpRs) {
      // every epilogue thread's P2P stores, then one system fence (cumulative over the barrier)
      named_bar_sync(1, EPI_THREADS);
      if (warp == 2 && lane == 0) {
        __threadfence_system();
        for (int d = 0; d < p.tp; ++d)
          if (push_count[d]) atomicAdd_system(p.rs_counter[d], (unsigned)push_count[d]);
      }
    }
  } else if constexpr (MODE != kTpRs) {
    // ------------------------------------------------------------ gather (AG)
    // One elected thread streams each remote m-tile (its 128 rows, then its
    // scale atoms: two contiguous ranges) from the peer's symmetric buffer
    // into the same rows here: bulk loads peer -> shared memory (two 8 KB
    // slots, both in flight) and bulk stores shared -> local memory. Then it
    // releases the m-tile's ready word for the TMA producers of every CTA.
    if (threadIdx.x == 10 * 32) {
      const int remote_tiles = (p.tp - 1) * tpr;
      int seen_peer = -1;
      uint32_t gph[2] = {0u, 0u};
      bool pend[2] = {false, false};  // a bulk load into the slot is issued and not yet waited for
      bool ok = true;
      for (int g = blockIdx.x; g < remote_tiles && ok; g += gridDim.x) {
        const int o = (p.rank + 1 + g / tpr) % p.tp;  // nearest peer first
        const int tm = o * tpr + g % tpr;
        if (o != seen_peer) {
          if (!wait_word<true>(p.flag_peer[o], p.epoch, p.err)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();  // the bulk loads below read what the acquire made visible
          seen_peer = o;
        }
        const size_t a_off = (size_t)tm * BM * p.K, a_len = (size_t)BM * p.K;
        const size_t s_off = (size_t)tm * num_k * 512, s_len = (size_t)num_k * 512;
        const size_t total = a_len + s_len;
        const int pieces = (int)((total + kTpGatherPiece - 1) / kTpGatherPiece);
        auto src_of = [&](int i) -> const uint8_t* {
          const size_t off = (size_t)i * kTpGatherPiece;
          return off < a_len ? p.a_peer[o] + a_off + off : p.sfa_peer[o] + s_off + (off - a_len);
        };
        auto dst_of = [&](int i) -> uint8_t* {
          const size_t off = (size_t)i * kTpGatherPiece;
          return off < a_len ? p.a_local + a_off + off : p.sfa_local + s_off + (off - a_len);
        };
        // pieces never straddle the A / scale boundary: a_len is a multiple of the piece size
        auto size_of = [&](int i) -> uint32_t {
          const size_t off = (size_t)i * kTpGatherPiece;
          const size_t end = off < a_len ? a_len : total;
          return (uint32_t)min((size_t)kTpGatherPiece, end - off);
        };
        auto issue = [&](int i) {
          const int slot = i & 1;
          mbar_arrive_expect_tx(&gbar[slot], size_of(i));
          bulk_load(gstage + slot * kTpGatherPiece, src_of(i), size_of(i), &gbar[slot]);
          pend[slot] = true;
        };
        issue(0);
        if (pieces > 1) issue(1);
        for (int i = 0; i < pieces; ++i) {
          const int slot = i & 1;
          if (!mbar_wait(&gbar[slot], gph[slot], p.err, kErrTimeoutPeer)) {
            ok = false;
            break;
          }
          gph[slot] ^= 1u;
          pend[slot] = false;
          bulk_store(dst_of(i), gstage + slot * kTpGatherPiece, size_of(i));
          bulk_commit();
          if (i + 2 < pieces) {
            bulk_wait_read<0>();  // the slot's bytes have left shared memory
            issue(i + 2);
          }
        }
        bulk_wait<0>();  // every store of this m-tile is in local memory
        if (!ok) break;
        fence_proxy_async_global();
        st_release_gpu(&p.tile_ready[tm], p.epoch);
      }
      // on a timeout, wait (bounded) for the loads still landing in shared memory
      for (int slot = 0; slot < 2; ++slot)
        if (pend[slot] && mbar_wait(&gbar[slot], gph[slot], p.err, kErrTimeoutPeer)) gph[slot] ^= 1u;
      bulk_wait<0>();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc<TMEM_COLS>(tmem_base);
  }
}

// ---------------------------------------------------------------- reduce + norm
// One warp per local row; each lane owns 8 columns of every 256-column slab.
// With `tp_slots` > 0 the CTA first waits for every source's tiles; the row is
// then residual + sum of the slots. The result is the new residual row; its
// RMSNorm goes out as e4m3 + UE8M0 atoms into this rank's rows of the
// symmetric A buffer. The last CTA to finish raises this rank's flag.
template <int H>
__global__ void rs_reduce_norm_kernel(const __nv_bfloat16* __restrict__ slots, int tp_slots, int rpr,
                                      const uint32_t* __restrict__ counters, uint32_t want,
                                      __nv_bfloat16* __restrict__ resid, const __nv_bfloat16* __restrict__ w,
                                      float eps, uint8_t* __restrict__ a_sym, uint8_t* __restrict__ sf_sym,
                                      int row0, uint32_t* __restrict__ done_ctr, uint32_t done_want,
                                      uint32_t* __restrict__ flag, uint32_t epoch, int* err) {
  constexpr int SLABS = H / 256;
  __shared__ int go;
  if (threadIdx.x == 0) {
    int ok = 1;
    for (int s = 0; s < tp_slots && ok; ++s) ok = wait_word<true>(&counters[s], want, err) ? 1 : 0;
    go = ok;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (go && r < rpr) {
    float v[SLABS][8];
    float ss = 0.f;
#pragma unroll
    for (int s = 0; s < SLABS; ++s) {
      ld_bf16x8f(resid + (size_t)r * H + s * 256 + lane * 8, v[s]);
      for (int k = 0; k < tp_slots; ++k) {
        float u[8];
        ld_bf16x8f(slots + ((size_t)k * rpr + r) * H + s * 256 + lane * 8, u);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[s][i] += u[i];
      }
      if (tp_slots) st_bf16x8(resid + (size_t)r * H + s * 256 + lane * 8, v[s]);
      // the stored residual is bf16: normalize what was stored
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[s][i] = __bfloat162float(__float2bfloat16(v[s][i]));
        ss += v[s][i] * v[s][i];
      }
    }
    ss = warp_sum(ss);
    const float rinv = rsqrtf(ss / H + eps);
    const int m = row0 + r;  // row in the full [M, H] symmetric buffer
#pragma unroll
    for (int s = 0; s < SLABS; ++s) {
      float wv[8];
      ld_bf16x8f(w + s * 256 + lane * 8, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[s][i] = v[s][i] * rinv * wv[i];
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[s][i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const uint8_t e = ue8m0_of(amax);
      const float inv = ue8m0_inv(e);
      __nv_fp8x4_e4m3 a(make_float4(v[s][0] * inv, v[s][1] * inv, v[s][2] * inv, v[s][3] * inv));
      __nv_fp8x4_e4m3 b(make_float4(v[s][4] * inv, v[s][5] * inv, v[s][6] * inv, v[s][7] * inv));
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&a);
      pk.y = *reinterpret_cast<uint32_t*>(&b);
      *reinterpret_cast<uint2*>(a_sym + (size_t)m * H + s * 256 + lane * 8) = pk;
      if ((lane & 3) == 0) {
        const int j = s * 8 + (lane >> 2);  // 32-wide K block
        sf_sym[((size_t)(m >> 7) * (H / 128) + (j >> 2)) * 512 + (m & 31) * 16 + ((m & 127) >> 5) * 4 + (j & 3)] = e;
      }
    }
  }
  // last CTA out raises this rank's shard-ready flag for the peers
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // the CTA's rows (ordered by the barrier) before the count and the flag
    const uint32_t prev = atomicAdd(done_ctr, 1u);
    if (prev + 1 == done_want) st_release_sys(flag, epoch);
  }
}

// ------------------------------------------------------------------ host side

struct TpBuffers {
  std::vector<int64_t> a_peer, sfa_peer, flag_peer, rs_slot, rs_counter;
};

static void fill_ptrs(TpParams& p, const std::vector<int64_t>& a, const std::vector<int64_t>& sfa,
                      const std::vector<int64_t>& flag, const std::vector<int64_t>& slot,
                      const std::vector<int64_t>& ctr) {
  for (int i = 0; i < kTpMax; ++i) {
    p.a_peer[i] = i < (int)a.size() ? reinterpret_cast<const uint8_t*>(a[i]) : nullptr;
    p.sfa_peer[i] = i < (int)sfa.size() ? reinterpret_cast<const uint8_t*>(sfa[i]) : nullptr;
    p.flag_peer[i] = i < (int)flag.size() ? reinterpret_cast<const uint32_t*>(flag[i]) : nullptr;
    p.rs_slot[i] = i < (int)slot.size() ? reinterpret_cast<__nv_bfloat16*>(slot[i]) : nullptr;
    p.rs_counter[i] = i < (int)ctr.size() ? reinterpret_cast<uint32_t*>(ctr[i]) : nullptr;
  }
}

template <int MODE>
static void launch_tp(const CUtensorMap& ta, const CUtensorMap& tb, TpParams& p, cudaStream_t st, int dev) {
  // AG modes: 4 stages + the gather's staging; RS: 3 stages + 8 KB of row staging per epilogue warp
  constexpr int smem = MODE == kTpRs ? mx_pipeline_smem(3) + 64 + 256 + 8 * 8192
                                     : mx_pipeline_smem(kMxStages) + 64 + kTpGatherSmem;
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(tp_gemm_mx_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev] = true;
  }
  const int tiles = p.num_m_tiles * p.num_n_tiles;
  tp_gemm_mx_kernel<MODE><<<std::min(tiles, num_sms(dev)), kTpThreads, smem, st>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// AG -> GEMM. a_local: this rank's symmetric A buffer [M, K] e4m3 (its own
// rows already written); sfa_local its scale atoms; peers' buffers and flags
// by pointer. mode 0: out bf16 [M, N]; mode 1: SwiGLU out e4m3 [M, N/2] + atoms.
void tp_ag_gemm(const torch::Tensor& a_local, const torch::Tensor& sfa_local, const std::vector<int64_t>& a_peer,
                const std::vector<int64_t>& sfa_peer, const std::vector<int64_t>& flag_peer,
                const torch::Tensor& tile_ready, int64_t epoch, int64_t rank, int64_t rpr, const torch::Tensor& b,
                const torch::Tensor& sfb, int64_t mode, torch::Tensor& out, const c10::optional<torch::Tensor>& out_sf) {
  const int M = a_local.size(0), K = a_local.size(1), N = b.size(0);
  const int tp = (int)a_peer.size();
  TORCH_CHECK(tp >= 1 && tp <= kTpMax && rpr % 128 == 0 && (int64_t)M == rpr * tp, "tp_ag_gemm: M = tp x rpr");
  TORCH_CHECK(K % 128 == 0 && N % 16 == 0, "tp_ag_gemm: K % 128, N % 16");
  TORCH_CHECK(tile_ready.numel() >= M / 128 && tile_ready.scalar_type() == at::kInt, "tile_ready words");
  const int dev = a_local.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  TpParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.rank = (int)rank;
  p.tp = tp;
  p.rpr = (int)rpr;
  p.epoch = (uint32_t)epoch;
  fill_ptrs(p, a_peer, sfa_peer, flag_peer, {}, {});
  p.a_local = reinterpret_cast<uint8_t*>(a_local.data_ptr());
  p.sfa_local = sfa_local.data_ptr<uint8_t>();
  p.sfa = p.sfa_local;
  p.tile_ready = reinterpret_cast<uint32_t*>(tile_ready.data_ptr<int>());
  p.sfb = sfb.data_ptr<uint8_t>();
  p.err = device_error_word(dev);
  p.num_m_tiles = M / 128;
  p.num_n_tiles = (N + kMxBN - 1) / kMxBN;
  CUtensorMap ta = make_tmap_2d(a_local.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, a_local.stride(0), 128,
                                128, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, b.stride(0), 128, kMxBN,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  if (mode == 0) {
    TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.size(0) == M && out.size(1) == N, "bf16 out [M, N]");
    p.D = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    p.ldd = out.stride(0);
    launch_tp<kTpAgBf16>(ta, tb, p, st, dev);
  } else {
    TORCH_CHECK(N % kMxBN == 0 && out.scalar_type() == at::kFloat8_e4m3fn && out.size(1) == N / 2 && out_sf.has_value(),
                "SwiGLU e4m3 out [M, N/2] + scale atoms");
    p.Y = reinterpret_cast<uint8_t*>(out.data_ptr());
    p.ldy = out.stride(0);
    p.Ysf = out_sf->data_ptr<uint8_t>();
    launch_tp<kTpAgSwiglu>(ta, tb, p, st, dev);
  }
}

// GEMM -> RS: a [M, K] e4m3 (local), output rows pushed to their owner's slot.
void tp_gemm_rs(const torch::Tensor& a, const torch::Tensor& sfa, const torch::Tensor& b, const torch::Tensor& sfb,
                const std::vector<int64_t>& slot_ptrs, int64_t ld_slot, const std::vector<int64_t>& counter_ptrs,
                int64_t rank, int64_t rpr) {
  const int M = a.size(0), K = a.size(1), N = b.size(0);
  const int tp = (int)slot_ptrs.size();
  TORCH_CHECK(tp >= 1 && tp <= kTpMax && (int64_t)M == rpr * tp && rpr % 128 == 0, "tp_gemm_rs: M = tp x rpr");
  TORCH_CHECK(K % 128 == 0 && N % kMxBN == 0 && ld_slot % 8 == 0, "tp_gemm_rs shapes: K % 128, N % 256");
  const int dev = a.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  TpParams p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.rank = (int)rank;
  p.tp = tp;
  p.rpr = (int)rpr;
  fill_ptrs(p, {}, {}, {}, slot_ptrs, counter_ptrs);
  p.ld_slot = (int)ld_slot;
  p.sfa = sfa.data_ptr<uint8_t>();
  p.sfb = sfb.data_ptr<uint8_t>();
  p.err = device_error_word(dev);
  p.num_m_tiles = M / 128;
  p.num_n_tiles = (N + kMxBN - 1) / kMxBN;
  CUtensorMap ta = make_tmap_2d(a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, a.stride(0), 128, 128,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(b.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, N, b.stride(0), 128, kMxBN,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  launch_tp<kTpRs>(ta, tb, p, st, dev);
}

void tp_reduce_norm(const torch::Tensor& slots, int64_t tp_slots, const torch::Tensor& counters, int64_t want,
                    torch::Tensor& resid, const torch::Tensor& w, double eps, torch::Tensor& a_sym,
                    torch::Tensor& sf_sym, int64_t row0, torch::Tensor& done_ctr, int64_t done_base,
                    torch::Tensor& flag, int64_t epoch) {
  const int rpr = resid.size(0), H = resid.size(1);
  TORCH_CHECK(resid.scalar_type() == at::kBFloat16 && resid.is_contiguous(), "residual rows bf16");
  const int dev = resid.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  const int rows_per_cta = 8;
  const int grid = (rpr + rows_per_cta - 1) / rows_per_cta;
  auto sp = reinterpret_cast<const __nv_bfloat16*>(slots.data_ptr());
#define QB_RS_CASE(HH)                                                                                           \
  if (H == HH) {                                                                                                 \
    rs_reduce_norm_kernel<HH><<<grid, rows_per_cta * 32, 0, st>>>(                                               \
        sp, (int)tp_slots, rpr, reinterpret_cast<const uint32_t*>(counters.data_ptr<int>()), (uint32_t)want,     \
        reinterpret_cast<__nv_bfloat16*>(resid.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), \
        (float)eps, reinterpret_cast<uint8_t*>(a_sym.data_ptr()), sf_sym.data_ptr<uint8_t>(), (int)row0,         \
        reinterpret_cast<uint32_t*>(done_ctr.data_ptr<int>()), (uint32_t)(done_base + grid),                    \
        reinterpret_cast<uint32_t*>(flag.data_ptr<int>()), (uint32_t)epoch, device_error_word(dev));            \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                              \
    return;                                                                                                      \
  }
  QB_RS_CASE(1024)
  QB_RS_CASE(2048)
  QB_RS_CASE(2560)
  QB_RS_CASE(4096)
  QB_RS_CASE(5120)
#undef QB_RS_CASE
  TORCH_CHECK(false, "tp_reduce_norm: unsupported hidden size ", H);
}

}  // namespace qb
