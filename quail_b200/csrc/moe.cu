// K11: mixture-of-experts layer with expert parallelism fused into the
// grouped expert GEMMs (Qwen3-MoE: softmax router, top-k, renormalized
// weights, SwiGLU experts).
//
// W ranks (W = 1 .. 8) each hold E / W experts (Epr) and route their own
// tokens. Per layer, on every rank, in stream order:
//
//   moe_route     one warp per token: softmax over the router logits, top-k,
//                 renormalized weights; each (token, k) takes a slot among
//                 this rank's rows for its expert (atomic per expert count).
//   moe_plan      one CTA: publishes this rank's per-expert counts to every
//                 peer (P2P stores + a per-layer-parity flag), waits (bounded)
//                 for all peers' counts, then derives from the full W x E count
//                 matrix (the same on every rank): where this rank's rows of
//                 expert e land in the owner's receive buffer, the dispatch
//                 units of this rank (32 rows of one expert each, ordered by
//                 local expert index then owner, so every owner's first expert
//                 completes first), and the tile table of this rank's own
//                 experts (expert, first row, valid rows per 128-row tile).
//   moe_sort      lists this rank's (token, k) items expert by expert.
//   moe_gate_up   persistent MX GEMM over the tile table with two dispatch
//                 warps per CTA: they copy token rows (e4m3 + scale atoms +
//                 home/weight metadata) into the owners' receive buffers with
//                 plain P2P stores and count the rows per expert on the owner
//                 (release at system scope). The TMA producer waits (bounded)
//                 until its tile's expert has all rows, then loads the tile
//                 from local memory. Epilogue: SwiGLU -> e4m3 + MX scales.
//   moe_down      persistent MX GEMM over the same tiles; the epilogue scales
//                 each row by its routing weight and stores it as bf16 straight
//                 into the home rank's combine buffer at (token, k), then adds
//                 the row count to the home's counter.
//   moe_combine   one warp per token waits (bounded) for all rows of this rank's
//                 tokens, sums the K expert rows into the residual and, when a
//                 norm weight is given, writes the next layer's RMSNorm as e4m3 +
//                 MX scale atoms.
//
// The count exchange of layer l + 1 cannot start on any rank before every
// rank finished reading the counts of layer l - 1, so the counts and flags are
// double-buffered by layer parity, and the receive / combine buffers of a
// layer are only rewritten after every rank passed the next count exchange.
// All counters are monotonic (cumulative rows, epochs): nothing is reset.
//
// TMA here reads only this GPU's memory; peer memory is only written, by
// st.global from the dispatch warps and the down-GEMM epilogue.
//
// Reference: the MoE block runs vLLM's fused Triton experts on one GPU with
// no expert parallelism (quail/backends/quail/executor/moe.py:12-87,
// FP8Experts asserts tp == ep == dp == 1).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "gemm_sm100.h"
#include "mx_common.cuh"
#include "peer_sync.cuh"

namespace qb {

constexpr int kMoeMaxRanks = 8;
constexpr int kMoeMaxExperts = 256;
constexpr int kUnitRows = 32;

// int32 plan buffer: a header, then per-expert tables, then the tile table
struct PlanView {
  int* num_tiles;    // [0]
  int* num_units;    // [1]
  int* send_base;    // [E] row of this rank's first row of expert e in the owner's receive buffer
  int* src_off;      // [E] offset of expert e's items in this rank's sorted item list
  int* cnt_local;    // [E] this rank's rows for expert e
  int* unit_start;   // [E + 1] dispatch units, prefix over order o = le * W + owner
  int* recv_target;  // [Epr] cumulative rows expected for each local expert
  int* tile_le;      // [Tcap]
  int* tile_row0;    // [Tcap]
  int* tile_valid;   // [Tcap]
};

__host__ __device__ inline int plan_ints(int E, int Epr, int tcap) { return 8 + 4 * E + 1 + Epr + 3 * tcap; }

__host__ __device__ inline PlanView plan_view(int* base, int E, int Epr, int tcap) {
  PlanView v;
  v.num_tiles = base;
  v.num_units = base + 1;
  v.send_base = base + 8;
  v.src_off = v.send_base + E;
  v.cnt_local = v.src_off + E;
  v.unit_start = v.cnt_local + E;
  v.recv_target = v.unit_start + E + 1;
  v.tile_le = v.recv_target + Epr;
  v.tile_row0 = v.tile_le + tcap;
  v.tile_valid = v.tile_row0 + tcap;
  return v;
}

// byte offset of row r, 128-wide K chunk kc in MX scale atoms with kchunks chunks per row block
__device__ __forceinline__ size_t sf_word_offset(int r, int kc, int kchunks) {
  return ((size_t)(r >> 7) * kchunks + kc) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4;
}

// ------------------------------------------------------------------ route
// logits bf16 [M, ldl] (first E columns), one warp per token.
__global__ void moe_route_kernel(const __nv_bfloat16* __restrict__ logits, int ldl, int M, int E, int K,
                                 int* __restrict__ ids, float* __restrict__ wts, int* __restrict__ pos,
                                 int* __restrict__ counts) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= M) return;
  constexpr int VPL = kMoeMaxExperts / 32;
  float v[VPL];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? __bfloat162float(logits[(size_t)t * ldl + e]) : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < E ? expf(v[i] - mx) : -1.f;  // probabilities; -1 marks absent / taken
    sum += e < E ? v[i] : 0.f;
  }
  sum = warp_sum(sum);
  int my_id = 0;
  float my_p = 0.f, top_sum = 0.f;
  for (int k = 0; k < K; ++k) {
    float bv = -1.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (v[i] > bv) {  // ascending i: the lowest expert index wins a tie within the lane
        bv = v[i];
        bi = i * 32 + lane;
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) {
#pragma unroll
      for (int i = 0; i < VPL; ++i)
        if (i == (bi >> 5)) v[i] = -1.f;
    }
    if (lane == k) {
      my_id = bi;
      my_p = bv / sum;
    }
    top_sum += bv / sum;
  }
  if (lane < K) {
    const size_t o = (size_t)t * K + lane;
    ids[o] = my_id;
    wts[o] = my_p / top_sum;
    pos[o] = atomicAdd(&counts[my_id], 1);
  }
}

// exclusive prefix sum of v(0 .. n-1) by one warp (each lane a run of
// consecutive items); out(i, prefix) per item; returns the total
template <class V, class O>
__device__ __forceinline__ int warp_scan_excl(int n, int lane, V v, O out) {
  const int per = (n + 31) / 32;
  int local = 0;
  for (int k = 0; k < per; ++k) {
    const int i = lane * per + k;
    if (i < n) local += v(i);
  }
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  int run = incl - local;
  for (int k = 0; k < per; ++k) {
    const int i = lane * per + k;
    if (i < n) {
      out(i, run);
      run += v(i);
    }
  }
  return __shfl_sync(0xffffffffu, incl, 31);
}

// ------------------------------------------------------------------ plan
struct PlanParams {
  int* counts;                             // local per-expert counts (zeroed here after use)
  int* counts_all_peer[kMoeMaxRanks];      // each rank's [2][W][E] count matrix
  uint32_t* cflag_peer[kMoeMaxRanks];      // each rank's [2][W] flags
  const int* counts_all_local;
  const uint32_t* cflag_local;
  int* plan;
  int* cum;                                // [Epr] cumulative rows per local expert
  int rank, W, E, Epr, tcap;
  uint32_t epoch;
  int* err;
};

__global__ void __launch_bounds__(256) moe_plan_kernel(const PlanParams p) {
  __shared__ int cnt[kMoeMaxRanks][kMoeMaxExperts];
  __shared__ int total[kMoeMaxExperts];
  __shared__ int base[kMoeMaxExperts];
  __shared__ int tile_start[kMoeMaxExperts + 1];
  __shared__ int ok;
  const int t = threadIdx.x;
  const int parity = p.epoch & 1;
  const PlanView pv = plan_view(p.plan, p.E, p.Epr, p.tcap);
  if (t == 0) ok = 1;
  if (p.W > 1) {
    for (int e = t; e < p.E; e += blockDim.x) {
      const int c = p.counts[e];
      for (int d = 0; d < p.W; ++d) p.counts_all_peer[d][((size_t)parity * p.W + p.rank) * p.E + e] = c;
    }
    // the CTA's count stores, then one release per peer (cumulative over the barrier)
    __syncthreads();
    if (t < p.W) {
      __threadfence_system();
      st_release_sys(&p.cflag_peer[t][parity * p.W + p.rank], p.epoch);
    }
    if (t < p.W && !wait_word<true>(&p.cflag_local[parity * p.W + t], p.epoch, p.err)) ok = 0;
    __syncthreads();
    for (int i = t; i < p.W * p.E; i += blockDim.x)
      cnt[i / p.E][i % p.E] = ok ? p.counts_all_local[(size_t)parity * p.W * p.E + i] : 0;
  } else {
    for (int e = t; e < p.E; e += blockDim.x) cnt[0][e] = p.counts[e];
  }
  __syncthreads();
  for (int e = t; e < p.E; e += blockDim.x) {
    int s = 0;
    for (int r = 0; r < p.W; ++r) s += cnt[r][e];
    total[e] = s;
    p.counts[e] = 0;  // ready for the next layer's route
  }
  __syncthreads();
  const int warp = t >> 5, lane = t & 31;
  // owner `warp`'s receive buffer: its experts' rows back to back, each padded to 128
  if (warp < p.W) {
    const int d = warp;
    warp_scan_excl(p.Epr, lane, [&](int le) { return (total[d * p.Epr + le] + 127) & ~127; },
                   [&](int le, int v) { base[d * p.Epr + le] = v; });
  }
  __syncthreads();
  if (warp == 0) {
    // this rank's dispatch units in order o = le * W + owner
    const int u = warp_scan_excl(
        p.E, lane, [&](int o) { return (cnt[p.rank][(o % p.W) * p.Epr + o / p.W] + kUnitRows - 1) / kUnitRows; },
        [&](int o, int v) { pv.unit_start[o] = v; });
    if (lane == 0) {
      pv.unit_start[p.E] = u;
      *pv.num_units = ok ? u : 0;
    }
  } else if (warp == 1) {
    // item offsets of this rank's sorted list, same order
    warp_scan_excl(p.E, lane, [&](int o) { return cnt[p.rank][(o % p.W) * p.Epr + o / p.W]; },
                   [&](int o, int v) { pv.src_off[(o % p.W) * p.Epr + o / p.W] = v; });
  } else if (warp == 2) {
    const int ts = warp_scan_excl(p.Epr, lane, [&](int le) { return (total[p.rank * p.Epr + le] + 127) >> 7; },
                                  [&](int le, int v) { tile_start[le] = v; });
    if (lane == 0) {
      tile_start[p.Epr] = ts;
      *pv.num_tiles = (ok && ts <= p.tcap) ? ts : 0;
      if (ts > p.tcap) atomicCAS(p.err, 0, kErrCapacity);
    }
  }
  __syncthreads();
  for (int e = t; e < p.E; e += blockDim.x) {
    int before = 0;
    for (int r = 0; r < p.rank; ++r) before += cnt[r][e];
    pv.send_base[e] = base[e] + before;
    pv.cnt_local[e] = cnt[p.rank][e];
  }
  for (int le = t; le < p.Epr; le += blockDim.x) {
    const int tot = total[p.rank * p.Epr + le];
    p.cum[le] += tot;
    pv.recv_target[le] = p.cum[le];
  }
  // tile table: one warp per local expert
  for (int le = warp; le < p.Epr; le += blockDim.x >> 5) {
    const int e = p.rank * p.Epr + le;
    const int tot = total[e];
    for (int i = lane; tile_start[le] + i < tile_start[le + 1]; i += 32) {
      const int ti = tile_start[le] + i;
      if (ti >= p.tcap) break;
      pv.tile_le[ti] = le;
      pv.tile_row0[ti] = base[e] + i * 128;
      pv.tile_valid[ti] = min(128, tot - i * 128);
    }
  }
}

// ------------------------------------------------------------------ sort
__global__ void moe_sort_kernel(const int* __restrict__ ids, const int* __restrict__ pos, int n,
                                const int* __restrict__ plan_src_off, int* __restrict__ src_list) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) src_list[plan_src_off[ids[i]] + pos[i]] = i;
}

// ------------------------------------------------------------------ grouped GEMMs
enum MoeMode : int { kMoeGateUp = 0, kMoeDown = 1 };

struct MoeGemmParams {
  int N, K;              // per-expert output rows of B, reduction length
  int H, topk;           // hidden size (dispatch row bytes / combine row width), routing top-k
  int rank, W, E, Epr, tcap;
  const int* plan;
  // dispatch (gate_up)
  const uint8_t* x8;     // this rank's normalized tokens [M, H] e4m3
  const uint8_t* xsf;    // their scale atoms
  const int* src_list;
  const float* wts;
  uint8_t* recv_a_peer[kMoeMaxRanks];
  uint8_t* recv_sf_peer[kMoeMaxRanks];
  int2* recv_meta_peer[kMoeMaxRanks];
  uint32_t* recv_count_peer[kMoeMaxRanks];
  const uint32_t* recv_count;  // local
  // A of this GEMM (local): its scale atoms
  const uint8_t* sfa;
  const uint8_t* sfb;
  // gate_up output
  uint8_t* Y;
  uint8_t* Ysf;
  int ldy;
  // down epilogue
  const int2* recv_meta;
  __nv_bfloat16* comb_peer[kMoeMaxRanks];
  uint32_t* comb_counter_peer[kMoeMaxRanks];
  int* err;
  int act;               // gate activation: 0 SiLU (SwiGLU), 1 GELU tanh form (GeGLU)
};

constexpr int kMoeWarps = 12;  // producer, MMA, 8 epilogue, 2 dispatch
constexpr int kMoeThreads = kMoeWarps * 32;
constexpr int kMoeExtraSmem = 64 + 4 * (kMoeMaxExperts + 1);

template <int MODE>
__global__ void __launch_bounds__(kMoeThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const MoeGemmParams p) {
  // the down GEMM stages its output rows in shared memory for coalesced
  // stores to the tokens' homes (64 KB), so it keeps three pipeline stages
  constexpr int BM = 128, BN = kMxBN, STAGES = MODE == kMoeDown ? 3 : kMxStages;
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
  int* push_count = reinterpret_cast<int*>(tmem_slot + 4);  // [kMoeMaxRanks]
  int* s_unit = push_count + kMoeMaxRanks;                  // [E + 1] dispatch unit prefix
  uint8_t* rstage = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(s_unit + kMoeMaxExperts + 1) + 127) & ~static_cast<uintptr_t>(127));  // down: 8 x 8 KB

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_k = p.K / 128;
  const PlanView pv = plan_view(const_cast<int*>(p.plan), p.E, p.Epr, p.tcap);
  const int num_tiles_m = *pv.num_tiles;
  const int num_n = p.N / BN;
  const int num_tiles = num_tiles_m * num_n;
  const int n_chunks_b = p.N / 128;  // B scale chunks per expert

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, EPI_THREADS);
    mbar_init(done_bar, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (threadIdx.x < kMoeMaxRanks) push_count[threadIdx.x] = 0;
  if constexpr (MODE == kMoeGateUp)
    for (int i = threadIdx.x; i <= p.E; i += blockDim.x) s_unit[i] = pv.unit_start[i];
  if (warp == 1) tmem_alloc<TMEM_COLS>(tmem_slot);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // tile t -> (m-tile index in the table, n-tile): n fastest, so one CTA's
  // consecutive tiles share the expert's A rows
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
      int waited_le = -1;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        const int ti = t / num_n, tn = t % num_n;
        const int le = pv.tile_le[ti], row0 = pv.tile_row0[ti];
        if (MODE == kMoeGateUp && le != waited_le) {
          // every row of this expert is in the local receive buffer
          if (!wait_word<true>(&p.recv_count[le], (uint32_t)pv.recv_target[le], p.err)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
          waited_le = le;
        }
        for (int kb = 0; kb < num_k; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kMxABytes + kMxBBytes + kMxSfaBytes + 2 * 512);
          tma_load_2d(&tmA, &full[stage], sA + stage * kMxABytes, kb * 128, row0);
          tma_load_2d(&tmB, &full[stage], sB + stage * kMxBBytes, kb * 128, le * p.N + tn * BN);
          bulk_load(sSFA + stage * kMxSfaBytes, p.sfa + ((size_t)(row0 >> 7) * num_k + kb) * 512, 512, &full[stage]);
#pragma unroll
          for (int c = 0; c < 2; ++c)
            bulk_load(sSFB + stage * kMxSfbBytes + c * 512,
                      p.sfb + ((size_t)(le * n_chunks_b + tn * 2 + c) * num_k + kb) * 512, 512, &full[stage]);
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
      const int ti = t / num_n, tn = t % num_n;
      const int row0 = pv.tile_row0[ti], valid = pv.tile_valid[ti];
      const int m = row0 + row;
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
      if constexpr (MODE == kMoeDown) {
        // each row: weighted by its routing weight, stored at (token, k) of its home's combine buffer
        const bool live = row < valid;
        int home = 0, item = 0;
        if (live) {
          const int2 meta = p.recv_meta[m];
          home = (int)((uint32_t)meta.x >> 28);
          item = meta.x & 0x0fffffff;
          const float w = __int_as_float(meta.y);
#pragma unroll
          for (int i = 0; i < 128; ++i) acc[i] *= w;
          atomicAdd(&push_count[home], 1);
        }
        const int n0 = tn * BN + h * 128;
        warp_push_rows(acc, rstage + ew * 8192, lane, [&](int r) -> __nv_bfloat16* {
          const int hr = __shfl_sync(0xffffffffu, home, r);
          const int ir = __shfl_sync(0xffffffffu, item, r);
          const bool lv = __shfl_sync(0xffffffffu, (int)live, r) != 0;
          return lv ? p.comb_peer[hr] + (size_t)ir * p.N + n0 : nullptr;
        });
        continue;
      }
      if (row >= valid) continue;
      {
        // gate = acc[0..63], up = acc[64..127] of outputs out0 .. out0+63
        const int out0 = tn * (BN / 2) + h * 64;
        if (p.act == 1) {
#pragma unroll
          for (int i = 0; i < 64; ++i) acc[i] = gelu_tanh_f(acc[i]) * acc[64 + i];
        } else {
#pragma unroll
          for (int i = 0; i < 64; ++i) acc[i] = silu_f(acc[i]) * acc[64 + i];
        }
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
    if constexpr (MODE == kMoeDown) {
      // every epilogue thread's stores, then one system fence (cumulative over the barrier) before the counts
      named_bar_sync(1, EPI_THREADS);
      if (warp == 2 && lane == 0) {
        __threadfence_system();
        for (int d = 0; d < p.W; ++d)
          if (push_count[d]) atomicAdd_system(p.comb_counter_peer[d], (unsigned)push_count[d]);
      }
    }
  } else if constexpr (MODE == kMoeGateUp) {
    // ------------------------------------------------------------ dispatch warps
    const int gw = blockIdx.x * 2 + (warp - 10);
    const int nw = gridDim.x * 2;
    const int units = *pv.num_units;
    const int hk = p.H / 128;       // scale words per row
    const int h16 = p.H / 16;       // 16-byte pieces per row
    for (int u = gw; u < units; u += nw) {
      // order o of this unit: the last o with unit_start[o] <= u
      int lo = 0, hi = p.E;
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_unit[mid] <= u) lo = mid; else hi = mid;
      }
      const int o = lo;
      const int d = o % p.W, le = o / p.W;
      const int e = d * p.Epr + le;
      const int j0 = (u - s_unit[o]) * kUnitRows;
      const int n = min(kUnitRows, pv.cnt_local[e] - j0);
      const int rbase = pv.send_base[e] + j0;
      const int* items = p.src_list + pv.src_off[e] + j0;
      uint8_t* dst_a = p.recv_a_peer[d];
      uint8_t* dst_sf = p.recv_sf_peer[d];
      for (int r = 0; r < n; ++r) {
        const int item = items[r];
        const int tok = item / p.topk;
        const int R = rbase + r;
        const uint4* src = reinterpret_cast<const uint4*>(p.x8 + (size_t)tok * p.H);
        uint4* dst = reinterpret_cast<uint4*>(dst_a + (size_t)R * p.H);
        for (int i = lane; i < h16; i += 32) dst[i] = src[i];
        if (lane < hk)
          *reinterpret_cast<uint32_t*>(dst_sf + sf_word_offset(R, lane, hk)) =
              *reinterpret_cast<const uint32_t*>(p.xsf + sf_word_offset(tok, lane, hk));
        if (lane == 31)
          p.recv_meta_peer[d][R] = make_int2((int)(((uint32_t)p.rank << 28) | (uint32_t)item), __float_as_int(p.wts[item]));
      }
      __syncwarp();
      if (lane == 0) {
        __threadfence_system();  // the warp's row stores (ordered by the warp barrier) before the count
        atomicAdd_system(p.recv_count_peer[d] + le, (unsigned)n);
      }
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

// ------------------------------------------------------------------ combine + norm
// One CTA of H / 8 threads per token (8 columns each): waits for all K rows of
// every token of this rank, then resid[t] += sum_k comb[t * K + k]; with a
// norm weight, also the next layer's RMSNorm of the new residual as e4m3 +
// MX scale atoms (4 threads share a 32-column scale block).
template <int H>
__global__ void __launch_bounds__(H / 8) moe_combine_kernel(const __nv_bfloat16* __restrict__ comb, int M, int K,
                                                           const uint32_t* __restrict__ counter, uint32_t want,
                                                           __nv_bfloat16* __restrict__ resid,
                                                           const __nv_bfloat16* __restrict__ w, float eps,
                                                           uint8_t* __restrict__ y8, uint8_t* __restrict__ ysf,
                                                           int* err) {
  constexpr int NT = H / 8, NW = NT / 32;
  __shared__ int go;
  __shared__ float red[NW];
  if (threadIdx.x == 0) go = wait_word<true>(counter, want, err) ? 1 : 0;
  __syncthreads();
  const int r = blockIdx.x;
  if (!go || r >= M) return;
  const int c0 = threadIdx.x * 8;
  float v[8];
  ld_bf16x8f(resid + (size_t)r * H + c0, v);
  for (int k = 0; k < K; ++k) {
    float u[8];
    ld_bf16x8f(comb + ((size_t)r * K + k) * H + c0, u);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] += u[i];
  }
  st_bf16x8(resid + (size_t)r * H + c0, v);
  if (w == nullptr) return;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = __bfloat162float(__float2bfloat16(v[i]));
    ss += v[i] * v[i];
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < NW; ++i) tot += red[i];
  const float rinv = rsqrtf(tot / H + eps);
  float wv[8];
  ld_bf16x8f(w + c0, wv);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = v[i] * rinv * wv[i];
    amax = fmaxf(amax, fabsf(v[i]));
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  const uint8_t e = ue8m0_of(amax);
  const float inv = ue8m0_inv(e);
  __nv_fp8x4_e4m3 a(make_float4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv));
  __nv_fp8x4_e4m3 b(make_float4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv));
  uint2 pk;
  pk.x = *reinterpret_cast<uint32_t*>(&a);
  pk.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(y8 + (size_t)r * H + c0) = pk;
  if ((threadIdx.x & 3) == 0) {
    const int j = c0 / 32;
    ysf[((size_t)(r >> 7) * (H / 128) + (j >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (j & 3)] = e;
  }
}

// ------------------------------------------------------------------ host side

static int* i32(const torch::Tensor& t) { return t.data_ptr<int>(); }

void moe_route(const torch::Tensor& logits, int64_t E, int64_t topk, torch::Tensor& ids, torch::Tensor& wts,
               torch::Tensor& pos, torch::Tensor& counts) {
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(1) == 1, "moe_route: bf16 logits");
  TORCH_CHECK(E <= kMoeMaxExperts && topk <= 32 && topk <= E, "moe_route: E <= 256, top-k <= 32");
  const int M = logits.size(0);
  TORCH_CHECK(ids.numel() >= M * topk && wts.numel() >= M * topk && pos.numel() >= M * topk && counts.numel() >= E,
              "moe_route: output sizes");
  if (M == 0) return;
  const int dev = logits.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  moe_route_kernel<<<(M + 7) / 8, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()),
                                                (int)logits.stride(0), M, (int)E, (int)topk, i32(ids),
                                                wts.data_ptr<float>(), i32(pos), i32(counts));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t moe_plan_ints(int64_t E, int64_t Epr, int64_t tcap) { return plan_ints((int)E, (int)Epr, (int)tcap); }

void moe_plan(torch::Tensor& counts, const std::vector<int64_t>& counts_all_peer,
              const std::vector<int64_t>& cflag_peer, const torch::Tensor& counts_all_local,
              const torch::Tensor& cflag_local, torch::Tensor& plan, torch::Tensor& cum, int64_t rank, int64_t E,
              int64_t tcap, int64_t epoch) {
  const int W = std::max<int>(1, (int)counts_all_peer.size());
  TORCH_CHECK(W <= kMoeMaxRanks && E % W == 0 && E <= kMoeMaxExperts, "moe_plan: ranks / experts");
  TORCH_CHECK(plan.numel() >= plan_ints((int)E, (int)E / W, (int)tcap) && cum.numel() >= E / W, "moe_plan: sizes");
  const int dev = counts.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  PlanParams p{};
  p.counts = i32(counts);
  for (int i = 0; i < kMoeMaxRanks; ++i) {
    p.counts_all_peer[i] = i < (int)counts_all_peer.size() ? reinterpret_cast<int*>(counts_all_peer[i]) : nullptr;
    p.cflag_peer[i] = i < (int)cflag_peer.size() ? reinterpret_cast<uint32_t*>(cflag_peer[i]) : nullptr;
  }
  p.counts_all_local = W > 1 ? i32(counts_all_local) : nullptr;
  p.cflag_local = W > 1 ? reinterpret_cast<const uint32_t*>(cflag_local.data_ptr<int>()) : nullptr;
  p.plan = i32(plan);
  p.cum = i32(cum);
  p.rank = (int)rank;
  p.W = W;
  p.E = (int)E;
  p.Epr = (int)E / W;
  p.tcap = (int)tcap;
  p.epoch = (uint32_t)epoch;
  p.err = device_error_word(dev);
  moe_plan_kernel<<<1, 256, 0, st>>>(p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_sort(const torch::Tensor& ids, const torch::Tensor& pos, int64_t n, const torch::Tensor& plan, int64_t E,
              torch::Tensor& src_list) {
  if (n == 0) return;
  const int dev = ids.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  moe_sort_kernel<<<(n + 255) / 256, 256, 0, st>>>(i32(ids), i32(pos), (int)n, i32(plan) + 8 + E, i32(src_list));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int MODE>
static void launch_moe(const CUtensorMap& ta, const CUtensorMap& tb, MoeGemmParams& p, int grid, cudaStream_t st,
                       int dev) {
  constexpr int smem = MODE == kMoeDown ? mx_pipeline_smem(3) + kMoeExtraSmem + 128 + 8 * 8192
                                       : kMxSmem + kMoeExtraSmem;
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(moe_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev] = true;
  }
  moe_gemm_kernel<MODE><<<grid, kMoeThreads, smem, st>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static void fill_peers(const std::vector<int64_t>& v, uint8_t** out) {
  for (int i = 0; i < kMoeMaxRanks; ++i) out[i] = i < (int)v.size() ? reinterpret_cast<uint8_t*>(v[i]) : nullptr;
}

// Dispatch fused into the grouped gate_up GEMM.
// x8 [M, H] e4m3 + xsf atoms: this rank's normalized tokens. recv_a / recv_sf /
// recv_count: this rank's receive buffer (the TMA source), peers' by pointer.
// w_gu [Epr * 2I, H] e4m3 (per-expert gate/up rows interleaved for SwiGLU) + atoms.
// y [Rcap, I] e4m3 + ysf atoms: SwiGLU outputs in receive-buffer row order.
void moe_gate_up(const torch::Tensor& x8, const torch::Tensor& xsf, const torch::Tensor& src_list,
                 const torch::Tensor& wts, const torch::Tensor& plan, int64_t rank, int64_t E, int64_t topk,
                 int64_t tcap, const std::vector<int64_t>& recv_a_peer, const std::vector<int64_t>& recv_sf_peer,
                 const std::vector<int64_t>& recv_meta_peer, const std::vector<int64_t>& recv_count_peer,
                 const torch::Tensor& recv_a, const torch::Tensor& recv_sf, const torch::Tensor& recv_count,
                 const torch::Tensor& w_gu, const torch::Tensor& s_gu, torch::Tensor& y, torch::Tensor& ysf,
                 int64_t act) {
  const int W = (int)recv_a_peer.size();
  const int H = x8.size(1), N = w_gu.size(0) / (E / W), Rcap = recv_a.size(0);
  TORCH_CHECK(W >= 1 && W <= kMoeMaxRanks && E % W == 0, "moe_gate_up: ranks");
  TORCH_CHECK(H % 128 == 0 && H <= 8192 && N % kMxBN == 0 && recv_a.size(1) == H && w_gu.size(1) == H,
              "moe_gate_up: H % 128, 2I % 256");
  TORCH_CHECK(y.size(0) == Rcap && y.size(1) == N / 2 && y.stride(0) % 16 == 0, "moe_gate_up: y [Rcap, I]");
  TORCH_CHECK(Rcap >= tcap * 128, "moe_gate_up: receive rows >= 128 x tile capacity");
  const int dev = x8.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  MoeGemmParams p{};
  p.N = N;
  p.K = H;
  p.H = H;
  p.topk = (int)topk;
  p.rank = (int)rank;
  p.W = W;
  p.E = (int)E;
  p.Epr = (int)E / W;
  p.tcap = (int)tcap;
  p.act = (int)act;
  p.plan = i32(plan);
  p.x8 = reinterpret_cast<const uint8_t*>(x8.data_ptr());
  p.xsf = xsf.data_ptr<uint8_t>();
  p.src_list = i32(src_list);
  p.wts = wts.data_ptr<float>();
  fill_peers(recv_a_peer, p.recv_a_peer);
  fill_peers(recv_sf_peer, p.recv_sf_peer);
  for (int i = 0; i < kMoeMaxRanks; ++i) {
    p.recv_meta_peer[i] = i < W ? reinterpret_cast<int2*>(recv_meta_peer[i]) : nullptr;
    p.recv_count_peer[i] = i < W ? reinterpret_cast<uint32_t*>(recv_count_peer[i]) : nullptr;
  }
  p.recv_count = reinterpret_cast<const uint32_t*>(recv_count.data_ptr<int>());
  p.sfa = recv_sf.data_ptr<uint8_t>();
  p.sfb = s_gu.data_ptr<uint8_t>();
  p.Y = reinterpret_cast<uint8_t*>(y.data_ptr());
  p.Ysf = ysf.data_ptr<uint8_t>();
  p.ldy = y.stride(0);
  p.err = device_error_word(dev);
  CUtensorMap ta = make_tmap_2d(recv_a.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, H, Rcap, recv_a.stride(0), 128,
                                128, CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(w_gu.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, H, w_gu.size(0), w_gu.stride(0), 128,
                                kMxBN, CU_TENSOR_MAP_SWIZZLE_128B);
  // every CTA dispatches, so the grid is the whole GPU (one CTA per SM, all resident)
  launch_moe<kMoeGateUp>(ta, tb, p, num_sms(dev), st, dev);
}

// Combine fused into the grouped down GEMM epilogue.
// y [Rcap, I] e4m3 + ysf; w_d [Epr * H, I] e4m3 + atoms; comb_peer: each
// rank's combine buffer [M_home * topk, H] bf16; comb_counter_peer: their counters.
void moe_down(const torch::Tensor& y, const torch::Tensor& ysf, const torch::Tensor& plan, int64_t E, int64_t tcap,
              const torch::Tensor& recv_meta, const torch::Tensor& w_d, const torch::Tensor& s_d,
              const std::vector<int64_t>& comb_peer, const std::vector<int64_t>& comb_counter_peer) {
  const int W = (int)comb_peer.size();
  const int I = y.size(1), Rcap = y.size(0), H = w_d.size(0) / (E / W);
  TORCH_CHECK(W >= 1 && W <= kMoeMaxRanks && E % W == 0, "moe_down: ranks");
  TORCH_CHECK(I % 128 == 0 && H % kMxBN == 0 && w_d.size(1) == I, "moe_down: I % 128, H % 256");
  const int dev = y.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  MoeGemmParams p{};
  p.N = H;
  p.K = I;
  p.H = H;
  p.W = W;
  p.E = (int)E;
  p.Epr = (int)E / W;
  p.tcap = (int)tcap;
  p.plan = i32(plan);
  p.sfa = ysf.data_ptr<uint8_t>();
  p.sfb = s_d.data_ptr<uint8_t>();
  p.recv_meta = reinterpret_cast<const int2*>(recv_meta.data_ptr());
  for (int i = 0; i < kMoeMaxRanks; ++i) {
    p.comb_peer[i] = i < W ? reinterpret_cast<__nv_bfloat16*>(comb_peer[i]) : nullptr;
    p.comb_counter_peer[i] = i < W ? reinterpret_cast<uint32_t*>(comb_counter_peer[i]) : nullptr;
  }
  p.err = device_error_word(dev);
  CUtensorMap ta = make_tmap_2d(y.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, I, Rcap, y.stride(0), 128, 128,
                                CU_TENSOR_MAP_SWIZZLE_128B);
  CUtensorMap tb = make_tmap_2d(w_d.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, I, w_d.size(0), w_d.stride(0), 128,
                                kMxBN, CU_TENSOR_MAP_SWIZZLE_128B);
  launch_moe<kMoeDown>(ta, tb, p, num_sms(dev), st, dev);
}

void moe_combine(const torch::Tensor& comb, int64_t M, int64_t topk, const torch::Tensor& counter, int64_t want,
                 torch::Tensor& resid, const c10::optional<torch::Tensor>& w, double eps,
                 const c10::optional<torch::Tensor>& y8, const c10::optional<torch::Tensor>& ysf) {
  const int H = resid.size(1);
  TORCH_CHECK(resid.scalar_type() == at::kBFloat16 && resid.is_contiguous() && resid.size(0) >= M, "moe_combine: resid");
  TORCH_CHECK(!w.has_value() || (y8.has_value() && ysf.has_value()), "moe_combine: norm outputs");
  if (M == 0) return;
  const int dev = resid.get_device();
  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t st = at::cuda::getCurrentCUDAStream(dev);
  auto cp = reinterpret_cast<const __nv_bfloat16*>(comb.data_ptr());
  auto wp = w.has_value() ? reinterpret_cast<const __nv_bfloat16*>(w->data_ptr()) : nullptr;
  uint8_t* yp = y8.has_value() ? reinterpret_cast<uint8_t*>(y8->data_ptr()) : nullptr;
  uint8_t* sp = ysf.has_value() ? ysf->data_ptr<uint8_t>() : nullptr;
#define QB_MOE_CASE(HH)                                                                                      \
  if (H == HH) {                                                                                             \
    moe_combine_kernel<HH><<<(int)M, HH / 8, 0, st>>>(                                                     \
        cp, (int)M, (int)topk, reinterpret_cast<const uint32_t*>(counter.data_ptr<int>()), (uint32_t)want,  \
        reinterpret_cast<__nv_bfloat16*>(resid.data_ptr()), wp, (float)eps, yp, sp, device_error_word(dev)); \
    C10_CUDA_KERNEL_LAUNCH_CHECK();                                                                          \
    return;                                                                                                  \
  }
  QB_MOE_CASE(1024)
  QB_MOE_CASE(2048)
  QB_MOE_CASE(2816)
  QB_MOE_CASE(4096)
#undef QB_MOE_CASE
  TORCH_CHECK(false, "moe_combine: unsupported hidden size ", H);
}

}  // namespace qb
