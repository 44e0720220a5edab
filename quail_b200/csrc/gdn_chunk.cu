// K13b: the Gated DeltaNet recurrence in 64-token chunks on the tensor cores.
//
// Per token the rule is (state S: d_k x d_v, fp32; a = exp(g) the decay):
//   S <- a S;  u = beta (v - S^T k);  S <- S + k u^T;  o = S^T q
// Within a chunk of C tokens entering with state S0, write G_i for the
// cumulative log decay (G_i = g_1 + ... + g_i) and gamma_i = exp(G_i). By
// induction S_i = gamma_i S0 + sum_{j<=i} exp(G_i - G_j) k_j u_j^T, so the
// chunk's u rows solve one lower-triangular system:
//   (I + A) U = diag(beta) (V - diag(gamma) K S0),
//   A_ij = beta_i exp(G_i - G_j) k_i.k_j   (j < i, else 0)
// Splitting the right-hand side, U = U~ - W S0 with
//   [W | U~] = (I + A)^-1 [diag(beta gamma) K | diag(beta) V],
// and then
//   O    = diag(gamma) Q S0 + (M o Q K^T) U,   M_ij = exp(G_i - G_j) (j <= i)
//   S_C  = gamma_C S0 + K^T diag(exp(G_C - G_j)) U.
// (The derivation is this file's own, from the recurrence above.)
//
// One CTA of 8 warps per (sequence, value head) walks the sequence's chunks:
//   load    q, k rows -> bf16 tiles; gates -> log decay g and beta; G by a warp scan
//   mma     K K^T and Q K^T (64 x 64, k = 128)  -> A (fp32) and M o QK^T (bf16)
//   solve   (I + A) X = R by forward substitution, one thread per column of
//           R (256 columns: W's 128 and U~'s 128), X in registers, A rows read
//           as broadcasts; no barrier inside
//   mma     U = U~ + (-W) S0 and Q S0 (k = d_k), then O += (M o QK^T) U (k = 64)
//   mma     S = gamma_C S + K^T Us   (Us = U rows scaled by exp(G_C - G_j));
//           each warp keeps 16 rows of S in fp32 accumulator registers
// The tensor-core operands are bf16 (S0 is rounded to bf16 for the products;
// the state itself accumulates in fp32); every mma is m16n8k16 with fp32
// accumulation, operands through ldmatrix from padded shared-memory rows.
//
// Only d_k = d_v = 128 (every Qwen3.5 / 3.6 / 3.8 spec). Reference: the
// reference runs the chunked form through FLA's Triton kernels
// (quail/backends/quail/executor/gdn.py:27-1088).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace qb {

namespace {

constexpr int kCh = 64;            // tokens per chunk
constexpr int kD = 128;            // d_k = d_v
constexpr int kP = kD + 8;         // bf16 pitch of [*][128] tiles (272 B rows)
constexpr int kPm = kCh + 8;       // bf16 pitch of the [64][64] tile (144 B rows)
constexpr int kPa = kCh + 4;       // fp32 pitch of A (68: float4-aligned rows)
constexpr int kPu = kD + 4;        // fp32 pitch of U~
constexpr int kChSeqInts = 12;

struct GcSmem {
  static constexpr int Q = 0;                       // bf16 [64][kP]
  static constexpr int K = Q + kCh * kP * 2;        // bf16 [64][kP]
  static constexpr int S = K + kCh * kP * 2;        // bf16 [128][kP] S0, [d_k][d_v]
  static constexpr int W = S + kD * kP * 2;         // bf16 [64][kP] -W
  static constexpr int U = W + kCh * kP * 2;        // bf16 [64][kP]
  static constexpr int Us = U + kCh * kP * 2;       // bf16 [64][kP] decayed U
  static constexpr int M = Us + kCh * kP * 2;       // bf16 [64][kPm] masked decayed Q K^T
  static constexpr int A = M + kCh * kPm * 2;       // fp32 [64][kPa]
  static constexpr int Ut = A + kCh * kPa * 4;      // fp32 [64][kPu] U~
  static constexpr int G = Ut + kCh * kPu * 4;      // fp32 [64] cumulative log decay
  static constexpr int B = G + kCh * 4;             // fp32 [64] beta
  static constexpr int BYTES = B + kCh * 4;
};

__device__ __forceinline__ void gc_ldsm4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void gc_ldsm4t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void gc_mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t gc_pack(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Fragment addresses (lane l) for a 16x16 A tile at (m0, k0) and a pair of
// 16x8 B tiles at (k0, n0), n0 + 8, by how the operand is stored:
//   A from [M][K] rows:  row m0 + (l & 15),               col k0 + (l >> 4) * 8
//   A from [K][M] rows:  row k0 + (l & 7) + (l >> 4) * 8, col m0 + ((l >> 3) & 1) * 8  (.trans)
//   B from [N][K] rows:  row n0 + (l & 7) + (l >> 4) * 8, col k0 + ((l >> 3) & 1) * 8
//   B from [K][N] rows:  row k0 + (l & 7) + ((l >> 3) & 1) * 8, col n0 + (l >> 4) * 8  (.trans)
// The B forms return {b0, b1} of tile n0 then {b0, b1} of tile n0 + 8.
__device__ __forceinline__ uint32_t a_rows(uint32_t base, int pitch, int m0, int k0, int l) {
  return base + (m0 + (l & 15)) * pitch + (k0 + (l >> 4) * 8) * 2;
}
__device__ __forceinline__ uint32_t a_cols(uint32_t base, int pitch, int m0, int k0, int l) {
  return base + (k0 + (l & 7) + (l >> 4) * 8) * pitch + (m0 + ((l >> 3) & 1) * 8) * 2;
}
__device__ __forceinline__ uint32_t b_rows(uint32_t base, int pitch, int n0, int k0, int l) {
  return base + (n0 + (l & 7) + (l >> 4) * 8) * pitch + (k0 + ((l >> 3) & 1) * 8) * 2;
}
__device__ __forceinline__ uint32_t b_cols(uint32_t base, int pitch, int n0, int k0, int l) {
  return base + (k0 + (l & 7) + ((l >> 3) & 1) * 8) * pitch + (n0 + (l >> 4) * 8) * 2;
}

// conv_out fp32 [T, C]: q at hk*128, k at qk/2 + hk*128, v at qk + h*128.
// ab bf16 [T, ldab]: b at b_col + h, a at a_col + h. out fp32 [T, Hv*128].
__global__ void __launch_bounds__(256, 1) gdn_chunk_kernel(
    const float* __restrict__ conv_out, int C, int qk_channels, const __nv_bfloat16* __restrict__ ab, int ldab,
    int b_col, int a_col, const float* __restrict__ A_log, const float* __restrict__ dt_bias, int Hv, int Hk,
    const int* __restrict__ seqs, const int* __restrict__ sio, float* __restrict__ ssm_state, int gi, int G,
    float* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16* sW = reinterpret_cast<__nv_bfloat16*>(smem + GcSmem::W);
  float* sA = reinterpret_cast<float*>(smem + GcSmem::A);
  float* sUt = reinterpret_cast<float*>(smem + GcSmem::Ut);
  float* sG = reinterpret_cast<float*>(smem + GcSmem::G);
  float* sB = reinterpret_cast<float*>(smem + GcSmem::B);
  const uint32_t base = smem_u32(smem);
  const uint32_t aQ = base + GcSmem::Q, aK = base + GcSmem::K, aS = base + GcSmem::S, aW = base + GcSmem::W;
  const uint32_t aU = base + GcSmem::U, aUs = base + GcSmem::Us, aM = base + GcSmem::M;
  constexpr int P2 = kP * 2, Pm2 = kPm * 2;

  const int s = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, t4 = lane & 3;
  const int hk = h / (Hv / Hk);
  const int q0 = seqs[s * kChSeqInts], n = seqs[s * kChSeqInts + 1];
  const int src = sio[2 * s], dst = sio[2 * s + 1];
  const size_t slot_stride = (size_t)G * Hv * kD * kD;
  const size_t head_off = ((size_t)gi * Hv + h) * kD * kD;
  const float Aexp = -__expf(A_log[h]);
  const float dtb = dt_bias[h];
  const int kofs = qk_channels / 2 + hk * kD, qofs = hk * kD, vofs = qk_channels + h * kD;

  // state: warp w owns rows [16w, 16w + 16) of S, all 128 columns (16 n-tiles)
  float Sacc[16][4];
  const int r_lo = 16 * warp + g, r_hi = r_lo + 8;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = nt * 8 + 2 * t4;
    if (src >= 0) {
      const float* S0 = ssm_state + (size_t)src * slot_stride + head_off;
      const float2 lo = *reinterpret_cast<const float2*>(S0 + (size_t)r_lo * kD + c);
      const float2 hi = *reinterpret_cast<const float2*>(S0 + (size_t)r_hi * kD + c);
      Sacc[nt][0] = lo.x; Sacc[nt][1] = lo.y; Sacc[nt][2] = hi.x; Sacc[nt][3] = hi.y;
    } else {
      Sacc[nt][0] = Sacc[nt][1] = Sacc[nt][2] = Sacc[nt][3] = 0.f;
    }
  }
  auto store_state_bf16 = [&]() {
    uint32_t* sS32 = reinterpret_cast<uint32_t*>(smem + GcSmem::S);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int c = nt * 8 + 2 * t4;
      sS32[(r_lo * kP + c) >> 1] = gc_pack(Sacc[nt][0], Sacc[nt][1]);
      sS32[(r_hi * kP + c) >> 1] = gc_pack(Sacc[nt][2], Sacc[nt][3]);
    }
  };
  store_state_bf16();

  const int mt = warp & 3;       // phases 1, 3, 4: the warp's 16 rows of the chunk
  const int nh = warp >> 2;      // and its half of the columns

  for (int c0 = 0; c0 < n; c0 += kCh) {
    const int cn = min(kCh, n - c0);
    // ---- load q, k (bf16) and the gates
    for (int idx = tid; idx < kCh * (kD / 4); idx += 256) {
      const int row = idx >> 5, col = (idx & 31) * 4;
      float4 q = make_float4(0.f, 0.f, 0.f, 0.f), k = q;
      if (row < cn) {
        const float* r = conv_out + (size_t)(q0 + c0 + row) * C;
        q = *reinterpret_cast<const float4*>(r + qofs + col);
        k = *reinterpret_cast<const float4*>(r + kofs + col);
      }
      uint32_t* dq = reinterpret_cast<uint32_t*>(smem + GcSmem::Q + row * P2 + col * 2);
      uint32_t* dk = reinterpret_cast<uint32_t*>(smem + GcSmem::K + row * P2 + col * 2);
      dq[0] = gc_pack(q.x, q.y);
      dq[1] = gc_pack(q.z, q.w);
      dk[0] = gc_pack(k.x, k.y);
      dk[1] = gc_pack(k.z, k.w);
    }
    if (tid < kCh) {
      float gl = 0.f, beta = 0.f;
      if (tid < cn) {
        const size_t r = (size_t)(q0 + c0 + tid) * ldab;
        const float a = __bfloat162float(ab[r + a_col + h]) + dtb;
        const float sp = a > 20.f ? a : log1pf(__expf(a));  // softplus
        gl = Aexp * sp;                                      // log decay, <= 0
        const float b = __bfloat162float(ab[r + b_col + h]);
        beta = 1.f / (1.f + __expf(-b));
      }
      sG[tid] = gl;
      sB[tid] = beta;
    }
    __syncthreads();
    if (warp == 0) {
      // inclusive prefix sum of the log decays, two per lane
      const float x0 = sG[2 * lane], x1 = sG[2 * lane + 1];
      float p = x0 + x1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, p, o);
        if (lane >= o) p += y;
      }
      const float excl = p - (x0 + x1);
      sG[2 * lane] = excl + x0;
      sG[2 * lane + 1] = excl + x0 + x1;
    }
    __syncthreads();

    // ---- K K^T and Q K^T: rows 16 mt.., columns 32 nh.. (4 n-tiles)
    {
      float accP[4][4], accQ[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) accP[i][e] = accQ[i][e] = 0.f;
#pragma unroll
      for (int k0 = 0; k0 < kD; k0 += 16) {
        uint32_t ak[4], aq[4];
        gc_ldsm4(a_rows(aK, P2, 16 * mt, k0, lane), ak);
        gc_ldsm4(a_rows(aQ, P2, 16 * mt, k0, lane), aq);
#pragma unroll
        for (int np = 0; np < 2; ++np) {
          uint32_t b[4];
          gc_ldsm4(b_rows(aK, P2, 32 * nh + 16 * np, k0, lane), b);
          gc_mma(accP[2 * np], ak, b[0], b[1]);
          gc_mma(accP[2 * np + 1], ak, b[2], b[3]);
          gc_mma(accQ[2 * np], aq, b[0], b[1]);
          gc_mma(accQ[2 * np + 1], aq, b[2], b[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int i = 16 * mt + g + 8 * hf;
          const int j = 32 * nh + 8 * nt + 2 * t4;
          const float gi_ = sG[i], bi = sB[i];
          const float d0 = j <= i ? __expf(gi_ - sG[j]) : 0.f;
          const float d1 = j + 1 <= i ? __expf(gi_ - sG[j + 1]) : 0.f;
          sA[i * kPa + j] = j < i ? bi * d0 * accP[nt][2 * hf] : 0.f;
          sA[i * kPa + j + 1] = j + 1 < i ? bi * d1 * accP[nt][2 * hf + 1] : 0.f;
          *reinterpret_cast<uint32_t*>(smem + GcSmem::M + i * Pm2 + j * 2) =
              gc_pack(d0 * accQ[nt][2 * hf], d1 * accQ[nt][2 * hf + 1]);
        }
    }
    __syncthreads();

    // ---- (I + A) X = R, one thread per column: X = [W | U~]
    {
      const int col = tid;
      const bool kside = col < kD;
      const int gofs = kside ? kofs + col : vofs + (col - kD);
      float x[kCh];
#pragma unroll
      for (int i = 0; i < kCh; ++i) x[i] = 0.f;
#pragma unroll
      for (int i = 0; i < kCh; ++i) {
        float r = 0.f;
        if (i < cn) {
          const float v = conv_out[(size_t)(q0 + c0 + i) * C + gofs];
          r = sB[i] * (kside ? __expf(sG[i]) : 1.f) * v;
        }
        const float4* arow = reinterpret_cast<const float4*>(sA + i * kPa);
#pragma unroll
        for (int j4 = 0; j4 < (i + 3) / 4; ++j4) {
          const float4 a = arow[j4];
          r -= a.x * x[4 * j4] + a.y * x[4 * j4 + 1] + a.z * x[4 * j4 + 2] + a.w * x[4 * j4 + 3];
        }
        x[i] = r;
      }
      if (kside) {
#pragma unroll
        for (int i = 0; i < kCh; ++i) sW[i * kP + col] = __float2bfloat16(-x[i]);
      } else {
#pragma unroll
        for (int i = 0; i < kCh; ++i) sUt[i * kPu + (col - kD)] = x[i];
      }
    }
    __syncthreads();

    // ---- U = U~ + (-W) S0 and Oq = Q S0: rows 16 mt.., columns 64 nh.. (8 n-tiles)
    float accO[8][4];
    {
      float accU[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int c = 64 * nh + 8 * nt + 2 * t4;
        const int i0 = 16 * mt + g;
        accU[nt][0] = sUt[i0 * kPu + c];
        accU[nt][1] = sUt[i0 * kPu + c + 1];
        accU[nt][2] = sUt[(i0 + 8) * kPu + c];
        accU[nt][3] = sUt[(i0 + 8) * kPu + c + 1];
        accO[nt][0] = accO[nt][1] = accO[nt][2] = accO[nt][3] = 0.f;
      }
#pragma unroll
      for (int k0 = 0; k0 < kD; k0 += 16) {
        uint32_t aw[4], aq[4];
        gc_ldsm4(a_rows(aW, P2, 16 * mt, k0, lane), aw);
        gc_ldsm4(a_rows(aQ, P2, 16 * mt, k0, lane), aq);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b[4];
          gc_ldsm4t(b_cols(aS, P2, 64 * nh + 16 * np, k0, lane), b);
          gc_mma(accU[2 * np], aw, b[0], b[1]);
          gc_mma(accU[2 * np + 1], aw, b[2], b[3]);
          gc_mma(accO[2 * np], aq, b[0], b[1]);
          gc_mma(accO[2 * np + 1], aq, b[2], b[3]);
        }
      }
      const float Gl = sG[kCh - 1];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int i = 16 * mt + g + 8 * hf;
        const float gam = __expf(sG[i]), tail = __expf(Gl - sG[i]);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int c = 64 * nh + 8 * nt + 2 * t4;
          const float u0 = accU[nt][2 * hf], u1 = accU[nt][2 * hf + 1];
          *reinterpret_cast<uint32_t*>(smem + GcSmem::U + i * P2 + c * 2) = gc_pack(u0, u1);
          *reinterpret_cast<uint32_t*>(smem + GcSmem::Us + i * P2 + c * 2) = gc_pack(tail * u0, tail * u1);
          accO[nt][2 * hf] *= gam;
          accO[nt][2 * hf + 1] *= gam;
        }
      }
    }
    __syncthreads();

    // ---- O += (M o Q K^T) U, then the chunk's output rows
#pragma unroll
    for (int k0 = 0; k0 < kCh; k0 += 16) {
      uint32_t am[4];
      gc_ldsm4(a_rows(aM, Pm2, 16 * mt, k0, lane), am);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        gc_ldsm4t(b_cols(aU, P2, 64 * nh + 16 * np, k0, lane), b);
        gc_mma(accO[2 * np], am, b[0], b[1]);
        gc_mma(accO[2 * np + 1], am, b[2], b[3]);
      }
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int i = 16 * mt + g + 8 * hf;
      if (i < cn) {
        float* orow = out + (size_t)(q0 + c0 + i) * Hv * kD + h * kD;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int c = 64 * nh + 8 * nt + 2 * t4;
          *reinterpret_cast<float2*>(orow + c) = make_float2(accO[nt][2 * hf], accO[nt][2 * hf + 1]);
        }
      }
    }

    // ---- S = gamma_C S + K^T Us: the warp's rows 16 w.. of d_k, all of d_v
    {
      const float gC = __expf(sG[kCh - 1]);
#pragma unroll
      for (int nt = 0; nt < 16; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) Sacc[nt][e] *= gC;
#pragma unroll
      for (int k0 = 0; k0 < kCh; k0 += 16) {
        uint32_t ak[4];
        gc_ldsm4t(a_cols(aK, P2, 16 * warp, k0, lane), ak);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t b[4];
          gc_ldsm4t(b_cols(aUs, P2, 16 * np, k0, lane), b);
          gc_mma(Sacc[2 * np], ak, b[0], b[1]);
          gc_mma(Sacc[2 * np + 1], ak, b[2], b[3]);
        }
      }
      store_state_bf16();   // S0 of the next chunk; phase 3 (its only reader) is behind a barrier
    }
    __syncthreads();
  }
  if (dst < 0) return;   // the state is not kept
  float* Sd = ssm_state + (size_t)dst * slot_stride + head_off;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = nt * 8 + 2 * t4;
    *reinterpret_cast<float2*>(Sd + (size_t)r_lo * kD + c) = make_float2(Sacc[nt][0], Sacc[nt][1]);
    *reinterpret_cast<float2*>(Sd + (size_t)r_hi * kD + c) = make_float2(Sacc[nt][2], Sacc[nt][3]);
  }
}

// ------------------------------------------------------------------ split form
// The same algebra in two kernels, so the state-free work (gates, K K^T, Q K^T,
// the triangular solve) runs in parallel over every chunk of the pass:
//   gdn_chunk_index   the pass's chunk list (sequence, first token) and each
//                     sequence's first chunk, by a block-wide scan
//   gdn_conv_chunk    the causal conv, token-parallel, into a bf16 [T, C] buffer
//                     that the two kernels below read (q, k, v rows)
//   gdn_chunk_prep    one CTA per (chunk, value head): writes the chunk's record
//                     -W, U~ (bf16 [64][128]), M o QK^T (bf16 [64][64]), G (fp32 [64])
//   gdn_chunk_scan    one CTA per (sequence, value head): walks the records with
//                     the state: U = U~ + (-W) S0, O, S update (as above); the
//                     next record streams into shared memory (cp.async, two
//                     buffers) while the current one is in the tensor cores
constexpr int kRecW = 0;                      // bf16 [64][128] -W
constexpr int kRecU = kRecW + kCh * kD * 2;   // bf16 [64][128] U~
constexpr int kRecM = kRecU + kCh * kD * 2;   // bf16 [64][64] M o QK^T
constexpr int kRecG = kRecM + kCh * kCh * 2;  // fp32 [64] G
constexpr int kRecBytes = kRecG + kCh * 4;    // 41,216 B = 161 x 256
static_assert(kRecBytes % 256 == 0, "records stay 256-byte aligned");

// ws ints: [0] chunk count, [4, 4 + 2 maxc) the (sequence, first token) list,
// then first[S] (each sequence's first chunk index), then order[S]: the
// sequences by chunk count, most first (the scan kernel's CTAs start the
// longest sequences first, so short ones fill in behind them)
__device__ __forceinline__ void gc_block_scan256(int* v, int* total) {
  // exclusive scan of 256 shared ints by warp 0 (8 per lane)
  const int t = threadIdx.x;
  if (t < 32) {
    int x[8], sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] = v[t * 8 + i];
      sum += x[i];
    }
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (t >= o) incl += y;
    }
    int run = incl - sum;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[t * 8 + i] = run;
      run += x[i];
    }
    if (t == 31 && total) *total = incl;
  }
}

__global__ void __launch_bounds__(256) gdn_chunk_index_kernel(const int* __restrict__ seqs, int S, int maxc,
                                                              int* __restrict__ ws) {
  __shared__ int part[256], hist[256];
  const int t = threadIdx.x, per = (S + 255) / 256;
  const int a = min(S, t * per), b = min(S, a + per);
  hist[t] = 0;
  __syncthreads();
  int cnt = 0;
  for (int s = a; s < b; ++s) {
    const int c = (seqs[s * kChSeqInts + 1] + kCh - 1) / kCh;
    cnt += c;
    atomicAdd(&hist[255 - min(c, 255)], 1);
  }
  part[t] = cnt;
  __syncthreads();
  gc_block_scan256(hist, nullptr);
  __syncthreads();
  int* order = ws + 4 + 2 * maxc + S;
  for (int s = a; s < b; ++s) {
    const int c = (seqs[s * kChSeqInts + 1] + kCh - 1) / kCh;
    order[atomicAdd(&hist[255 - min(c, 255)], 1)] = s;
  }
  gc_block_scan256(part, ws);
  __syncthreads();
  int off = part[t];
  int2* list = reinterpret_cast<int2*>(ws + 4);
  int* first = ws + 4 + 2 * maxc;
  for (int s = a; s < b; ++s) {
    const int n = seqs[s * kChSeqInts + 1];
    first[s] = off;
    for (int c0 = 0; c0 < n; c0 += kCh) list[off++] = make_int2(s, c0);
  }
}

struct GpSmem {
  static constexpr int Q = 0;
  static constexpr int K = Q + kCh * kP * 2;
  static constexpr int V = K + kCh * kP * 2;        // bf16 [64][kP]: the solve's right-hand side
  static constexpr int A = V + kCh * kP * 2;
  static constexpr int G = A + kCh * kPa * 4;
  static constexpr int B = G + kCh * 4;
  static constexpr int BYTES = B + kCh * 4;
};

__global__ void __launch_bounds__(256, 2) gdn_chunk_prep_kernel(
    const __nv_bfloat16* __restrict__ cv, int C, int qk_channels, const __nv_bfloat16* __restrict__ ab, int ldab,
    int b_col, int a_col, const float* __restrict__ A_log, const float* __restrict__ dt_bias, int Hv, int Hk,
    const int* __restrict__ seqs, const int* __restrict__ ws, uint8_t* __restrict__ recs) {
  const int ci = blockIdx.x, h = blockIdx.y;
  if (ci >= ws[0]) return;
  extern __shared__ __align__(16) uint8_t smem[];
  float* sA = reinterpret_cast<float*>(smem + GpSmem::A);
  float* sG = reinterpret_cast<float*>(smem + GpSmem::G);
  float* sB = reinterpret_cast<float*>(smem + GpSmem::B);
  const uint32_t base = smem_u32(smem);
  const uint32_t aQ = base + GpSmem::Q, aK = base + GpSmem::K;
  constexpr int P2 = kP * 2;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t4 = lane & 3;
  const int2 e = reinterpret_cast<const int2*>(ws + 4)[ci];
  const int s = e.x, c0 = e.y;
  const int q0 = seqs[s * kChSeqInts], n = seqs[s * kChSeqInts + 1];
  const int cn = min(kCh, n - c0);
  const int hk = h / (Hv / Hk);
  const int kofs = qk_channels / 2 + hk * kD, qofs = hk * kD, vofs = qk_channels + h * kD;
  uint8_t* rec = recs + ((size_t)ci * Hv + h) * kRecBytes;

  for (int idx = tid; idx < kCh * (kD / 8); idx += 256) {
    const int row = idx >> 4, col = (idx & 15) * 8;
    uint4 q = make_uint4(0, 0, 0, 0), k = q, v = q;
    if (row < cn) {
      const __nv_bfloat16* r = cv + (size_t)(q0 + c0 + row) * C;
      q = *reinterpret_cast<const uint4*>(r + qofs + col);
      k = *reinterpret_cast<const uint4*>(r + kofs + col);
      v = *reinterpret_cast<const uint4*>(r + vofs + col);
    }
    *reinterpret_cast<uint4*>(smem + GpSmem::Q + row * P2 + col * 2) = q;
    *reinterpret_cast<uint4*>(smem + GpSmem::K + row * P2 + col * 2) = k;
    *reinterpret_cast<uint4*>(smem + GpSmem::V + row * P2 + col * 2) = v;
  }
  if (tid < kCh) {
    float gl = 0.f, beta = 0.f;
    if (tid < cn) {
      const size_t r = (size_t)(q0 + c0 + tid) * ldab;
      const float a = __bfloat162float(ab[r + a_col + h]) + dt_bias[h];
      const float sp = a > 20.f ? a : log1pf(__expf(a));  // softplus
      gl = -__expf(A_log[h]) * sp;                         // log decay, <= 0
      beta = 1.f / (1.f + __expf(-__bfloat162float(ab[r + b_col + h])));
    }
    sG[tid] = gl;
    sB[tid] = beta;
  }
  __syncthreads();
  if (warp == 0) {
    const float x0 = sG[2 * lane], x1 = sG[2 * lane + 1];
    float p = x0 + x1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, p, o);
      if (lane >= o) p += y;
    }
    const float excl = p - (x0 + x1);
    sG[2 * lane] = excl + x0;
    sG[2 * lane + 1] = excl + x0 + x1;
    reinterpret_cast<float2*>(rec + kRecG)[lane] = make_float2(excl + x0, excl + x0 + x1);
  }
  __syncthreads();

  {
    const int mt = warp & 3, nh = warp >> 2;
    float accP[4][4], accQ[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) accP[i][j] = accQ[i][j] = 0.f;
#pragma unroll
    for (int k0 = 0; k0 < kD; k0 += 16) {
      uint32_t ak[4], aq[4];
      gc_ldsm4(a_rows(aK, P2, 16 * mt, k0, lane), ak);
      gc_ldsm4(a_rows(aQ, P2, 16 * mt, k0, lane), aq);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b[4];
        gc_ldsm4(b_rows(aK, P2, 32 * nh + 16 * np, k0, lane), b);
        gc_mma(accP[2 * np], ak, b[0], b[1]);
        gc_mma(accP[2 * np + 1], ak, b[2], b[3]);
        gc_mma(accQ[2 * np], aq, b[0], b[1]);
        gc_mma(accQ[2 * np + 1], aq, b[2], b[3]);
      }
    }
    uint32_t* Mrec = reinterpret_cast<uint32_t*>(rec + kRecM);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int i = 16 * mt + g + 8 * hf;
        const int j = 32 * nh + 8 * nt + 2 * t4;
        const float gi_ = sG[i], bi = sB[i];
        const float d0 = j <= i ? __expf(gi_ - sG[j]) : 0.f;
        const float d1 = j + 1 <= i ? __expf(gi_ - sG[j + 1]) : 0.f;
        sA[i * kPa + j] = j < i ? bi * d0 * accP[nt][2 * hf] : 0.f;
        sA[i * kPa + j + 1] = j + 1 < i ? bi * d1 * accP[nt][2 * hf + 1] : 0.f;
        Mrec[(i * kCh + j) >> 1] = gc_pack(d0 * accQ[nt][2 * hf], d1 * accQ[nt][2 * hf + 1]);
      }
  }
  __syncthreads();

  {
    const int col = tid;
    const bool kside = col < kD;
    // the right-hand side from the staged bf16 rows (rows past the chunk are zeros)
    const __nv_bfloat16* rhs =
        reinterpret_cast<const __nv_bfloat16*>(smem + (kside ? GpSmem::K : GpSmem::V)) + (col & (kD - 1));
    float x[kCh];
#pragma unroll
    for (int i = 0; i < kCh; ++i) x[i] = 0.f;
#pragma unroll
    for (int i = 0; i < kCh; ++i) {
      float r = sB[i] * (kside ? __expf(sG[i]) : 1.f) * __bfloat162float(rhs[i * kP]);
      const float4* arow = reinterpret_cast<const float4*>(sA + i * kPa);
#pragma unroll
      for (int j4 = 0; j4 < (i + 3) / 4; ++j4) {
        const float4 a = arow[j4];
        r -= a.x * x[4 * j4] + a.y * x[4 * j4 + 1] + a.z * x[4 * j4 + 2] + a.w * x[4 * j4 + 3];
      }
      x[i] = r;
    }
    __nv_bfloat16* dstp = reinterpret_cast<__nv_bfloat16*>(rec + (kside ? kRecW : kRecU)) + (kside ? col : col - kD);
#pragma unroll
    for (int i = 0; i < kCh; ++i) dstp[i * kD] = __float2bfloat16(kside ? -x[i] : x[i]);
  }
}

struct GsSmem {
  // two buffers of one record's tiles (padded rows), then the state and U tiles
  static constexpr int Q = 0;
  static constexpr int K = Q + kCh * kP * 2;
  static constexpr int W = K + kCh * kP * 2;
  static constexpr int Ut = W + kCh * kP * 2;
  static constexpr int M = Ut + kCh * kP * 2;
  static constexpr int G = M + kCh * kPm * 2;
  static constexpr int BUF = G + kCh * 4;            // 79,104 B
  static constexpr int S = 2 * BUF;
  static constexpr int U = S + kD * kP * 2;
  static constexpr int Us = U + kCh * kP * 2;
  static constexpr int BYTES = Us + kCh * kP * 2;    // 227,840 B
};

__device__ __forceinline__ void gc_cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void gc_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void gc_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void gc_cp16z(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}

// one chunk into buffer `buf`: its q and k rows from the bf16 conv buffer (rows
// past the chunk's end zero-filled), the record's -W and U~ tiles, M and G (16 B pieces)
__device__ __forceinline__ void gc_fetch_record(uint32_t sbuf, const uint8_t* rec, const __nv_bfloat16* qrows,
                                                const __nv_bfloat16* krows, int C, int cn, int tid) {
  constexpr int P2 = kP * 2, Pm2 = kPm * 2;
  for (int idx = tid; idx < 2 * kCh * 16; idx += 256) {
    const int tile = idx >> 10, row = (idx >> 4) & 63, c16 = idx & 15;
    const bool valid = row < cn;
    const __nv_bfloat16* src = (tile == 0 ? qrows : krows) + (size_t)(valid ? row : 0) * C + c16 * 8;
    gc_cp16z(sbuf + (tile == 0 ? GsSmem::Q : GsSmem::K) + row * P2 + c16 * 16, src, valid);
  }
  for (int idx = tid; idx < 2 * kCh * 16; idx += 256) {
    const int tile = idx >> 10, row = (idx >> 4) & 63, c16 = idx & 15;
    const int src = tile == 0 ? kRecW : kRecU;
    const int dst = tile == 0 ? GsSmem::W : GsSmem::Ut;
    gc_cp16(sbuf + dst + row * P2 + c16 * 16, rec + src + row * kD * 2 + c16 * 16);
  }
  for (int idx = tid; idx < kCh * 8; idx += 256) {
    const int row = idx >> 3, c16 = idx & 7;
    gc_cp16(sbuf + GsSmem::M + row * Pm2 + c16 * 16, rec + kRecM + row * kCh * 2 + c16 * 16);
  }
  if (tid < 16) gc_cp16(sbuf + GsSmem::G + tid * 16, rec + kRecG + tid * 16);
}

__global__ void __launch_bounds__(256, 1) gdn_chunk_scan_kernel(
    int Hv, int Hk, const int* __restrict__ seqs, const int* __restrict__ sio, float* __restrict__ ssm_state, int gi,
    int G, const int* __restrict__ ws, int maxc, const uint8_t* __restrict__ recs, const __nv_bfloat16* __restrict__ cv,
    int C, int qk_channels, float* __restrict__ out) {
  extern __shared__ __align__(16) uint8_t smem[];
  const uint32_t base = smem_u32(smem);
  const uint32_t aS = base + GsSmem::S, aU = base + GsSmem::U, aUs = base + GsSmem::Us;
  constexpr int P2 = kP * 2, Pm2 = kPm * 2;

  const int S = gridDim.y, h = blockIdx.x, tid = threadIdx.x;
  const int s = ws[4 + 2 * maxc + S + blockIdx.y];   // longest sequences first
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, t4 = lane & 3;
  const int q0 = seqs[s * kChSeqInts], n = seqs[s * kChSeqInts + 1];
  const int src = sio[2 * s], dst = sio[2 * s + 1];
  const int first = ws[4 + 2 * maxc + s];
  const int nch = (n + kCh - 1) / kCh;
  const size_t slot_stride = (size_t)G * Hv * kD * kD;
  const size_t head_off = ((size_t)gi * Hv + h) * kD * kD;
  auto record = [&](int c) { return recs + ((size_t)(first + c) * Hv + h) * kRecBytes; };
  const int hk = h / (Hv / Hk);
  const __nv_bfloat16* qbase = cv + (size_t)q0 * C + hk * kD;
  const __nv_bfloat16* kbase = cv + (size_t)q0 * C + qk_channels / 2 + hk * kD;
  auto fetch = [&](uint32_t sbuf, int c) {
    gc_fetch_record(sbuf, record(c), qbase + (size_t)c * kCh * C, kbase + (size_t)c * kCh * C, C,
                    min(kCh, n - c * kCh), tid);
  };
  if (nch > 0) {
    fetch(base, 0);
    gc_commit();
  }

  float Sacc[16][4];
  const int r_lo = 16 * warp + g, r_hi = r_lo + 8;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = nt * 8 + 2 * t4;
    if (src >= 0) {
      const float* S0 = ssm_state + (size_t)src * slot_stride + head_off;
      const float2 lo = *reinterpret_cast<const float2*>(S0 + (size_t)r_lo * kD + c);
      const float2 hi = *reinterpret_cast<const float2*>(S0 + (size_t)r_hi * kD + c);
      Sacc[nt][0] = lo.x; Sacc[nt][1] = lo.y; Sacc[nt][2] = hi.x; Sacc[nt][3] = hi.y;
    } else {
      Sacc[nt][0] = Sacc[nt][1] = Sacc[nt][2] = Sacc[nt][3] = 0.f;
    }
  }
  uint32_t* sS32 = reinterpret_cast<uint32_t*>(smem + GsSmem::S);
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = nt * 8 + 2 * t4;
    sS32[(r_lo * kP + c) >> 1] = gc_pack(Sacc[nt][0], Sacc[nt][1]);
    sS32[(r_hi * kP + c) >> 1] = gc_pack(Sacc[nt][2], Sacc[nt][3]);
  }
  const int mt = warp & 3, nh = warp >> 2;

  for (int c = 0; c < nch; ++c) {
    const int c0 = c * kCh, cn = min(kCh, n - c0);
    const uint32_t boff = (c & 1) * GsSmem::BUF;
    if (c + 1 < nch) {
      fetch(base + (boff ^ GsSmem::BUF), c + 1);
      gc_commit();
      gc_wait<1>();
    } else {
      gc_wait<0>();
    }
    __syncthreads();
    const uint32_t aQ = base + boff + GsSmem::Q, aK = base + boff + GsSmem::K, aW = base + boff + GsSmem::W;
    const uint32_t aM = base + boff + GsSmem::M;
    const uint8_t* sUt = smem + boff + GsSmem::Ut;
    const float* sG = reinterpret_cast<const float*>(smem + boff + GsSmem::G);

    float accO[8][4];
    {
      float accU[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int cc = 64 * nh + 8 * nt + 2 * t4;
        const int i0 = 16 * mt + g;
        const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(sUt + i0 * P2 + cc * 2);
        const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(sUt + (i0 + 8) * P2 + cc * 2);
        accU[nt][0] = __low2float(lo);
        accU[nt][1] = __high2float(lo);
        accU[nt][2] = __low2float(hi);
        accU[nt][3] = __high2float(hi);
        accO[nt][0] = accO[nt][1] = accO[nt][2] = accO[nt][3] = 0.f;
      }
#pragma unroll
      for (int k0 = 0; k0 < kD; k0 += 16) {
        uint32_t aw[4], aq[4];
        gc_ldsm4(a_rows(aW, P2, 16 * mt, k0, lane), aw);
        gc_ldsm4(a_rows(aQ, P2, 16 * mt, k0, lane), aq);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b[4];
          gc_ldsm4t(b_cols(aS, P2, 64 * nh + 16 * np, k0, lane), b);
          gc_mma(accU[2 * np], aw, b[0], b[1]);
          gc_mma(accU[2 * np + 1], aw, b[2], b[3]);
          gc_mma(accO[2 * np], aq, b[0], b[1]);
          gc_mma(accO[2 * np + 1], aq, b[2], b[3]);
        }
      }
      const float Gl = sG[kCh - 1];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int i = 16 * mt + g + 8 * hf;
        const float gam = __expf(sG[i]), tail = __expf(Gl - sG[i]);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int cc = 64 * nh + 8 * nt + 2 * t4;
          const float u0 = accU[nt][2 * hf], u1 = accU[nt][2 * hf + 1];
          *reinterpret_cast<uint32_t*>(smem + GsSmem::U + i * P2 + cc * 2) = gc_pack(u0, u1);
          *reinterpret_cast<uint32_t*>(smem + GsSmem::Us + i * P2 + cc * 2) = gc_pack(tail * u0, tail * u1);
          accO[nt][2 * hf] *= gam;
          accO[nt][2 * hf + 1] *= gam;
        }
      }
    }
    __syncthreads();

#pragma unroll
    for (int k0 = 0; k0 < kCh; k0 += 16) {
      uint32_t am[4];
      gc_ldsm4(a_rows(aM, Pm2, 16 * mt, k0, lane), am);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        gc_ldsm4t(b_cols(aU, P2, 64 * nh + 16 * np, k0, lane), b);
        gc_mma(accO[2 * np], am, b[0], b[1]);
        gc_mma(accO[2 * np + 1], am, b[2], b[3]);
      }
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int i = 16 * mt + g + 8 * hf;
      if (i < cn) {
        float* orow = out + (size_t)(q0 + c0 + i) * Hv * kD + h * kD;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int cc = 64 * nh + 8 * nt + 2 * t4;
          *reinterpret_cast<float2*>(orow + cc) = make_float2(accO[nt][2 * hf], accO[nt][2 * hf + 1]);
        }
      }
    }
    {
      const float gC = __expf(sG[kCh - 1]);
#pragma unroll
      for (int nt = 0; nt < 16; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) Sacc[nt][e] *= gC;
#pragma unroll
      for (int k0 = 0; k0 < kCh; k0 += 16) {
        uint32_t ak[4];
        gc_ldsm4t(a_cols(aK, P2, 16 * warp, k0, lane), ak);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
          uint32_t b[4];
          gc_ldsm4t(b_cols(aUs, P2, 16 * np, k0, lane), b);
          gc_mma(Sacc[2 * np], ak, b[0], b[1]);
          gc_mma(Sacc[2 * np + 1], ak, b[2], b[3]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        const int cc = nt * 8 + 2 * t4;
        sS32[(r_lo * kP + cc) >> 1] = gc_pack(Sacc[nt][0], Sacc[nt][1]);
        sS32[(r_hi * kP + cc) >> 1] = gc_pack(Sacc[nt][2], Sacc[nt][3]);
      }
    }
    __syncthreads();
  }
  if (dst < 0) return;   // the state is not kept
  float* Sd = ssm_state + (size_t)dst * slot_stride + head_off;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = nt * 8 + 2 * t4;
    *reinterpret_cast<float2*>(Sd + (size_t)r_lo * kD + c) = make_float2(Sacc[nt][0], Sacc[nt][1]);
    *reinterpret_cast<float2*>(Sd + (size_t)r_hi * kD + c) = make_float2(Sacc[nt][2], Sacc[nt][3]);
  }
}

// ------------------------------------------------------------------ conv, token-parallel
// The causal depthwise conv (width 4) + SiLU + q/k L2 norm, one warp per
// (token, 128-channel block), 4 channels per lane: a token reads its own
// input row and the 3 before it (the source slot's window before the
// sequence's first token), so tokens are independent; a 128-channel block
// of q or k is one head, so its norm is a warp reduction. CTAs walk the
// chunk list (64 tokens each). The new windows are written afterwards by
// gdn_conv_window (a sequence's source and destination slot may be the same).
__global__ void __launch_bounds__(256) gdn_conv_chunk_kernel(
    const __nv_bfloat16* __restrict__ mixed, int ldm, int C, int qk_channels, const float* __restrict__ wconv,
    const int* __restrict__ seqs, const int* __restrict__ sio, const float* __restrict__ conv_state, int gi, int G,
    float q_scale, const int* __restrict__ ws, __nv_bfloat16* __restrict__ out) {
  const int ci = blockIdx.x;
  if (ci >= ws[0]) return;
  const int2 e = reinterpret_cast<const int2*>(ws + 4)[ci];
  const int s = e.x, c0 = e.y;
  const int q0 = seqs[s * kChSeqInts], n = seqs[s * kChSeqInts + 1];
  const int cn = min(kCh, n - c0);
  const int src = sio[2 * s];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cb = blockIdx.y * 128, ch = cb + lane * 4;
  const bool is_qk = cb < qk_channels, is_q = cb < qk_channels / 2;
  float w[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 v = *reinterpret_cast<const float4*>(wconv + (size_t)(ch + j) * 4);
    w[j][0] = v.x; w[j][1] = v.y; w[j][2] = v.z; w[j][3] = v.w;
  }
  const float* win = src >= 0 ? conv_state + ((size_t)src * G + gi) * 3 * C : nullptr;
  // input row `pos` of the sequence (the source window before its first token)
  auto load_in = [&](int pos, float* x) {
    x[0] = x[1] = x[2] = x[3] = 0.f;
    if (pos >= 0) {
      const uint2 raw = *reinterpret_cast<const uint2*>(mixed + (size_t)(q0 + pos) * ldm + ch);
      const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
      const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
      x[0] = __low2float(a); x[1] = __high2float(a); x[2] = __low2float(b); x[3] = __high2float(b);
    } else if (win != nullptr) {
      const float4 v = *reinterpret_cast<const float4*>(win + (size_t)(3 + pos) * C + ch);
      x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    }
  };
  // each warp takes 8 consecutive tokens and slides the 4-row window over them,
  // loading one new input row per token
  const int t_lo = warp * 8, t_hi = min(cn, t_lo + 8);
  float hist[3][4];
  if (t_lo < t_hi)
#pragma unroll
    for (int k = 0; k < 3; ++k) load_in(c0 + t_lo - 3 + k, hist[k]);
  for (int tt = t_lo; tt < t_hi; ++tt) {
    const int t = c0 + tt;
    float cur[4];
    load_in(t, cur);
    float acc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      acc[j] = w[j][0] * hist[0][j] + w[j][1] * hist[1][j] + w[j][2] * hist[2][j] + w[j][3] * cur[j];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      hist[0][j] = hist[1][j];
      hist[1][j] = hist[2][j];
      hist[2][j] = cur[j];
    }
    float y[4], ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      y[j] = acc[j] / (1.f + __expf(-acc[j]));   // SiLU
      ss += y[j] * y[j];
    }
    if (is_qk) {
      ss = warp_sum(ss);
      const float r = rsqrtf(fmaxf(ss, 1e-12f)) * (is_q ? q_scale : 1.f);
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] *= r;
    }
    *reinterpret_cast<uint2*>(out + (size_t)(q0 + t) * C + ch) = make_uint2(gc_pack(y[0], y[1]), gc_pack(y[2], y[3]));
  }
}

// The destination window of each sequence: its last 3 inputs (older ones from
// the source window when it has fewer than 3 new tokens). One thread per channel.
__global__ void __launch_bounds__(128) gdn_conv_window_kernel(const __nv_bfloat16* __restrict__ mixed, int ldm,
                                                              int C, const int* __restrict__ seqs,
                                                              const int* __restrict__ sio,
                                                              float* __restrict__ conv_state, int gi, int G) {
  const int s = blockIdx.x, c = blockIdx.y * 128 + threadIdx.x;
  if (c >= C) return;
  const int q0 = seqs[s * kChSeqInts], n = seqs[s * kChSeqInts + 1];
  const int src = sio[2 * s], dst = sio[2 * s + 1];
  float v[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int pos = n - 3 + j;
    v[j] = pos >= 0 ? __bfloat162float(mixed[(size_t)(q0 + pos) * ldm + c])
                    : (src >= 0 ? conv_state[(((size_t)src * G + gi) * 3 + (3 + pos)) * C + c] : 0.f);
  }
  if (dst < 0) return;   // the state is not kept
#pragma unroll
  for (int j = 0; j < 3; ++j) conv_state[(((size_t)dst * G + gi) * 3 + j) * C + c] = v[j];
}

}  // namespace

// The chunked recurrence for one Gated DeltaNet layer (d_k = d_v = 128); the
// caller (gdn_layer) has run the conv phase into conv_out.
void launch_gdn_chunk(const float* conv_out, int C, int qk_channels, const __nv_bfloat16* ab, int ldab, int b_col,
                      int a_col, const float* A_log, const float* dt_bias, int Hv, int Hk, const int* seqs,
                      const int* sio, int S, float* ssm_state, int gi, int G, float* out, int dev,
                      cudaStream_t st) {
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        GcSmem::BYTES));
    configured[dev] = true;
  }
  dim3 grid(S, Hv);
  gdn_chunk_kernel<<<grid, 256, GcSmem::BYTES, st>>>(conv_out, C, qk_channels, ab, ldab, b_col, a_col, A_log,
                                                     dt_bias, Hv, Hk, seqs, sio, ssm_state, gi, G, out);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Bytes of the split form's workspace for a pass of T tokens in S sequences.
int64_t gdn_chunk_ws_bytes(int64_t T, int64_t S, int64_t Hv, int64_t C) {
  const int64_t maxc = T / kCh + S + 1;
  const int64_t ints = ((4 + 2 * maxc + 2 * S) * 4 + 255) / 256 * 256;
  const int64_t cvb = (T * C * 2 + 255) / 256 * 256;
  return ints + cvb + maxc * Hv * kRecBytes;
}

void launch_gdn_chunk_split(const __nv_bfloat16* mixed, const float* wconv, float* conv_state, float q_scale,
                            float* conv_out, int C, int qk_channels, const __nv_bfloat16* ab, int ldab,
                            int b_col, int a_col, const float* A_log, const float* dt_bias, int Hv, int Hk,
                            const int* seqs, const int* sio, int T, int S, float* ssm_state, int gi, int G,
                            float* out, uint8_t* ws, int dev, cudaStream_t st) {
  static bool configured[64] = {false};
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        GpSmem::BYTES));
    C10_CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        GsSmem::BYTES));
    configured[dev] = true;
  }
  const int maxc = T / kCh + S + 1;
  const int64_t ints = ((4 + 2 * (int64_t)maxc + 2 * S) * 4 + 255) / 256 * 256;
  int* wsi = reinterpret_cast<int*>(ws);
  __nv_bfloat16* cv = reinterpret_cast<__nv_bfloat16*>(ws + ints);
  uint8_t* recs = ws + ints + ((int64_t)T * C * 2 + 255) / 256 * 256;
  gdn_chunk_index_kernel<<<1, 256, 0, st>>>(seqs, S, maxc, wsi);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  gdn_conv_chunk_kernel<<<dim3(maxc, C / 128), 256, 0, st>>>(mixed, ldab, C, qk_channels, wconv, seqs, sio,
                                                              conv_state, gi, G, q_scale, wsi, cv);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  gdn_conv_window_kernel<<<dim3(S, C / 128), 128, 0, st>>>(mixed, ldab, C, seqs, sio, conv_state, gi, G);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  gdn_chunk_prep_kernel<<<dim3(maxc, Hv), 256, GpSmem::BYTES, st>>>(cv, C, qk_channels, ab, ldab, b_col,
                                                                     a_col, A_log, dt_bias, Hv, Hk, seqs, wsi, recs);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  gdn_chunk_scan_kernel<<<dim3(Hv, S), 256, GsSmem::BYTES, st>>>(Hv, Hk, seqs, sio, ssm_state, gi, G, wsi, maxc,
                                                                  recs, cv, C, qk_channels, out);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace qb
