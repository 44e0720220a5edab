// Epilogue selector of the tcgen05 GEMM kernel.
#pragma once

namespace qb {

enum Epi : int {
  kEpiBf16 = 0,        // D = acc (bf16)
  kEpiResidual = 1,    // D = acc + R (bf16; R may alias D)
  kEpiSwigluFp8 = 2,   // Y = e4m3(silu(g) * u), one fp32 scale per 128 outputs
  kEpiSwigluBf16 = 3,  // D = silu(g) * u (bf16)
  kEpiQkvRope = 4,     // per 128-column head: q/k RMSNorm + NeoX RoPE; q -> q_out, k/v -> paged cache
  kEpiResidualMx = 5,  // D = acc + R (bf16), and D as e4m3 + UE8M0 per 32 columns, row sums of squares
  kEpiGegluBf16 = 6,   // D = gelu_tanh(g) * u (bf16), gate/up interleaved as for SwiGLU
  kEpiGegluFp8 = 7,    // MX GEMM: Y = e4m3(gelu_tanh(g) * u) + UE8M0 scales, as kEpiSwigluFp8
};

}  // namespace qb
