// Tile order of the persistent GEMM schedules.
#pragma once

namespace qb {

// Tile order of the persistent schedule. The CTAs in flight at one time read
// the A rows of their m-tiles and the B rows of their n-tiles; when A is the
// larger operand (M > N, e.g. the down projection of a 16k-token pass, A =
// 160 MB) n runs fastest, so the ~148 tiles in flight share ~15 m-tiles of A
// (each read from HBM once, then from L2 by the other n-tiles) and all of B
// stays in L2; otherwise m runs fastest and B is the shared operand.
__device__ __forceinline__ void tile_coords(int t, int num_m_tiles, int num_n_tiles, int n_fast, int& tm,
                                            int& tn) {
  if (n_fast) {
    tm = t / num_n_tiles;
    tn = t % num_n_tiles;
  } else {
    tm = t % num_m_tiles;
    tn = t / num_m_tiles;
  }
}

}  // namespace qb
