// The 16 two-input logic gates of CompactLogic, in the three forms the kernels need.
//
// Gate ids follow the reference truth table (compactlogic/cuda/utils.cuh:122-139): reading the id
// as a 4-bit number, bit 3 is the output for (A,B)=(0,0), bit 2 for (0,1), bit 1 for (1,0) and
// bit 0 for (1,1).  E.g. id 1 = AND (only (1,1) is true), id 6 = XOR, id 8 = NOR.
//
// * Real relaxation (utils.cuh:180-207): the multilinear extension of the truth table,
//     f(a,b) = t00 (1-a)(1-b) + t01 (1-a) b + t10 a (1-b) + t11 a b
//            = c0 + c1 a + c2 b + c3 a b,
//   with c0 = t00, c1 = t10 - t00, c2 = t01 - t00, c3 = t00 - t01 - t10 + t11.  The coefficients
//   are derived from the id bits here instead of being read from a per-gate constant table, so a
//   warp whose lanes hold different gate ids issues no divergent constant-cache loads.
// * Derivatives (utils.cuh:209-243): df/da = c1 + c3 b, df/db = c2 + c3 a.
// * Bitwise form on packed words (64 samples per uint64): a branch-free two-level multiplexer
//   over the four truth-table bits, used by the bit-packed discrete inference.
#pragma once

#include <stdint.h>

namespace clb {

struct GatePoly {
    float c0, c1, c2, c3;
};

__host__ __device__ __forceinline__ GatePoly gate_poly(int id) {
    const float t00 = (float)((id >> 3) & 1);
    const float t01 = (float)((id >> 2) & 1);
    const float t10 = (float)((id >> 1) & 1);
    const float t11 = (float)(id & 1);
    GatePoly g;
    g.c0 = t00;
    g.c1 = t10 - t00;
    g.c2 = t01 - t00;
    g.c3 = t00 - t01 - t10 + t11;
    return g;
}

// out bit = truth_table(id)[a bit][b bit], for all bit positions at once.
template <typename W>
__host__ __device__ __forceinline__ W gate_word(int id, W a, W b) {
    const W m00 = (W)0 - (W)((id >> 3) & 1);
    const W m01 = (W)0 - (W)((id >> 2) & 1);
    const W m10 = (W)0 - (W)((id >> 1) & 1);
    const W m11 = (W)0 - (W)(id & 1);
    const W lo = m00 ^ ((m00 ^ m10) & a);  // b = 0: select by a
    const W hi = m01 ^ ((m01 ^ m11) & a);  // b = 1: select by a
    return lo ^ ((lo ^ hi) & b);
}

}  // namespace clb
