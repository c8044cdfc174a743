// The softmax step shared by the tcgen05 exact kernels (attn_tc.cu, attn_tc1.cu):
// one thread owns one query row (one TMEM lane) of a block of NC keys (128, or a 64-key half).
#pragma once

#include "tc.cuh"

namespace fpx {
namespace tc {

// One NC-column row of P: x = s * scale_log2 - m, p = 2^x, packed to bf16 into TMEM (16
// columns at a time); returns the row sum of p (fp32, before rounding, as the reference's
// tile_denominator). kEmu of every 8 pairs use the FMA-pipe exp2.
template <int kEmu, int NC = 128>
FPX_INLINE float softmax_row(const float (&sv)[NC], float sl2, float neg, uint32_t p_addr) {
  const uint64_t sl2x2 = pk2(sl2, sl2), negx2 = pk2(neg, neg);
  uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
  for (int q4 = 0; q4 < NC / 32; ++q4) {
    uint32_t pk[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint64_t xx = ffma2(pk2(sv[32 * q4 + 2 * c], sv[32 * q4 + 2 * c + 1]), sl2x2, negx2);
      uint64_t pp;
      if ((c & 7) < kEmu) {
        pp = exp2_poly2(xx);
      } else {
        float a, e;
        up2(xx, a, e);
        pp = pk2(ex2(a), ex2(e));
      }
      acc[c & 3] = fadd2(acc[c & 3], pp);
      pk[c] = cvt_bf16x2(pp);
    }
    tmem_st16u(p_addr + 16 * q4, pk);
  }
  float a0, a1, a2, a3, b0, b1, b2, b3;
  up2(acc[0], a0, b0);
  up2(acc[1], a1, b1);
  up2(acc[2], a2, b2);
  up2(acc[3], a3, b3);
  return ((a0 + b0) + (a1 + b1)) + ((a2 + b2) + (a3 + b3));
}

}  // namespace tc
}  // namespace fpx
