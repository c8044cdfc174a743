// Exact block-sparse causal attention, mma.sync (m16n8k16 bf16) version.
//
// Reference: upstream/flashprefill_native_forward.py:215-354 (_flash_forward). One CTA per
// (batch, query head, 128-row query tile) walks the tile's selected 128-key blocks in
// ascending order as 64-key sub-tiles (cp.async double buffering), with an online softmax
// in exp2 units; the diagonal block is causally masked; P is rounded to bf16 before the P.V
// product (upstream:338); O is written bf16 and the log-sum-exp in natural-log units
// (upstream:349). Rows with no key get O = 0 and LSE = -inf, as the reference does.
//
// This kernel is the portable path used for the reference-layout entry point and as the
// cross-check of the tcgen05 kernel; 8 warps x 16 rows, K/V sub-tiles of 64 x 128 bf16.
#include "attn.cuh"

namespace fpx {

constexpr int kSubKeys = 64;
constexpr int kAttnThreads = 256;

// XOR-swizzled [rows][128] bf16 tile: 16-byte chunk c of row r lives at chunk c ^ (r & 7).
FPX_INLINE int swz(int r, int chunk) { return r * kHeadDim + ((chunk ^ (r & 7)) << 3); }

template <int kMode>
__global__ void __launch_bounds__(kAttnThreads, 1) exact_mma_kernel(ExactParams p) {
  const int t = p.tile_begin + (gridDim.x - 1 - blockIdx.x);
  const int h = p.head_begin + blockIdx.y;
  const int b = blockIdx.z;
  const int kvh = h / p.group;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16 *sq = reinterpret_cast<__nv_bfloat16 *>(smem);
  __nv_bfloat16 *sk = sq + kBlock * kHeadDim;          // [2][64][128]
  __nv_bfloat16 *sv = sk + 2 * kSubKeys * kHeadDim;    // [2][64][128]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;

  // The tile's block list.
  int count;
  const int32_t *list32 = nullptr;
  const int64_t *list64 = nullptr;
  int64_t list_stride = 1;
  if (kMode == kExactLists) {
    const int64_t rrow = p.route.row(b, h, t, p.H);
    count = p.route.counts[rrow];
    list32 = p.route.lists + rrow * p.route.nb;
  } else if (kMode == kExactRefLayout) {
    count = p.ref_counts[((int64_t)b * p.nb + t) * p.H + h];
    list64 = p.ref_indices + ((int64_t)b * p.nb + t) * p.nb * p.H + h;
    list_stride = p.H;
  } else {
    count = t + 1;
  }
  auto block_at = [&](int i) -> int {
    if (kMode == kExactLists) return list32[i];
    if (kMode == kExactRefLayout) return (int)list64[i * list_stride];
    return i;
  };

  const __nv_bfloat16 *qbase = p.q + b * p.q_sb + h * p.q_sh;
  const __nv_bfloat16 *kbase = p.k + b * p.k_sb + kvh * p.k_sh;
  const __nv_bfloat16 *vbase = p.v + b * p.v_sb + kvh * p.v_sh;
  const int row0 = t * kBlock;

  // Query tile -> smem (rows past L zero-filled).
  for (int i = tid; i < kBlock * 16; i += kAttnThreads) {
    const int r = i >> 4, ch = i & 15;
    const int pos = row0 + r;
    const bool ok = pos < p.L;
    cp_async16(sq + swz(r, ch), qbase + (int64_t)(ok ? pos : 0) * p.q_sl + ch * 8, ok);
  }
  cp_async_commit();

  auto load_sub = [&](int s, int stage) {
    const int blk = block_at(s >> 1);
    const int key0 = blk * kBlock + (s & 1) * kSubKeys;
    __nv_bfloat16 *dk = sk + stage * kSubKeys * kHeadDim;
    __nv_bfloat16 *dv = sv + stage * kSubKeys * kHeadDim;
    for (int i = tid; i < kSubKeys * 16; i += kAttnThreads) {
      const int r = i >> 4, ch = i & 15;
      const int pos = key0 + r;
      const bool ok = pos < p.L;
      const int64_t src = (int64_t)(ok ? pos : 0);
      cp_async16(dk + swz(r, ch), kbase + src * p.k_sl + ch * 8, ok);
      cp_async16(dv + swz(r, ch), vbase + src * p.v_sl + ch * 8, ok);
    }
  };

  const int subs = 2 * count;
  if (subs > 0) load_sub(0, 0);
  cp_async_commit();
  cp_async_wait<1>();
  __syncthreads();

  // Q fragments for this warp's 16 rows (ldmatrix x4: rows +0/+8, k chunks 2kk / 2kk+1).
  uint32_t qf[8][4];
  {
    const int m = lane >> 3;
    const int r = 16 * warp + ((m & 1) << 3) + (lane & 7);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      ldmatrix_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], smem_u32(sq + swz(r, 2 * kk + (m >> 1))));
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  float lrow[2] = {0.f, 0.f};
  const int qpos0 = row0 + 16 * warp + g;

  for (int s = 0; s < subs; ++s) {
    if (s + 1 < subs) load_sub(s + 1, (s + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const int stage = s & 1;
    const __nv_bfloat16 *ck = sk + stage * kSubKeys * kHeadDim;
    const __nv_bfloat16 *cv = sv + stage * kSubKeys * kHeadDim;
    const int blk = block_at(s >> 1);
    const int key0 = blk * kBlock + (s & 1) * kSubKeys;

    float sacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
    for (int kk2 = 0; kk2 < 4; ++kk2) {
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3, smem_u32(ck + swz(8 * nt + (lane & 7), 4 * kk2 + (lane >> 3))));
        mma_bf16_16816(sacc[nt], qf[2 * kk2], b0, b1);
        mma_bf16_16816(sacc[nt], qf[2 * kk2 + 1], b2, b3);
      }
    }
    // Scale, causal mask on the diagonal block, online softmax (exp2 units).
    const bool diag = blk == t;
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kpos = key0 + 8 * nt + 2 * tq + (e & 1);
        const int qpos = qpos0 + ((e >> 1) << 3);
        float x = sacc[nt][e] * p.scale_log2;
        if (diag && kpos > qpos) x = -INFINITY;
        sacc[nt][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      corr[r] = (mrow[r] == -INFINITY) ? (mx[r] == -INFINITY ? 1.f : 0.f) : exp2f(mrow[r] - mx[r]);
      mrow[r] = mx[r];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = mx[e >> 1];
        pv[e] = (m == -INFINITY) ? 0.f : exp2f(sacc[nt][e] - m);
        rs[e >> 1] += pv[e];
      }
      pa[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16(pv[0], pv[1]);
      pa[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16(pv[2], pv[3]);
    }
    lrow[0] = lrow[0] * corr[0] + rs[0];
    lrow[1] = lrow[1] * corr[1] + rs[1];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= corr[0]; o[i][1] *= corr[0];
      o[i][2] *= corr[1]; o[i][3] *= corr[1];
    }
    // O += P V. pa[kk] = A fragment of keys 16kk..16kk+15: {row g lo, row g+8 lo, row g hi,
    // row g+8 hi} — rearranged from the accumulator layout of n-tiles 2kk and 2kk+1.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t af2[4] = {pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3]};
#pragma unroll
      for (int dn2 = 0; dn2 < 8; ++dn2) {
        uint32_t b0, b1, b2, b3;
        const int vr = 16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3);
        ldmatrix_x4_trans(b0, b1, b2, b3, smem_u32(cv + swz(vr, 2 * dn2 + (lane >> 4))));
        mma_bf16_16816(o[2 * dn2], af2, b0, b1);
        mma_bf16_16816(o[2 * dn2 + 1], af2, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // Finalise: full row sums, O / l, natural LSE = m ln 2 + ln l.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  float inv[2], lse[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const bool none = mrow[r] == -INFINITY;
    inv[r] = none ? 0.f : 1.f / lrow[r];
    lse[r] = none ? -INFINITY : mrow[r] * kLn2 + logf(lrow[r]);
  }
  // Stage the bf16 output tile in the (now free) Q buffer, then 16-byte row stores.
  __syncthreads();
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = 8 * nt + 2 * tq;
    const int r0 = 16 * warp + g;
    *reinterpret_cast<uint32_t *>(sq + swz(r0, c >> 3) + (c & 7)) =
        pack_bf16(o[nt][0] * inv[0], o[nt][1] * inv[0]);
    *reinterpret_cast<uint32_t *>(sq + swz(r0 + 8, c >> 3) + (c & 7)) =
        pack_bf16(o[nt][2] * inv[1], o[nt][3] * inv[1]);
  }
  if (tq == 0) {
    if (p.lse) {
      if (qpos0 < p.L) p.lse[((int64_t)b * p.L + qpos0) * p.H + h] = lse[0];
      if (qpos0 + 8 < p.L) p.lse[((int64_t)b * p.L + qpos0 + 8) * p.H + h] = lse[1];
    }
  }
  __syncwarp();
  for (int i = lane; i < 16 * 16; i += 32) {
    const int r = 16 * warp + (i >> 4), ch = i & 15;
    const int pos = row0 + r;
    if (pos < p.L)
      *reinterpret_cast<uint4 *>(p.out + b * p.o_sb + (int64_t)pos * p.o_sl + h * p.o_sh + ch * 8) =
          *reinterpret_cast<const uint4 *>(sq + swz(r, ch));
  }
}

size_t exact_mma_smem() { return (size_t)(kBlock + 4 * kSubKeys) * kHeadDim * 2; }

int launch_exact_mma(const ExactParams &p, int mode, int tiles, int heads, int B, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  const size_t smem = exact_mma_smem();
  dim3 grid(tiles, heads, B);
#define FPX_EXACT_LAUNCH(M)                                                                  \
  do {                                                                                       \
    cudaFuncSetAttribute(exact_mma_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                         (int)smem);                                                         \
    exact_mma_kernel<M><<<grid, kAttnThreads, smem, s>>>(p);                                 \
  } while (0)
  if (mode == kExactLists)
    FPX_EXACT_LAUNCH(kExactLists);
  else if (mode == kExactRefLayout)
    FPX_EXACT_LAUNCH(kExactRefLayout);
  else
    FPX_EXACT_LAUNCH(kExactDense);
#undef FPX_EXACT_LAUNCH
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

}  // namespace fpx
