// The new selectors' routing (kernels.py:49-126) on the 5th-generation tensor core, fused with
// their selection (kernels.py:129-151).
//
// For query tile t of head h and every visible block kb < t (a full block, n = 128):
//   ell0 = (q . mean_k) * scale + ln 128
//   u    = max((q^2 . var_k) * scale^2, 0)        (cgf_mean, dispersion_mean)
//   logit = ell0 (+ u / 2)
//   p     = softmax over kb of the row's logits
//   score = mean over the tile's rows of p (x sqrt(u) x sigma_v for dispersion_mean)
//   keep  = score > 0 and score >= alpha * max score, plus the protected blocks.
//
// The products run on the tensor core over 128-block chunks:
//   pass 1, row layout (TMEM lane = query row): S = Q . mean_K^T (and Q^2 . var_K^T); each
//     thread keeps its row's running max and sum, giving the row's log-sum-exp;
//   column sums of the probabilities, in one of two ways:
//   - a tile with at most two chunks (t <= 256, every tile of a 32K layer): pass 1 writes each
//     2^(logit - running max) back into its accumulator column (and dispersion_mean's sqrt(u)
//     weight into the u column), keeping each 32-column slice's max; both chunks stay resident
//     in the two TMEM buffers, and once the row LSEs are known a probability is one multiply by
//     2^(slice max - LSE); each warp sums its 32 rows of every column with a 5-round shuffle
//     butterfly (32 columns per 31 shuffles), the four warps meeting in shared memory. No
//     product or exponential runs twice;
//   - longer tiles: pass 2, transposed (TMEM lane = block): S^T = mean_K . Q^T (and
//     var_K . (Q^2)^T); each thread owns one block and adds up its rows' probabilities (row
//     LSEs from shared memory), so the column sums need no cross-thread reduction.
// Precision: the fp32 descriptors enter as bf16 high + low halves (mean_k = hi + lo, lo the
// rounding remainder), and Q^2 (exact in fp32: a bf16 square has 16 significant bits) splits
// exactly into bf16 hi + lo; u accumulates Q2hi.VKhi + Q2lo.VKhi + Q2hi.VKlo. Logits carry about
// 16 mantissa bits of the descriptors, against fp32's 24 in the reference.
//
// One CTA per (b, h, t); 384 threads:
//   warp 0       TMA: Q, then the operand ring (chunk by chunk: mean-K hi, lo, var-K hi, lo)
//   warp 1       MMA issuer (one lane), TMEM owner
//   warps 2..11  first square Q into Q2hi / Q2lo together (same swizzled layout: squaring is
//                elementwise; the var-K products wait for it)
//   warps 4..11  then the epilogue, two warpgroups splitting each chunk's columns (pass 1) or
//                rows (pass 2); then warpgroup 0 runs the selection
// TMEM: two buffers x (logit accumulator, u accumulator) x 128 columns.
// Waits are bounded; a failed wait flags the CTA and the device error word and the row is
// written with count 0.
#include <cuda.h>

#include "route.cuh"
#include "tc.cuh"

namespace fpx {

namespace {

using namespace tc;

constexpr int kThreads = 384;
constexpr int kMaxBlocks = 2048;
constexpr uint32_t kHalf = 128 * 128;
constexpr uint32_t kTile = 2 * kHalf;
constexpr uint32_t kIdesc = idesc_bf16(128, 128, false);
constexpr float kLn128 = 4.852030263919617f;

// kQ2: the squared-query tiles exist (cgf_mean, dispersion_mean). mean_balanced keeps 96 KB of
// shared memory and 256 TMEM columns, so two of its CTAs share an SM.
template <bool kQ2>
struct alignas(1024) SelSmem {
  uint8_t q[kTile];
  uint8_t q2h[kQ2 ? kTile : 16], q2l[kQ2 ? kTile : 16];
  alignas(1024) uint8_t ring[2][kTile];
  uint64_t q_full, q2_full, r_full[2], r_empty[2], acc_full[2], acc_empty[2], drain;
  uint32_t tmem_base;
  int abort;
  float lse[128];
  float part_m[2][128], part_s[2][128];  // the two warpgroups' halves
  float colpart[2][4][64];              // resident path: [warpgroup][warp][column] partial sums
  float red[2][8];
  int scan[2][4 * (kMaxBlocks / 128)];
  float sc[kMaxBlocks];
};

FPX_INLINE uint64_t desc_kmajor(const uint8_t *tile, int kk) {
  return smem_desc_sw128(smem_u32(tile) + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}

// 8 MMAs: D (+)= A . B^T over K = 128, both K-major SW128 tiles.
FPX_INLINE void mma_tile(uint32_t d, const uint8_t *a, const uint8_t *b, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) mma_ss(d, desc_kmajor(a, kk), desc_kmajor(b, kk), kIdesc, (accumulate || kk > 0) ? 1u : 0u);
}

template <int kSel>
FPX_INLINE float sel_logit(float dot, float udot, float scale, float scale2) {
  const float ell0 = __fadd_rn(__fmul_rn(dot, scale), kLn128);
  if (kSel == 0) return ell0;
  const float u = fmaxf(__fmul_rn(udot, scale2), 0.f);
  return __fadd_rn(ell0, 0.5f * u);
}

}  // namespace

// mean_balanced's CTA is small enough for two per SM (shared memory, TMEM): its registers are
// held to that.
template <int kSel>  // 0 mean_balanced, 1 cgf_mean, 2 dispersion_mean
__global__ void __launch_bounds__(kThreads, kSel == 0 ? 2 : 1)
    selector_route_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_mkh,
                             const __grid_constant__ CUtensorMap tm_mkl, const __grid_constant__ CUtensorMap tm_vkh,
                             const __grid_constant__ CUtensorMap tm_vkl, SelParams p, int *device_error) {
  constexpr int kTilesPerChunk = kSel == 0 ? 2 : 4;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  constexpr uint32_t kCols = kSel == 0 ? 256 : 512;       // TMEM columns
  constexpr uint32_t kAccStride = kSel == 0 ? 128 : 256;  // per accumulator buffer
  SelSmem<(kSel > 0)> &sh = *reinterpret_cast<SelSmem<(kSel > 0)> *>(smem_raw + pad);
  volatile int *abort = &sh.abort;
  const int t = p.tile_begin + (gridDim.x - 1 - blockIdx.x);
  const int h = p.head_begin + blockIdx.y;
  const int b = blockIdx.z;
  const int kvh = h / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = (t + 127) / 128;  // visible blocks kb < t
  // At most two chunks: their logits stay resident in the two TMEM buffers, no second pass.
  const bool resident = chunks <= 2;
  const int units = resident ? chunks : 2 * chunks;  // pass 1 (then pass 2), chunk by chunk

  if (threadIdx.x == 0) {
    mbar_init(&sh.q_full, 1);
    mbar_init(&sh.q2_full, kThreads - 64);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh.r_full[s], 1);
      mbar_init(&sh.r_empty[s], 1);
      mbar_init(&sh.acc_full[s], 1);
      mbar_init(&sh.acc_empty[s], 256);
    }
    mbar_init(&sh.drain, 1);
    sh.abort = *reinterpret_cast<volatile int *>(device_error) != 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    int n = 0;  // operand tiles issued
    bool ok = !*abort && chunks > 0;
    if (ok && lane == 0) {
      mbar_expect_tx(&sh.q_full, kTile);
      tma_load_4d(sh.q, &tm_q, &sh.q_full, 0, h, t * 128, b);
      tma_load_4d(sh.q + kHalf, &tm_q, &sh.q_full, 64, h, t * 128, b);
    }
    for (int u = 0; u < units && ok; ++u) {
      const int c = u % chunks;
      for (int j = 0; j < kTilesPerChunk && ok; ++j, ++n) {
        const int s = n & 1;
        if (n >= 2 && !(ok = mbar_wait_warp(&sh.r_empty[s], ((n >> 1) - 1) & 1, abort))) break;
        if (lane == 0) {
          const CUtensorMap *map = j == 0 ? &tm_mkh : j == 1 ? &tm_mkl : j == 2 ? &tm_vkh : &tm_vkl;
          mbar_expect_tx(&sh.r_full[s], kTile);
          tma_load_4d(sh.ring[s], map, &sh.r_full[s], 0, kvh, c * 128, b);
          tma_load_4d(sh.ring[s] + kHalf, map, &sh.r_full[s], 64, kvh, c * 128, b);
        }
      }
    }
    __syncwarp();
    if (*abort && chunks > 0) {  // drain copies in flight before the shared memory goes away
      int never = 0;
      mbar_wait(&sh.q_full, 0, &never);
      for (int s = 0; s < 2; ++s) {
        const int issued = n / 2 + (s < (n & 1) ? 1 : 0);
        if (issued > 0) mbar_wait(&sh.r_full[s], (issued - 1) & 1, &never);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    bool ok = !*abort && chunks > 0;
    if (ok) ok = mbar_wait_warp(&sh.q_full, 0, abort);
    bool have_q2 = kSel == 0;  // Q^2 is awaited only before its first product
    int n = 0;
    for (int u = 0; u < units && ok; ++u) {
      const bool transposed = u >= chunks;
      const int a = u & 1;
      if (u >= 2 && !(ok = mbar_wait_warp(&sh.acc_empty[a], ((u >> 1) - 1) & 1, abort))) break;
      const uint32_t acc_l = tmem + kAccStride * a, acc_u = acc_l + 128;
      for (int j = 0; j < kTilesPerChunk && ok; ++j, ++n) {
        const int s = n & 1;
        if (!(ok = mbar_wait_warp(&sh.r_full[s], (n >> 1) & 1, abort))) break;
        if (j >= 2 && !have_q2) {
          if (!(ok = mbar_wait_warp(&sh.q2_full, 0, abort))) break;
          have_q2 = true;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint8_t *x = sh.ring[s];
          if (!transposed) {  // rows x blocks
            if (j < 2) {
              mma_tile(acc_l, sh.q, x, j == 1);
            } else if (j == 2) {
              mma_tile(acc_u, sh.q2h, x, false);
              mma_tile(acc_u, sh.q2l, x, true);
            } else {
              mma_tile(acc_u, sh.q2h, x, true);
            }
          } else {  // blocks x rows
            if (j < 2) {
              mma_tile(acc_l, x, sh.q, j == 1);
            } else if (j == 2) {
              mma_tile(acc_u, x, sh.q2h, false);
              mma_tile(acc_u, x, sh.q2l, true);
            } else {
              mma_tile(acc_u, x, sh.q2h, true);
            }
          }
          tc_commit(&sh.r_empty[s]);
          if (j == kTilesPerChunk - 1) tc_commit(&sh.acc_full[a]);
        }
        __syncwarp();
      }
    }
    if (*abort && chunks > 0) {
      int never = 0;
      if (lane == 0) tc_commit(&sh.drain);
      __syncwarp();
      mbar_wait(&sh.drain, 0, &never);
    }
  } else {
    // ------------------------------------------------------------------ Q^2 = hi + lo
    // Warps 2..11 together: the epilogue warps have nothing to do until pass 1's first
    // accumulators, and the var-K products wait for Q^2.
    if (kSel > 0 && chunks > 0) {
      const bool ok = mbar_wait(&sh.q_full, 0, abort);
      if (ok) {
        const int tid = threadIdx.x - 64;
        for (int i = tid; i < (int)(kTile / 16); i += kThreads - 64) {
          const uint4 v = reinterpret_cast<const uint4 *>(sh.q)[i];
          const uint32_t *w = reinterpret_cast<const uint32_t *>(&v);
          uint4 hi4, lo4;
          uint32_t *hw = reinterpret_cast<uint32_t *>(&hi4), *lw = reinterpret_cast<uint32_t *>(&lo4);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[k]));
            const float s0 = f.x * f.x, s1 = f.y * f.y;  // exact: 16 significant bits
            const __nv_bfloat16 h0 = __float2bfloat16_rn(s0), h1 = __float2bfloat16_rn(s1);
            const __nv_bfloat16 l0 = __float2bfloat16_rn(s0 - __bfloat162float(h0));
            const __nv_bfloat16 l1 = __float2bfloat16_rn(s1 - __bfloat162float(h1));
            hw[k] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
            lw[k] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
          }
          reinterpret_cast<uint4 *>(sh.q2h)[i] = hi4;
          reinterpret_cast<uint4 *>(sh.q2l)[i] = lo4;
        }
      }
      fence_proxy_async();  // generic writes -> read by the tensor core
      mbar_arrive(&sh.q2_full);
    }
  }
  if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    // Two warpgroups: in pass 1 group g reduces columns [64 g, 64 g + 64) of every chunk for
    // its row, in pass 2 rows [64 g, 64 g + 64) for its block; the halves meet in shared memory.
    const int g = (warp - 4) >> 2;
    const int ew = warp & 3;
    const int e = ew * 32 + lane;                    // TMEM lane: row (pass 1) or block (pass 2)
    const uint32_t lane_off = (uint32_t)(ew * 32) << 16;
    const int rows = min(kBlock, p.L - t * kBlock);  // valid query rows
    const float scale = p.scale, scale2 = p.scale2;
    bool ok = !*abort;
    int red_k = 0;
    auto all_sync = [&]() { named_sync(1, 256); };
    auto grp_sync = [&]() { named_sync(2, 128); };  // group 0 only (the selection)
    // Pass 1: running max / sum of this half of row e (log2 units), 32 columns at a time.
    float m = -INFINITY, ssum = 0.f;
    // Resident path: each slice's running max after it, so that the kept 2^(logit - max)
    // become probabilities with one multiply once the row LSE is known.
    float sm0 = -INFINITY, sm1 = -INFINITY, sm2 = -INFINITY, sm3 = -INFINITY;
    auto slice_max = [&](int k) { return k == 0 ? sm0 : k == 1 ? sm1 : k == 2 ? sm2 : sm3; };
    for (int u = 0; u < chunks; ++u) {
      const int a = u & 1;
      if (ok) ok = mbar_wait_warp(&sh.acc_full[a], (u >> 1) & 1, abort);
      tc_fence_after();
      const int ncol = min(128, t - 128 * u);  // visible columns of this chunk
      if (ok && 64 * g < ncol) {
#pragma unroll 1
        for (int q2 = 0; q2 < 2; ++q2) {
          const int c0 = 64 * g + 32 * q2;
          float vl[32], vu[32];
          tmem_ld32(tmem + lane_off + kAccStride * a + c0, vl);
          if (kSel > 0) tmem_ld32(tmem + lane_off + kAccStride * a + 128 + c0, vu);
          tmem_wait_ld();
          float cmax = -INFINITY;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float x = c0 + c < ncol ? sel_logit<kSel>(vl[c], kSel > 0 ? vu[c] : 0.f, scale, scale2) * kLog2e
                                          : -INFINITY;
            if (kSel == 2) vu[c] = sqrtf(fmaxf(__fmul_rn(vu[c], scale2), 0.f));  // dispersion weight
            vl[c] = x;
            cmax = fmaxf(cmax, x);
          }
          const float mn = fmaxf(m, cmax);
          if (mn != -INFINITY) {
            float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const float e0 = ex2(vl[c] - mn), e1 = ex2(vl[c + 1] - mn);
              acc0 += e0;
              acc1 += e1;
              vl[c] = e0;
              vl[c + 1] = e1;
            }
            ssum = (m == -INFINITY ? 0.f : ssum * ex2(m - mn)) + (acc0 + acc1);
            m = mn;
          } else {
#pragma unroll
            for (int c = 0; c < 32; ++c) vl[c] = 0.f;
          }
          if (resident) {  // keep 2^(logit - mn) (and the weights) for the column sums
            tmem_st32(tmem + lane_off + kAccStride * a + c0, vl);
            if (kSel == 2) tmem_st32(tmem + lane_off + kAccStride * a + 128 + c0, vu);
            const int k = 2 * u + q2;
            if (k == 0) sm0 = mn; else if (k == 1) sm1 = mn; else if (k == 2) sm2 = mn; else sm3 = mn;
          }
        }
      }
      if (resident) {
        tmem_wait_st();
      } else {
        tc_fence_before();
        mbar_arrive(&sh.acc_empty[a]);
      }
    }
    sh.part_m[g][e] = m;
    sh.part_s[g][e] = ssum;
    all_sync();
    if (g == 0) {
      const float m0 = sh.part_m[0][e], m1 = sh.part_m[1][e];
      const float mm = fmaxf(m0, m1);
      const float s0 = m0 == -INFINITY ? 0.f : sh.part_s[0][e] * ex2(m0 - mm);
      const float s1 = m1 == -INFINITY ? 0.f : sh.part_s[1][e] * ex2(m1 - mm);
      sh.lse[e] = mm + __log2f(s0 + s1);
    }
    all_sync();
    // Resident path: p = 2^(logit - LSE) from the kept exponentials; warp ew sums its 32 rows of each
    // 32-column slice by a shuffle butterfly (after the rounds lane l holds column l), the
    // four warps' partials meet in shared memory, and group 0 forms block kb = 128 c + e.
    for (int c = 0; resident && c < chunks; ++c) {
      const int ncol = min(128, t - 128 * c);
      const float lse_row = sh.lse[e];
      const bool row_ok = e < rows;
#pragma unroll 1
      for (int q2 = 0; q2 < 2; ++q2) {
        const int c0 = 64 * g + 32 * q2;
        float v[32];
        if (ok && c0 < ncol) {
          float w[32];
          tmem_ld32(tmem + lane_off + kAccStride * c + c0, v);
          if (kSel == 2) tmem_ld32(tmem + lane_off + kAccStride * c + 128 + c0, w);
          tmem_wait_ld();
          // p = 2^(logit - mn) x 2^(mn - LSE); columns past the visible ones hold 0.
          const float f = row_ok ? ex2(slice_max(2 * c + q2) - lse_row) : 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            float x = v[i] * f;
            if (kSel == 2) x *= w[i];
            v[i] = x;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
          const bool upper = (lane & o) != 0;
#pragma unroll
          for (int i = 0; i < o; ++i) {
            const float send = upper ? v[i] : v[i + o];
            const float keep = upper ? v[i + o] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
        }
        sh.colpart[g][ew][32 * q2 + lane] = v[0];
      }
      all_sync();
      if (g == 0 && 128 * c + e < p.nb) {
        const int kb = 128 * c + e, gc = e >> 6, col = e & 63;
        float score = 0.f;
        if (kb < t) {
          float total = (sh.colpart[gc][0][col] + sh.colpart[gc][1][col]) +
                        (sh.colpart[gc][2][col] + sh.colpart[gc][3][col]);
          if (kSel == 2) total *= p.sigma_v[((int64_t)b * p.nb + kb) * p.Hkv + kvh];
          score = total / (float)rows;
        }
        sh.sc[kb] = score;
      }
      all_sync();
    }
    // Pass 2: block kb = 128 c + e sums the probabilities of this group's rows.
    for (int u = chunks; !resident && u < 2 * chunks; ++u) {
      const int a = u & 1, c = u - chunks;
      if (ok) ok = mbar_wait_warp(&sh.acc_full[a], (u >> 1) & 1, abort);
      tc_fence_after();
      const int kb = 128 * c + e;
      float colsum = 0.f;
      if (ok && 128 * c + 32 * ew < t && 64 * g < rows) {  // some block of this warp is visible
#pragma unroll 1
        for (int q2 = 0; q2 < 2; ++q2) {
          const int r0 = 64 * g + 32 * q2;
          float vl[32], vu[32];
          tmem_ld32(tmem + lane_off + kAccStride * a + r0, vl);
          if (kSel > 0) tmem_ld32(tmem + lane_off + kAccStride * a + 128 + r0, vu);
          tmem_wait_ld();
          float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
          for (int r = 0; r < 32; ++r) {
            const int row = r0 + r;
            const float l = sel_logit<kSel>(vl[r], kSel > 0 ? vu[r] : 0.f, scale, scale2) * kLog2e;
            float w = ex2(l - sh.lse[row]);
            if (kSel == 2) w *= sqrtf(fmaxf(__fmul_rn(vu[r], scale2), 0.f));
            w = row < rows ? w : 0.f;
            if (r & 1) acc1 += w; else acc0 += w;
          }
          colsum += acc0 + acc1;
        }
      }
      tc_fence_before();
      mbar_arrive(&sh.acc_empty[a]);
      if (g == 1) sh.part_s[1][e] = colsum;
      all_sync();
      if (g == 0 && kb < p.nb) {
        float score = 0.f;
        if (kb < t) {
          float total = colsum + sh.part_s[1][e];
          if (kSel == 2) total *= p.sigma_v[((int64_t)b * p.nb + kb) * p.Hkv + kvh];
          score = total / (float)rows;
        }
        sh.sc[kb] = score;
      }
      all_sync();
    }
    if (g == 1) {  // the selection is group 0's; group 1 only reports whether its waits held
      sh.part_m[1][e] = ok ? 1.f : 0.f;
      all_sync();
    } else {
      all_sync();
      ok = ok && sh.part_m[1][e] == 1.f;
    for (int kb = 128 * chunks + e; kb < p.nb; kb += 128) sh.sc[kb] = 0.f;
    // Selection (kernels.py:129-151): keep = score > 0 and score >= alpha * max score, plus
    // the protected blocks; the group agrees on success before anything is written.
    float lx = 0.f;
    for (int kb = e; kb < p.nb; kb += 128) lx = fmaxf(lx, sh.sc[kb]);
    lx = warp_max(lx);
    float *red = sh.red[red_k & 1];
    if (lane == 0) {
      red[ew] = lx;
      red[4 + ew] = ok ? 1.f : 0.f;
    }
    grp_sync();
    ++red_k;
    const float smax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const bool wg_ok = (red[4] + red[5]) + (red[6] + red[7]) == 4.f;
    if (p.scores && wg_ok)
      for (int kb = e; kb < p.nb; kb += 128) p.scores[(((int64_t)b * p.nb + t) * p.nb + kb) * p.H + h] = sh.sc[kb];
    const SelectArgs &sa = p.sel;
    if (sa.route.lists) {
      const float thr = smax * sa.alpha;
      const int64_t rrow = sa.route.row(b, h, t, sa.H);
      int32_t *list = sa.route.lists + rrow * sa.route.nb;
      uint32_t *tail = sa.route.tail + rrow * sa.route.words;
      auto active_at = [&](int kb) {
        if (kb >= sa.nb || kb > t) return false;
        const float s = sh.sc[kb];
        return sa.all_causal || (s >= thr && s > 0.f) || is_protected(t, kb, sa.nb, sa.sink, sa.window, sa.last_full);
      };
      const int nch = (sa.nb + 127) / 128;
      int *cnt = sh.scan[red_k & 1];
      for (int j = 0; j < nch; ++j) {
        const unsigned bal = __ballot_sync(0xffffffffu, active_at(128 * j + e));
        if (lane == 0) cnt[4 * j + ew] = __popc(bal);
      }
      grp_sync();
      ++red_k;
      int base = 0;
      for (int j = 0; j < nch; ++j) {
        const int kb = 128 * j + e;
        const bool active = active_at(kb);
        const unsigned bal = __ballot_sync(0xffffffffu, active);
        int pre = 0;
        for (int w = 0; w < ew; ++w) pre += cnt[4 * j + w];
        if (active && wg_ok) list[base + pre + __popc(bal & ((1u << lane) - 1u))] = kb;
        const unsigned tb = __ballot_sync(0xffffffffu, kb < sa.nb && kb < t && !active);
        if (lane == 0 && kb < sa.nb && wg_ok) tail[kb >> 5] = tb;
        base += (cnt[4 * j] + cnt[4 * j + 1]) + (cnt[4 * j + 2] + cnt[4 * j + 3]);
      }
      if (e == 0) sa.route.counts[rrow] = wg_ok ? base : 0;
    }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && sh.abort) atomicExch(device_error, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

template <int kSel>
size_t selector_route_tc_smem() { return sizeof(SelSmem<(kSel > 0)>) + 1024; }

int launch_selector_route_tc(const SelParams &p, int selector, int tiles, int heads, int B, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  if (p.nb > kMaxBlocks) return FPX_ERR_UNSUPPORTED;
  if (!p.mk_hi || !p.mk_lo || !p.vk_hi || !p.vk_lo) return FPX_ERR_INVALID;
  int *device_error = device_error_word();
  if (!device_error) return FPX_ERR_CUDA;
  const int64_t d = kHeadDim, dstride = (int64_t)p.Hkv * kHeadDim, bstride = (int64_t)p.nb * dstride;
  CUtensorMap tq, tmkh, tmkl, tvkh, tvkl;
  if (!encode_4d(&tq, p.q, d, p.H, p.L, B, p.q_sh, p.q_sl, p.q_sb) ||
      !encode_4d(&tmkh, p.mk_hi, d, p.Hkv, p.nb, B, kHeadDim, dstride, bstride) ||
      !encode_4d(&tmkl, p.mk_lo, d, p.Hkv, p.nb, B, kHeadDim, dstride, bstride) ||
      !encode_4d(&tvkh, p.vk_hi, d, p.Hkv, p.nb, B, kHeadDim, dstride, bstride) ||
      !encode_4d(&tvkl, p.vk_lo, d, p.Hkv, p.nb, B, kHeadDim, dstride, bstride))
    return FPX_ERR_INVALID;
  const dim3 grid(tiles, heads, B);
#define FPX_SEL_TC(K)                                                                                   \
  do {                                                                                                  \
    const size_t smem = selector_route_tc_smem<K>();                                                    \
    cudaFuncSetAttribute(selector_route_tc_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    selector_route_tc_kernel<K><<<grid, kThreads, smem, s>>>(tq, tmkh, tmkl, tvkh, tvkl, p, device_error); \
  } while (0)
  if (selector == FPX_METHOD_MEAN_BALANCED)
    FPX_SEL_TC(0);
  else if (selector == FPX_METHOD_CGF_MEAN)
    FPX_SEL_TC(1);
  else if (selector == FPX_METHOD_DISPERSION_MEAN)
    FPX_SEL_TC(2);
  else
    return FPX_ERR_INVALID;
#undef FPX_SEL_TC
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

}  // namespace fpx
