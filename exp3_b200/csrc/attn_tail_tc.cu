// Block-mean tail on the 5th-generation tensor core, merged into the exact output in place.
//
// Reference: kernels.py:179-230 (mean_tail) and kernels.py:312-325 (merge_exact_mean). For
// query tile t of head h the tail is every block kb < t that the routing did not select; each
// tail block is one pseudo-key with key mean_k[kb] and value mean_v[kb] (fp32 descriptors) and
// logit q . mean_k[kb] * scale + ln n_kb. Tail blocks lie strictly before the tile, so they are
// full blocks: n_kb = 128 and the ln 128 only shifts the tail's LSE. The tail's softmax output
// and LSE are merged with the exact path's by logaddexp, in place on the exact output.
//
// The pseudo-keys of a tile are processed as chunks of 128 consecutive blocks, as if they were
// keys: S = Q . mean_K^T for every block of the chunk, columns outside the tail masked. The
// fp32 mean K enters as two bf16 halves, mean_K = hi + lo (lo = the rounding remainder), and S
// is accumulated from Q . hi^T + Q . lo^T, so the logits carry ~16 mantissa bits of mean_K
// rather than bf16's 8. P (bf16, as the exact path rounds it) multiplies the bf16 mean V.
//
// Structure as the exact kernel (attn_tc.cu), with its work units (exact_unit): one CTA runs
// two tiles of one KV group, two heads at the same query tile or the last head of an odd group
// at tiles t and t - 1, sharing every chunk; 384 threads —
//   warps 0..3 / 4..7  softmax of tiles A / B (thread = query row = TMEM lane), then the merge
//   warp 8  TMA: Q, then the mean-K ring (stage 0 = high halves, stage 1 = low halves)
//   warp 9  MMA issuer      warp 10  TMA: the mean-V ring      warp 11  idle
// TMEM: S_A, S_B, O_A, O_B (128 columns each); P overwrites the first 64 columns of S.
// The merge loads the exact output tile by TMA into the tile's Q buffer (free once its last
// product is done), merges row by row and stores it back by TMA.
// Waits are bounded as in the exact kernel: a wait that gives up flags the CTA and the device
// error word; roles drain their copies and MMAs and exit.
#include <cuda.h>

#include <algorithm>

#include "attn.cuh"
#include "tc.cuh"

namespace fpx {

namespace {

using namespace tc;

constexpr uint32_t kHalf = 128 * 128;
constexpr uint32_t kTile = 2 * kHalf;
constexpr uint32_t kIdescQK = idesc_bf16(128, 128, false);
constexpr uint32_t kIdescPV = idesc_bf16(128, 128, true);
constexpr int kThreads = 384;
constexpr int kSoftmaxRegs = 216, kControlRegs = 64;
constexpr int kMaxBlocks = 2048;
constexpr int kMaxChunks = kMaxBlocks / 128;
constexpr float kRescaleThreshold = 8.f;
constexpr float kLn128 = 4.852030263919617f;

struct alignas(1024) Smem {
  uint8_t q[2][kTile];  // Q of tiles A and B; then each tile's exact output for the merge
  uint8_t k[2][kTile];  // mean K of one chunk: [0] high halves, [1] low halves
  uint8_t v[2][kTile];  // mean V ring
  uint64_t q_full, k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], p_full[2], o_done[2], oe_full[2], drain;
  uint32_t tmem_base;
  int abort, n_union;
  uint32_t bits[2][kMaxBlocks / 32];
  uint8_t u_chunk[kMaxChunks], u_flags[kMaxChunks];
};

FPX_INLINE uint64_t desc_kmajor(const uint8_t *tile, int kk) {
  return smem_desc_sw128(smem_u32(tile) + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}
FPX_INLINE uint64_t desc_v(const uint8_t *tile, int kk) {
  return smem_desc_sw128(smem_u32(tile) + kk * 2048, kHalf, 1024);
}
FPX_INLINE uint32_t sw128_offset(int row, int col) {
  const int half = col >> 6, chunk = (col & 63) >> 3;
  return half * kHalf + row * 128 + ((chunk ^ (row & 7)) << 4) + ((col & 7) << 1);
}

// One row of P for a chunk: p = 2^(s * scale_log2 - m) (masked columns hold -inf and give 0),
// packed to bf16 into TMEM; returns the fp32 row sum before rounding.
FPX_INLINE float tail_row(const float (&sv)[128], float sl2, float neg, uint32_t p_addr) {
  const uint64_t sl2x2 = pk2(sl2, sl2), negx2 = pk2(neg, neg);
  uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    uint32_t pk[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      const uint64_t xx = ffma2(pk2(sv[32 * q4 + 2 * c], sv[32 * q4 + 2 * c + 1]), sl2x2, negx2);
      float a, e;
      up2(xx, a, e);
      const uint64_t pp = pk2(ex2(a), ex2(e));
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

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    mean_tail_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_mkh,
                        const __grid_constant__ CUtensorMap tm_mkl, const __grid_constant__ CUtensorMap tm_mv,
                        const __grid_constant__ CUtensorMap tm_o, MeanParams p, int tiles, int kv_count,
                        float scale_log2,
                        int *device_error) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem &sh = *reinterpret_cast<Smem *>(smem_raw + pad);
  volatile int *abort = &sh.abort;

  // x: (KV group, head pair), fastest; y: tile, longest tail first; z: batch.
  // The exact kernel's work units and launch order (exact_unit): a head pair at one tile, or the
  // last head of an odd group at tiles t and t - 1, whose tails are nearly the same blocks.
  const ExactUnit unit = exact_unit(blockIdx.x, p.tile_begin, tiles, p.head_begin / p.group, kv_count, p.group);
  const int kvh = unit.kvh;
  const int b = blockIdx.z;
  const int hA = unit.h[0], hB = unit.h[1], tA = unit.t[0], tB = unit.t[1];
  const bool has_b = unit.has_b;
  auto head_of = [&](int x) { return x ? hB : hA; };
  auto tile_of = [&](int x) { return x ? tB : tA; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int words = p.route.words;
  const bool failed = *reinterpret_cast<volatile int *>(device_error) != 0;
  if (failed) return;
  // A tile has a tail iff some block kb < t went unselected: its selected count (blocks <= t,
  // the diagonal always among them) is then below t + 1. A CTA whose tiles both have none
  // leaves before it touches the bitmaps or a barrier: the exact output stands.
  {
    const int c_a = p.route.counts[p.route.row(b, hA, tA, p.H)];
    const int c_b = has_b ? p.route.counts[p.route.row(b, hB, tB, p.H)] : tB + 1;
    if (c_a >= tA + 1 && c_b >= tB + 1) return;
  }

  // Tail bits of both tiles, then the chunks that hold any tail column (ascending, with flags).
  for (int x = 0; x < 2; ++x) {
    const bool live = (x == 0 || has_b) && !failed;
    const uint32_t *src = p.route.tail + p.route.row(b, live ? head_of(x) : hA, live ? tile_of(x) : tA, p.H) * words;
    for (int w = threadIdx.x; w < kMaxBlocks / 32; w += kThreads) sh.bits[x][w] = (live && w < words) ? src[w] : 0u;
  }
  __syncthreads();
  if (warp == 0) {
    const int chunks = (p.nb + 127) / 128;
    int flags = 0;
    if (lane < chunks)
      for (int x = 0; x < 2; ++x) {
        const uint32_t *w4 = sh.bits[x] + 4 * lane;
        if (w4[0] | w4[1] | w4[2] | w4[3]) flags |= 1 << x;
      }
    const unsigned any = __ballot_sync(0xffffffffu, flags != 0);
    if (flags) {
      const int pos = __popc(any & ((1u << lane) - 1u));
      sh.u_chunk[pos] = (uint8_t)lane;
      sh.u_flags[pos] = (uint8_t)flags;
    }
    if (lane == 0) sh.n_union = __popc(any);
  }
  __syncthreads();
  const int n_union = sh.n_union;
  if (n_union == 0) return;  // no tail in either tile: the exact output stands

  if (threadIdx.x == 0) {
    mbar_init(&sh.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh.k_full[s], 1);
      mbar_init(&sh.k_empty[s], 1);
      mbar_init(&sh.v_full[s], 1);
      mbar_init(&sh.v_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&sh.s_full[x], 1);
      mbar_init(&sh.p_full[x], 128);
      mbar_init(&sh.o_done[x], 1);
      mbar_init(&sh.oe_full[x], 1);
    }
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(&sh.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const int n_tiles = has_b ? 2 : 1;

  if (warp >= 8) {
    regs_dec<kControlRegs>();
    if (warp == 8 || warp == 10) {
      // ------------------------------------------------------------ TMA producers
      const bool is_k = warp == 8;
      int issued[2] = {0, 0};
      if (is_k && lane == 0) {
        mbar_expect_tx(&sh.q_full, kTile * n_tiles);
        for (int x = 0; x < n_tiles; ++x) {
          tma_load_4d(sh.q[x], &tm_q, &sh.q_full, 0, head_of(x), tile_of(x) * 128, b);
          tma_load_4d(sh.q[x] + kHalf, &tm_q, &sh.q_full, 64, head_of(x), tile_of(x) * 128, b);
        }
      }
      bool ok = true;
      for (int u = 0; u < n_union && ok; ++u) {
        const int c = sh.u_chunk[u];
        if (is_k) {  // both halves of chunk u: stage 0 <- high, stage 1 <- low
          for (int part = 0; part < 2 && ok; ++part) {
            if (u > 0 && !(ok = mbar_wait_warp(&sh.k_empty[part], (u - 1) & 1, abort))) break;
            if (lane == 0) {
              const CUtensorMap *map = part ? &tm_mkl : &tm_mkh;
              mbar_expect_tx(&sh.k_full[part], kTile);
              tma_load_4d(sh.k[part], map, &sh.k_full[part], 0, kvh, c * 128, b);
              tma_load_4d(sh.k[part] + kHalf, map, &sh.k_full[part], 64, kvh, c * 128, b);
            }
            issued[part] = u + 1;
          }
        } else {
          const int s = u & 1, n = u >> 1;
          if (n > 0 && !(ok = mbar_wait_warp(&sh.v_empty[s], (n - 1) & 1, abort))) break;
          if (lane == 0) {
            mbar_expect_tx(&sh.v_full[s], kTile);
            tma_load_4d(sh.v[s], &tm_mv, &sh.v_full[s], 0, kvh, c * 128, b);
            tma_load_4d(sh.v[s] + kHalf, &tm_mv, &sh.v_full[s], 64, kvh, c * 128, b);
          }
          issued[s] = n + 1;
        }
      }
      __syncwarp();
      if (*abort) {  // drain copies still in flight before the shared memory goes away
        int never = 0;
        if (is_k) mbar_wait(&sh.q_full, 0, &never);
        for (int s = 0; s < 2; ++s)
          if (issued[s] > 0) mbar_wait(is_k ? &sh.k_full[s] : &sh.v_full[s], (issued[s] - 1) & 1, &never);
      }
    } else if (warp == 9) {
      // ------------------------------------------------------------ MMA issuer (lane 0 alone)
      // One thread issues every product, without warp votes around its waits, and it waits for
      // a chunk's mean-V stage before it waits for that chunk's P (the stage lands long before).
      if (lane == 0 && mbar_wait(&sh.q_full, 0, abort)) {
        int pend[2] = {-1, -1}, n_pv[2] = {0, 0};
        auto flush = [&](int x) -> bool {  // P_x . V of tile x's pending chunk
          const int u = pend[x], s = u & 1;
          if (!mbar_wait(&sh.v_full[s], (u >> 1) & 1, abort)) return false;
          if (!mbar_wait(&sh.p_full[x], n_pv[x] & 1, abort)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ts(tmem + 256 + 128 * x, tmem + 128 * x + 8 * kk, desc_v(sh.v[s], kk), kIdescPV,
                   (n_pv[x] > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sh.o_done[x]);
          if (pend[x ^ 1] != u) tc_commit(&sh.v_empty[s]);
          ++n_pv[x];
          pend[x] = -1;
          return true;
        };
        bool ok = true;
        for (int u = 0; u < n_union && ok; ++u) {
          for (int x = 0; x < 2 && ok; ++x)
            if (u >= 2 && pend[x] == u - 2) ok = flush(x);
          const int flags = sh.u_flags[u];
          for (int x = 0; x < 2 && ok; ++x)
            if ((flags & (1 << x)) && pend[x] >= 0) ok = flush(x);
          for (int part = 0; part < 2 && ok; ++part) {
            if (!(ok = mbar_wait(&sh.k_full[part], u & 1, abort))) break;
            tc_fence_after();
            for (int x = 0; x < 2; ++x) {
              if (!(flags & (1 << x))) continue;
#pragma unroll
              for (int kk = 0; kk < 8; ++kk)
                mma_ss(tmem + 128 * x, desc_kmajor(sh.q[x], kk), desc_kmajor(sh.k[part], kk), kIdescQK,
                       (part > 0 || kk > 0) ? 1u : 0u);
              if (part == 1) tc_commit(&sh.s_full[x]);
            }
            tc_commit(&sh.k_empty[part]);
          }
          if (ok)
            for (int x = 0; x < 2; ++x)
              if (flags & (1 << x)) pend[x] = u;
        }
        for (int x = 0; x < 2 && ok && !*abort; ++x)
          if (pend[x] >= 0) ok = flush(x);
        if (*abort) {
          int never = 0;
          tc_commit(&sh.drain);
          mbar_wait(&sh.drain, 0, &never);
        }
      }
      __syncwarp();
    }
  } else {
    regs_inc<kSoftmaxRegs>();
    // -------------------------------------------------------------- softmax of tile x, merge
    const int x = warp >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + 128 * x;
    const uint32_t o_addr = tmem + lane_off + 256 + 128 * x;
    const bool live = x == 0 || has_b;
    const int h = head_of(x);
    const int qrow = tile_of(x) * 128 + r;
    int n_x = 0;  // chunks of this tile (the same for the whole warpgroup)
    for (int u = 0; u < n_union; ++u) n_x += (sh.u_flags[u] >> x) & 1;
    float m = -INFINITY, l = 0.f;
    bool ok = live;
    int i = 0;  // chunks of this tile so far
    for (int u = 0; u < n_union && ok; ++u) {
      if (!(sh.u_flags[u] & (1 << x))) continue;
      if (!mbar_wait_warp(&sh.s_full[x], i & 1, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + 32 * c, *reinterpret_cast<float(*)[32]>(&sv[32 * c]));
      tmem_wait_ld();
      const uint32_t *w4 = sh.bits[x] + 4 * sh.u_chunk[u];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const uint32_t w = w4[q4];
#pragma unroll
        for (int c = 0; c < 32; ++c) sv[32 * q4 + c] = ((w >> c) & 1u) ? sv[32 * q4 + c] : -INFINITY;
      }
      float mx[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mx[c] = sv[c];
#pragma unroll
      for (int c = 8; c < 128; ++c) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
      const float bmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * scale_log2;
      const float mn = fmaxf(m, bmax);
      float corr = 1.f;
      // Each row decides for itself (rows never influence one another's rounding); rows that
      // keep their max rescale O by exactly 1 when another row of the warp moves.
      const bool move = mn > m + kRescaleThreshold || m == -INFINITY;
      if (move) {
        corr = (m == -INFINITY) ? 0.f : ex2(m - mn);
        l *= corr;
        m = mn;
      }
      l += tail_row(sv, scale_log2, -m, s_addr);
      if (i > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tmem_ld32(o_addr + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= corr;
          tmem_st32(o_addr + 32 * c, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&sh.p_full[x]);
      ++i;
    }
    if (live && n_x > 0) {
      // merge_exact_mean (kernels.py:318-325): the exact tile comes in by TMA over Q_x.
      if (ok && !mbar_wait_warp(&sh.o_done[x], (n_x - 1) & 1, abort)) ok = false;
      tc_fence_after();
      if (ok) {
        if (r == 0) {
          mbar_expect_tx(&sh.oe_full[x], kTile);
          tma_load_4d(sh.q[x], &tm_o, &sh.oe_full[x], 0, h, tile_of(x) * 128, b);
          tma_load_4d(sh.q[x] + kHalf, &tm_o, &sh.oe_full[x], 64, h, tile_of(x) * 128, b);
        }
        if (!mbar_wait_warp(&sh.oe_full[x], 0, abort)) ok = false;
      }
      if (ok) {
        const int64_t lrow = ((int64_t)b * p.L + qrow) * p.H + h;
        const bool in = qrow < p.L;
        const float lse_m = m * kLn2 + logf(l) + kLn128;
        const float lse_e = in ? p.lse[lrow] : 0.f;
        const float total = logaddexp(lse_e, lse_m);
        const float we = expf(lse_e - total), wm = expf(lse_m - total);
        const float inv = 1.f / l;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float o[32];
          tmem_ld32(o_addr + 32 * c, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint8_t *ptr = sh.q[x] + sw128_offset(r, 32 * c + 8 * e);
            uint4 v4 = *reinterpret_cast<const uint4 *>(ptr);
            uint32_t *w = reinterpret_cast<uint32_t *>(&v4);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 ex = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[j]));
              w[j] = pack_bf16(ex.x * we + o[8 * e + 2 * j] * inv * wm, ex.y * we + o[8 * e + 2 * j + 1] * inv * wm);
            }
            *reinterpret_cast<uint4 *>(ptr) = v4;
          }
        }
        if (in) p.lse[lrow] = total;
      }
      fence_proxy_async();
      named_sync(1 + x, 128);
      if (r == 0 && ok && !*abort) {
        tma_store_4d(&tm_o, sh.q[x], 0, h, tile_of(x) * 128, b);
        tma_store_4d(&tm_o, sh.q[x] + kHalf, 64, h, tile_of(x) * 128, b);
        bulk_commit();
        bulk_wait0();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && sh.abort) atomicExch(device_error, 1);
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

size_t mean_tail_tc_smem() { return sizeof(Smem) + 1024; }

int launch_mean_tail_tc(const MeanParams &p, int B, int tiles, int heads, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  if (p.nb > kMaxBlocks) return FPX_ERR_UNSUPPORTED;
  if (!p.mk_hi || !p.mk_lo || !p.mv_hi) return FPX_ERR_INVALID;
  int *device_error = device_error_word();
  if (!device_error) return FPX_ERR_CUDA;
  const int64_t d = kHeadDim, dstride = (int64_t)p.Hkv * kHeadDim, bstride = (int64_t)p.nb * dstride;
  // The block means exist only for the blocks before the launch's last tile (a shard computes
  // no more), and a chunk of 128 blocks reaches past them: the maps end there, so the copy
  // fills those rows with zeros instead of reading stale workspace (whose NaNs would survive
  // the masked columns' P = 0 in P.V).
  const int64_t mean_blocks = std::min<int64_t>(p.nb, (int64_t)p.tile_begin + tiles);
  CUtensorMap tq, tmkh, tmkl, tmv, to;
  if (!encode_4d(&tq, p.q, d, p.H, p.L, B, p.q_sh, p.q_sl, p.q_sb) ||
      !encode_4d(&tmkh, p.mk_hi, d, p.Hkv, mean_blocks, B, kHeadDim, dstride, bstride) ||
      !encode_4d(&tmkl, p.mk_lo, d, p.Hkv, mean_blocks, B, kHeadDim, dstride, bstride) ||
      !encode_4d(&tmv, p.mv_hi, d, p.Hkv, mean_blocks, B, kHeadDim, dstride, bstride) ||
      !encode_4d(&to, p.out, d, p.H, p.L, B, p.o_sh, p.o_sl, p.o_sb))
    return FPX_ERR_INVALID;
  const int kv_count = heads / p.group;
  const dim3 grid(exact_units(tiles, kv_count, p.group), 1, B);
  const size_t smem = mean_tail_tc_smem();
  cudaFuncSetAttribute(mean_tail_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  mean_tail_tc_kernel<<<grid, kThreads, smem, s>>>(tq, tmkh, tmkl, tmv, to, p, tiles, kv_count, p.scale * kLog2e,
                                                   device_error);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

}  // namespace fpx
