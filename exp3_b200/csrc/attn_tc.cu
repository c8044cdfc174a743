// Exact block-sparse causal attention on the 5th-generation tensor core (tcgen05 + TMEM + TMA).
//
// Reference semantics: upstream/flashprefill_native_forward.py:215-354 (_flash_forward) — for
// query tile t (128 rows) of head h, attend over the tile's selected 128-key blocks in ascending
// order with an online softmax in exp2 units, causal mask on the diagonal block, P rounded to
// bf16 before P.V, bf16 output and natural-log LSE.
//
// One CTA runs two query tiles of one KV group that read nearly the same K/V blocks, so every
// block loaded serves both (GQA sharing inside the CTA; no cluster multicast): heads
// hA = kv*G + 2*pair and hA + 1 at the same query tile t, or, for the last head of an odd
// group, that head at tiles t and t - 1. A CTA holding one tile runs the same per-block chain
// as a pair (the softmax, then the tile's own products), so pairing the odd head across
// neighbouring tiles removes a whole CTA's worth of time per two tiles. 384 threads in three
// warpgroups:
//   warps 0..3   softmax of tile A       warps 4..7   softmax of tile B
//   warp 8       TMA: Q, then the K ring warp 10      TMA: the V ring
//   warp 9       MMA issuer (one elected lane)        warp 11 idle
// The K and V rings stream the union of the two heads' block lists (each two stages, 128-byte
// swizzle); a K stage is released as soon as the block's QK^T products are done, a V stage once
// its P.V products are, so loads run well ahead of the tensor core. The MMA warp issues tile X's
// products only for blocks in X's own list:
//   S_X = Q_X K^T   (A = Q_X, B = K: both K-major in shared memory) into TMEM S_X,
//   O_X += P_X V    (A = P_X read from TMEM, B = V MN-major in shared memory) into TMEM O_X.
// TMEM: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512) fp32 columns x 128 lanes;
// P_X (bf16, two per column) overwrites the first 64 columns of S_X once the softmax has read it.
// While one tile runs its softmax the tensor core works on the other tile.
//
// Ordering facts the protocol relies on: a thread's tcgen05 MMAs complete in issue order and a
// commit tracks all of the thread's earlier MMAs. So when s_full[X] fires for a block, the
// previous P_X.V product has finished: O_X is stable and P_X's columns are free.
//
// Softmax (thread = query row = TMEM lane): the row max only moves when a block's max exceeds it
// by more than 8 (log2 units), so P stays below 2^8 and O is rescaled rarely; O / l at the end is
// exact either way. Scores are scaled with packed f32x2 FMAs; a fixed share of the exp2 pairs is
// computed on the FMA pipe (exp2_poly2) to offload the special-function unit.
//
// Every mbarrier wait is bounded (about 1 s); a wait that gives up flags the CTA and the device
// error word, the roles drain their in-flight copies and MMAs and exit, and later CTAs skip
// their work, so a failed launch ends quickly and the host sees fpx_device_error() != 0.
#include <cuda.h>

#include <mutex>

#include "attn.cuh"
#include "softmax_tc.cuh"
#include "tc.cuh"

namespace fpx {

__device__ int g_device_error;  // 0 = ok; 1 = a bounded wait in a tcgen05 kernel gave up

namespace {

using namespace tc;

constexpr uint32_t kHalf = 128 * 128;  // 128 rows x 64 bf16: one SW128 half tile
constexpr uint32_t kTile = 2 * kHalf;  // 128 x 128 bf16
constexpr uint32_t kIdescQK = idesc_bf16(128, 128, false);
constexpr uint32_t kIdescPV = idesc_bf16(128, 128, true);
constexpr int kKStages = 2, kVStages = 2;
constexpr int kThreads = 384;
// Launched at 168 registers per thread (384 x 168 = 64512). The control warpgroup gives
// registers up so each softmax thread holds a full 128-column row of S without spilling:
// 2 x 128 x 216 + 128 x 64 = 63488 <= 64512, and per SM sub-partition 216 + 216 + 64 <= 512.
constexpr int kSoftmaxRegs = 216, kControlRegs = 64;
constexpr int kMaxBlocks = 2048;  // union list capacity: L <= 262144
constexpr float kRescaleThreshold = 8.f;

struct alignas(1024) Smem {
  uint8_t q[2][kTile];  // Q of tiles A and B; reused to stage each tile's output
  uint8_t k[kKStages][kTile];
  uint8_t v[kVStages][kTile];
  uint64_t q_full, k_full[kKStages], k_empty[kKStages], v_full[kVStages], v_empty[kVStages];
  uint64_t s_full[2], p_full[2], o_done[2], drain;
  uint32_t tmem_base;
  int abort, n_union, n_tile[2], diag_tile[2];
  uint32_t bits[2][kMaxBlocks / 32];
  uint16_t u_blk[kMaxBlocks];
  uint8_t u_flags[kMaxBlocks];
};

// K-major SW128 operand (Q, K) at K offset 16*kk: halves of 64 columns sit kHalf apart,
// 16 columns = 32 bytes inside a half; 8-row groups 1024 B apart.
FPX_INLINE uint64_t desc_kmajor(const uint8_t *tile, int kk) {
  return smem_desc_sw128(smem_u32(tile) + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}
// MN-major SW128 V operand at key offset 16*kk: 16 keys = 16 rows of 128 B; the two 64-column
// halves (MN atoms) kHalf apart, 8-key groups 1024 B apart.
FPX_INLINE uint64_t desc_v(const uint8_t *tile, int kk) {
  return smem_desc_sw128(smem_u32(tile) + kk * 2048, kHalf, 1024);
}
// Descriptor low-word steps (desc_join in tc.cuh) of K-step kk: K-major (Q, K) and MN-major V, as desc_kmajor / desc_v place them.
constexpr uint32_t kmajor_step(int kk) { return (uint32_t)(((kk >> 2) * kHalf + (kk & 3) * 32) >> 4); }
constexpr uint32_t v_step(int kk) { return (uint32_t)(kk * 2048 >> 4); }
// Byte offset of (row, col) inside a 128 x 128 bf16 SW128 K-major tile.
FPX_INLINE uint32_t sw128_offset(int row, int col) {
  const int half = col >> 6, chunk = (col & 63) >> 3;
  return half * kHalf + row * 128 + ((chunk ^ (row & 7)) << 4) + ((col & 7) << 1);
}

}  // namespace

template <int kEmu>
__global__ void __launch_bounds__(kThreads, 1)
    exact_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                    ExactParams p, int tiles, int kv_count) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem &sh = *reinterpret_cast<Smem *>(smem_raw + pad);
  volatile int *abort = &sh.abort;

  // x: the work unit in launch order (longest tiles first, a KV group's units side by side, so
  // they read the same K/V blocks at about the same time); z: batch.
  const ExactUnit unit = exact_unit(blockIdx.x, p.tile_begin, tiles, p.head_begin / p.group, kv_count, p.group);
  const int kvh = unit.kvh;
  const int b = blockIdx.z;
  const int hA = unit.h[0];
  const bool has_b = unit.has_b;
  // Tile x's head and query tile (128 rows), chosen by select so that nothing goes to local memory.
  const int hB = unit.h[1], tA = unit.t[0], tB = unit.t[1];
  auto head_of = [&](int x) { return x ? hB : hA; };
  auto tile_of = [&](int x) { return x ? tB : tA; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool failed = *reinterpret_cast<volatile int *>(&g_device_error) != 0;
  // Block lists: the fused path's compact lists, or the reference's [B, nb, nb, H] int64
  // indices with [B, nb, H] counts (fpx_exact_attention); entries past the tile are dropped,
  // as the reference's causal mask leaves them no key.
  const bool ref = p.ref_indices != nullptr;
  const int nb = ref ? p.nb : p.route.nb;
  int cnt[2];
  const int32_t *lists[2];
  for (int x = 0; x < 2; ++x) {
    const bool live = x == 0 || has_b;
    const int h = live ? head_of(x) : hA, tx = live ? tile_of(x) : tA;
    const int64_t rr = ref ? 0 : p.route.row(b, h, tx, p.H);
    cnt[x] = (live && !failed) ? (ref ? p.ref_counts[((int64_t)b * nb + tx) * p.H + h] : p.route.counts[rr]) : 0;
    cnt[x] = min(max(cnt[x], 0), nb);
    lists[x] = ref ? nullptr : p.route.lists + rr * p.route.nb;
  }
  const int words = (nb + 31) / 32;

  if (threadIdx.x == 0) {
    mbar_init(&sh.q_full, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&sh.k_full[s], 1);
      mbar_init(&sh.k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&sh.v_full[s], 1);
      mbar_init(&sh.v_empty[s], 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(&sh.s_full[x], 1);
      mbar_init(&sh.p_full[x], 128);
      mbar_init(&sh.o_done[x], 1);
    }
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  for (int w = threadIdx.x; w < 2 * (kMaxBlocks / 32); w += kThreads) (&sh.bits[0][0])[w] = 0u;
  if (warp == 9) {
    tmem_alloc(&sh.tmem_base, 512);
    tmem_relinquish();
  }
  __syncthreads();
  for (int x = 0; x < 2; ++x)
    for (int i = threadIdx.x; i < cnt[x]; i += kThreads) {
      const int blk = ref ? (int)p.ref_indices[(((int64_t)b * nb + tile_of(x)) * nb + i) * p.H + head_of(x)] : lists[x][i];
      if (blk >= 0 && blk <= tile_of(x)) atomicOr(&sh.bits[x][blk >> 5], 1u << (blk & 31));
    }
  __syncthreads();
  if (warp == 8) {  // union of the two lists, ascending, with per-tile flags
    int base = 0;
    for (int w0 = 0; w0 < words; w0 += 32) {
      const int w = w0 + lane;
      const uint32_t a = w < words ? sh.bits[0][w] : 0u, c = w < words ? sh.bits[1][w] : 0u;
      const uint32_t u = a | c;
      const int n = __popc(u);
      int incl = n;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int pos = base + incl - n;
      for (uint32_t bits = u; bits; bits &= bits - 1) {
        const int bit = __ffs(bits) - 1;
        sh.u_blk[pos] = (uint16_t)(32 * w + bit);
        sh.u_flags[pos] = (uint8_t)(((a >> bit) & 1u) | (((c >> bit) & 1u) << 1));
        ++pos;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) sh.n_union = base;
    // Per tile: the number of blocks it runs and whether the diagonal block is among them
    // (ascending order puts it last).
    for (int x = 0; x < 2; ++x) {
      int nx = 0;
      for (int w = lane; w < words; w += 32) nx += __popc(sh.bits[x][w]);
      nx = __reduce_add_sync(0xffffffffu, nx);
      if (lane == 0) {
        sh.n_tile[x] = nx;
        sh.diag_tile[x] = (sh.bits[x][tile_of(x) >> 5] >> (tile_of(x) & 31)) & 1u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const int n_union = sh.n_union;
  const int n_tiles = has_b ? 2 : 1;

  if (warp >= 8) {
    regs_dec<kControlRegs>();
    if (warp == 8 || warp == 10) {
      // ------------------------------------------------------------ TMA producers (K / V rings)
      const bool is_k = warp == 8;
      const int stages = is_k ? kKStages : kVStages;
      uint64_t *full = is_k ? sh.k_full : sh.v_full;
      uint64_t *empty = is_k ? sh.k_empty : sh.v_empty;
      const CUtensorMap *map = is_k ? &tm_k : &tm_v;
      int issued[2] = {0, 0};
      if (n_union > 0) {
        if (is_k && lane == 0) {
          mbar_expect_tx(&sh.q_full, kTile * n_tiles);
          for (int x = 0; x < n_tiles; ++x) {
            tma_load_4d(sh.q[x], &tm_q, &sh.q_full, 0, head_of(x), tile_of(x) * 128, b);
            tma_load_4d(sh.q[x] + kHalf, &tm_q, &sh.q_full, 64, head_of(x), tile_of(x) * 128, b);
          }
        }
        for (int u = 0; u < n_union; ++u) {
          const int s = u % stages, n = u / stages;
          if (n > 0 && !mbar_wait_warp(&empty[s], (n - 1) & 1, abort)) break;
          const int blk = sh.u_blk[u];
          uint8_t *dst = is_k ? sh.k[s] : sh.v[s];
          if (lane == 0) {
            mbar_expect_tx(&full[s], kTile);
            tma_load_4d(dst, map, &full[s], 0, kvh, blk * 128, b);
            tma_load_4d(dst + kHalf, map, &full[s], 64, kvh, blk * 128, b);
          }
          issued[s] = n + 1;
        }
        __syncwarp();
        if (*abort) {  // drain copies still in flight before the shared memory goes away
          int never = 0;
          if (is_k) mbar_wait(&sh.q_full, 0, &never);
          for (int s = 0; s < stages; ++s)
            if (issued[s] > 0) mbar_wait(&full[s], (issued[s] - 1) & 1, &never);
        }
      }
    } else if (warp == 9) {
      // ------------------------------------------------------------ MMA issuer (lane 0 alone)
      // The issuing thread is on the critical path, so it runs alone, without warp votes,
      // with every descriptor's fixed part computed here, and waits for the K and V stages
      // before it waits for P: a stage has landed long before P is written, so those waits
      // stay off the softmax -> P.V -> QK^T chain.
      if (lane == 0 && n_union > 0 && mbar_wait(&sh.q_full, 0, abort)) {
        int pend[2] = {-1, -1}, n_pv[2] = {0, 0};
        static_assert(kKStages == 2 && kVStages == 2, "the stage bases below are chosen by select");
        const uint32_t hi_km = desc_hi(desc_kmajor(sh.q[0], 0)), hi_v = desc_hi(desc_v(sh.v[0], 0));
        const uint32_t q_lo0 = desc_lo(desc_kmajor(sh.q[0], 0)), q_lo1 = desc_lo(desc_kmajor(sh.q[1], 0));
        const uint32_t k_lo0 = desc_lo(desc_kmajor(sh.k[0], 0)), k_lo1 = desc_lo(desc_kmajor(sh.k[1], 0));
        const uint32_t v_lo0 = desc_lo(desc_v(sh.v[0], 0)), v_lo1 = desc_lo(desc_v(sh.v[1], 0));
        // P.V of tile x for its pending block; frees the V stage once no tile still needs it.
        auto flush = [&](int x) -> bool {
          const int u = pend[x], s = u % kVStages;
          if (!mbar_wait(&sh.v_full[s], (u / kVStages) & 1, abort)) return false;
          if (!mbar_wait(&sh.p_full[x], n_pv[x] & 1, abort)) return false;
          tc_fence_after();
          const uint32_t v_lo = s ? v_lo1 : v_lo0, o_tm = tmem + 256 + 128 * x, p_tm = tmem + 128 * x;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ts(o_tm, p_tm + 8 * kk, desc_join(v_lo + v_step(kk), hi_v), kIdescPV,
                   (n_pv[x] > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sh.o_done[x]);
          if (pend[x ^ 1] != u) tc_commit(&sh.v_empty[s]);
          ++n_pv[x];
          pend[x] = -1;
          return true;
        };
        bool ok = true;
        for (int u = 0; u < n_union && ok; ++u) {
          const int s = u % kKStages;
          // The V producer refills this block's V stage only after block u - kVStages's P.V.
          for (int x = 0; x < 2 && ok; ++x)
            if (u >= kVStages && pend[x] == u - kVStages) ok = flush(x);
          if (!ok || !(ok = mbar_wait(&sh.k_full[s], (u / kKStages) & 1, abort))) break;
          const int flags = sh.u_flags[u];
          for (int x = 0; x < 2 && ok; ++x) {
            if (!(flags & (1 << x))) continue;
            if (pend[x] >= 0 && !(ok = flush(x))) break;
            tc_fence_after();
            const uint32_t q_lo = x ? q_lo1 : q_lo0, k_lo = s ? k_lo1 : k_lo0, s_tm = tmem + 128 * x;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_ss(s_tm, desc_join(q_lo + kmajor_step(kk), hi_km), desc_join(k_lo + kmajor_step(kk), hi_km),
                     kIdescQK, kk > 0 ? 1u : 0u);
            tc_commit(&sh.s_full[x]);
            pend[x] = u;
          }
          if (ok) tc_commit(&sh.k_empty[s]);  // both tiles' QK^T of block u issued: refill its K stage
        }
        for (int x = 0; x < 2 && ok && !*abort; ++x)
          if (pend[x] >= 0) ok = flush(x);
        if (*abort) {  // let every MMA this thread issued finish before TMEM is released
          int never = 0;
          tc_commit(&sh.drain);
          mbar_wait(&sh.drain, 0, &never);
        }
      }
      __syncwarp();
    }
  } else {
    regs_inc<kSoftmaxRegs>();
    // -------------------------------------------------------------- softmax of tile x
    const int x = warp >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + 128 * x;
    const uint32_t o_addr = tmem + lane_off + 256 + 128 * x;
    const bool live = x == 0 || has_b;
    const int h = head_of(x);
    const int n = sh.n_tile[x];
    const int qrow = tile_of(x) * 128 + r;
    const float sl2 = p.scale_log2;
    // Blocks run in ascending order and end at most at t, so only the last can be the diagonal.
    const bool last_is_diag = n > 0 && sh.diag_tile[x];
    float m = -INFINITY, l = 0.f;
    bool ok = live;
    for (int i = 0; i < n && ok; ++i) {
      if (!mbar_wait_warp(&sh.s_full[x], i & 1, abort)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + 32 * c, *reinterpret_cast<float(*)[32]>(&sv[32 * c]));
      tmem_wait_ld();
      const bool diag = last_is_diag && i == n - 1;
      if (diag) {  // key j of the diagonal block is visible to row r iff j <= r
#pragma unroll
        for (int c = 0; c < 128; ++c) sv[c] = c <= r ? sv[c] : -INFINITY;
      }
      // Row max over the 128 columns: eight running maxima, two columns folded in per step.
      float mx[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mx[c] = sv[c];
#pragma unroll
      for (int c = 8; c < 120; c += 16)
#pragma unroll
        for (int j = 0; j < 8; ++j) mx[j] = fmax3(mx[j], sv[c + j], sv[c + 8 + j]);
#pragma unroll
      for (int j = 0; j < 8; ++j) mx[j] = fmaxf(mx[j], sv[120 + j]);
      const float bmax = fmaxf(fmax3(mx[0], mx[1], mx[2]), fmax3(fmax3(mx[3], mx[4], mx[5]), mx[6], mx[7])) * sl2;
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
      const float neg = (m == -INFINITY) ? 0.f : -m;
      // The diagonal block's masked entries are -inf: the MUFU returns exactly 0 for them.
      l += diag ? softmax_row<0>(sv, sl2, neg, s_addr) : softmax_row<kEmu>(sv, sl2, neg, s_addr);
      // O_X holds blocks < i and no P.V runs until p_full: rescale it for the moved max.
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
    }
    if (live) {
      // Epilogue: O / l -> bf16 -> swizzled tile (in this tile's Q buffer) -> TMA store; LSE.
      if (ok && n > 0 && !mbar_wait_warp(&sh.o_done[x], (n - 1) & 1, abort)) ok = false;
      tc_fence_after();
      const bool none = !(ok && n > 0) || m == -INFINITY;
      const float inv = none ? 0.f : 1.f / l;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float o[32];
        if (ok && n > 0) {
          tmem_ld32(o_addr + 32 * c, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint4 v4 = make_uint4(pack_bf16(o[8 * e] * inv, o[8 * e + 1] * inv),
                                      pack_bf16(o[8 * e + 2] * inv, o[8 * e + 3] * inv),
                                      pack_bf16(o[8 * e + 4] * inv, o[8 * e + 5] * inv),
                                      pack_bf16(o[8 * e + 6] * inv, o[8 * e + 7] * inv));
          *reinterpret_cast<uint4 *>(sh.q[x] + sw128_offset(r, 32 * c + 8 * e)) = v4;
        }
      }
      if (p.lse && qrow < p.L) p.lse[((int64_t)b * p.L + qrow) * p.H + h] = none ? -INFINITY : m * kLn2 + logf(l);
      fence_proxy_async();
      named_sync(1 + x, 128);
      if (r == 0 && !*abort) {
        tma_store_4d(&tm_o, sh.q[x], 0, h, tile_of(x) * 128, b);
        tma_store_4d(&tm_o, sh.q[x] + kHalf, 64, h, tile_of(x) * 128, b);
        bulk_commit();
        bulk_wait0();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && sh.abort) atomicExch(&g_device_error, 1);
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

namespace {

// cuTensorMapEncodeTiled, resolved through the runtime so the library loads without libcuda.
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(ptr);
  }();
  return fn;
}

}  // namespace

// [B, rows, heads, d] bf16 with element strides -> 4-D map (d, head, row, batch), box 64 x 1 x box_rows x 1.
bool encode_4d(CUtensorMap *map, const void *base, int64_t d, int64_t heads, int64_t rows, int64_t batch,
               int64_t sh, int64_t sl, int64_t sb, int box_rows) {
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)heads, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)(sh * 2), (cuuint64_t)(sl * 2), (cuuint64_t)(sb * 2)};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  // A size-1 dimension may carry any stride; keep it a valid multiple of 16 bytes.
  if (heads == 1) strides[0] = 16;
  if (batch == 1) strides[2] = strides[1] * (cuuint64_t)rows;
  const EncodeTiledFn encode = encode_fn();
  if (!encode) return false;
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

template <int kEmu>
void launch_variant(dim3 grid, size_t smem, cudaStream_t s, const CUtensorMap &tq, const CUtensorMap &tk,
                    const CUtensorMap &tv, const CUtensorMap &to, const ExactParams &p, int tiles, int kv_count) {
  cudaFuncSetAttribute(exact_tc_kernel<kEmu>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  exact_tc_kernel<kEmu><<<grid, kThreads, smem, s>>>(tq, tk, tv, to, p, tiles, kv_count);
}

}  // namespace

size_t exact_tc_smem() { return sizeof(Smem) + 1024; }

int launch_exact_tc(const ExactParams &p, int B, int L, int Hkv, int tiles, int heads, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  if ((p.ref_indices ? p.nb : p.route.nb) > kMaxBlocks) return FPX_ERR_UNSUPPORTED;
  CUtensorMap tq, tk, tv, to;
  if (!encode_4d(&tq, p.q, kHeadDim, p.H, L, B, p.q_sh, p.q_sl, p.q_sb) ||
      !encode_4d(&tk, p.k, kHeadDim, Hkv, L, B, p.k_sh, p.k_sl, p.k_sb) ||
      !encode_4d(&tv, p.v, kHeadDim, Hkv, L, B, p.v_sh, p.v_sl, p.v_sb) ||
      !encode_4d(&to, p.out, kHeadDim, p.H, L, B, p.o_sh, p.o_sl, p.o_sb))
    return FPX_ERR_INVALID;
  const int kv_count = heads / p.group;
  const dim3 grid(exact_units(tiles, kv_count, p.group), 1, B);
  const size_t smem = exact_tc_smem();
  switch (get_option(kOptExpEmulation)) {
    case 0: launch_variant<0>(grid, smem, s, tq, tk, tv, to, p, tiles, kv_count); break;
    case 3: launch_variant<3>(grid, smem, s, tq, tk, tv, to, p, tiles, kv_count); break;
    default: launch_variant<2>(grid, smem, s, tq, tk, tv, to, p, tiles, kv_count); break;
  }
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

int *device_error_word() {
  static std::mutex mu;
  static int *cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void *ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_device_error) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int *>(ptr);
  }
  return cache[dev];
}

}  // namespace fpx

extern "C" int fpx_device_error(int *code, int reset) {
  if (!code) return FPX_ERR_INVALID;
  if (cudaMemcpyFromSymbol(code, fpx::g_device_error, sizeof(int)) != cudaSuccess) return FPX_ERR_CUDA;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(fpx::g_device_error, &zero, sizeof(int)) != cudaSuccess) return FPX_ERR_CUDA;
  }
  return FPX_OK;
}
