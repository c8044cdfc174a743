// Exact block-sparse causal attention on the 5th-generation tensor core (tcgen05 + TMEM + TMA).
//
// Reference semantics: upstream/flashprefill_native_forward.py:215-354 (_flash_forward) —
// for query tile t (128 rows) of head h, attend over the tile's selected 128-key blocks in
// ascending order with an online softmax in exp2 units, causal mask on the diagonal block,
// P rounded to bf16 before P.V, bf16 output and natural-log LSE.
//
// One CTA per (batch, head, query tile), 192 threads in three roles:
//   warp 0      TMA producer: Q once, then K and V of each selected block into a 2-stage ring;
//   warp 1      MMA issuer (one elected lane): S = Q K^T into a double-buffered TMEM S, then
//               O += P V into TMEM O once the softmax has published P;
//   warps 2..5  softmax (thread = query row = TMEM lane): read S from TMEM, mask, online
//               softmax, rescale O in TMEM when the row max grows, write P (bf16) into a
//               swizzled shared tile, and finally normalise O and store it with TMA.
// TMEM: columns [0,128) S0, [128,256) S1, [256,384) O (fp32, 128 lanes). Every mbarrier wait
// is bounded; a wait that gives up flags the CTA, the roles drain and exit, and the host sees
// FPX_ERR_TIMEOUT through fpx_device_error().
#include <cuda.h>

#include <algorithm>

#include "attn.cuh"
#include "tc.cuh"

namespace fpx {

__device__ int g_device_error;  // 0 = ok; 1 = a bounded wait in a tcgen05 kernel gave up

namespace {

using namespace tc;

constexpr int kStages = 2;
constexpr int kThreads = 192;
constexpr uint32_t kHalf = 128 * 128;  // 128 rows x 64 bf16 (one SW128 half tile)
constexpr uint32_t kTile = 2 * kHalf;  // 128 x 128 bf16
constexpr uint32_t kIdescQK = idesc_bf16(128, 128, false);
constexpr uint32_t kIdescPV = idesc_bf16(128, 128, true);

struct alignas(1024) Smem {
  uint8_t q[kTile];
  uint8_t k[kStages][kTile];
  uint8_t v[kStages][kTile];
  uint8_t p[kTile];
  uint64_t q_full, k_full[kStages], v_full[kStages], kv_empty[kStages];
  uint64_t s_full[2], s_empty[2], p_full, o_done, drain;
  uint32_t tmem_base;
  int abort;
};

// K-major SW128 operand (Q, K, P) at K offset 16*kk: halves of 64 columns sit kHalf apart,
// 16 columns = 32 bytes inside a half.
FPX_INLINE uint64_t desc_kmajor(const uint8_t *tile, int kk) {
  const uint32_t a = smem_u32(tile) + (kk >> 2) * kHalf + (kk & 3) * 32;
  return smem_desc_sw128(a, 16, 1024);
}
// MN-major SW128 V operand at key offset 16*kk: 16 keys = 16 rows of 128 bytes.
FPX_INLINE uint64_t desc_v(const uint8_t *tile, int kk) {
  return smem_desc_sw128(smem_u32(tile) + kk * 2048, kHalf, 1024);
}

// Byte offset of (row, col) inside a 128 x 128 bf16 SW128 K-major tile.
FPX_INLINE uint32_t sw128_offset(int row, int col) {
  const int half = col >> 6, chunk = (col & 63) >> 3;
  return half * kHalf + row * 128 + ((chunk ^ (row & 7)) << 4) + ((col & 7) << 1);
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    exact_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                    ExactParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem &sh = *reinterpret_cast<Smem *>(smem_raw + pad);
  volatile int *abort = &sh.abort;

  const int t = p.tile_begin + (gridDim.x - 1 - blockIdx.x);
  const int h = p.head_begin + blockIdx.y;
  const int b = blockIdx.z;
  const int kvh = h / p.group;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rrow = p.route.row(b, h, t, p.H);
  // Once any CTA has given up on a wait, the rest skip their work (the launch is failed).
  const int count = *reinterpret_cast<volatile int *>(&g_device_error) ? 0 : p.route.counts[rrow];
  const int32_t *list = p.route.lists + rrow * p.route.nb;

  if (threadIdx.x == 0) {
    mbar_init(&sh.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.k_full[s], 1);
      mbar_init(&sh.v_full[s], 1);
      mbar_init(&sh.kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh.s_full[s], 1);
      mbar_init(&sh.s_empty[s], 128);
    }
    mbar_init(&sh.p_full, 128);
    mbar_init(&sh.o_done, 1);
    mbar_init(&sh.drain, 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    int issued[kStages] = {0, 0};
    if (count > 0) {
      if (lane == 0) {
        mbar_expect_tx(&sh.q_full, kTile);
        tma_load_4d(sh.q, &tm_q, &sh.q_full, 0, h, t * 128, b);
        tma_load_4d(sh.q + kHalf, &tm_q, &sh.q_full, 64, h, t * 128, b);
      }
      for (int j = 0; j < count; ++j) {
        const int s = j % kStages, n = j / kStages;
        if (n > 0 && !mbar_wait_warp(&sh.kv_empty[s], (n - 1) & 1, abort)) break;
        const int blk = list[j];
        if (lane == 0) {
          mbar_expect_tx(&sh.k_full[s], kTile);
          tma_load_4d(sh.k[s], &tm_k, &sh.k_full[s], 0, kvh, blk * 128, b);
          tma_load_4d(sh.k[s] + kHalf, &tm_k, &sh.k_full[s], 64, kvh, blk * 128, b);
          mbar_expect_tx(&sh.v_full[s], kTile);
          tma_load_4d(sh.v[s], &tm_v, &sh.v_full[s], 0, kvh, blk * 128, b);
          tma_load_4d(sh.v[s] + kHalf, &tm_v, &sh.v_full[s], 64, kvh, blk * 128, b);
        }
        issued[s] = n + 1;
      }
      __syncwarp();
      if (*abort) {  // drain copies still in flight before the CTA's shared memory goes away
        int never = 0;
        mbar_wait(&sh.q_full, 0, &never);
        for (int s = 0; s < kStages; ++s)
          if (issued[s] > 0) {
            mbar_wait(&sh.k_full[s], (issued[s] - 1) & 1, &never);
            mbar_wait(&sh.v_full[s], (issued[s] - 1) & 1, &never);
          }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (count > 0 && mbar_wait_warp(&sh.q_full, 0, abort)) {
      auto issue_pv = [&](int i) -> bool {
        const int s = i % kStages;
        if (!mbar_wait_warp(&sh.p_full, i & 1, abort)) return false;
        if (!mbar_wait_warp(&sh.v_full[s], (i / kStages) & 1, abort)) return false;
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss(tmem + 256, desc_kmajor(sh.p, kk), desc_v(sh.v[s], kk), kIdescPV, (i > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sh.kv_empty[s]);
          tc_commit(&sh.o_done);
        }
        __syncwarp();
        return true;
      };
      bool ok = true;
      for (int j = 0; j < count && ok; ++j) {
        const int s = j % kStages, sb = j & 1;
        if (!mbar_wait_warp(&sh.k_full[s], (j / kStages) & 1, abort)) break;
        if (j >= 2 && !mbar_wait_warp(&sh.s_empty[sb], ((j >> 1) - 1) & 1, abort)) break;
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ss(tmem + sb * 128, desc_kmajor(sh.q, kk), desc_kmajor(sh.k[s], kk), kIdescQK, kk > 0 ? 1u : 0u);
          tc_commit(&sh.s_full[sb]);
        }
        __syncwarp();
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok && !*abort) issue_pv(count - 1);
      if (*abort) {  // let every MMA this thread issued finish before TMEM is released
        int never = 0;
        if (lane == 0) tc_commit(&sh.drain);
        __syncwarp();
        mbar_wait(&sh.drain, 0, &never);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax warpgroup
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row in the tile == TMEM lane
    const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
    const int qrow = t * 128 + r;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < count && ok; ++j) {
      const int sb = j & 1;
      if (!mbar_wait_warp(&sh.s_full[sb], (j >> 1) & 1, abort)) { ok = false; break; }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(lane_addr + sb * 128 + 32 * c, *reinterpret_cast<float(*)[32]>(&s[32 * c]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&sh.s_empty[sb]);
      const int blk = list[j];
      const int kmax = (blk == t) ? (r) : 127;  // diagonal block: key j <= row
      float mx = m;
#pragma unroll
      for (int i = 0; i < 128; ++i) {
        const float x = (i <= kmax) ? s[i] * p.scale_log2 : -INFINITY;
        s[i] = x;
        mx = fmaxf(mx, x);
      }
      float rs = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float a = (mx == -INFINITY) ? 0.f : exp2f(s[2 * i] - mx);
        const float c = (mx == -INFINITY) ? 0.f : exp2f(s[2 * i + 1] - mx);
        rs += a + c;
        pk[i] = pack_bf16(a, c);
      }
      const float corr = (m == -INFINITY) ? (mx == -INFINITY ? 1.f : 0.f) : exp2f(m - mx);
      if (j > 0) {
        if (!mbar_wait_warp(&sh.o_done, (j - 1) & 1, abort)) { ok = false; break; }
        if (__any_sync(0xffffffffu, corr != 1.f)) {  // tcgen05.ld/st are warp-collective
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32(lane_addr + 256 + 32 * c, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tmem_st32(lane_addr + 256 + 32 * c, o);
          }
          tmem_wait_st();
        }
      }
      l = l * corr + rs;
      m = mx;
      // P row -> swizzled K-major tile (16-byte chunks).
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 v4 = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        *reinterpret_cast<uint4 *>(sh.p + sw128_offset(r, 8 * c)) = v4;
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(&sh.p_full);
    }
    // Epilogue: O / l -> bf16 -> swizzled tile (in the Q buffer) -> TMA store; LSE.
    if (ok && count > 0) {
      if (!mbar_wait_warp(&sh.o_done, (count - 1) & 1, abort)) ok = false;
    }
    tc_fence_after();
    const bool none = !(ok && count > 0) || m == -INFINITY;
    const float inv = none ? 0.f : 1.f / l;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float o[32];
      if (ok && count > 0) {
        tmem_ld32(lane_addr + 256 + 32 * c, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 v4 = make_uint4(pack_bf16(o[8 * i] * inv, o[8 * i + 1] * inv), pack_bf16(o[8 * i + 2] * inv, o[8 * i + 3] * inv),
                              pack_bf16(o[8 * i + 4] * inv, o[8 * i + 5] * inv), pack_bf16(o[8 * i + 6] * inv, o[8 * i + 7] * inv));
        *reinterpret_cast<uint4 *>(sh.q + sw128_offset(r, 32 * c + 8 * i)) = v4;
      }
    }
    if (p.lse && qrow < p.L) p.lse[((int64_t)b * p.L + qrow) * p.H + h] = none ? -INFINITY : m * kLn2 + logf(l);
    fence_proxy_async();
    named_sync(1, 128);
    if (threadIdx.x == 64 && !*abort) {
      tma_store_4d(&tm_o, sh.q, 0, h, t * 128, b);
      tma_store_4d(&tm_o, sh.q + kHalf, 64, h, t * 128, b);
      bulk_commit();
      bulk_wait0();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && sh.abort) atomicExch(&g_device_error, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================================
// Two query tiles per CTA: heads hA = kv*G + 2*pair and hB = hA + 1 of one KV group, same
// query tile t, so every K/V block loaded serves both. 320 threads:
//   warps 0..3  softmax of tile A      warps 4..7  softmax of tile B
//   warp 8      TMA producer           warp 9      MMA issuer
// The producer streams the union of the two heads' block lists; the MMA warp issues tile X's
// QK / PV only for blocks in X's own list. TMEM columns: S_A [0,128), S_B [128,256),
// O_A [256,384), O_B [384,512); P_X (bf16, two per column) overwrites the first 64 columns of
// S_X after the softmax has read S_X, and feeds P.V straight from TMEM. With both tiles in
// flight the tensor core works on one tile while the other's softmax runs.
//
// Ordering facts the protocol relies on: the MMAs of one issuing thread complete in issue
// order, and a commit tracks every earlier MMA of that thread. So when s_full[X] fires for
// block i, PV_X(i-1) has finished: O_X is stable and P_X's columns are free.
// The softmax keeps a running row max m and only moves it (rescaling O and l) when the block
// max exceeds it by more than 8 (log2 units), so P stays below 2^8 and O is rarely touched;
// O / l at the end is exact either way.
namespace v2 {

constexpr int kStages = 2;
constexpr int kThreads = 320;
constexpr int kMaxBlocks = 2048;  // union list capacity: L <= 262144
constexpr float kRescaleThreshold = 8.f;

struct alignas(1024) Smem {
  uint8_t q[2][kTile];  // Q of tiles A and B; reused to stage each tile's output
  uint8_t k[kStages][kTile];
  uint8_t v[kStages][kTile];
  uint64_t q_full, k_full[kStages], v_full[kStages], kv_empty[kStages];
  uint64_t s_full[2], p_full[2], o_done[2], drain;
  uint32_t tmem_base;
  int abort, n_union;
  uint32_t bits[2][kMaxBlocks / 32];
  uint16_t u_blk[kMaxBlocks];
  uint8_t u_flags[kMaxBlocks];
};

}  // namespace v2

__global__ void __launch_bounds__(v2::kThreads, 1)
    exact_tc2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                     ExactParams p, int pairs) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  v2::Smem &sh = *reinterpret_cast<v2::Smem *>(smem_raw + pad);
  volatile int *abort = &sh.abort;

  const int t = p.tile_begin + (gridDim.x - 1 - blockIdx.x);
  const int pair = blockIdx.y % pairs;
  const int kvh = p.head_begin / p.group + blockIdx.y / pairs;
  const int b = blockIdx.z;
  const int hA = kvh * p.group + 2 * pair;
  const bool has_b = 2 * pair + 1 < p.group;
  const int heads[2] = {hA, hA + 1};
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool failed = *reinterpret_cast<volatile int *>(&g_device_error) != 0;
  int cnt[2];
  const int32_t *lists[2];
  for (int x = 0; x < 2; ++x) {
    const bool live = x == 0 || has_b;
    const int64_t rr = p.route.row(b, live ? heads[x] : hA, t, p.H);
    cnt[x] = (live && !failed) ? p.route.counts[rr] : 0;
    lists[x] = p.route.lists + rr * p.route.nb;
  }
  const int words = (p.route.nb + 31) / 32;

  if (threadIdx.x == 0) {
    mbar_init(&sh.q_full, 1);
    for (int s = 0; s < v2::kStages; ++s) {
      mbar_init(&sh.k_full[s], 1);
      mbar_init(&sh.v_full[s], 1);
      mbar_init(&sh.kv_empty[s], 1);
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
  for (int w = threadIdx.x; w < 2 * (v2::kMaxBlocks / 32); w += v2::kThreads) (&sh.bits[0][0])[w] = 0u;
  if (warp == 9) {
    tmem_alloc(&sh.tmem_base, 512);
    tmem_relinquish();
  }
  __syncthreads();
  for (int x = 0; x < 2; ++x)
    for (int i = threadIdx.x; i < cnt[x]; i += v2::kThreads) {
      const int blk = lists[x][i];
      atomicOr(&sh.bits[x][blk >> 5], 1u << (blk & 31));
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
      for (uint32_t x = u; x; x &= x - 1) {
        const int bit = __ffs(x) - 1;
        sh.u_blk[pos] = (uint16_t)(32 * w + bit);
        sh.u_flags[pos] = (uint8_t)(((a >> bit) & 1u) | (((c >> bit) & 1u) << 1));
        ++pos;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) sh.n_union = base;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const int n_union = sh.n_union;
  const int n_tiles = has_b ? 2 : 1;

  if (warp == 8) {
    // ---------------------------------------------------------------- TMA producer
    int issued[v2::kStages] = {0, 0};
    if (n_union > 0) {
      if (lane == 0) {
        mbar_expect_tx(&sh.q_full, kTile * n_tiles);
        for (int x = 0; x < n_tiles; ++x) {
          tma_load_4d(sh.q[x], &tm_q, &sh.q_full, 0, heads[x], t * 128, b);
          tma_load_4d(sh.q[x] + kHalf, &tm_q, &sh.q_full, 64, heads[x], t * 128, b);
        }
      }
      for (int u = 0; u < n_union; ++u) {
        const int s = u % v2::kStages, n = u / v2::kStages;
        if (n > 0 && !mbar_wait_warp(&sh.kv_empty[s], (n - 1) & 1, abort)) break;
        const int blk = sh.u_blk[u];
        if (lane == 0) {
          mbar_expect_tx(&sh.k_full[s], kTile);
          tma_load_4d(sh.k[s], &tm_k, &sh.k_full[s], 0, kvh, blk * 128, b);
          tma_load_4d(sh.k[s] + kHalf, &tm_k, &sh.k_full[s], 64, kvh, blk * 128, b);
          mbar_expect_tx(&sh.v_full[s], kTile);
          tma_load_4d(sh.v[s], &tm_v, &sh.v_full[s], 0, kvh, blk * 128, b);
          tma_load_4d(sh.v[s] + kHalf, &tm_v, &sh.v_full[s], 64, kvh, blk * 128, b);
        }
        issued[s] = n + 1;
      }
      __syncwarp();
      if (*abort) {
        int never = 0;
        mbar_wait(&sh.q_full, 0, &never);
        for (int s = 0; s < v2::kStages; ++s)
          if (issued[s] > 0) {
            mbar_wait(&sh.k_full[s], (issued[s] - 1) & 1, &never);
            mbar_wait(&sh.v_full[s], (issued[s] - 1) & 1, &never);
          }
      }
    }
  } else if (warp == 9) {
    // ---------------------------------------------------------------- MMA issuer
    if (n_union > 0 && mbar_wait_warp(&sh.q_full, 0, abort)) {
      int pend[2] = {-1, -1}, n_pv[2] = {0, 0};
      // P.V of tile x for its pending block; releases the K/V stage once no tile needs it.
      auto flush = [&](int x) -> bool {
        const int u = pend[x], s = u % v2::kStages;
        if (!mbar_wait_warp(&sh.p_full[x], n_pv[x] & 1, abort)) return false;
        if (!mbar_wait_warp(&sh.v_full[s], (u / v2::kStages) & 1, abort)) return false;
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_ts(tmem + 256 + 128 * x, tmem + 128 * x + 8 * kk, desc_v(sh.v[s], kk), kIdescPV,
                   (n_pv[x] > 0 || kk > 0) ? 1u : 0u);
          tc_commit(&sh.o_done[x]);
          if (pend[x ^ 1] != u) tc_commit(&sh.kv_empty[s]);
        }
        __syncwarp();
        ++n_pv[x];
        pend[x] = -1;
        return true;
      };
      bool ok = true;
      for (int u = 0; u < n_union && ok; ++u) {
        const int s = u % v2::kStages;
        for (int x = 0; x < 2 && ok; ++x)
          if (u >= v2::kStages && pend[x] == u - v2::kStages) ok = flush(x);
        if (!ok || !mbar_wait_warp(&sh.k_full[s], (u / v2::kStages) & 1, abort)) break;
        const int flags = sh.u_flags[u];
        for (int x = 0; x < 2 && ok; ++x) {
          if (!(flags & (1 << x))) continue;
          if (pend[x] >= 0 && !(ok = flush(x))) break;
          tc_fence_after();
          if (lane == 0) {
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_ss(tmem + 128 * x, desc_kmajor(sh.q[x], kk), desc_kmajor(sh.k[s], kk), kIdescQK,
                     kk > 0 ? 1u : 0u);
            tc_commit(&sh.s_full[x]);
          }
          __syncwarp();
          pend[x] = u;
        }
      }
      for (int x = 0; x < 2 && ok && !*abort; ++x)
        if (pend[x] >= 0) ok = flush(x);
      if (*abort) {
        int never = 0;
        if (lane == 0) tc_commit(&sh.drain);
        __syncwarp();
        mbar_wait(&sh.drain, 0, &never);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax, tile x
    const int x = warp >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_off + 128 * x;
    const uint32_t o_addr = tmem + lane_off + 256 + 128 * x;
    const bool live = x == 0 || has_b;
    const int h = heads[x];
    const int n = cnt[x];
    const int32_t *list = lists[x];
    const int qrow = t * 128 + r;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = live;
    for (int i = 0; i < n && ok; ++i) {
      if (!mbar_wait_warp(&sh.s_full[x], i & 1, abort)) { ok = false; break; }
      tc_fence_after();
      float sv[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + 32 * c, *reinterpret_cast<float(*)[32]>(&sv[32 * c]));
      tmem_wait_ld();
      if (list[i] == t) {  // diagonal block: key j visible to row r iff j <= r
#pragma unroll
        for (int c = 0; c < 128; ++c) sv[c] = c <= r ? sv[c] : -INFINITY;
      }
      float mx[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mx[c] = sv[c];
#pragma unroll
      for (int c = 8; c < 128; ++c) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
      const float bmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * sl2;
      const float mn = fmaxf(m, bmax);
      float corr = 1.f;
      const bool move = __any_sync(0xffffffffu, mn > m + v2::kRescaleThreshold || m == -INFINITY);
      if (move) {
        corr = (m == -INFINITY) ? 0.f : ex2(m - mn);
        l *= corr;
        m = mn;
      }
      const float neg = (m == -INFINITY) ? 0.f : -m;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {  // 32 scores -> 16 packed columns of P at a time
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float a = ex2(fmaf(sv[32 * q4 + 2 * c], sl2, neg));
          const float e = ex2(fmaf(sv[32 * q4 + 2 * c + 1], sl2, neg));
          acc[c & 3] += a + e;
          pk[c] = pack_bf16(a, e);
        }
        tmem_st16u(s_addr + 16 * q4, pk);
      }
      l += (acc[0] + acc[1]) + (acc[2] + acc[3]);
      // O_X holds blocks < i and no P.V runs until p_full: rescale it for the moved max.
      if (move && i > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
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
          uint4 v4 = make_uint4(pack_bf16(o[8 * e] * inv, o[8 * e + 1] * inv),
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
        tma_store_4d(&tm_o, sh.q[x], 0, h, t * 128, b);
        tma_store_4d(&tm_o, sh.q[x] + kHalf, 64, h, t * 128, b);
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

bool encode_4d(CUtensorMap *map, const void *base, int64_t d, int64_t heads, int64_t rows, int64_t batch, int64_t sh,
               int64_t sl, int64_t sb) {
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)heads, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)(sh * 2), (cuuint64_t)(sl * 2), (cuuint64_t)(sb * 2)};
  cuuint32_t box[4] = {64, 1, 128, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  // A size-1 dimension may carry any stride; keep it a valid multiple of 16 bytes.
  if (heads == 1) strides[0] = 16;
  if (batch == 1) strides[2] = strides[1] * (cuuint64_t)rows;
  const EncodeTiledFn encode = encode_fn();
  if (!encode) return false;
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void *>(base), dims, strides,
                                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t exact_tc_smem() { return sizeof(Smem) + 1024; }
size_t exact_tc2_smem() { return sizeof(v2::Smem) + 1024; }

int launch_exact_tc(const ExactParams &p, int B, int L, int Hkv, int tiles, int heads, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  CUtensorMap tq, tk, tv, to;
  if (!encode_4d(&tq, p.q, kHeadDim, p.H, L, B, p.q_sh, p.q_sl, p.q_sb) ||
      !encode_4d(&tk, p.k, kHeadDim, Hkv, L, B, p.k_sh, p.k_sl, p.k_sb) ||
      !encode_4d(&tv, p.v, kHeadDim, Hkv, L, B, p.v_sh, p.v_sl, p.v_sb) ||
      !encode_4d(&to, p.out, kHeadDim, p.H, L, B, p.o_sh, p.o_sl, p.o_sb))
    return FPX_ERR_INVALID;
  if (get_option(kOptExactKernel) == kExactKernelTcgen05Single) {
    const size_t smem = exact_tc_smem();
    cudaFuncSetAttribute(exact_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    exact_tc_kernel<<<dim3(tiles, heads, B), kThreads, smem, s>>>(tq, tk, tv, to, p);
  } else {
    if (p.route.nb > v2::kMaxBlocks) return FPX_ERR_UNSUPPORTED;
    const int pairs = (p.group + 1) / 2;
    const size_t smem = exact_tc2_smem();
    cudaFuncSetAttribute(exact_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    exact_tc2_kernel<<<dim3(tiles, (heads / p.group) * pairs, B), v2::kThreads, smem, s>>>(tq, tk, tv, to, p,
                                                                                            pairs);
  }
  FPX_CHECK_LAUNCH();
  return FPX_OK;
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
