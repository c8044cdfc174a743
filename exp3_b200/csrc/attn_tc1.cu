// Exact block-sparse causal attention, one query tile per CTA, on the tcgen05 tensor core, for
// head dim D = 128 and D = 256 (the Qwen3.5 shape: 16 query heads over 4 KV heads,
// check_qwen35_math.py:93-185).
//
// Reference semantics are those of upstream/flashprefill_native_forward.py:215-354 (and of the
// two-tile kernel in attn_tc.cu): for query tile t of head h, an online softmax in exp2 units
// over the tile's selected 128-key blocks in ascending order, causal mask on the diagonal
// block, P rounded to bf16 before P.V, bf16 output, natural LSE.
//
// One CTA runs ONE query tile (the G heads of a KV group run as neighbouring CTAs, which read
// the same K/V blocks from L2) and double-buffers S, so the softmax never waits for the tensor
// core to turn P(i) into S(i + 1):
//   TMEM: S0 [0,128), S1 [128,256), O [256,256+D) fp32 columns x 128 lanes;
//   P of block i (bf16, two per column) overwrites the first 64 columns of S(i & 1).
// The tensor core computes QK^T of block i + 1 while the softmax works on block i:
//   issue order  QK0, QK1, PV0, QK2, PV1, ..., QK(n-1), PV(n-2), PV(n-1).
// Shared memory: Q (128 x D bf16, D/64 128-byte-swizzled 64-column atoms) and a ring of
// stages, each holding 64 keys x D of K or of V, loaded in the order the tensor core consumes
// them (K halves of block i + 1, then V halves of block i): twelve 16 KB stages at D = 128,
// five 32 KB stages at D = 256 (Q + ring = 224 KB either way). 192 threads:
//   warps 0..3  softmax (thread = query row = TMEM lane)
//   warp 4      TMA producer (Q, then the K / V ring)       warp 5  MMA issuer, TMEM owner
//
// Ordering facts the protocol relies on: MMAs of one thread complete in issue order and a commit
// tracks all earlier MMAs of the thread. So when s_full fires for block i, P(i-2).V has finished
// (it was issued before QK(i)); the softmax only touches O when a row's max moves, and then
// first waits for P(i-1).V on o_done[(i-1) & 1]. Two o_done barriers (one per parity of the
// block) keep every wait within one phase of its barrier.
//
// Every wait is bounded (about 1 s); a wait that gives up flags the CTA and the device error
// word, the roles drain their copies and MMAs in flight, and the CTA exits.
#include <cuda.h>

#include "attn.cuh"
#include "softmax_tc.cuh"
#include "tc.cuh"

namespace fpx {
namespace {

using namespace tc;

constexpr uint32_t kQAtom = 128 * 128;  // 128 rows x 64 bf16: one 128-byte-swizzled atom column
constexpr uint32_t kKvAtom = 64 * 128;  // 64 rows x 64 bf16
constexpr int kThreads1 = 192;
constexpr uint32_t kIdescQK = idesc_bf16(128, 64, false);
constexpr float kRescaleThreshold1 = 8.f;

template <int D>
struct Geometry {
  static constexpr int kAtoms = D / 64;
  static constexpr uint32_t kQBytes = kAtoms * kQAtom;       // 128 x D bf16
  static constexpr uint32_t kStageBytes = kAtoms * kKvAtom;  // 64 keys x D bf16
  static constexpr int kStages = D == 128 ? 12 : 5;
  static constexpr uint32_t kIdescPV = idesc_bf16(128, D, true);
};

template <int D>
struct alignas(1024) Smem1 {
  uint8_t q[Geometry<D>::kQBytes];  // Q; reused to stage the output tile
  uint8_t ring[Geometry<D>::kStages][Geometry<D>::kStageBytes];
  uint64_t q_full, full[Geometry<D>::kStages], empty[Geometry<D>::kStages], s_full[2], p_full[2], o_done[2], drain;
  uint32_t tmem_base;
  int abort, n, diag;
};

// K-major operands at K offset 16 * kk: 64-column atoms `atom` bytes apart, 32 B per K step
// inside an atom, 8-row groups 1024 B apart.
FPX_INLINE uint64_t desc_q1(const uint8_t *q, int kk) {
  return smem_desc_sw128(smem_u32(q) + (kk >> 2) * kQAtom + (kk & 3) * 32, 16, 1024);
}
FPX_INLINE uint64_t desc_k1(const uint8_t *stage, int kk) {
  return smem_desc_sw128(smem_u32(stage) + (kk >> 2) * kKvAtom + (kk & 3) * 32, 16, 1024);
}
// MN-major V (N = D) at key offset 16 * kk: 16 keys = 2048 B; the 64-column MN atoms kKvAtom
// apart; 8-key groups 1024 B apart.
FPX_INLINE uint64_t desc_v1(const uint8_t *stage, int kk) {
  return smem_desc_sw128(smem_u32(stage) + kk * 2048, kKvAtom, 1024);
}
// Descriptor low-word steps (desc_join in tc.cuh) of K-step kk, as desc_q1 / desc_k1 / desc_v1
// place them.
constexpr uint32_t q1_step(int kk) { return (uint32_t)(((kk >> 2) * kQAtom + (kk & 3) * 32) >> 4); }
constexpr uint32_t k1_step(int kk) { return (uint32_t)(((kk >> 2) * kKvAtom + (kk & 3) * 32) >> 4); }
constexpr uint32_t v1_step(int kk) { return (uint32_t)(kk * 2048 >> 4); }
// Byte offset of (row, col) in the 128 x D output tile (swizzled 64-column atoms).
FPX_INLINE uint32_t out_offset(int row, int col) {
  const int atom = col >> 6, chunk = (col & 63) >> 3;
  return atom * kQAtom + row * 128 + ((chunk ^ (row & 7)) << 4) + ((col & 7) << 1);
}

// Walks the valid entries of one tile's block list, 32 entries per step across the warp.
// A trusted list (the fused path's own) takes every entry below its count; a reference-layout
// list keeps entries with 0 <= blk <= t that are above the entry before them (the reference's
// lists are ascending, so this drops the sentinel and anything past the tile).
struct ListCursor {
  const int32_t *lst;
  const int64_t *ref;
  int64_t ref_stride;
  int cnt, t;
  bool trusted;
  int base, val, prev_last;
  uint32_t mask;

  FPX_INLINE void load(int lane) {
    const int i = base + lane;
    int v = -1;
    if (i < cnt) v = ref ? (int)ref[(int64_t)i * ref_stride] : lst[i];
    int prev = __shfl_up_sync(0xffffffffu, v, 1);
    if (lane == 0) prev = prev_last;
    const bool ok = i < cnt && (trusted || (v >= 0 && v <= t && v > prev));
    val = v;
    mask = __ballot_sync(0xffffffffu, ok);
    prev_last = __shfl_sync(0xffffffffu, v, 31);
  }
  FPX_INLINE void start(int lane) {
    base = 0;
    prev_last = -1;
    load(lane);
  }
  // Next valid block (warp-uniform), or -1 past the end.
  FPX_INLINE int next(int lane) {
    while (mask == 0u) {
      base += 32;
      if (base >= cnt) return -1;
      load(lane);
    }
    const int bit = __ffs(mask) - 1;
    mask &= mask - 1u;
    return __shfl_sync(0xffffffffu, val, bit);
  }
};

}  // namespace

template <int D, int kEmu>
__global__ void __launch_bounds__(kThreads1, 1)
    exact_tc1_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                     ExactParams p, int *err) {
  using Geo = Geometry<D>;
  constexpr int kStages = Geo::kStages;
  constexpr int kAtoms = Geo::kAtoms;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem1<D> &sh = *reinterpret_cast<Smem1<D> *>(smem_raw + pad);
  volatile int *abort = &sh.abort;

  // x: (KV group, head), fastest, so a group's heads are adjacent and read the same K/V blocks
  // at about the same time; y: tile, longest first over the whole grid; z: batch.
  const int G = p.group;
  const int kv_local = blockIdx.x / G;
  const int b = blockIdx.z;
  const int kvh = p.head_begin / G + kv_local;
  const int head = kvh * G + blockIdx.x % G;
  const int t = p.tile_begin + (gridDim.y - 1 - blockIdx.y);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool failed = err && *reinterpret_cast<volatile int *>(err) != 0;

  const bool ref = p.ref_indices != nullptr;
  const int nb = ref ? p.nb : p.route.nb;
  ListCursor cur{};
  if (ref) {
    cur.ref = p.ref_indices + ((int64_t)b * nb + t) * nb * p.H + head;
    cur.ref_stride = p.H;
    cur.cnt = failed ? 0 : min(max(p.ref_counts[((int64_t)b * nb + t) * p.H + head], 0), nb);
    cur.trusted = false;
  } else {
    const int64_t rr = p.route.row(b, head, t, p.H);
    cur.lst = p.route.lists + rr * p.route.nb;
    cur.cnt = failed ? 0 : min(max(p.route.counts[rr], 0), nb);
    cur.trusted = true;
  }
  cur.t = t;

  if (threadIdx.x == 0) {
    mbar_init(&sh.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
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
  if (warp == 4) {  // the tile's block count and whether its last block is the diagonal
    int n = 0, last = -1;
    if (cur.trusted) {
      n = cur.cnt;
      if (n > 0) last = cur.lst[n - 1];
    } else {
      cur.start(lane);
      for (int blk = cur.next(lane); blk >= 0; blk = cur.next(lane)) {
        ++n;
        last = blk;
      }
    }
    if (lane == 0) {
      sh.n = n;
      sh.diag = last == t;
    }
  }
  if (warp == 5) {
    tmem_alloc(&sh.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const int n = sh.n;

  if (warp == 4) {
    // ---------------------------------------------------------------- TMA producer
    if (n > 0) {
      if (lane == 0) {
        mbar_expect_tx(&sh.q_full, Geo::kQBytes);
        for (int a = 0; a < kAtoms; ++a) tma_load_4d(sh.q + a * kQAtom, &tm_q, &sh.q_full, 64 * a, head, t * 128, b);
      }
      int j = 0;
      int issued[kStages];
#pragma unroll
      for (int s = 0; s < kStages; ++s) issued[s] = 0;
      bool ok = true;
      // Two halves (64 keys each) of block blk's K or V into the next two ring stages.
      auto load_block = [&](const CUtensorMap *map, int blk) {
        for (int half = 0; half < 2 && ok; ++half, ++j) {
          const int s = j % kStages, use = j / kStages;
          if (use > 0 && !(ok = mbar_wait_warp(&sh.empty[s], (use - 1) & 1, abort))) break;
          if (lane == 0) {
            mbar_expect_tx(&sh.full[s], Geo::kStageBytes);
            for (int a = 0; a < kAtoms; ++a)
              tma_load_4d(sh.ring[s] + a * kKvAtom, map, &sh.full[s], 64 * a, kvh, blk * 128 + 64 * half, b);
          }
          issued[s] = use + 1;
        }
      };
      ListCursor kc = cur, vc = cur;
      kc.start(lane);
      vc.start(lane);
      load_block(&tm_k, kc.next(lane));
      for (int i = 0; i < n && ok; ++i) {
        if (i + 1 < n) load_block(&tm_k, kc.next(lane));
        load_block(&tm_v, vc.next(lane));
      }
      __syncwarp();
      if (*abort) {  // drain copies still in flight before the shared memory goes away
        int never = 0;
        mbar_wait(&sh.q_full, 0, &never);
        for (int s = 0; s < kStages; ++s)
          if (issued[s] > 0) mbar_wait(&sh.full[s], (issued[s] - 1) & 1, &never);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer
    if (n > 0 && mbar_wait_warp(&sh.q_full, 0, abort)) {
      int j = 0;
      bool ok = true;
      // Descriptors: fixed parts computed once; a ring stage moves the low word by its size.
      const uint32_t hi_km = desc_hi(desc_q1(sh.q, 0)), hi_v = desc_hi(desc_v1(sh.ring[0], 0));
      const uint32_t q_lo = desc_lo(desc_q1(sh.q, 0)), k_lo0 = desc_lo(desc_k1(sh.ring[0], 0));
      const uint32_t v_lo0 = desc_lo(desc_v1(sh.ring[0], 0));
      constexpr uint32_t kStageStep = Geo::kStageBytes >> 4;
      auto qk = [&](int i) {
        const int buf = i & 1;
        for (int half = 0; half < 2 && ok; ++half, ++j) {
          const int s = j % kStages;
          if (!(ok = mbar_wait_warp(&sh.full[s], (j / kStages) & 1, abort))) break;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t k_lo = k_lo0 + (uint32_t)s * kStageStep, s_tm = tmem + 128 * buf + 64 * half;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              mma_ss(s_tm, desc_join(q_lo + q1_step(kk), hi_km), desc_join(k_lo + k1_step(kk), hi_km), kIdescQK,
                     kk > 0 ? 1u : 0u);
            tc_commit(&sh.empty[s]);
          }
          __syncwarp();
        }
        if (ok) {
          if (lane == 0) tc_commit(&sh.s_full[buf]);
          __syncwarp();
        }
      };
      auto pv = [&](int i) {
        const int buf = i & 1;
        if (!(ok = mbar_wait_warp(&sh.p_full[buf], (i >> 1) & 1, abort))) return;
        for (int half = 0; half < 2 && ok; ++half, ++j) {
          const int s = j % kStages;
          if (!(ok = mbar_wait_warp(&sh.full[s], (j / kStages) & 1, abort))) break;
          tc_fence_after();
          if (lane == 0) {
            const uint32_t v_lo = v_lo0 + (uint32_t)s * kStageStep, p_tm = tmem + 128 * buf + 32 * half;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_ts(tmem + 256, p_tm + 8 * kk, desc_join(v_lo + v1_step(kk), hi_v), Geo::kIdescPV,
                     (i > 0 || half > 0 || kk > 0) ? 1u : 0u);
            tc_commit(&sh.empty[s]);
          }
          __syncwarp();
        }
        if (ok) {
          if (lane == 0) tc_commit(&sh.o_done[i & 1]);
          __syncwarp();
        }
      };
      qk(0);
      for (int i = 0; i < n && ok; ++i) {
        if (i + 1 < n) qk(i + 1);
        if (ok) pv(i);
      }
      if (*abort) {  // let every MMA this thread issued finish before TMEM is released
        int never = 0;
        if (lane == 0) tc_commit(&sh.drain);
        __syncwarp();
        mbar_wait(&sh.drain, 0, &never);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int r = warp * 32 + lane;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    const uint32_t o_addr = tmem + lane_off + 256;
    const int qrow = t * 128 + r;
    const float sl2 = p.scale_log2;
    const bool last_is_diag = n > 0 && sh.diag;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < n && ok; ++i) {
      const int buf = i & 1;
      const uint32_t s_addr = tmem + lane_off + 128 * buf;
      if (!(ok = mbar_wait_warp(&sh.s_full[buf], (i >> 1) & 1, abort))) break;
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
      float mx[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mx[c] = sv[c];
#pragma unroll
      for (int c = 8; c < 128; ++c) mx[c & 7] = fmaxf(mx[c & 7], sv[c]);
      const float bmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * sl2;
      const float mn = fmaxf(m, bmax);
      float corr = 1.f;
      // Each row decides for itself, as in the d = 128 kernel.
      const bool move = mn > m + kRescaleThreshold1 || m == -INFINITY;
      if (move) {
        corr = (m == -INFINITY) ? 0.f : ex2(m - mn);
        l *= corr;
        m = mn;
      }
      const float neg = (m == -INFINITY) ? 0.f : -m;
      l += diag ? softmax_row<0>(sv, sl2, neg, s_addr) : softmax_row<kEmu>(sv, sl2, neg, s_addr);
      if (i > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
        // O must hold blocks < i before it is rescaled: wait for P(i-1).V.
        if (!(ok = mbar_wait_warp(&sh.o_done[(i - 1) & 1], ((i - 1) >> 1) & 1, abort))) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
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
      mbar_arrive(&sh.p_full[buf]);
    }
    // Epilogue: O / l -> bf16 -> swizzled tile (in the Q buffer) -> TMA store; LSE.
    if (ok && n > 0 && !mbar_wait_warp(&sh.o_done[(n - 1) & 1], ((n - 1) >> 1) & 1, abort)) ok = false;
    tc_fence_after();
    const bool none = !(ok && n > 0) || m == -INFINITY;
    const float inv = none ? 0.f : 1.f / l;
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
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
        *reinterpret_cast<uint4 *>(sh.q + out_offset(r, 32 * c + 8 * e)) = v4;
      }
    }
    if (p.lse && qrow < p.L) p.lse[((int64_t)b * p.L + qrow) * p.H + head] = none ? -INFINITY : m * kLn2 + logf(l);
    fence_proxy_async();
    named_sync(1, 128);
    if (r == 0 && !*abort) {
      for (int a = 0; a < kAtoms; ++a) tma_store_4d(&tm_o, sh.q + a * kQAtom, 64 * a, head, t * 128, b);
      bulk_commit();
      bulk_wait0();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && sh.abort && err) atomicExch(err, 1);
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

namespace {
template <int D, int kEmu>
void launch_variant1(dim3 grid, cudaStream_t s, const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv,
                     const CUtensorMap &to, const ExactParams &p, int *err) {
  const size_t smem = sizeof(Smem1<D>) + 1024;
  cudaFuncSetAttribute(exact_tc1_kernel<D, kEmu>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  exact_tc1_kernel<D, kEmu><<<grid, kThreads1, smem, s>>>(tq, tk, tv, to, p, err);
}

template <int D>
void launch_d(dim3 grid, cudaStream_t s, const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv,
              const CUtensorMap &to, const ExactParams &p, int *err) {
  switch (get_option(kOptExpEmulation)) {
    case 0: launch_variant1<D, 0>(grid, s, tq, tk, tv, to, p, err); break;
    case 3: launch_variant1<D, 3>(grid, s, tq, tk, tv, to, p, err); break;
    default: launch_variant1<D, 2>(grid, s, tq, tk, tv, to, p, err); break;
  }
}
}  // namespace

int launch_exact_tc1(const ExactParams &p, int d, int B, int L, int Hkv, int tiles, int heads, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  if (d != 128 && d != 256) return FPX_ERR_UNSUPPORTED;
  if (p.group <= 0 || heads % p.group || p.head_begin % p.group) return FPX_ERR_SHAPE;
  CUtensorMap tq, tk, tv, to;
  if (!encode_4d(&tq, p.q, d, p.H, L, B, p.q_sh, p.q_sl, p.q_sb, 128) ||
      !encode_4d(&tk, p.k, d, Hkv, L, B, p.k_sh, p.k_sl, p.k_sb, 64) ||
      !encode_4d(&tv, p.v, d, Hkv, L, B, p.v_sh, p.v_sl, p.v_sb, 64) ||
      !encode_4d(&to, p.out, d, p.H, L, B, p.o_sh, p.o_sl, p.o_sb, 128))
    return FPX_ERR_INVALID;
  ExactParams q = p;
  q.kv_count = heads / p.group;
  const dim3 grid(p.group * q.kv_count, tiles, B);
  int *err = device_error_word();
  if (d == 128)
    launch_d<128>(grid, s, tq, tk, tv, to, q, err);
  else
    launch_d<256>(grid, s, tq, tk, tv, to, q, err);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

}  // namespace fpx
