// V1 routing on the 5th-generation tensor core: block scores, per-(tile, block) max / mass,
// normalisation and the threshold + protected selection, fused, for every (b, KV group, query
// tile) of a layer.
//
// Reference semantics (upstream/flashprefill_native_forward.py):
//   :147-161  x = fp32(mk_b . q_i) * scale * log2 e for rows i of tile t with i >= 128 b + 127
//   :162-164  M = max_i x, S = sum_i exp2(x - M)
//   :410-417  score = S exp2(M - max M) / (sum + 1e-9), blocks with M = -inf score 0
//   :366-385  keep score >= alpha * max score, plus the sink / window / last-blocks protection
//
// The product is computed transposed, D = mean_K . Q^T, so TMEM lane = key block and column =
// query row: one thread owns one block and reduces its 128 query rows without any shuffle.
// A persistent CTA walks work items (b, KV group, tile t), longest tiles first, and inside an
// item the G heads of the group; each (head, 128-block chunk) is one unit of d / 16 MMAs
// (M = 128 blocks, N = 128 rows, K = d; head dim 128 or 256). 320 threads:
//   warp 0       TMA: Q tiles (3-stage ring at d = 128, one stage at d = 256, whose 64 KB
//                tiles leave room for two resident block-mean chunks) and block-mean chunks
//   warp 1       MMA issuer (one elected lane), TMEM owner
//   warps 2..9   epilogue, two warpgroups taking alternate heads: thread = block (TMEM lane),
//                then the head's normalisation and selection over the group's named barrier
// TMEM holds four 128-column accumulators, so the tensor core runs up to four units ahead of
// the epilogue. Up to 256 blocks the group's block means stay resident for the whole item
// (both chunks load once, every head reuses them); past that each unit streams its chunk.
//
// Every mbarrier wait is bounded; a wait that gives up sets the CTA's abort flag and the
// device error word, every role then runs out its loops without waiting (the epilogue still
// meets each named barrier), in-flight copies and MMAs are drained and TMEM is freed.
#include <cuda.h>

#include "route.cuh"
#include "tc.cuh"

namespace fpx {

namespace {

using namespace tc;

constexpr int kThreads = 320;
constexpr int kAcc = 4;                   // 128-column accumulators in 512 TMEM columns:
                                          // slots 2g, 2g + 1 belong to epilogue warpgroup g
constexpr uint32_t kHalf = 128 * 128;     // 128 rows x 64 bf16, one SW128 atom
constexpr uint32_t kIdesc = idesc_bf16(128, 128, false);

// Per head dim: Q ring depth and the longest layer (blocks) the score arrays hold.
template <int D>
struct RouteGeo {
  static constexpr int kAtoms = D / 64;                    // 64-column SW128 atoms per tile
  static constexpr uint32_t kTile = kAtoms * kHalf;         // 128 x D bf16
  static constexpr int kQStages = D == 128 ? 3 : 1;
  static constexpr int kMaxBlocks = D == 128 ? 2048 : 512;  // L <= 262144 / 65536
};

template <int D>
struct alignas(1024) Smem {
  static constexpr int kQStages = RouteGeo<D>::kQStages, kMaxBlocks = RouteGeo<D>::kMaxBlocks;
  uint8_t q[kQStages][RouteGeo<D>::kTile];
  uint8_t mk[2][RouteGeo<D>::kTile];
  uint64_t q_full[kQStages], q_empty[kQStages], mk_full[2], mk_empty[2], acc_full[kAcc], acc_empty[kAcc];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  float red[2][2][8];                     // [warpgroup][parity][partials]
  int scan[2][2][4 * (kMaxBlocks / 128)];  // [warpgroup][parity][chunk x warp]
  float bm[2][kMaxBlocks], bs[2][kMaxBlocks], sc[2][kMaxBlocks];
};

FPX_INLINE uint64_t desc_kmajor(const uint8_t *tile, int kk) {
  return smem_desc_sw128(smem_u32(tile) + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
}

// Max and mass of one block's 128 query rows (this thread's TMEM lane, 128 fp32 columns at
// taddr), in two warp-uniform passes over TMEM: M = fp32(max dot * scale_log2), then
// S = sum exp2(x - M) with x = fp32(dot * scale_log2) rounded before the subtraction, as the
// reference forms it. kRagged: only the first nrows rows exist. `last` = row 127's dot.
template <bool kRagged>
FPX_INLINE void block_mass(uint32_t taddr, int nrows, float sl2, float &M, float &S, float &last) {
  float mx[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) mx[j] = -INFINITY;
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    float v[32];
    tmem_ld32(taddr + 32 * q4, v);
    tmem_wait_ld();
#pragma unroll
    for (int r = 0; r < 32; ++r)
      if (!kRagged || 32 * q4 + r < nrows) mx[r & 7] = fmaxf(mx[r & 7], v[r]);
    if (q4 == 3) last = v[31];
  }
  M = __fmul_rn(fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))),
                sl2);
  const uint64_t sl2x2 = pk2(sl2, sl2), negm = pk2(-M, -M);
  uint64_t acc2[4] = {0, 0, 0, 0};
#pragma unroll
  for (int q4 = 0; q4 < 4; ++q4) {
    float v[32];
    tmem_ld32(taddr + 32 * q4, v);
    tmem_wait_ld();
#pragma unroll
    for (int r = 0; r < 32; r += 2) {
      float x0, x1;
      up2(fadd2(fmul2(pk2(v[r], v[r + 1]), sl2x2), negm), x0, x1);
      if (kRagged) {  // rows past the end of the sequence take no part
        x0 = 32 * q4 + r < nrows ? x0 : -INFINITY;
        x1 = 32 * q4 + r + 1 < nrows ? x1 : -INFINITY;
      }
      acc2[(r >> 1) & 3] = fadd2(acc2[(r >> 1) & 3], pk2(ex2(x0), ex2(x1)));
    }
  }
  float s[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) up2(acc2[j], s[2 * j], s[2 * j + 1]);
  S = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

struct Item {
  int b, kvh, t, nblk, chunks, h0, h1;  // heads [h0, h1) of the group, as offsets in it
  bool resident;
};

// Item i: tile (last - i / (B kv_groups splits)), then batch, then KV group, then the split of
// the group's G heads into `splits` runs (more items when a launch has few tiles).
FPX_INLINE Item item_at(int i, int B, int tiles, int kv_groups, int kv_begin, int tile_begin, int G, int splits) {
  const int per_tile = kv_groups * B * splits;
  const int rank = i / per_tile, rem = i % per_tile;
  const int sp = rem % splits, rest = rem / splits;
  Item it;
  it.t = tile_begin + tiles - 1 - rank;
  it.b = rest / kv_groups;
  it.kvh = kv_begin + rest % kv_groups;
  it.h0 = sp * G / splits;
  it.h1 = (sp + 1) * G / splits;
  it.nblk = it.t + 1;
  it.chunks = (it.nblk + 127) / 128;
  it.resident = it.chunks <= 2;
  return it;
}

}  // namespace

// Items run longest tile first; CTA c takes items c, c + gridDim.x, ...
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    v1_route_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_mk,
                       V1Params p, int B, int tiles, int kv_groups, int splits, int n_items, int *device_error) {
  constexpr int kQStages = RouteGeo<D>::kQStages, kAtoms = RouteGeo<D>::kAtoms;
  constexpr uint32_t kTile = RouteGeo<D>::kTile;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  Smem<D> &sh = *reinterpret_cast<Smem<D> *>(smem_raw + pad);
  volatile int *abort = &sh.abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv_begin = p.head_begin / p.group;
  const int G = p.group;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(&sh.q_full[s], 1);
      mbar_init(&sh.q_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sh.mk_full[s], 1);
      mbar_init(&sh.mk_empty[s], 1);
    }
    for (int a = 0; a < kAcc; ++a) {
      mbar_init(&sh.acc_full[a], 1);
      mbar_init(&sh.acc_empty[a], 128);
    }
    mbar_init(&sh.drain, 1);
    sh.abort = *reinterpret_cast<volatile int *>(device_error) != 0;
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
    // ------------------------------------------------------------------ TMA producer
    int q_n = 0, mk_use[2] = {0, 0}, mk_rr = 0;
    bool ok = !*abort;
    auto load_mk = [&](int slot, const Item &it, int c) -> bool {
      if (mk_use[slot] > 0 && !mbar_wait_warp(&sh.mk_empty[slot], (mk_use[slot] - 1) & 1, abort)) return false;
      if (lane == 0) {
        mbar_expect_tx(&sh.mk_full[slot], kTile);
        for (int at = 0; at < kAtoms; ++at)
          tma_load_4d(sh.mk[slot] + at * kHalf, &tm_mk, &sh.mk_full[slot], 64 * at, it.kvh, c * 128, it.b);
      }
      ++mk_use[slot];
      return true;
    };
    for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
      const Item it = item_at(i, B, tiles, kv_groups, kv_begin, p.tile_begin, G, splits);
      for (int hi = it.h0; hi < it.h1 && ok; ++hi) {
        const int s = q_n % kQStages;
        if (q_n >= kQStages && !(ok = mbar_wait_warp(&sh.q_empty[s], (q_n / kQStages - 1) & 1, abort))) break;
        if (lane == 0) {
          const int h = it.kvh * G + hi;
          mbar_expect_tx(&sh.q_full[s], kTile);
          for (int at = 0; at < kAtoms; ++at)
            tma_load_4d(sh.q[s] + at * kHalf, &tm_q, &sh.q_full[s], 64 * at, h, it.t * 128, it.b);
        }
        ++q_n;
        if (it.resident) {
          if (hi == it.h0)
            for (int c = 0; c < it.chunks && ok; ++c) ok = load_mk(c, it, c);
        } else {
          for (int c = 0; c < it.chunks && ok; ++c) ok = load_mk(mk_rr++ & 1, it, c);
        }
      }
    }
    __syncwarp();
    if (*abort) {  // drain copies still in flight before the shared memory goes away
      int never = 0;
      for (int s = 0; s < kQStages; ++s) {
        const int n = q_n / kQStages + (s < q_n % kQStages ? 1 : 0);
        if (n > 0) mbar_wait(&sh.q_full[s], (n - 1) & 1, &never);
      }
      for (int s = 0; s < 2; ++s)
        if (mk_use[s] > 0) mbar_wait(&sh.mk_full[s], (mk_use[s] - 1) & 1, &never);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    // Each warpgroup's two slots are filled and drained strictly in turn, so no wait on a slot is
    // ever more than one phase ahead of it (a parity wait cannot tell phases two apart).
    int q_n = 0, mk_use[2] = {0, 0}, mk_rr = 0, issued[2] = {0, 0}, hseq = 0;
    bool ok = !*abort;
    for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
      const Item it = item_at(i, B, tiles, kv_groups, kv_begin, p.tile_begin, G, splits);
      for (int hi = it.h0; hi < it.h1 && ok; ++hi, ++hseq) {
        const int g = hseq & 1;  // the warpgroup that reduces this head
        const int s = q_n % kQStages;
        if (!(ok = mbar_wait_warp(&sh.q_full[s], (q_n / kQStages) & 1, abort))) break;
        for (int c = 0; c < it.chunks && ok; ++c) {
          const int slot = it.resident ? c : (mk_rr & 1);
          if ((!it.resident || hi == it.h0) && !(ok = mbar_wait_warp(&sh.mk_full[slot], mk_use[slot] & 1, abort)))
            break;
          const int a = 2 * g + (issued[g] & 1), use = issued[g] >> 1;
          if (use > 0 && !(ok = mbar_wait_warp(&sh.acc_empty[a], (use - 1) & 1, abort))) break;
          tc_fence_after();
          if (lane == 0) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk)
              mma_ss(tmem + 128 * a, desc_kmajor(sh.mk[slot], kk), desc_kmajor(sh.q[s], kk), kIdesc,
                     kk > 0 ? 1u : 0u);
            tc_commit(&sh.acc_full[a]);
            if (!it.resident) tc_commit(&sh.mk_empty[slot]);
          }
          __syncwarp();
          if (!it.resident) {
            ++mk_use[slot];
            ++mk_rr;
          }
          ++issued[g];
        }
        if (!ok) break;
        if (lane == 0) tc_commit(&sh.q_empty[s]);
        __syncwarp();
        ++q_n;
      }
      if (ok && it.resident) {
        if (lane == 0)
          for (int c = 0; c < it.chunks; ++c) tc_commit(&sh.mk_empty[c]);
        __syncwarp();
        for (int c = 0; c < it.chunks; ++c) ++mk_use[c];
      }
    }
    if (*abort) {  // let every MMA this thread issued finish before TMEM is released
      int never = 0;
      if (lane == 0) tc_commit(&sh.drain);
      __syncwarp();
      mbar_wait(&sh.drain, 0, &never);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    // Two warpgroups take alternate heads (the CTA's running head count decides), so one runs
    // a head's selection while the other reduces the next head's accumulators.
    const int g = (warp - 2) >> 2;         // warpgroup: 0 = warps 2..5, 1 = warps 6..9
    const int ew = warp & 3;               // TMEM lane quarter this warp may access
    const int e = ew * 32 + lane;          // block within a chunk == TMEM lane
    const uint32_t lane_off = (uint32_t)(ew * 32) << 16;
    const float sl2 = p.scale_log2;
    const SelectArgs &a = p.sel;
    float *bm = sh.bm[g], *bs = sh.bs[g], *sc = sh.sc[g];
    int done = 0, hseq = 0, red_k = 0;  // done: units this warpgroup has reduced
    bool ok = !*abort;
    auto grp_sync = [&]() { named_sync(1 + g, 128); };
    for (int i = blockIdx.x; i < n_items; i += gridDim.x) {
      const Item it = item_at(i, B, tiles, kv_groups, kv_begin, p.tile_begin, G, splits);
      const int t = it.t;
      const int nrows = min(kBlock, p.L - t * kBlock);  // valid query rows of the tile
      for (int hi = it.h0; hi < it.h1; ++hi, ++hseq) {
        if ((hseq & 1) != g) continue;
        const int h = it.kvh * G + hi;
        for (int c = 0; c < it.chunks; ++c, ++done) {
          const int ac = 2 * g + (done & 1);
          if (ok) ok = mbar_wait_warp(&sh.acc_full[ac], (done >> 1) & 1, abort);
          tc_fence_after();
          const int kb = c * 128 + e;
          const uint32_t taddr = tmem + lane_off + 128 * ac;
          float M = -INFINITY, S = 0.f;
          if (ok && c * 128 + ew * 32 <= t) {  // some block of this warp is visible
            float last;
            if (nrows == kBlock)
              block_mass<false>(taddr, nrows, sl2, M, S, last);
            else
              block_mass<true>(taddr, nrows, sl2, M, S, last);
            if (kb == t) {  // the diagonal block is seen by the tile's last row only
              const bool seen = nrows == kBlock;
              M = seen ? __fmul_rn(last, sl2) : -INFINITY;
              S = seen ? 1.f : 0.f;
            } else if (kb > t) {
              M = -INFINITY;
              S = 0.f;
            }
          }
          tc_fence_before();
          mbar_arrive(&sh.acc_empty[ac]);
          bm[kb] = M;
          bs[kb] = S;
        }
        // normalize_scores (upstream:410-417), then the selection (upstream:366-385). Thread e
        // handles blocks e, e + 128, ...: the same blocks it wrote above, so bm / bs / sc need
        // no barrier of their own. score = r / total with r = S exp2(M - max M); max score is
        // (max r) / total exactly, as rounding is monotonic.
        // The group agrees on whether every warp's waits succeeded before anything is written,
        // so a row is either complete or has count 0 (never a count over unwritten entries).
        float lm = -INFINITY;
        for (int kb = e; kb < it.nblk; kb += 128) lm = fmaxf(lm, bm[kb]);
        lm = warp_max(lm);
        float *red = sh.red[g][red_k & 1];
        if (lane == 0) {
          red[ew] = lm;
          red[4 + ew] = ok ? 1.f : 0.f;
        }
        grp_sync();
        ++red_k;
        const float gmax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        const bool wg_ok = (red[4] + red[5]) + (red[6] + red[7]) == 4.f;
        float ls = 0.f, lr = 0.f;
        for (int kb = e; kb < it.nblk; kb += 128) {
          const float m = bm[kb];
          const float r = (m != -INFINITY) ? __fmul_rn(bs[kb], ex2(m - gmax)) : 0.f;
          sc[kb] = r;
          ls += r;
          lr = fmaxf(lr, r);
        }
        ls = warp_sum(ls);
        lr = warp_max(lr);
        red = sh.red[g][red_k & 1];
        if (lane == 0) {
          red[ew] = ls;
          red[4 + ew] = lr;
        }
        grp_sync();
        ++red_k;
        const float total = ((red[0] + red[1]) + (red[2] + red[3])) + 1e-9f;
        const float smax = fmaxf(fmaxf(red[4], red[5]), fmaxf(red[6], red[7])) / total;
        if (p.scores && wg_ok)
          for (int kb = e; kb < p.nb; kb += 128)
            p.scores[(((int64_t)it.b * p.nb + t) * p.nb + kb) * p.H + h] = kb < it.nblk ? sc[kb] / total : 0.f;
        if (a.route.lists) {
          const float thr = smax * a.alpha;
          const int64_t rrow = a.route.row(it.b, h, t, a.H);
          int32_t *list = a.route.lists + rrow * a.route.nb;
          uint32_t *tail = a.route.tail + rrow * a.route.words;
          auto active_at = [&](int kb) {
            return kb < a.nb && kb <= t &&
                   (a.all_causal || sc[kb] / total >= thr || is_protected(t, kb, a.nb, a.sink, a.window, a.last_full));
          };
          // One exchange for the whole row: per-(chunk, warp) counts, then each warp's offsets.
          const int nch = (a.nb + 127) / 128;
          int *cnt = sh.scan[g][red_k & 1];
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
            const unsigned tb = __ballot_sync(0xffffffffu, kb < a.nb && kb < t && !active);
            if (lane == 0 && kb < a.nb && wg_ok) tail[kb >> 5] = tb;
            base += (cnt[4 * j] + cnt[4 * j + 1]) + (cnt[4 * j + 2] + cnt[4 * j + 3]);
          }
          if (e == 0) a.route.counts[rrow] = wg_ok ? base : 0;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && sh.abort) atomicExch(device_error, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
size_t v1_route_tc_smem() { return sizeof(Smem<D>) + 1024; }

template <int D>
static int launch_v1_route_tc_d(const V1Params &p, int B, int tiles, int heads, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  if (heads % p.group || p.head_begin % p.group) return FPX_ERR_SHAPE;
  if (p.nb > RouteGeo<D>::kMaxBlocks) return FPX_ERR_UNSUPPORTED;
  const int kv_groups = heads / p.group;
  // Split each group's heads over more items when the launch has fewer than two items per SM
  // (a tile range of one rank, a short sequence): an item's heads run one after another.
  CUtensorMap tq, tmk;
  if (!encode_4d(&tq, p.q, D, p.H, p.L, B, p.q_sh, p.q_sl, p.q_sb) ||
      !encode_4d(&tmk, p.mean_k, D, p.Hkv, p.nb, B, D, (int64_t)p.Hkv * D, (int64_t)p.nb * p.Hkv * D))
    return FPX_ERR_INVALID;
  int *device_error = device_error_word();
  if (!device_error) return FPX_ERR_CUDA;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return FPX_ERR_CUDA;
  const int base_items = B * tiles * kv_groups;
  const int splits = std::max(1, std::min(p.group, (2 * sms + base_items - 1) / base_items));
  const int n_items = base_items * splits;
  const int grid = std::min(n_items, sms);
  const size_t smem = v1_route_tc_smem<D>();
  cudaFuncSetAttribute(v1_route_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  v1_route_tc_kernel<D><<<grid, kThreads, smem, s>>>(tq, tmk, p, B, tiles, kv_groups, splits, n_items, device_error);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

int launch_v1_route_tc(const V1Params &p, int B, int tiles, int heads, cudaStream_t s) {
  return p.d == 256 ? launch_v1_route_tc_d<256>(p, B, tiles, heads, s)
                    : launch_v1_route_tc_d<128>(p, B, tiles, heads, s);
}

bool v1_route_tc_supports(int d, int nb) {
  return d == 256 ? nb <= RouteGeo<256>::kMaxBlocks : nb <= RouteGeo<128>::kMaxBlocks;
}

}  // namespace fpx
