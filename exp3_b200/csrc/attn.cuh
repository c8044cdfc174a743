// Parameter blocks and launchers of the exact-path and mean-tail kernels.
#pragma once

#include "common.cuh"

namespace fpx {

enum ExactMode { kExactLists = 0, kExactRefLayout = 1, kExactDense = 2 };

struct ExactParams {
  const __nv_bfloat16 *q, *k, *v;
  int64_t q_sb, q_sl, q_sh, k_sb, k_sl, k_sh, v_sb, v_sl, v_sh;
  __nv_bfloat16 *out;
  int64_t o_sb, o_sl, o_sh;
  float *lse;                       // [B][L][H] or null
  int L, nb, H, group, head_begin, tile_begin;
  float scale_log2;
  RouteView route;                  // kExactLists
  const int64_t *ref_indices;       // kExactRefLayout: [B][nb][nb][H]
  const int32_t *ref_counts;        //                  [B][nb][H]
  int kv_count;                     // KV groups in the launch (set by the d = 256 launcher)
};

int launch_exact_mma(const ExactParams &p, int mode, int tiles, int heads, int B, cudaStream_t s);
// tcgen05 / TMEM / TMA exact kernel over internal lists (kExactLists).
int launch_exact_tc(const ExactParams &p, int B, int L, int Hkv, int tiles, int heads, cudaStream_t s);
// One query tile per CTA with double-buffered S (attn_tc1.cu), head dim d = 128 or 256, lists
// or reference layout.
int launch_exact_tc1(const ExactParams &p, int d, int B, int L, int Hkv, int tiles, int heads, cudaStream_t s);

// Process-wide options (fpx_set_option): which exact kernel the fused path runs, how many
// of every 8 exp2 pairs the tcgen05 kernel computes on the FMA pipe (0, 2 or 3), which V1
// routing kernel, mean-tail kernel and new-selector routing kernel run.
enum Option { kOptExactKernel = 1, kOptExpEmulation = 2, kOptRouteKernel = 3, kOptMeanKernel = 4,
              kOptSelectorKernel = 5 };
enum ExactKernel { kExactKernelTcgen05 = 0, kExactKernelMmaSync = 1, kExactKernelTcgen05Single = 2 };
enum RouteKernel { kRouteKernelTcgen05 = 0, kRouteKernelMmaSync = 1 };
enum MeanKernel { kMeanKernelTcgen05 = 0, kMeanKernelFp32 = 1 };
enum SelectorKernel { kSelectorKernelTcgen05 = 0, kSelectorKernelFp32 = 1 };
int get_option(int key);

enum MeanMode { kMeanMergeInPlace = 0, kMeanStandalone = 1 };

struct MeanParams {
  const __nv_bfloat16 *q;
  int64_t q_sb, q_sl, q_sh;
  const float *mean_k, *mean_v;     // [B][nb][Hkv][d]
  // bf16 splits of the same descriptors for the tensor-core tail: mean_k = mk_hi + mk_lo
  // (lo = bf16 of the rounding remainder), mv_hi = bf16(mean_v)
  const __nv_bfloat16 *mk_hi, *mk_lo, *mv_hi;
  int L, nb, H, Hkv, group, head_begin, tile_begin;
  float scale;
  RouteView route;                  // kMeanMergeInPlace: tail bits
  const uint8_t *mask;              // kMeanStandalone: selected [B][nb][nb][H]
  // kMeanMergeInPlace: exact output (bf16, merged in place) and its LSE (updated in place)
  __nv_bfloat16 *out;
  int64_t o_sb, o_sl, o_sh;
  float *lse;
  // kMeanStandalone: fp32 mean-tail output [B][L][H][d] and LSE [B][L][H]
  float *mean_out, *mean_lse;
  // rescue tails: K / V and the chosen token of every (b, h, t, kb), [B][H][nb][nb]
  const __nv_bfloat16 *k, *v;
  int64_t k_sb, k_sl, k_sh, v_sb, v_sl, v_sh;
  uint8_t *choice;
  // rescue choice: fp32 query means [B][nb][H][d] filled by the choice launch itself (one pass
  // over Q), or null to have each choice CTA form its group's means from Q
  float *qmean;
  int d;                            // head dim: 128 (0 reads as 128) or 256 (block-mean tail only)
};

// keys: 0 block means (mean_tail), 1 rescue tokens, 2 rescue tokens + remainder means.
int launch_mean_tail(const MeanParams &p, int mode, int tiles, int heads, int B, cudaStream_t s, int keys = 0);
// Rescue token of every tail block (kernels.py:276-285) into p.choice; the tail comes from the
// route's bits (kMeanMergeInPlace) or from the mask (kMeanStandalone).
int launch_rescue_choice(const MeanParams &p, int mode, int tiles, int kv_count, int B, cudaStream_t s);
// Rescue tails (keys 1 / 2) on the tensor core, merged in place (rescue_tc.cu); needs choice,
// k, v, mean_k, mean_v, route (tail bits), out and lse.
int launch_rescue_tail_tc(const MeanParams &p, int keys, int B, int L, int tiles, int heads, cudaStream_t s);
// tcgen05 / TMEM / TMA tail, merged in place (attn_tail_tc.cu); needs mk_hi, mk_lo, mv_hi.
int launch_mean_tail_tc(const MeanParams &p, int B, int tiles, int heads, cudaStream_t s);
int launch_merge(const __nv_bfloat16 *exact_out, const float *exact_lse, const float *mean_out,
                 const float *mean_lse, int64_t rows, __nv_bfloat16 *out, float *lse,
                 cudaStream_t s, int d = kHeadDim);

// The two-tile kernels' work units (attn_tc.cu, attn_tail_tc.cu): two query tiles of one KV group
// that read nearly the same blocks, heads hA and hA + 1 at one tile, or the last head of an odd
// group at tiles t and t - 1. Launch order: per two tiles (longest first) the U = kv_count * G/2
// head pairs of the longer tile, then (G odd) the kv_count units of the last head at both
// tiles, then the U head pairs of the shorter tile. Returns the unit's two (tile, head) and
// whether the second exists.
struct ExactUnit {
  int kvh, t[2], h[2];
  bool has_b;
};
FPX_INLINE ExactUnit exact_unit(int idx, int tile_begin, int tiles, int kv_begin, int kv_count, int G) {
  const int full = G / 2, U = kv_count * full, V = (G & 1) ? kv_count : 0;
  const int j = idx / (2 * U + V), r = idx % (2 * U + V);
  const int y = r < U + V ? 2 * j : 2 * j + 1;
  const int slot = r < U + V ? r : r - (U + V);
  const int t0 = tile_begin + tiles - 1 - y;
  ExactUnit e;
  if (slot < U) {
    e.kvh = kv_begin + slot / full;
    e.h[0] = e.kvh * G + 2 * (slot % full);
    e.h[1] = e.h[0] + 1;
    e.t[0] = e.t[1] = t0;
    e.has_b = true;
  } else {
    e.kvh = kv_begin + (slot - U);
    e.h[0] = e.h[1] = e.kvh * G + G - 1;
    e.has_b = t0 - 1 >= tile_begin;
    e.t[0] = t0;
    e.t[1] = e.has_b ? t0 - 1 : t0;  // an absent tile keeps a valid index
  }
  return e;
}
__host__ __device__ inline int exact_units(int tiles, int kv_count, int G) {
  return tiles * kv_count * (G / 2) + ((tiles + 1) / 2) * ((G & 1) ? kv_count : 0);
}

}  // namespace fpx
