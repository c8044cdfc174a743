// Parameter blocks and launchers of the routing kernels (route.cu).
#pragma once

#include "common.cuh"

namespace fpx {

struct StatsParams {
  const __nv_bfloat16 *k, *v;
  int64_t k_sb, k_sl, k_sh, v_sb, v_sl, v_sh;
  int L, nb, Hkv, kv_begin;
  __nv_bfloat16 *mean_bf16;                      // [B][nb][Hkv][d] (V1 block mean)
  float *mean_k, *mean_v, *var_k, *sigma_v;      // fp32 descriptors
  __nv_bfloat16 *mk_hi, *mk_lo, *mv_hi;          // bf16 splits for the tensor-core tail, or null
  __nv_bfloat16 *vk_hi, *vk_lo;                  // bf16 splits of var_k for the tensor-core selectors
  int32_t *counts;                               // [nb] or null
  int d;                                         // head dim: 128 (0 reads as 128) or 256
};

// What the selection epilogue needs (compact lists are written when route.lists != null).
struct SelectArgs {
  RouteView route;
  int nb, H, sink, window, last_full;
  float alpha;
  bool all_causal;
};

struct V1Params {
  const __nv_bfloat16 *q;
  int64_t q_sb, q_sl, q_sh;
  const __nv_bfloat16 *mean_k;  // [B][nb][Hkv][d]
  int L, nb, H, Hkv, group, head_begin, tile_begin;
  float scale_log2;             // fp32(scale) * fp32(log2 e), as the reference kernel forms it
  float *scores;                // reference layout [B][nb][nb][H], or null
  SelectArgs sel;
  int d;                        // head dim: 128 (0 reads as 128) or 256
};

struct SelParams {
  const __nv_bfloat16 *q;
  int64_t q_sb, q_sl, q_sh;
  const float *mean_k, *var_k, *sigma_v;
  // bf16 high + low halves of mean_k and var_k for the tensor-core kernel (null for the fp32 one)
  const __nv_bfloat16 *mk_hi, *mk_lo, *vk_hi, *vk_lo;
  int L, nb, H, Hkv, group, head_begin, tile_begin;
  float scale, scale2;          // fp32(scale), fp32(scale * scale)
  float *scores;
  SelectArgs sel;
  int d;                        // head dim: 128 (0 reads as 128) or 256 (the fp32 kernel only)
};

struct ColumnSelectParams {
  const float *scores;
  int nb, H, sink, window, last_full, min_budget, mode;
  float alpha;
  bool all_causal;
  int64_t *indices;
  int32_t *counts;
  uint8_t *mask;
};

int launch_block_stats(const StatsParams &p, int blocks, int kv_count, int B, bool bf16_mean,
                       bool desc, cudaStream_t s);
int launch_v1_route(const V1Params &p, int tiles, int heads, int B, cudaStream_t s);
// tcgen05 form (route_tc.cu): persistent CTAs over (b, KV group, tile) items.
int launch_v1_route_tc(const V1Params &p, int B, int tiles, int heads, cudaStream_t s);
// Whether the tcgen05 routing kernel holds a layer of nb blocks at head dim d.
bool v1_route_tc_supports(int d, int nb);
// The kernel fpx_set_option(3, ...) selects.
int launch_v1_route_selected(const V1Params &p, int tiles, int heads, int B, cudaStream_t s);
// tcgen05 form (route_sel_tc.cu): needs the bf16 splits in p (the fused path's workspace).
int launch_selector_route_tc(const SelParams &p, int selector, int tiles, int heads, int B, cudaStream_t s);
int launch_selector_route(const SelParams &p, int selector, int tiles, int heads, int B,
                          cudaStream_t s);
int launch_causal_route(const RouteView &r, int H, int head_begin, int heads, int tile_begin,
                        int tiles, int B, cudaStream_t s);
int launch_export_routing(const RouteView &r, int H, int B, uint8_t *mask, int64_t *indices,
                          int32_t *counts, cudaStream_t s);

}  // namespace fpx
