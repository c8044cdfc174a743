// The fused prefill path (attention.py:210-333) and the C ABI of the exact / mean / merge ops.
//
// fpx_prefill_attention runs, on one stream and a caller-provided workspace:
//   route  — block statistics + the method's scores + selection into compact lists;
//   exact  — block-sparse attention over the lists, bf16 output + natural LSE;
//   mean   — for mean methods, the block-mean tail merged into the exact output in place.
#include <algorithm>

#include "attn.cuh"
#include "route.cuh"

namespace fpx {

struct Workspace {
  int32_t *lists, *counts;
  uint32_t *tail;
  __nv_bfloat16 *mk16, *mkh, *mkl, *mvh, *vkh, *vkl;
  uint8_t *choice;  // rescue token of every (b, h, t, kb), [B][H][nb][nb]
  float *mk, *mv, *vk, *sv, *lse;
  float *qmean;     // rescue choice: fp32 query means, [B][nb][H][d]
  size_t bytes;
};

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static Workspace carve(void *base, int B, int L, int H, int Hkv, int d = kHeadDim) {
  const int64_t nb = (L + kBlock - 1) / kBlock, words = (nb + 31) / 32;
  Workspace w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t *p = base ? static_cast<uint8_t *>(base) + off : nullptr;
    off += align256(bytes);
    return p;
  };
  w.lists = reinterpret_cast<int32_t *>(take((size_t)B * H * nb * nb * 4));
  w.counts = reinterpret_cast<int32_t *>(take((size_t)B * H * nb * 4));
  w.tail = reinterpret_cast<uint32_t *>(take((size_t)B * H * nb * words * 4));
  const size_t desc = (size_t)B * nb * Hkv * d;
  w.mk16 = reinterpret_cast<__nv_bfloat16 *>(take(desc * 2));
  w.mkh = reinterpret_cast<__nv_bfloat16 *>(take(desc * 2));
  w.mkl = reinterpret_cast<__nv_bfloat16 *>(take(desc * 2));
  w.mvh = reinterpret_cast<__nv_bfloat16 *>(take(desc * 2));
  w.vkh = reinterpret_cast<__nv_bfloat16 *>(take(desc * 2));
  w.vkl = reinterpret_cast<__nv_bfloat16 *>(take(desc * 2));
  w.mk = reinterpret_cast<float *>(take(desc * 4));
  w.mv = reinterpret_cast<float *>(take(desc * 4));
  w.vk = reinterpret_cast<float *>(take(desc * 4));
  w.sv = reinterpret_cast<float *>(take((size_t)B * nb * Hkv * 4));
  w.lse = reinterpret_cast<float *>(take((size_t)B * L * H * 4));
  w.choice = static_cast<uint8_t *>(take((size_t)B * H * nb * nb));
  w.qmean = reinterpret_cast<float *>(take((size_t)B * nb * H * d * 4));
  w.bytes = off;
  return w;
}

static bool aligned16(const void *p) { return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
static bool strides_ok(int64_t a, int64_t b, int64_t c) { return a % 8 == 0 && b % 8 == 0 && c % 8 == 0; }

static bool is_rescue_method(int m) {
  return m == FPX_METHOD_FP_V1_RESCUE || m == FPX_METHOD_FP_V1_RESCUE_V2;
}

static bool is_mean_method(int m) {
  return m == FPX_METHOD_MEAN_NATIVE || m == FPX_METHOD_MEAN_BALANCED || m == FPX_METHOD_CGF_MEAN ||
         m == FPX_METHOD_DISPERSION_MEAN;
}

}  // namespace fpx

using namespace fpx;

extern "C" const char *fpx_status_string(int status) {
  switch (status) {
    case FPX_OK: return "ok";
    case FPX_ERR_INVALID: return "invalid argument";
    case FPX_ERR_SHAPE: return "inconsistent shapes";
    case FPX_ERR_UNSUPPORTED: return "unsupported head_dim, block size or method";
    case FPX_ERR_CUDA: return "CUDA launch failed";
    case FPX_ERR_WORKSPACE: return "workspace too small or misaligned";
    case FPX_ERR_TIMEOUT: return "device-side wait timed out";
    default: return "unknown status";
  }
}

extern "C" int fpx_version(void) { return 1; }

namespace fpx {
static int g_options[6] = {0, kExactKernelTcgen05, 0, kRouteKernelTcgen05, kMeanKernelTcgen05,
                           kSelectorKernelTcgen05};
int get_option(int key) { return (key > 0 && key < 6) ? g_options[key] : 0; }
}  // namespace fpx

extern "C" int fpx_set_option(int key, int value) {
  if ((key == kOptExactKernel && (value == kExactKernelTcgen05 || value == kExactKernelMmaSync ||
                                  value == kExactKernelTcgen05Single)) ||
      (key == kOptExpEmulation && (value == 0 || value == 2 || value == 3)) ||
      (key == kOptRouteKernel && (value == kRouteKernelTcgen05 || value == kRouteKernelMmaSync)) ||
      (key == kOptMeanKernel && (value == kMeanKernelTcgen05 || value == kMeanKernelFp32)) ||
      (key == kOptSelectorKernel && (value == kSelectorKernelTcgen05 || value == kSelectorKernelFp32))) {
    g_options[key] = value;
    return FPX_OK;
  }
  return FPX_ERR_INVALID;
}

extern "C" size_t fpx_prefill_workspace_bytes(int method, int B, int L, int H, int Hkv, int d,
                                              int block) {
  (void)method; (void)block;
  if (B <= 0 || L <= 0 || H <= 0 || Hkv <= 0 || (d != kHeadDim && d != 256)) return 0;
  return carve(nullptr, B, L, H, Hkv, d).bytes;
}

extern "C" int fpx_prefill_attention(int method, double alpha, int sink, int window, int last_full,
                                     const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                     const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                     const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                                     int B, int L, int H, int Hkv, int d, int block, double scale,
                                     int kv_begin, int kv_end, int tile_begin, int tile_end,
                                     void *out, int64_t o_sb, int64_t o_sl, int64_t o_sh,
                                     float *lse, void *workspace, size_t workspace_bytes,
                                     int stages, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (method < 0 || method > FPX_METHOD_FP_V1_RESCUE_V2) return FPX_ERR_INVALID;
  if (block != kBlock) return FPX_ERR_UNSUPPORTED;
  // Head dim 128, or 256 (the Qwen3.5 path, check_qwen35_math.py).
  if (d != kHeadDim && d != 256) return FPX_ERR_UNSUPPORTED;
  if (B <= 0 || L <= 0 || H <= 0 || Hkv <= 0 || !aligned16(q) || !aligned16(k) || !aligned16(v) ||
      !aligned16(out))
    return FPX_ERR_INVALID;
  if (H % Hkv || !strides_ok(q_sb, q_sl, q_sh) || !strides_ok(k_sb, k_sl, k_sh) ||
      !strides_ok(v_sb, v_sl, v_sh) || !strides_ok(o_sb, o_sl, o_sh))
    return FPX_ERR_SHAPE;
  const int nb = (L + kBlock - 1) / kBlock;
  if (kv_begin < 0 || kv_end > Hkv || kv_begin >= kv_end || tile_begin < 0 || tile_end > nb ||
      tile_begin >= tile_end)
    return FPX_ERR_SHAPE;
  const Workspace ws = carve(workspace, B, L, H, Hkv, d);
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) || workspace_bytes < ws.bytes)
    return FPX_ERR_WORKSPACE;
  cudaStream_t s = stream;
  const int G = H / Hkv;
  const int head_begin = kv_begin * G, heads = (kv_end - kv_begin) * G;
  const int tiles = tile_end - tile_begin;
  const int kv_count = kv_end - kv_begin;
  float *lse_out = lse ? lse : ws.lse;
  RouteView rv{ws.lists, ws.counts, ws.tail, nb, (nb + 31) / 32};
  const auto *qb = static_cast<const __nv_bfloat16 *>(q);
  const auto *kb = static_cast<const __nv_bfloat16 *>(k);
  const auto *vb = static_cast<const __nv_bfloat16 *>(v);
  int rc = FPX_OK;

  if (stages & FPX_STAGE_ROUTE) {
    SelectArgs sel{};
    sel.route = rv; sel.nb = nb; sel.H = H; sel.sink = sink; sel.window = window;
    sel.last_full = last_full; sel.alpha = (float)alpha; sel.all_causal = false;
    StatsParams st{};
    st.k = kb; st.k_sb = k_sb; st.k_sl = k_sl; st.k_sh = k_sh;
    st.v = vb; st.v_sb = v_sb; st.v_sl = v_sl; st.v_sh = v_sh;
    st.L = L; st.nb = nb; st.Hkv = Hkv; st.kv_begin = kv_begin;
    st.mean_bf16 = ws.mk16; st.mean_k = ws.mk; st.mean_v = ws.mv; st.var_k = ws.vk;
    st.sigma_v = ws.sv; st.counts = nullptr;
    st.mk_hi = ws.mkh; st.mk_lo = ws.mkl; st.mv_hi = ws.mvh; st.vk_hi = ws.vkh; st.vk_lo = ws.vkl;
    st.d = d;
    if (method == FPX_METHOD_DENSE) {
      rc = launch_causal_route(rv, H, head_begin, heads, tile_begin, tiles, B, s);
    } else if (method == FPX_METHOD_FP_V1 || method == FPX_METHOD_MEAN_NATIVE || is_rescue_method(method)) {
      // V1 routing (attention.py:25); mean_native and the rescue tails also use the fp32 means
      rc = launch_block_stats(st, tile_end, kv_count, B, true, method != FPX_METHOD_FP_V1, s);
      if (rc) return rc;
      V1Params vp{};
      vp.q = qb; vp.q_sb = q_sb; vp.q_sl = q_sl; vp.q_sh = q_sh;
      vp.mean_k = ws.mk16; vp.L = L; vp.nb = nb; vp.H = H; vp.Hkv = Hkv; vp.group = G;
      vp.head_begin = head_begin; vp.tile_begin = tile_begin;
      vp.scale_log2 = (float)scale * kLog2e;
      vp.scores = nullptr; vp.sel = sel; vp.d = d;
      rc = launch_v1_route_selected(vp, tiles, heads, B, s);
    } else {
      rc = launch_block_stats(st, tile_end, kv_count, B, false, true, s);
      if (rc) return rc;
      if (alpha == 0.0) {
        rc = launch_causal_route(rv, H, head_begin, heads, tile_begin, tiles, B, s);
      } else {
        SelParams sp{};
        sp.q = qb; sp.q_sb = q_sb; sp.q_sl = q_sl; sp.q_sh = q_sh;
        sp.mean_k = ws.mk; sp.var_k = ws.vk; sp.sigma_v = ws.sv;
        sp.L = L; sp.nb = nb; sp.H = H; sp.Hkv = Hkv; sp.group = G;
        sp.head_begin = head_begin; sp.tile_begin = tile_begin;
        sp.scale = (float)scale; sp.scale2 = (float)(scale * scale);
        sp.scores = nullptr; sp.sel = sel;
        sp.mk_hi = ws.mkh; sp.mk_lo = ws.mkl; sp.vk_hi = ws.vkh; sp.vk_lo = ws.vkl;
        sp.d = d;
        // The tensor-core selector kernel is written for head dim 128; 256 takes the fp32 one.
        rc = (get_option(kOptSelectorKernel) == kSelectorKernelFp32 || d == 256)
                 ? launch_selector_route(sp, method, tiles, heads, B, s)
                 : launch_selector_route_tc(sp, method, tiles, heads, B, s);
      }
    }
    if (rc) return rc;
  }
  if (stages & FPX_STAGE_EXACT) {
    ExactParams ep{};
    ep.q = qb; ep.k = kb; ep.v = vb;
    ep.q_sb = q_sb; ep.q_sl = q_sl; ep.q_sh = q_sh;
    ep.k_sb = k_sb; ep.k_sl = k_sl; ep.k_sh = k_sh;
    ep.v_sb = v_sb; ep.v_sl = v_sl; ep.v_sh = v_sh;
    ep.out = static_cast<__nv_bfloat16 *>(out); ep.o_sb = o_sb; ep.o_sl = o_sl; ep.o_sh = o_sh;
    ep.lse = lse_out; ep.L = L; ep.nb = nb; ep.H = H; ep.group = G;
    ep.head_begin = head_begin; ep.tile_begin = tile_begin;
    ep.scale_log2 = (float)scale * kLog2e;
    ep.route = rv;
    const int ek = get_option(kOptExactKernel);
    rc = (d == 256 || ek == kExactKernelTcgen05Single) ? launch_exact_tc1(ep, d, B, L, Hkv, tiles, heads, s)
         : ek == kExactKernelMmaSync ? launch_exact_mma(ep, kExactLists, tiles, heads, B, s)
                                     : launch_exact_tc(ep, B, L, Hkv, tiles, heads, s);
    if (rc) return rc;
  }
  if ((stages & FPX_STAGE_MEAN) && is_mean_method(method)) {
    MeanParams mp{};
    mp.q = qb; mp.q_sb = q_sb; mp.q_sl = q_sl; mp.q_sh = q_sh;
    mp.mean_k = ws.mk; mp.mean_v = ws.mv;
    mp.mk_hi = ws.mkh; mp.mk_lo = ws.mkl; mp.mv_hi = ws.mvh;
    mp.L = L; mp.nb = nb; mp.H = H; mp.Hkv = Hkv; mp.group = G;
    mp.head_begin = head_begin; mp.tile_begin = tile_begin;
    mp.scale = (float)scale; mp.route = rv;
    mp.out = static_cast<__nv_bfloat16 *>(out); mp.o_sb = o_sb; mp.o_sl = o_sl; mp.o_sh = o_sh;
    mp.lse = lse_out; mp.d = d;
    // The tensor-core tail is written for head dim 128; head dim 256 takes the fp32 tail.
    rc = (get_option(kOptMeanKernel) == kMeanKernelFp32 || d == 256)
             ? launch_mean_tail(mp, kMeanMergeInPlace, tiles, heads, B, s)
             : launch_mean_tail_tc(mp, B, tiles, heads, s);
  }
  if ((stages & FPX_STAGE_MEAN) && is_rescue_method(method)) {
    // attention.py:306-331: rescue tail (kernels.py:233-309), merged in place like the mean tail
    MeanParams mp{};
    mp.q = qb; mp.q_sb = q_sb; mp.q_sl = q_sl; mp.q_sh = q_sh;
    mp.k = kb; mp.k_sb = k_sb; mp.k_sl = k_sl; mp.k_sh = k_sh;
    mp.v = vb; mp.v_sb = v_sb; mp.v_sl = v_sl; mp.v_sh = v_sh;
    mp.mean_k = ws.mk; mp.mean_v = ws.mv; mp.choice = ws.choice;
    mp.L = L; mp.nb = nb; mp.H = H; mp.Hkv = Hkv; mp.group = G;
    mp.head_begin = head_begin; mp.tile_begin = tile_begin;
    mp.scale = (float)scale; mp.route = rv;
    mp.out = static_cast<__nv_bfloat16 *>(out); mp.o_sb = o_sb; mp.o_sl = o_sl; mp.o_sh = o_sh;
    mp.lse = lse_out; mp.d = d;
    mp.qmean = ws.qmean;
    rc = launch_rescue_choice(mp, kMeanMergeInPlace, tiles, kv_count, B, s);
    if (rc) return rc;
    const int keys = method == FPX_METHOD_FP_V1_RESCUE_V2 ? 2 : 1;
    // The tensor-core rescue tail is written for head dim 128; 256 takes the fp32 tail.
    rc = (get_option(kOptMeanKernel) == kMeanKernelFp32 || d == 256)
             ? launch_mean_tail(mp, kMeanMergeInPlace, tiles, heads, B, s, keys)
             : launch_rescue_tail_tc(mp, keys, B, L, tiles, heads, s);
  }
  return rc;
}

extern "C" int fpx_prefill_export_routing(int method, int B, int L, int H, int Hkv, int d, int block,
                                          const void *workspace, size_t workspace_bytes,
                                          uint8_t *selected, int64_t *indices, int32_t *counts,
                                          fpx_stream_t stream) {
  FPX_BIND(stream);
  (void)method;
  if ((d != kHeadDim && d != 256) || block != kBlock) return FPX_ERR_UNSUPPORTED;
  if (B <= 0 || L <= 0 || H <= 0 || Hkv <= 0 || (!selected && !indices)) return FPX_ERR_INVALID;
  const Workspace ws = carve(const_cast<void *>(workspace), B, L, H, Hkv, d);
  if (!workspace || workspace_bytes < ws.bytes) return FPX_ERR_WORKSPACE;
  const int nb = (L + kBlock - 1) / kBlock;
  RouteView rv{ws.lists, ws.counts, ws.tail, nb, (nb + 31) / 32};
  if (selected && cudaMemsetAsync(selected, 0, (size_t)B * nb * nb * H, stream) != cudaSuccess)
    return FPX_ERR_CUDA;
  return launch_export_routing(rv, H, B, selected, indices, counts, stream);
}

extern "C" int fpx_exact_attention(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                   const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                   const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                                   const int64_t *indices, const int32_t *counts, int B, int L,
                                   int H, int Hkv, int d, int block, double scale, void *out,
                                   float *lse, fpx_stream_t stream) {
  FPX_BIND(stream);
  if ((d != kHeadDim && d != 256) || block != kBlock) return FPX_ERR_UNSUPPORTED;
  if (B <= 0 || L <= 0 || H <= 0 || Hkv <= 0 || !aligned16(q) || !aligned16(k) || !aligned16(v) ||
      !aligned16(out) || !indices || !counts || !lse)
    return FPX_ERR_INVALID;
  if (H % Hkv || !strides_ok(q_sb, q_sl, q_sh) || !strides_ok(k_sb, k_sl, k_sh) ||
      !strides_ok(v_sb, v_sl, v_sh))
    return FPX_ERR_SHAPE;
  const int nb = (L + kBlock - 1) / kBlock;
  ExactParams ep{};
  ep.q = static_cast<const __nv_bfloat16 *>(q);
  ep.k = static_cast<const __nv_bfloat16 *>(k);
  ep.v = static_cast<const __nv_bfloat16 *>(v);
  ep.q_sb = q_sb; ep.q_sl = q_sl; ep.q_sh = q_sh;
  ep.k_sb = k_sb; ep.k_sl = k_sl; ep.k_sh = k_sh;
  ep.v_sb = v_sb; ep.v_sl = v_sl; ep.v_sh = v_sh;
  ep.out = static_cast<__nv_bfloat16 *>(out);
  ep.o_sb = (int64_t)L * H * d; ep.o_sl = (int64_t)H * d; ep.o_sh = d;
  ep.lse = lse; ep.L = L; ep.nb = nb; ep.H = H; ep.group = H / Hkv;
  ep.head_begin = 0; ep.tile_begin = 0;
  ep.scale_log2 = (float)scale * kLog2e;
  ep.ref_indices = indices; ep.ref_counts = counts;
  if (d == 256 || get_option(kOptExactKernel) == kExactKernelTcgen05Single)
    return launch_exact_tc1(ep, d, B, L, Hkv, nb, H, stream);
  return get_option(kOptExactKernel) == kExactKernelMmaSync ? launch_exact_mma(ep, kExactRefLayout, nb, H, B, stream)
                                                            : launch_exact_tc(ep, B, L, Hkv, nb, H, stream);
}

extern "C" int fpx_mean_tail(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                             const float *mean_k, const float *mean_v, const int32_t *counts,
                             const uint8_t *selected, int B, int L, int H, int Hkv, int d,
                             int block, double scale, float *out, float *lse,
                             fpx_stream_t stream) {
  FPX_BIND(stream);
  (void)counts;  // n_kb follows from L
  if ((d != kHeadDim && d != 256) || block != kBlock) return FPX_ERR_UNSUPPORTED;
  if (B <= 0 || L <= 0 || H <= 0 || Hkv <= 0 || !aligned16(q) || !aligned16(mean_k) ||
      !aligned16(mean_v) || !selected || !aligned16(out) || !lse)
    return FPX_ERR_INVALID;
  if (H % Hkv || !strides_ok(q_sb, q_sl, q_sh)) return FPX_ERR_SHAPE;
  MeanParams mp{};
  mp.q = static_cast<const __nv_bfloat16 *>(q);
  mp.q_sb = q_sb; mp.q_sl = q_sl; mp.q_sh = q_sh;
  mp.mean_k = mean_k; mp.mean_v = mean_v;
  mp.L = L; mp.nb = (L + kBlock - 1) / kBlock; mp.H = H; mp.Hkv = Hkv; mp.group = H / Hkv;
  mp.head_begin = 0; mp.tile_begin = 0; mp.scale = (float)scale;
  mp.mask = selected; mp.mean_out = out; mp.mean_lse = lse; mp.d = d;
  return launch_mean_tail(mp, kMeanStandalone, mp.nb, H, B, stream);
}

namespace fpx {
struct RescueWorkspace {
  uint8_t *choice;
  float *mk, *mv, *vk, *sv;
  size_t bytes;
};
static RescueWorkspace carve_rescue(void *base, int B, int L, int H, int Hkv, int d = kHeadDim) {
  const int64_t nb = (L + kBlock - 1) / kBlock;
  const size_t desc = (size_t)B * nb * Hkv * d;
  RescueWorkspace w{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t *p = base ? static_cast<uint8_t *>(base) + off : nullptr;
    off += align256(bytes);
    return p;
  };
  w.choice = take((size_t)B * H * nb * nb);
  w.mk = reinterpret_cast<float *>(take(desc * 4));
  w.mv = reinterpret_cast<float *>(take(desc * 4));
  w.vk = reinterpret_cast<float *>(take(desc * 4));
  w.sv = reinterpret_cast<float *>(take((size_t)B * nb * Hkv * 4));
  w.bytes = off;
  return w;
}
}  // namespace fpx

extern "C" size_t fpx_rescue_tail_workspace_bytes(int B, int L, int H, int Hkv, int d, int block) {
  if ((d != kHeadDim && d != 256) || block != kBlock || B <= 0 || L <= 0 || H <= 0 || Hkv <= 0) return 0;
  return carve_rescue(nullptr, B, L, H, Hkv, d).bytes;
}

extern "C" int fpx_rescue_tail(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                               const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                               const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                               const uint8_t *selected, int B, int L, int H, int Hkv, int d, int block,
                               double scale, int remainder, float *out, float *lse, void *workspace,
                               size_t workspace_bytes, fpx_stream_t stream) {
  FPX_BIND(stream);
  if ((d != kHeadDim && d != 256) || block != kBlock) return FPX_ERR_UNSUPPORTED;
  if (B <= 0 || L <= 0 || H <= 0 || Hkv <= 0 || !aligned16(q) || !aligned16(k) || !aligned16(v) ||
      !selected || !aligned16(out) || !lse)
    return FPX_ERR_INVALID;
  if (H % Hkv || !strides_ok(q_sb, q_sl, q_sh) || !strides_ok(k_sb, k_sl, k_sh) || !strides_ok(v_sb, v_sl, v_sh))
    return FPX_ERR_SHAPE;
  const RescueWorkspace ws = carve_rescue(workspace, B, L, H, Hkv, d);
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255) || workspace_bytes < ws.bytes)
    return FPX_ERR_WORKSPACE;
  const int nb = (L + kBlock - 1) / kBlock;
  StatsParams st{};
  st.k = static_cast<const __nv_bfloat16 *>(k); st.k_sb = k_sb; st.k_sl = k_sl; st.k_sh = k_sh;
  st.v = static_cast<const __nv_bfloat16 *>(v); st.v_sb = v_sb; st.v_sl = v_sl; st.v_sh = v_sh;
  st.L = L; st.nb = nb; st.Hkv = Hkv; st.kv_begin = 0; st.d = d;
  st.mean_k = ws.mk; st.mean_v = ws.mv; st.var_k = ws.vk; st.sigma_v = ws.sv;
  int rc = launch_block_stats(st, nb, Hkv, B, false, true, stream);
  if (rc) return rc;
  MeanParams mp{};
  mp.q = static_cast<const __nv_bfloat16 *>(q); mp.q_sb = q_sb; mp.q_sl = q_sl; mp.q_sh = q_sh;
  mp.k = st.k; mp.k_sb = k_sb; mp.k_sl = k_sl; mp.k_sh = k_sh;
  mp.v = st.v; mp.v_sb = v_sb; mp.v_sl = v_sl; mp.v_sh = v_sh;
  mp.mean_k = ws.mk; mp.mean_v = ws.mv; mp.choice = ws.choice;
  mp.L = L; mp.nb = nb; mp.H = H; mp.Hkv = Hkv; mp.group = H / Hkv;
  mp.head_begin = 0; mp.tile_begin = 0; mp.scale = (float)scale;
  mp.mask = selected; mp.mean_out = out; mp.mean_lse = lse; mp.d = d;
  rc = launch_rescue_choice(mp, kMeanStandalone, nb, Hkv, B, stream);
  if (rc) return rc;
  return launch_mean_tail(mp, kMeanStandalone, nb, H, B, stream, remainder ? 2 : 1);
}

extern "C" int fpx_merge_exact_mean(const void *exact_out, const float *exact_lse,
                                    const float *mean_out, const float *mean_lse, int64_t rows,
                                    int d, void *out, float *lse, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (d != kHeadDim && d != 256) return FPX_ERR_UNSUPPORTED;
  if (rows < 0 || !aligned16(exact_out) || !exact_lse || !aligned16(mean_out) || !mean_lse ||
      !aligned16(out) || !lse)
    return FPX_ERR_INVALID;
  return launch_merge(static_cast<const __nv_bfloat16 *>(exact_out), exact_lse, mean_out, mean_lse,
                      rows, static_cast<__nv_bfloat16 *>(out), lse, stream, d);
}
