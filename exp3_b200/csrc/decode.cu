// Dense decode attention (q_len != k_len): every query row attends to all S cached keys,
// as the reference's decode call of F.scaled_dot_product_attention(is_causal=False,
// enable_gqa=True) does (attention.py:178-189).
//
// Split-K flash decode. Pass 1: one CTA per (key split, KV head, batch x query row)
// scores 128 keys at a time for all G query heads of the KV group (each K/V row is read
// once for the whole group), keeps an online softmax per head and writes a partial
// (o, m, l) per split. Pass 2 merges the splits into bf16 O and a natural-log LSE.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace fpx {

constexpr int kDecodeKeys = 128;
constexpr int kMaxGroup = 16;

struct DecodeParams {
  const __nv_bfloat16 *q, *k, *v;
  int64_t q_sb, q_sl, q_sh, k_sb, k_sl, k_sh, v_sb, v_sl, v_sh;
  __nv_bfloat16 *out;
  int64_t o_sb, o_sl, o_sh;
  float *lse;  // [B][Lq][H] or null
  int Lq, S, H, Hkv, group, splits, keys_per_split;
  float scale_log2;
  float *part_o;  // [B*Lq][H][splits][128]
  float *part_ml; // [B*Lq][H][splits][2]
};

__global__ void __launch_bounds__(128) decode_split_kernel(DecodeParams p) {
  const int split = blockIdx.x, kvh = blockIdx.y, bq = blockIdx.z;
  const int b = bq / p.Lq, row = bq % p.Lq;
  const int G = p.group, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __shared__ __align__(16) float qs[kMaxGroup][kHeadDim];
  __shared__ float ss[kMaxGroup][kDecodeKeys];
  __shared__ float mrow[kMaxGroup], lrow[kMaxGroup], corr[kMaxGroup];
  for (int i = tid; i < G * kHeadDim; i += 128) {
    const int g = i / kHeadDim, c = i % kHeadDim;
    const int h = kvh * G + g;
    qs[g][c] = __bfloat162float(p.q[b * p.q_sb + (int64_t)row * p.q_sl + h * p.q_sh + c]) * p.scale_log2;
  }
  if (tid < G) { mrow[tid] = -INFINITY; lrow[tid] = 0.f; }
  float o[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) o[g] = 0.f;
  const int k0 = split * p.keys_per_split;
  const int k1 = min(p.S, k0 + p.keys_per_split);
  const __nv_bfloat16 *kbase = p.k + b * p.k_sb + kvh * p.k_sh;
  const __nv_bfloat16 *vbase = p.v + b * p.v_sb + kvh * p.v_sh;
  __syncthreads();
  for (int c0 = k0; c0 < k1; c0 += kDecodeKeys) {
    const int n = min(kDecodeKeys, k1 - c0);
    // Scores: thread j takes key c0 + j.
    if (tid < n) {
      const uint4 *kr = reinterpret_cast<const uint4 *>(kbase + (int64_t)(c0 + tid) * p.k_sl);
      float acc[kMaxGroup];
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) acc[g] = 0.f;
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const uint4 u = kr[i];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[e]));
          const int c = 8 * i + 2 * e;
#pragma unroll
          for (int g = 0; g < kMaxGroup; ++g)
            if (g < G) acc[g] = fmaf(qs[g][c], kv.x, fmaf(qs[g][c + 1], kv.y, acc[g]));
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g)
        if (g < G) ss[g][tid] = acc[g];
    }
    __syncthreads();
    // Online softmax per head: warp w owns heads w, w+4, ...
    for (int g = warp; g < G; g += 4) {
      float m = -INFINITY;
      for (int j = lane; j < n; j += 32) m = fmaxf(m, ss[g][j]);
      m = warp_max(m);
      const float mn = fmaxf(mrow[g], m);
      float l = 0.f;
      for (int j = lane; j < n; j += 32) {
        const float e = exp2f(ss[g][j] - mn);
        ss[g][j] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        const float c = mrow[g] == -INFINITY ? 0.f : exp2f(mrow[g] - mn);
        corr[g] = c;
        lrow[g] = lrow[g] * c + l;
        mrow[g] = mn;
      }
    }
    __syncthreads();
    // O += P V: thread = output dimension.
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g)
      if (g < G) o[g] *= corr[g];
    for (int j = 0; j < n; ++j) {
      const float vv = __bfloat162float(vbase[(int64_t)(c0 + j) * p.v_sl + tid]);
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g)
        if (g < G) o[g] = fmaf(ss[g][j], vv, o[g]);
    }
    __syncthreads();
  }
  for (int g = 0; g < G; ++g) {
    const int h = kvh * G + g;
    const int64_t slot = ((int64_t)bq * p.H + h) * p.splits + split;
    p.part_o[slot * kHeadDim + tid] = o[g];
    if (tid == 0) {
      p.part_ml[2 * slot] = mrow[g];
      p.part_ml[2 * slot + 1] = lrow[g];
    }
  }
}

__global__ void __launch_bounds__(128) decode_combine_kernel(DecodeParams p) {
  const int h = blockIdx.x, bq = blockIdx.y;
  const int b = bq / p.Lq, row = bq % p.Lq;
  const int64_t base = ((int64_t)bq * p.H + h) * p.splits;
  float m = -INFINITY;
  for (int s = 0; s < p.splits; ++s) m = fmaxf(m, p.part_ml[2 * (base + s)]);
  float l = 0.f, o = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const float ms = p.part_ml[2 * (base + s)];
    if (ms == -INFINITY) continue;
    const float w = exp2f(ms - m);
    l += p.part_ml[2 * (base + s) + 1] * w;
    o += p.part_o[(base + s) * kHeadDim + threadIdx.x] * w;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  p.out[b * p.o_sb + (int64_t)row * p.o_sl + h * p.o_sh + threadIdx.x] = __float2bfloat16_rn(o * inv);
  if (p.lse && threadIdx.x == 0)
    p.lse[((int64_t)b * p.Lq + row) * p.H + h] = l > 0.f ? m * kLn2 + logf(l) : -INFINITY;
}

static int decode_splits(int B, int Lq, int Hkv, int S) {
  const int units = B * Lq * Hkv;
  const int want = (2 * 148 + units - 1) / units;
  const int most = (S + kDecodeKeys - 1) / kDecodeKeys;
  return std::max(1, std::min(want, most));
}

}  // namespace fpx

using namespace fpx;

extern "C" size_t fpx_decode_workspace_bytes(int B, int Lq, int H, int Hkv, int S, int d) {
  if (B <= 0 || Lq <= 0 || H <= 0 || Hkv <= 0 || S <= 0 || d != kHeadDim) return 0;
  const size_t splits = decode_splits(B, Lq, Hkv, S);
  return (size_t)B * Lq * H * splits * (kHeadDim + 2) * sizeof(float);
}

extern "C" int fpx_decode_attention(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                    const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                    const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                                    int B, int Lq, int S, int H, int Hkv, int d, double scale,
                                    void *out, int64_t o_sb, int64_t o_sl, int64_t o_sh, float *lse,
                                    void *workspace, size_t workspace_bytes, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (d != kHeadDim) return FPX_ERR_UNSUPPORTED;
  if (!q || !k || !v || !out || B <= 0 || Lq <= 0 || S <= 0 || H <= 0 || Hkv <= 0)
    return FPX_ERR_INVALID;
  if (H % Hkv || H / Hkv > kMaxGroup || k_sl % 8 || k_sb % 8 || k_sh % 8 ||
      (reinterpret_cast<uintptr_t>(k) & 15))
    return FPX_ERR_SHAPE;
  const size_t need = fpx_decode_workspace_bytes(B, Lq, H, Hkv, S, d);
  if (!workspace || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return FPX_ERR_WORKSPACE;
  DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16 *>(q);
  p.k = static_cast<const __nv_bfloat16 *>(k);
  p.v = static_cast<const __nv_bfloat16 *>(v);
  p.q_sb = q_sb; p.q_sl = q_sl; p.q_sh = q_sh;
  p.k_sb = k_sb; p.k_sl = k_sl; p.k_sh = k_sh;
  p.v_sb = v_sb; p.v_sl = v_sl; p.v_sh = v_sh;
  p.out = static_cast<__nv_bfloat16 *>(out); p.o_sb = o_sb; p.o_sl = o_sl; p.o_sh = o_sh;
  p.lse = lse; p.Lq = Lq; p.S = S; p.H = H; p.Hkv = Hkv; p.group = H / Hkv;
  p.splits = decode_splits(B, Lq, Hkv, S);
  p.keys_per_split = (((S + p.splits - 1) / p.splits) + kDecodeKeys - 1) / kDecodeKeys * kDecodeKeys;
  p.splits = (S + p.keys_per_split - 1) / p.keys_per_split;
  p.scale_log2 = (float)scale * kLog2e;
  p.part_o = static_cast<float *>(workspace);
  p.part_ml = p.part_o + (size_t)B * Lq * H * p.splits * kHeadDim;
  decode_split_kernel<<<dim3(p.splits, Hkv, B * Lq), 128, 0, stream>>>(p);
  FPX_CHECK_LAUNCH();
  decode_combine_kernel<<<dim3(H, B * Lq), 128, 0, stream>>>(p);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

// ---------------------------------------------------------------------------------------------
// Decode with no workspace argument and no allocation.
//
// Some callers cannot allocate device memory at the moment they decode: an inference engine
// that only hands out memory from its own pre-sized pool, a plug-in invoked from inside another
// runtime's step where calling the CUDA allocator is forbidden, or a C caller with no allocator
// at all. For them this entry point keeps the split-K partials in one fixed array compiled into
// the library (kDecodeScratchBytes per device, present on every GPU that loads the library
// until the process exits) instead of a caller-provided workspace.
//
// The first call on a device looks up the array's device address with cudaGetSymbolAddress (the
// array's name in host code is only a host-side stand-in, not a device address); make that
// first call before any stream capture. Every call shares the one array and it keeps the last
// call's contents: each call writes every partial it later reads, so nothing has to start at
// zero, but calls that overlap on the GPU (different streams, no ordering) race on the array.
namespace fpx {

constexpr size_t kDecodeScratchBytes = FPX_DECODE_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_decode_scratch[kDecodeScratchBytes];

static std::mutex g_decode_scratch_mutex;
static void *g_decode_scratch_address[64];

// Device address of g_decode_scratch on the current device (looked up once per device).
static int decode_scratch_address(void **out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return FPX_ERR_CUDA;
  if (dev < 0 || dev >= 64) return FPX_ERR_INVALID;
  std::lock_guard<std::mutex> lock(g_decode_scratch_mutex);
  if (!g_decode_scratch_address[dev]) {
    void *addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_decode_scratch) != cudaSuccess || !addr) return FPX_ERR_CUDA;
    g_decode_scratch_address[dev] = addr;
  }
  *out = g_decode_scratch_address[dev];
  return FPX_OK;
}

}  // namespace fpx

extern "C" int fpx_decode_attention_noalloc(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                            const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                            const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                                            int B, int Lq, int S, int H, int Hkv, int d, double scale,
                                            void *out, int64_t o_sb, int64_t o_sl, int64_t o_sh,
                                            float *lse, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (d != kHeadDim) return FPX_ERR_UNSUPPORTED;
  if (!q || !k || !v || !out || B <= 0 || Lq <= 0 || S <= 0 || H <= 0 || Hkv <= 0)
    return FPX_ERR_INVALID;
  if (H % Hkv || H / Hkv > kMaxGroup || k_sl % 8 || k_sb % 8 || k_sh % 8 ||
      (reinterpret_cast<uintptr_t>(k) & 15))
    return FPX_ERR_SHAPE;
  // Sizes whose partials do not fit the fixed array are refused before anything runs.
  if (fpx_decode_workspace_bytes(B, Lq, H, Hkv, S, d) > kDecodeScratchBytes) return FPX_ERR_WORKSPACE;
  void *scratch = nullptr;
  const int rc = decode_scratch_address(&scratch);
  if (rc != FPX_OK) return rc;
  DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16 *>(q);
  p.k = static_cast<const __nv_bfloat16 *>(k);
  p.v = static_cast<const __nv_bfloat16 *>(v);
  p.q_sb = q_sb; p.q_sl = q_sl; p.q_sh = q_sh;
  p.k_sb = k_sb; p.k_sl = k_sl; p.k_sh = k_sh;
  p.v_sb = v_sb; p.v_sl = v_sl; p.v_sh = v_sh;
  p.out = static_cast<__nv_bfloat16 *>(out); p.o_sb = o_sb; p.o_sl = o_sl; p.o_sh = o_sh;
  p.lse = lse; p.Lq = Lq; p.S = S; p.H = H; p.Hkv = Hkv; p.group = H / Hkv;
  p.splits = decode_splits(B, Lq, Hkv, S);
  p.keys_per_split = (((S + p.splits - 1) / p.splits) + kDecodeKeys - 1) / kDecodeKeys * kDecodeKeys;
  p.splits = (S + p.keys_per_split - 1) / p.keys_per_split;
  p.scale_log2 = (float)scale * kLog2e;
  p.part_o = static_cast<float *>(scratch);
  p.part_ml = p.part_o + (size_t)B * Lq * H * p.splits * kHeadDim;
  decode_split_kernel<<<dim3(p.splits, Hkv, B * Lq), 128, 0, stream>>>(p);
  FPX_CHECK_LAUNCH();
  decode_combine_kernel<<<dim3(H, B * Lq), 128, 0, stream>>>(p);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}
