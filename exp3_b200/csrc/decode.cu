// Dense decode attention (q_len != k_len): every query row attends to all S cached keys,
// as the reference's decode call of F.scaled_dot_product_attention(is_causal=False,
// enable_gqa=True) does (attention.py:178-189).
//
// Split-K flash decode. Pass 1: one CTA per (key split, KV head, batch x query row) streams
// its keys 64 at a time through a two-stage cp.async pipeline in shared memory, scores them
// for all G query heads of the KV group (each K/V row is read once for the whole group), keeps
// an online softmax per head and writes a partial (o, m, l) per split. Pass 2 merges the
// splits into bf16 O and a natural-log LSE.
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
  const int32_t *S_dev;  // if set, the number of keys is read here (S is then the capacity)
  float scale_log2;
  float *part_o;  // [B*Lq][H][splits][128]
  float *part_ml; // [B*Lq][H][splits][2]
};

constexpr int kDecodeChunk = 64;   // keys per pipeline stage
constexpr int kDecodeKPad = 136;   // bf16 per staged K row (272 B: rows start on distinct banks)
constexpr int kMaxSplits = 1024;

struct DecodeSmem {
  __nv_bfloat16 k[2][kDecodeChunk][kDecodeKPad];
  __nv_bfloat16 v[2][kDecodeChunk][kHeadDim];
  float qs[kMaxGroup][kHeadDim];
  float ss[kMaxGroup][kDecodeChunk];
  float mrow[kMaxGroup], lrow[kMaxGroup], corr[kMaxGroup];
};

__global__ void __launch_bounds__(128) decode_split_kernel(DecodeParams p) {
  const int split = blockIdx.x, kvh = blockIdx.y, bq = blockIdx.z;
  const int b = bq / p.Lq, row = bq % p.Lq;
  const int G = p.group, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  DecodeSmem &sh = *reinterpret_cast<DecodeSmem *>(smem_raw);
  for (int i = tid; i < G * kHeadDim; i += 128) {
    const int g = i / kHeadDim, c = i % kHeadDim;
    const int h = kvh * G + g;
    sh.qs[g][c] = __bfloat162float(p.q[b * p.q_sb + (int64_t)row * p.q_sl + h * p.q_sh + c]) * p.scale_log2;
  }
  if (tid < G) { sh.mrow[tid] = -INFINITY; sh.lrow[tid] = 0.f; }
  float o[kMaxGroup];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) o[g] = 0.f;
  const int S = p.S_dev ? min(*p.S_dev, p.S) : p.S;
  const int k0 = split * p.keys_per_split;
  const int k1 = min(S, k0 + p.keys_per_split);
  const int chunks = k1 > k0 ? (k1 - k0 + kDecodeChunk - 1) / kDecodeChunk : 0;
  const __nv_bfloat16 *kbase = p.k + b * p.k_sb + kvh * p.k_sh;
  const __nv_bfloat16 *vbase = p.v + b * p.v_sb + kvh * p.v_sh;
  // Stage chunk c's K and V rows (16-byte cp.async, rows past k1 zero-filled).
  auto stage = [&](int c) {
    const int st = c & 1, base = k0 + c * kDecodeChunk;
    for (int i = tid; i < kDecodeChunk * 16; i += 128) {
      const int r = i >> 4, ch = i & 15;
      const bool ok = base + r < k1;
      const int64_t key = ok ? base + r : k0;
      cp_async16(&sh.k[st][r][8 * ch], kbase + key * p.k_sl + 8 * ch, ok);
      cp_async16(&sh.v[st][r][8 * ch], vbase + key * p.v_sl + 8 * ch, ok);
    }
    cp_async_commit();
  };
  if (chunks > 0) stage(0);
  __syncthreads();
  for (int c = 0; c < chunks; ++c) {
    const int st = c & 1;
    const int n = min(kDecodeChunk, k1 - (k0 + c * kDecodeChunk));
    if (c + 1 < chunks) {
      stage(c + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // Scores: two threads per key, each over 64 dimensions, halves joined by a shuffle.
    {
      const int j = tid >> 1, half = tid & 1;
      float acc[kMaxGroup];
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) acc[g] = 0.f;
      const uint4 *kr = reinterpret_cast<const uint4 *>(&sh.k[st][j][64 * half]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 u = kr[i];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 kv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[e]));
          const int col = 64 * half + 8 * i + 2 * e;
#pragma unroll
          for (int g = 0; g < kMaxGroup; ++g)
            if (g < G) acc[g] = fmaf(sh.qs[g][col], kv.x, fmaf(sh.qs[g][col + 1], kv.y, acc[g]));
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g < G) {
          const float tot = acc[g] + __shfl_xor_sync(0xffffffffu, acc[g], 1);
          if (half == 0) sh.ss[g][j] = j < n ? tot : -INFINITY;
        }
      }
    }
    __syncthreads();
    // Online softmax per head: warp w owns heads w, w + 4, ...; lane covers keys lane, lane + 32.
    for (int g = warp; g < G; g += 4) {
      const float a = sh.ss[g][lane], bb = sh.ss[g][lane + 32];
      const float m = warp_max(fmaxf(a, bb));
      const float mn = fmaxf(sh.mrow[g], m);
      const float ea = a == -INFINITY ? 0.f : exp2f(a - mn), eb = bb == -INFINITY ? 0.f : exp2f(bb - mn);
      sh.ss[g][lane] = ea;
      sh.ss[g][lane + 32] = eb;
      const float l = warp_sum(ea + eb);
      if (lane == 0) {
        const float cr = sh.mrow[g] == -INFINITY ? 0.f : exp2f(sh.mrow[g] - mn);
        sh.corr[g] = cr;
        sh.lrow[g] = sh.lrow[g] * cr + l;
        sh.mrow[g] = mn;
      }
    }
    __syncthreads();
    // O += P V: thread = output dimension.
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g)
      if (g < G) o[g] *= sh.corr[g];
#pragma unroll 8
    for (int j = 0; j < kDecodeChunk; ++j) {
      const float vv = __bfloat162float(sh.v[st][j][tid]);
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g)
        if (g < G) o[g] = fmaf(sh.ss[g][j], vv, o[g]);
    }
    __syncthreads();  // stage st is refilled by the next iteration's prefetch
  }
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g >= G) break;
    const int h = kvh * G + g;
    const int64_t slot = ((int64_t)bq * p.H + h) * p.splits + split;
    p.part_o[slot * kHeadDim + tid] = o[g];
    if (tid == 0) {
      p.part_ml[2 * slot] = sh.mrow[g];
      p.part_ml[2 * slot + 1] = sh.lrow[g];
    }
  }
}

__global__ void __launch_bounds__(128) decode_combine_kernel(DecodeParams p) {
  const int h = blockIdx.x, bq = blockIdx.y;
  const int b = bq / p.Lq, row = bq % p.Lq;
  const int64_t base = ((int64_t)bq * p.H + h) * p.splits;
  __shared__ float w[kMaxSplits];
  __shared__ float red[4];
  float m = -INFINITY;
  for (int s = threadIdx.x; s < p.splits; s += 128) m = fmaxf(m, p.part_ml[2 * (base + s)]);
  m = block_max<128>(m, red);
  float l = 0.f;
  for (int s = threadIdx.x; s < p.splits; s += 128) {
    const float ms = p.part_ml[2 * (base + s)];
    const float ws = ms == -INFINITY ? 0.f : exp2f(ms - m);
    w[s] = ws;
    l += p.part_ml[2 * (base + s) + 1] * ws;
  }
  l = block_sum<128>(l, red);  // its barriers also publish w[]
  float o0 = 0.f, o1 = 0.f;
  int s = 0;
  for (; s + 1 < p.splits; s += 2) {
    o0 += p.part_o[(base + s) * kHeadDim + threadIdx.x] * w[s];
    o1 += p.part_o[(base + s + 1) * kHeadDim + threadIdx.x] * w[s + 1];
  }
  if (s < p.splits) o0 += p.part_o[(base + s) * kHeadDim + threadIdx.x] * w[s];
  const float o = o0 + o1;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  p.out[b * p.o_sb + (int64_t)row * p.o_sl + h * p.o_sh + threadIdx.x] = __float2bfloat16_rn(o * inv);
  if (p.lse && threadIdx.x == 0)
    p.lse[((int64_t)b * p.Lq + row) * p.H + h] = l > 0.f ? m * kLn2 + logf(l) : -INFINITY;
}

// Both decode kernels with the pipeline's shared memory.
static int decode_launch(const DecodeParams &p, int B, int Hkv, cudaStream_t stream) {
  if (p.splits > kMaxSplits) return FPX_ERR_UNSUPPORTED;
  const int smem = (int)sizeof(DecodeSmem);
  cudaFuncSetAttribute(decode_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  decode_split_kernel<<<dim3(p.splits, Hkv, B * p.Lq), 128, smem, stream>>>(p);
  FPX_CHECK_LAUNCH();
  decode_combine_kernel<<<dim3(p.H, B * p.Lq), 128, 0, stream>>>(p);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
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

static int decode_run(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh, const void *k, int64_t k_sb,
                      int64_t k_sl, int64_t k_sh, const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh, int B,
                      int Lq, int S, const int32_t *S_dev, int H, int Hkv, int d, double scale, void *out,
                      int64_t o_sb, int64_t o_sl, int64_t o_sh, float *lse, void *workspace,
                      size_t workspace_bytes, cudaStream_t stream) {
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
  p.lse = lse; p.Lq = Lq; p.S = S; p.S_dev = S_dev; p.H = H; p.Hkv = Hkv; p.group = H / Hkv;
  p.splits = decode_splits(B, Lq, Hkv, S);
  p.keys_per_split = (((S + p.splits - 1) / p.splits) + kDecodeKeys - 1) / kDecodeKeys * kDecodeKeys;
  p.splits = (S + p.keys_per_split - 1) / p.keys_per_split;
  p.scale_log2 = (float)scale * kLog2e;
  p.part_o = static_cast<float *>(workspace);
  p.part_ml = p.part_o + (size_t)B * Lq * H * p.splits * kHeadDim;
  return decode_launch(p, B, Hkv, stream);
}

extern "C" int fpx_decode_attention(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                    const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                    const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                                    int B, int Lq, int S, int H, int Hkv, int d, double scale,
                                    void *out, int64_t o_sb, int64_t o_sl, int64_t o_sh, float *lse,
                                    void *workspace, size_t workspace_bytes, fpx_stream_t stream) {
  FPX_BIND(stream);
  return decode_run(q, q_sb, q_sl, q_sh, k, k_sb, k_sl, k_sh, v, v_sb, v_sl, v_sh, B, Lq, S, nullptr, H, Hkv, d,
                    scale, out, o_sb, o_sl, o_sh, lse, workspace, workspace_bytes, stream);
}

// The key count is read from device memory (S_keys, at most S_max), so one launch sequence
// serves every step of a captured decode graph; the split layout follows S_max.
extern "C" int fpx_decode_attention_at(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                       const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                       const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                                       int B, int Lq, int S_max, const int32_t *S_keys, int H, int Hkv, int d,
                                       double scale, void *out, int64_t o_sb, int64_t o_sl, int64_t o_sh,
                                       float *lse, void *workspace, size_t workspace_bytes,
                                       fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!S_keys) return FPX_ERR_INVALID;
  return decode_run(q, q_sb, q_sl, q_sh, k, k_sb, k_sl, k_sh, v, v_sb, v_sl, v_sh, B, Lq, S_max, S_keys, H, Hkv,
                    d, scale, out, o_sb, o_sl, o_sh, lse, workspace, workspace_bytes, stream);
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
  return decode_launch(p, B, Hkv, stream);
}
