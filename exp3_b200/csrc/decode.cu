// Dense decode attention (q_len != k_len): every query row attends to all S cached keys,
// as the reference's decode call of F.scaled_dot_product_attention(is_causal=False,
// enable_gqa=True) does (attention.py:178-189).
//
// Split-K flash decode. Pass 1: one CTA per (key split, KV head, batch x query row) streams
// its keys 64 at a time through a two-stage cp.async pipeline in shared memory and runs them
// through mma.sync tiles with the G query heads of the KV group as the rows (each K/V row is
// read once for the whole group); every warp keeps an online softmax over its quarter of the
// keys, and the warps' partials are merged into one (o, m, l) per split. Pass 2 merges the
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
  float *part_o;  // [B*Lq][H][splits][d]
  float *part_ml; // [B*Lq][H][splits][2]
};

constexpr int kDecodeChunk = 64;   // keys per pipeline stage: 16 per warp
constexpr int kMaxSplits = 1024;

// XOR-swizzled [rows][D] bf16 tile: 16-byte chunk c of row r lives at chunk c ^ (r & 7).
template <int D>
FPX_INLINE int dswz(int r, int chunk) { return r * D + ((chunk ^ (r & 7)) << 3); }

template <int D>
struct DecodeSmem {
  __nv_bfloat16 q[16 * D];  // the group's query rows (rows >= G zero), swizzled
  union {
    struct {
      __nv_bfloat16 k[2][kDecodeChunk * D];  // swizzled K / V stages
      __nv_bfloat16 v[2][kDecodeChunk * D];
    } stage;
    struct {
      float o[4][16][D];  // each warp's O for the 16 rows
      float m[4][16], l[4][16];
    } merge;
  } u;
};

// Decode on the tensor core (mma.sync m16n8k16, bf16 in, fp32 accumulate): the G query heads of
// the KV group are the M = 16 rows (padded), keys stream 64 per stage through shared memory and
// warp w takes keys 16w..16w+15 of every stage with its own online softmax (exp2 units); P is
// rounded to bf16 for P.V. At the end the four warps' (m, l, O) are merged into the split's
// partial. D is the head dim (128 or 256).
template <int D>
__global__ void __launch_bounds__(128) decode_split_kernel(DecodeParams p) {
  constexpr int kChunks = D / 8;  // 16-byte pieces per row
  const int split = blockIdx.x, kvh = blockIdx.y, bq = blockIdx.z;
  const int b = bq / p.Lq, row = bq % p.Lq;
  const int G = p.group, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g8 = lane >> 2, tq = lane & 3;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  DecodeSmem<D> &sh = *reinterpret_cast<DecodeSmem<D> *>(smem_raw);
  for (int i = tid; i < 16 * kChunks; i += 128) {  // 16 rows x D/8 chunks of 8 bf16
    const int r = i / kChunks, ch = i % kChunks;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < G)
      val = *reinterpret_cast<const uint4 *>(p.q + b * p.q_sb + (int64_t)row * p.q_sl + (kvh * G + r) * p.q_sh + 8 * ch);
    *reinterpret_cast<uint4 *>(&sh.q[dswz<D>(r, ch)]) = val;
  }
  const int S = p.S_dev ? min(*p.S_dev, p.S) : p.S;
  const int k0 = split * p.keys_per_split;
  const int k1 = min(S, k0 + p.keys_per_split);
  const int chunks = k1 > k0 ? (k1 - k0 + kDecodeChunk - 1) / kDecodeChunk : 0;
  const __nv_bfloat16 *kbase = p.k + b * p.k_sb + kvh * p.k_sh;
  const __nv_bfloat16 *vbase = p.v + b * p.v_sb + kvh * p.v_sh;
  auto stage = [&](int c) {
    const int st = c & 1, base = k0 + c * kDecodeChunk;
    for (int i = tid; i < kDecodeChunk * kChunks; i += 128) {
      const int r = i / kChunks, ch = i % kChunks;
      const bool ok = base + r < k1;
      const int64_t key = ok ? base + r : k0;
      cp_async16(&sh.u.stage.k[st][dswz<D>(r, ch)], kbase + key * p.k_sl + 8 * ch, ok);
      cp_async16(&sh.u.stage.v[st][dswz<D>(r, ch)], vbase + key * p.v_sl + 8 * ch, ok);
    }
    cp_async_commit();
  };
  if (chunks > 0) stage(0);
  __syncthreads();
  uint32_t qf[D / 16][4];
  {
    const int m = lane >> 3;
    const int r = ((m & 1) << 3) + (lane & 7);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      ldmatrix_x4(qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], smem_u32(&sh.q[dswz<D>(r, 2 * kk + (m >> 1))]));
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  for (int c = 0; c < chunks; ++c) {
    const int st = c & 1;
    if (c + 1 < chunks) {
      stage(c + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __nv_bfloat16 *ck = sh.u.stage.k[st], *cv = sh.u.stage.v[st];
    const int key0 = k0 + c * kDecodeChunk + 16 * warp;  // this warp's 16 keys
    float sacc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
    for (int kk2 = 0; kk2 < D / 32; ++kk2) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(b0, b1, b2, b3, smem_u32(ck + dswz<D>(16 * warp + 8 * nt + (lane & 7), 4 * kk2 + (lane >> 3))));
        mma_bf16_16816(sacc[nt], qf[2 * kk2], b0, b1);
        mma_bf16_16816(sacc[nt], qf[2 * kk2 + 1], b2, b3);
      }
    }
    float mx[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + 8 * nt + 2 * tq + (e & 1);
        const float x = key < k1 ? sacc[nt][e] * p.scale_log2 : -INFINITY;
        sacc[nt][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      corr[r] = (mrow[r] == -INFINITY) ? (mx[r] == -INFINITY ? 1.f : 0.f) : exp2f(mrow[r] - mx[r]);
      mrow[r] = mx[r];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      float pv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float m = mx[e >> 1];
        pv[e] = (m == -INFINITY) ? 0.f : exp2f(sacc[nt][e] - m);
        rs[e >> 1] += pv[e];
      }
      pa[nt * 2 + 0] = pack_bf16(pv[0], pv[1]);
      pa[nt * 2 + 1] = pack_bf16(pv[2], pv[3]);
    }
    lrow[0] = lrow[0] * corr[0] + rs[0];
    lrow[1] = lrow[1] * corr[1] + rs[1];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= corr[0]; o[i][1] *= corr[0];
      o[i][2] *= corr[1]; o[i][3] *= corr[1];
    }
    const int vr = 16 * warp + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
    for (int dn2 = 0; dn2 < D / 16; ++dn2) {
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4_trans(b0, b1, b2, b3, smem_u32(cv + dswz<D>(vr, 2 * dn2 + (lane >> 4))));
      mma_bf16_16816(o[2 * dn2], pa, b0, b1);
      mma_bf16_16816(o[2 * dn2 + 1], pa, b2, b3);
    }
    __syncthreads();  // stage st is refilled by the next iteration's prefetch
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
    lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
  }
  // Merge the four warps (the staging buffers are free now).
  if (tq == 0) {
    sh.u.merge.m[warp][g8] = mrow[0];
    sh.u.merge.m[warp][g8 + 8] = mrow[1];
    sh.u.merge.l[warp][g8] = lrow[0];
    sh.u.merge.l[warp][g8 + 8] = lrow[1];
  }
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    const int col = 8 * dt + 2 * tq;
    sh.u.merge.o[warp][g8][col] = o[dt][0];
    sh.u.merge.o[warp][g8][col + 1] = o[dt][1];
    sh.u.merge.o[warp][g8 + 8][col] = o[dt][2];
    sh.u.merge.o[warp][g8 + 8][col + 1] = o[dt][3];
  }
  __syncthreads();
  for (int r = 0; r < G; ++r) {
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, sh.u.merge.m[w][r]);
    float ll = 0.f, oo[D / 128] = {};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float mw = sh.u.merge.m[w][r];
      if (mw == -INFINITY) continue;
      const float sc = exp2f(mw - mm);
      ll += sh.u.merge.l[w][r] * sc;
#pragma unroll
      for (int c = 0; c < D / 128; ++c) oo[c] += sh.u.merge.o[w][r][tid + 128 * c] * sc;
    }
    const int h = kvh * G + r;
    const int64_t slot = ((int64_t)bq * p.H + h) * p.splits + split;
#pragma unroll
    for (int c = 0; c < D / 128; ++c) p.part_o[slot * D + tid + 128 * c] = oo[c];
    if (tid == 0) {
      p.part_ml[2 * slot] = mm;
      p.part_ml[2 * slot + 1] = ll;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(D) decode_combine_kernel(DecodeParams p) {
  const int h = blockIdx.x, bq = blockIdx.y;
  const int b = bq / p.Lq, row = bq % p.Lq;
  const int64_t base = ((int64_t)bq * p.H + h) * p.splits;
  __shared__ float w[kMaxSplits];
  __shared__ float red[D / 32];
  float m = -INFINITY;
  for (int s = threadIdx.x; s < p.splits; s += D) m = fmaxf(m, p.part_ml[2 * (base + s)]);
  m = block_max<D>(m, red);
  float l = 0.f;
  for (int s = threadIdx.x; s < p.splits; s += D) {
    const float ms = p.part_ml[2 * (base + s)];
    const float ws = ms == -INFINITY ? 0.f : exp2f(ms - m);
    w[s] = ws;
    l += p.part_ml[2 * (base + s) + 1] * ws;
  }
  l = block_sum<D>(l, red);  // its barriers also publish w[]
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // eight loads in flight
  int s = 0;
  for (; s + 8 <= p.splits; s += 8) {
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] += p.part_o[(base + s + e) * D + threadIdx.x] * w[s + e];
  }
  for (; s < p.splits; ++s) acc[0] += p.part_o[(base + s) * D + threadIdx.x] * w[s];
  const float o = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
  const float inv = l > 0.f ? 1.f / l : 0.f;
  p.out[b * p.o_sb + (int64_t)row * p.o_sl + h * p.o_sh + threadIdx.x] = __float2bfloat16_rn(o * inv);
  if (p.lse && threadIdx.x == 0)
    p.lse[((int64_t)b * p.Lq + row) * p.H + h] = l > 0.f ? m * kLn2 + logf(l) : -INFINITY;
}

// Both decode kernels with the pipeline's shared memory.
template <int D>
static int decode_launch_d(const DecodeParams &p, int B, int Hkv, cudaStream_t stream) {
  const int smem = (int)sizeof(DecodeSmem<D>);
  cudaFuncSetAttribute(decode_split_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  decode_split_kernel<D><<<dim3(p.splits, Hkv, B * p.Lq), 128, smem, stream>>>(p);
  FPX_CHECK_LAUNCH();
  decode_combine_kernel<D><<<dim3(p.H, B * p.Lq), D, 0, stream>>>(p);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

static int decode_launch(const DecodeParams &p, int d, int B, int Hkv, cudaStream_t stream) {
  if (p.splits > kMaxSplits) return FPX_ERR_UNSUPPORTED;
  return d == 256 ? decode_launch_d<256>(p, B, Hkv, stream) : decode_launch_d<kHeadDim>(p, B, Hkv, stream);
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
  if (B <= 0 || Lq <= 0 || H <= 0 || Hkv <= 0 || S <= 0 || (d != kHeadDim && d != 256)) return 0;
  const size_t splits = decode_splits(B, Lq, Hkv, S);
  return (size_t)B * Lq * H * splits * (d + 2) * sizeof(float);
}

static int decode_run(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh, const void *k, int64_t k_sb,
                      int64_t k_sl, int64_t k_sh, const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh, int B,
                      int Lq, int S, const int32_t *S_dev, int H, int Hkv, int d, double scale, void *out,
                      int64_t o_sb, int64_t o_sl, int64_t o_sh, float *lse, void *workspace,
                      size_t workspace_bytes, cudaStream_t stream) {
  if (d != kHeadDim && d != 256) return FPX_ERR_UNSUPPORTED;
  if (!q || !k || !v || !out || B <= 0 || Lq <= 0 || S <= 0 || H <= 0 || Hkv <= 0)
    return FPX_ERR_INVALID;
  // Q, K and V rows move in 16-byte pieces: last dim contiguous, other strides multiples of 8.
  if (H % Hkv || H / Hkv > kMaxGroup || k_sl % 8 || k_sb % 8 || k_sh % 8 || v_sl % 8 || v_sb % 8 ||
      v_sh % 8 || q_sl % 8 || q_sb % 8 || q_sh % 8 || (reinterpret_cast<uintptr_t>(k) & 15) ||
      (reinterpret_cast<uintptr_t>(v) & 15) || (reinterpret_cast<uintptr_t>(q) & 15))
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
  p.part_ml = p.part_o + (size_t)B * Lq * H * p.splits * d;
  return decode_launch(p, d, B, Hkv, stream);
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
// first call before any stream capture. The address is cached per device index for the life of
// the process, so the library must not be used across a cudaDeviceReset (or any other teardown
// of the device's primary context): the cached address would then be stale. Every call shares
// the one array and it keeps the last call's contents: each call writes every partial it later
// reads, so nothing has to start at zero, but calls that overlap on the GPU (different streams,
// no ordering) race on the array.
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
  // Sizes whose partials do not fit the fixed array are refused before anything runs. Invalid
  // arguments size to 0 here and are refused by decode_run's own checks.
  if (fpx_decode_workspace_bytes(B, Lq, H, Hkv, S, d) > kDecodeScratchBytes) return FPX_ERR_WORKSPACE;
  void *scratch = nullptr;
  const int rc = decode_scratch_address(&scratch);
  if (rc != FPX_OK) return rc;
  return decode_run(q, q_sb, q_sl, q_sh, k, k_sb, k_sl, k_sh, v, v_sb, v_sl, v_sh, B, Lq, S, nullptr, H, Hkv, d,
                    scale, out, o_sb, o_sl, o_sh, lse, scratch, kDecodeScratchBytes, stream);
}
