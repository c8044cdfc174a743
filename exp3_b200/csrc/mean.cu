// Block-mean tail and the logaddexp merge.
//
// Reference: kernels.py:179-230 (mean_tail) and kernels.py:312-325 (merge_exact_mean).
// For query row i of tile t and head h, the tail is every block kb < t that the routing
// did not select. Each tail block acts as one pseudo-key with key mean_k[kb], value
// mean_v[kb] (fp32 descriptors) and logit (q_i . mean_k[kb]) * scale + ln n_kb; the tail's
// softmax output and log-sum-exp are merged with the exact path's by logaddexp. Selected
// blocks never enter the tail, so no block is counted twice.
//
// One CTA per (b, h, t) that has a tail; D / 64 threads per query row (two at head dim 128, four
// at 256), each holding 64 of the D dimensions (interleaved float4 chunks, so a row's threads
// read distinct banks). The tail blocks' pseudo-keys are staged 16 at a time; the softmax runs
// online in fp32.
//
// The same kernel runs the rescue tails of fp_v1_rescue / _v2 (kernels.py:233-309, kKeys 1 / 2):
// there the pseudo-key of tail block kb is its rescue token, the block's key row chosen by
// rescue_choice_kernel (bf16 K / V, exact in fp32) with weight 1; _v2 adds the block's other
// 127 tokens through their mean, K_rest = (sum K - k_rescue) / 127 (likewise V), with weight
// ln 127. Tail blocks are full, so sum K = 128 x mean_k exactly (a power-of-two scale).
#include "attn.cuh"

namespace fpx {

constexpr int kMeanChunk = 16;

template <int kMode, int kKeys, int D = kHeadDim>  // kKeys: 0 block means, 1 rescue, 2 rescue + remainder
__global__ void __launch_bounds__(2 * D) mean_tail_kernel(MeanParams p) {
  constexpr int TPR = D / 64;   // threads per query row
  constexpr int NT = 128 * TPR;
  constexpr int Q4 = D / 4;     // float4 pieces per row
  const int t = p.tile_begin + (gridDim.x - 1 - blockIdx.x);
  const int h = p.head_begin + blockIdx.y;
  const int b = blockIdx.z;
  const int kvh = h / p.group;
  extern __shared__ __align__(16) uint8_t smem[];
  float *smk = reinterpret_cast<float *>(smem);            // [16][D]
  float *smv = smk + kMeanChunk * D;                       // [16][D]
  float *slogn = smv + kMeanChunk * D;                     // [16]
  int *scratch = reinterpret_cast<int *>(slogn + kMeanChunk);  // [8]
  int *list = scratch + 8;                                 // [nb]
  const int tid = threadIdx.x;

  // Ascending list of the tail blocks of (b, h, t).
  int ntail = 0;
  if (kMode == kMeanMergeInPlace) {
    const uint32_t *bits = p.route.tail + p.route.row(b, h, t, p.H) * p.route.words;
    for (int w0 = 0; w0 < p.route.words; w0 += NT) {
      const int w = w0 + tid;
      const uint32_t word = w < p.route.words ? bits[w] : 0u;
      int total;
      int pos = block_exclusive_scan<NT>(__popc(word), scratch, &total);
      for (uint32_t x = word; x; x &= x - 1) list[ntail + pos++] = 32 * w + __ffs(x) - 1;
      ntail += total;
    }
  } else {
    const int64_t col = ((int64_t)b * p.nb + t) * p.nb * p.H + h;
    for (int c0 = 0; c0 < t; c0 += NT) {
      const int kb = c0 + tid;
      const bool in = kb < t && p.mask[col + (int64_t)kb * p.H] == 0;
      int total;
      const int pos = block_exclusive_scan<NT>(in ? 1 : 0, scratch, &total);
      if (in) list[ntail + pos] = kb;
      ntail += total;
    }
  }
  __syncthreads();

  const int rows = min(kBlock, p.L - t * kBlock);
  const int r = tid / TPR, half = tid % TPR;  // `half`: this thread's part of the row
  const bool valid = r < rows;
  const int pos = t * kBlock + min(r, rows - 1);
  if (ntail == 0) {
    if (kMode == kMeanStandalone && valid) {
      float4 *dst = reinterpret_cast<float4 *>(p.mean_out + (((int64_t)b * p.L + pos) * p.H + h) * D);
#pragma unroll
      for (int i = 0; i < 16; ++i) dst[TPR * i + half] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (half == 0) p.mean_lse[((int64_t)b * p.L + pos) * p.H + h] = -INFINITY;
    }
    return;
  }

  float q[64];
  {
    const __nv_bfloat16 *src = p.q + b * p.q_sb + (int64_t)pos * p.q_sl + h * p.q_sh;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint2 u = *reinterpret_cast<const uint2 *>(src + 4 * (TPR * i + half));
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
      const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
      q[4 * i] = a.x; q[4 * i + 1] = a.y; q[4 * i + 2] = c.x; q[4 * i + 3] = c.y;
    }
  }
  float o[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) o[i] = 0.f;
  float m = -INFINITY, s = 0.f;
  const int64_t dstride = (int64_t)p.Hkv * D;
  const float *mk_base = p.mean_k + ((int64_t)b * p.nb * p.Hkv + kvh) * D;
  const float *mv_base = p.mean_v + ((int64_t)b * p.nb * p.Hkv + kvh) * D;

  const int nkeys = kKeys == 2 ? 2 * ntail : ntail;  // pseudo-keys
  const uint8_t *choice = kKeys ? p.choice + (((int64_t)b * p.H + h) * p.nb + t) * p.nb : nullptr;
  for (int c0 = 0; c0 < nkeys; c0 += kMeanChunk) {
    const int cn = min(kMeanChunk, nkeys - c0);
    __syncthreads();
    for (int i = tid; i < cn * Q4; i += NT) {
      const int j = i / Q4, q4 = i % Q4;
      if (kKeys == 0) {
        const int kb = list[c0 + j];
        reinterpret_cast<float4 *>(smk + j * D)[q4] =
            reinterpret_cast<const float4 *>(mk_base + kb * dstride)[q4];
        reinterpret_cast<float4 *>(smv + j * D)[q4] =
            reinterpret_cast<const float4 *>(mv_base + kb * dstride)[q4];
      } else {
        const int key = c0 + j;
        const int kb = list[kKeys == 2 ? key >> 1 : key];
        const int64_t tok = (int64_t)kb * kBlock + choice[kb];
        const uint2 ku = *reinterpret_cast<const uint2 *>(p.k + b * p.k_sb + tok * p.k_sl + kvh * p.k_sh + 4 * q4);
        const uint2 vu = *reinterpret_cast<const uint2 *>(p.v + b * p.v_sb + tok * p.v_sl + kvh * p.v_sh + 4 * q4);
        const float2 k01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&ku.x));
        const float2 k23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&ku.y));
        const float2 v01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&vu.x));
        const float2 v23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&vu.y));
        float4 k4 = make_float4(k01.x, k01.y, k23.x, k23.y), v4 = make_float4(v01.x, v01.y, v23.x, v23.y);
        if (kKeys == 2 && (key & 1)) {  // the block's other tokens: (sum - rescue) / 127
          const float4 mk4 = reinterpret_cast<const float4 *>(mk_base + kb * dstride)[q4];
          const float4 mv4 = reinterpret_cast<const float4 *>(mv_base + kb * dstride)[q4];
          auto rest = [](float mean, float x) { return __fdiv_rn(__fsub_rn(__fmul_rn(mean, 128.f), x), 127.f); };
          k4 = make_float4(rest(mk4.x, k4.x), rest(mk4.y, k4.y), rest(mk4.z, k4.z), rest(mk4.w, k4.w));
          v4 = make_float4(rest(mv4.x, v4.x), rest(mv4.y, v4.y), rest(mv4.z, v4.z), rest(mv4.w, v4.w));
        }
        reinterpret_cast<float4 *>(smk + j * D)[q4] = k4;
        reinterpret_cast<float4 *>(smv + j * D)[q4] = v4;
      }
    }
    if (tid < cn) {
      if (kKeys == 0)
        slogn[tid] = logf((float)min(kBlock, p.L - list[c0 + tid] * kBlock));
      else
        slogn[tid] = (kKeys == 2 && ((c0 + tid) & 1)) ? logf((float)(kBlock - 1)) : 0.f;
    }
    __syncthreads();
    for (int j = 0; j < cn; ++j) {
      const float4 *mk4 = reinterpret_cast<const float4 *>(smk + j * D);
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 k4 = mk4[TPR * i + half];
        dot = fmaf(q[4 * i], k4.x, dot);
        dot = fmaf(q[4 * i + 1], k4.y, dot);
        dot = fmaf(q[4 * i + 2], k4.z, dot);
        dot = fmaf(q[4 * i + 3], k4.w, dot);
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      if (TPR == 4) dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      const float l = __fadd_rn(__fmul_rn(dot, p.scale), slogn[j]);
      if (l > m) {
        const float corr = expf(m - l);
        s *= corr;
#pragma unroll
        for (int i = 0; i < 64; ++i) o[i] *= corr;
        m = l;
      }
      const float w = expf(l - m);
      s += w;
      const float4 *mv4 = reinterpret_cast<const float4 *>(smv + j * D);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 v4 = mv4[TPR * i + half];
        o[4 * i] = fmaf(w, v4.x, o[4 * i]);
        o[4 * i + 1] = fmaf(w, v4.y, o[4 * i + 1]);
        o[4 * i + 2] = fmaf(w, v4.z, o[4 * i + 2]);
        o[4 * i + 3] = fmaf(w, v4.w, o[4 * i + 3]);
      }
    }
  }
  const float lse_m = m + logf(s);
  const float inv = 1.f / s;
  const int64_t lrow = ((int64_t)b * p.L + pos) * p.H + h;
  if (kMode == kMeanStandalone) {
    if (!valid) return;
    float4 *dst = reinterpret_cast<float4 *>(p.mean_out + lrow * D);
#pragma unroll
    for (int i = 0; i < 16; ++i)
      dst[TPR * i + half] = make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv,
                                        o[4 * i + 3] * inv);
    if (half == 0) p.mean_lse[lrow] = lse_m;
  } else {
    // merge_exact_mean (kernels.py:318-325), in place on the exact output row.
    const float lse_e = p.lse[lrow];
    __syncwarp();  // every thread of the row has read lse_e before it is overwritten
    if (!valid) return;
    const float total = logaddexp(lse_e, lse_m);
    const float we = expf(lse_e - total), wm = expf(lse_m - total);
    __nv_bfloat16 *dst = p.out + b * p.o_sb + (int64_t)pos * p.o_sl + h * p.o_sh;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      uint2 u = *reinterpret_cast<const uint2 *>(dst + 4 * (TPR * i + half));
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
      const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
      u.x = pack_bf16(a.x * we + o[4 * i] * inv * wm, a.y * we + o[4 * i + 1] * inv * wm);
      u.y = pack_bf16(c.x * we + o[4 * i + 2] * inv * wm, c.y * we + o[4 * i + 3] * inv * wm);
      *reinterpret_cast<uint2 *>(dst + 4 * (TPR * i + half)) = u;
    }
    if (half == 0) p.lse[lrow] = total;
  }
}

namespace {
template <int kMode, int kKeys, int D = kHeadDim>
void launch_tail_variant(const MeanParams &p, dim3 grid, size_t smem, cudaStream_t s) {
  cudaFuncSetAttribute(mean_tail_kernel<kMode, kKeys, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  mean_tail_kernel<kMode, kKeys, D><<<grid, 2 * D, smem, s>>>(p);
}
}  // namespace

int launch_mean_tail(const MeanParams &p, int mode, int tiles, int heads, int B, cudaStream_t s, int keys) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  const int d = p.d == 256 ? 256 : kHeadDim;
  const size_t smem = (size_t)2 * kMeanChunk * d * 4 + kMeanChunk * 4 + 32 + (size_t)p.nb * 4;
  if (smem > 200 * 1024) return FPX_ERR_UNSUPPORTED;
  if (keys != 0 && (!p.choice || !p.k || !p.v)) return FPX_ERR_INVALID;
  dim3 grid(tiles, heads, B);
  const bool merge = mode == kMeanMergeInPlace;
  if (d == 256) {  // head dim 256: block-mean and rescue tails on the fp32 kernel
    switch (keys) {
      case 0: merge ? launch_tail_variant<kMeanMergeInPlace, 0, 256>(p, grid, smem, s)
                    : launch_tail_variant<kMeanStandalone, 0, 256>(p, grid, smem, s); break;
      case 1: merge ? launch_tail_variant<kMeanMergeInPlace, 1, 256>(p, grid, smem, s)
                    : launch_tail_variant<kMeanStandalone, 1, 256>(p, grid, smem, s); break;
      case 2: merge ? launch_tail_variant<kMeanMergeInPlace, 2, 256>(p, grid, smem, s)
                    : launch_tail_variant<kMeanStandalone, 2, 256>(p, grid, smem, s); break;
      default: return FPX_ERR_INVALID;
    }
    FPX_CHECK_LAUNCH();
    return FPX_OK;
  }
  switch (keys) {
    case 0: merge ? launch_tail_variant<kMeanMergeInPlace, 0>(p, grid, smem, s)
                  : launch_tail_variant<kMeanStandalone, 0>(p, grid, smem, s); break;
    case 1: merge ? launch_tail_variant<kMeanMergeInPlace, 1>(p, grid, smem, s)
                  : launch_tail_variant<kMeanStandalone, 1>(p, grid, smem, s); break;
    case 2: merge ? launch_tail_variant<kMeanMergeInPlace, 2>(p, grid, smem, s)
                  : launch_tail_variant<kMeanStandalone, 2>(p, grid, smem, s); break;
    default: return FPX_ERR_INVALID;
  }
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

// merge_exact_mean (kernels.py:312-325) over rows of D: one thread per 4 elements.
template <int D>
__global__ void merge_kernel(const __nv_bfloat16 *eo, const float *el, const float *mo,
                             const float *ml, int64_t rows, __nv_bfloat16 *out, float *lse) {
  const int64_t n = rows * (D / 4);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / (D / 4);
    const float a = el[row], c = ml[row];
    const float total = logaddexp(a, c);
    const float we = expf(a - total), wm = expf(c - total);
    const uint2 u = reinterpret_cast<const uint2 *>(eo)[i];
    const float4 m4 = reinterpret_cast<const float4 *>(mo)[i];
    const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
    const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
    uint2 r;
    r.x = pack_bf16(x.x * we + m4.x * wm, x.y * we + m4.y * wm);
    r.y = pack_bf16(y.x * we + m4.z * wm, y.y * we + m4.w * wm);
    reinterpret_cast<uint2 *>(out)[i] = r;
    if ((i % (D / 4)) == 0) lse[row] = total;
  }
}

int launch_merge(const __nv_bfloat16 *exact_out, const float *exact_lse, const float *mean_out,
                 const float *mean_lse, int64_t rows, __nv_bfloat16 *out, float *lse,
                 cudaStream_t s, int d) {
  const int64_t n = rows * (d / 4);
  const int grid = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  if (grid <= 0) return FPX_OK;
  if (d == 256)
    merge_kernel<256><<<grid, 256, 0, s>>>(exact_out, exact_lse, mean_out, mean_lse, rows, out, lse);
  else
    merge_kernel<kHeadDim><<<grid, 256, 0, s>>>(exact_out, exact_lse, mean_out, mean_lse, rows, out, lse);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

}  // namespace fpx
