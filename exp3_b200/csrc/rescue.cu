// Rescue-token choice of fp_v1_rescue / fp_v1_rescue_v2 (kernels.py:276-285).
//
// For query tile t, head h and every tail block kb < t (unselected), the rescue token is the
// key of kb maximising q_mean . k_j, with q_mean the fp32 mean of the tile's valid query rows
// (torch.argmax: the first maximum on ties). The tail tokens then enter the rescue tail through
// mean_tail_kernel (mean.cu).
//
// kRescueSplits CTAs per (b, KV group, t), 256 threads each. On the fused path one pass over Q
// first forms every (b, t, h)'s query mean (fp32 sums of the valid rows, then divided by the
// row count) into the workspace and the split CTAs copy their group's means; otherwise each
// CTA forms them (the same arithmetic). Every CTA compacts the union of the group's tails into
// a list; CTA s of the split takes list entries
// s, s + kRescueSplits, ... For each of its blocks, thread pair (2j, 2j + 1) holds token j's key
// row in registers, 64 dimensions each (the next block's row is loaded while the current one is
// reduced), and forms one dot product per head with the broadcast means; a (value, index)
// maximum over the 128 tokens gives each head's choice.
#include "attn.cuh"

namespace fpx {

constexpr int kRescueMaxGroup = 16;
constexpr int kRescueSplits = 4;
constexpr int kChoiceThreads = 256;

// The fp32 mean of query tile t's valid rows of head h (kernels.py:278-279) into dst[D], by 256
// threads: warp w sums rows w, w + 8, ... for dimensions 4 lane + 128 c .. + 3, and the eight
// partial sums are added in warp order before the division by the row count. `part` is [8][D]
// of shared memory.
template <int D>
__device__ __forceinline__ void tile_query_mean(const MeanParams &p, int b, int t, int h, float *part, float *dst) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rows = min(kBlock, p.L - t * kBlock);
#pragma unroll
  for (int c = 0; c < D / 128; ++c) {
    const __nv_bfloat16 *src = p.q + b * p.q_sb + (int64_t)t * kBlock * p.q_sl + h * p.q_sh + 4 * lane + 128 * c;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll 4
    for (int r = warp; r < rows; r += 8) {
      const uint2 u = *reinterpret_cast<const uint2 *>(src + (int64_t)r * p.q_sl);
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.x));
      const float2 cc = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u.y));
      s0 += a.x; s1 += a.y; s2 += cc.x; s3 += cc.y;
    }
    *reinterpret_cast<float4 *>(part + warp * D + 4 * lane + 128 * c) = make_float4(s0, s1, s2, s3);
  }
  __syncthreads();
  if (tid < D) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += part[w * D + tid];
    dst[tid] = s / (float)rows;
  }
  __syncthreads();
}

// The query means of every (b, t, h) of the launch, once, for the choice CTAs to share.
template <int D>
__global__ void __launch_bounds__(256) rescue_qmean_kernel(MeanParams p) {
  __shared__ __align__(16) float part[8 * D];
  const int t = p.tile_begin + blockIdx.x, h = p.head_begin + blockIdx.y, b = blockIdx.z;
  if (t == 0) return;  // tile 0 has no earlier block to rescue from
  tile_query_mean<D>(p, b, t, h, part, p.qmean + (((int64_t)b * p.nb + t) * p.H + h) * D);
}

template <int kMode, int D = kHeadDim>
__global__ void __launch_bounds__(256, D == kHeadDim ? 2 : 1) rescue_choice_kernel(MeanParams p) {
  const int t = p.tile_begin + blockIdx.x;
  const int kvh = p.head_begin / p.group + blockIdx.y;
  const int b = blockIdx.z / kRescueSplits;
  const int split = blockIdx.z % kRescueSplits;
  const int G = p.group;
  if (t == 0) return;  // tile 0 has no earlier block
  extern __shared__ __align__(16) uint8_t smem[];
  float *qm = reinterpret_cast<float *>(smem);                                 // [G][D]
  float *part = qm + G * D;                                                    // [8][D]
  float *red_v = part + 8 * D;                                                 // [8][G]
  int *red_i = reinterpret_cast<int *>(red_v + 8 * G);                         // [8][G]
  const int words = (p.nb + 31) / 32;
  uint32_t *bits = reinterpret_cast<uint32_t *>(red_i + 8 * G);                // [G][words]
  uint16_t *ulist = reinterpret_cast<uint16_t *>(bits + G * words);            // [nb] union of the tails
  int *scratch = reinterpret_cast<int *>(ulist + ((p.nb + 1) & ~1));           // [8]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // Tail bits of the group's heads: the route's (fused path) or kb < t and not selected (op).
  for (int g = 0; g < G; ++g) {
    const int h = kvh * G + g;
    if (kMode == kMeanMergeInPlace) {
      const uint32_t *src = p.route.tail + p.route.row(b, h, t, p.H) * p.route.words;
      for (int w = tid; w < words; w += kChoiceThreads) bits[g * words + w] = src[w];
    } else {
      const int64_t col = ((int64_t)b * p.nb + t) * p.nb * p.H + h;
      for (int k0 = 0; k0 < 32 * words; k0 += kChoiceThreads) {
        const int kb = k0 + tid;
        const bool in = kb < t && p.mask[col + (int64_t)kb * p.H] == 0;
        const unsigned bal = __ballot_sync(0xffffffffu, in);
        if (lane == 0 && (kb >> 5) < words) bits[g * words + (kb >> 5)] = bal;
      }
    }
  }
  __syncthreads();
  // Union of the group's tails, ascending.
  int nu = 0;
  for (int w0 = 0; w0 < words; w0 += kChoiceThreads) {
    const int w = w0 + tid;
    uint32_t u = 0;
    if (w < words)
      for (int g = 0; g < G; ++g) u |= bits[g * words + w];
    int total;
    int pos = block_exclusive_scan<kChoiceThreads>(__popc(u), scratch, &total);
    for (uint32_t x = u; x; x &= x - 1) ulist[nu + pos++] = (uint16_t)(32 * w + __ffs(x) - 1);
    nu += total;
  }
  __syncthreads();
  if (split >= nu) return;  // nothing for this CTA of the split (uniform)
  // Query means (kernels.py:278-279): from the launch's shared pass when there is one, else
  // formed here (the same arithmetic).
  if (p.qmean) {
    for (int i = tid; i < G * D; i += kChoiceThreads)
      qm[i] = p.qmean[(((int64_t)b * p.nb + t) * p.H + kvh * G + i / D) * D + i % D];
    __syncthreads();
  } else {
    for (int g = 0; g < G; ++g) tile_query_mean<D>(p, b, t, kvh * G + g, part, qm + g * D);
  }

  // Thread pair (2 j, 2 j + 1) holds token j's key row, D / 2 dimensions each.
  const int tok = tid >> 1, half = tid & 1;
  uint8_t *choice = p.choice;
  auto load_row = [&](int kb, uint4 (&dst)[D / 16]) {
    const uint4 *row = reinterpret_cast<const uint4 *>(p.k + b * p.k_sb + ((int64_t)kb * kBlock + tok) * p.k_sl +
                                                       kvh * p.k_sh + (D / 2) * half);
#pragma unroll
    for (int i = 0; i < D / 16; ++i) dst[i] = row[i];
  };
  uint4 nxt[D / 16];
  load_row(ulist[split], nxt);
  for (int e = split; e < nu; e += kRescueSplits) {
    const int kb = ulist[e];
    // The next block's half row is requested before this block's dots.
    uint32_t kr[D / 4];
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
      kr[4 * i] = nxt[i].x; kr[4 * i + 1] = nxt[i].y; kr[4 * i + 2] = nxt[i].z; kr[4 * i + 3] = nxt[i].w;
    }
    if (e + kRescueSplits < nu) load_row(ulist[e + kRescueSplits], nxt);
    for (int g = 0; g < G; ++g) {
      if (!((bits[g * words + (kb >> 5)] >> (kb & 31)) & 1u)) continue;  // uniform per head
      const float4 *m4 = reinterpret_cast<const float4 *>(qm + g * D + (D / 2) * half);
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        const float4 m = m4[i];
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&kr[2 * i]));
        const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&kr[2 * i + 1]));
        dot = fmaf(m.x, a.x, dot);
        dot = fmaf(m.y, a.y, dot);
        dot = fmaf(m.z, c.x, dot);
        dot = fmaf(m.w, c.y, dot);
      }
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);  // the two halves, the same sum in both lanes
      // (value, index) maximum over the warp's 16 tokens, the lower index on ties.
      float bv = dot;
      int bi = tok;
#pragma unroll
      for (int o = 16; o > 1; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        red_v[warp * G + g] = bv;
        red_i[warp * G + g] = bi;
      }
    }
    __syncthreads();
    if (tid < G && ((bits[tid * words + (kb >> 5)] >> (kb & 31)) & 1u)) {
      float bv = red_v[tid];
      int bi = red_i[tid];
      for (int w = 1; w < 8; ++w) {
        const float v = red_v[w * G + tid];
        const int i = red_i[w * G + tid];
        if (v > bv || (v == bv && i < bi)) {
          bv = v;
          bi = i;
        }
      }
      const int h = kvh * G + tid;
      choice[(((int64_t)b * p.H + h) * p.nb + t) * p.nb + kb] = (uint8_t)bi;
    }
    __syncthreads();
  }
}

int launch_rescue_choice(const MeanParams &p, int mode, int tiles, int kv_count, int B, cudaStream_t s) {
  if (tiles <= 0 || kv_count <= 0) return FPX_OK;
  if (p.group > kRescueMaxGroup || !p.choice || !p.k) return FPX_ERR_UNSUPPORTED;
  const int d = p.d == 256 ? 256 : kHeadDim;
  const size_t smem = (size_t)p.group * d * 4 + 8 * d * 4 + 16 * p.group * 4 +
                      (size_t)p.group * ((p.nb + 31) / 32) * 4 + (size_t)((p.nb + 1) & ~1) * 2 + 32;
  if (smem > 200 * 1024) return FPX_ERR_UNSUPPORTED;
  const dim3 grid(tiles, kv_count, B * kRescueSplits);
  if (p.qmean) {  // one pass over Q for the query means, shared by the choice CTAs
    const dim3 mgrid(tiles, kv_count * p.group, B);
    if (d == 256)
      rescue_qmean_kernel<256><<<mgrid, kChoiceThreads, 0, s>>>(p);
    else
      rescue_qmean_kernel<kHeadDim><<<mgrid, kChoiceThreads, 0, s>>>(p);
  }
#define FPX_CHOICE_LAUNCH(MODE, DD)                                                                     \
  do {                                                                                                  \
    cudaFuncSetAttribute(rescue_choice_kernel<MODE, DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    rescue_choice_kernel<MODE, DD><<<grid, kChoiceThreads, smem, s>>>(p);                               \
  } while (0)
  if (mode == kMeanMergeInPlace) {
    if (d == 256) FPX_CHOICE_LAUNCH(kMeanMergeInPlace, 256); else FPX_CHOICE_LAUNCH(kMeanMergeInPlace, kHeadDim);
  } else {
    if (d == 256) FPX_CHOICE_LAUNCH(kMeanStandalone, 256); else FPX_CHOICE_LAUNCH(kMeanStandalone, kHeadDim);
  }
#undef FPX_CHOICE_LAUNCH
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

}  // namespace fpx
