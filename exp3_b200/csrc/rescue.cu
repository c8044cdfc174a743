// Rescue-token choice of fp_v1_rescue / fp_v1_rescue_v2 (kernels.py:276-285).
//
// For query tile t, head h and every tail block kb < t (unselected), the rescue token is the
// key of kb maximising q_mean . k_j, with q_mean the fp32 mean of the tile's valid query rows
// (torch.argmax: the first maximum on ties). The tail tokens then enter the rescue tail through
// mean_tail_kernel (mean.cu).
//
// One CTA per (b, KV group, t), 128 threads. The group's query means are formed in shared
// memory (thread = dimension; the rows are summed in order, then divided by the row count).
// For every block in the union of the group's tails, thread j loads token j's key row into
// registers and forms one dot product per head with the broadcast means; a (value, index)
// maximum over the 128 tokens gives each head's choice.
#include "attn.cuh"

namespace fpx {

constexpr int kRescueMaxGroup = 16;

template <int kMode>
__global__ void __launch_bounds__(128) rescue_choice_kernel(MeanParams p) {
  const int t = p.tile_begin + blockIdx.x;
  const int kvh = p.head_begin / p.group + blockIdx.y;
  const int b = blockIdx.z;
  const int G = p.group;
  if (t == 0) return;  // tile 0 has no earlier block
  extern __shared__ __align__(16) uint8_t smem[];
  float *qm = reinterpret_cast<float *>(smem);                                 // [G][128]
  float *red_v = qm + G * kHeadDim;                                            // [4][G]
  int *red_i = reinterpret_cast<int *>(red_v + 4 * G);                         // [4][G]
  const int words = (p.nb + 31) / 32;
  uint32_t *bits = reinterpret_cast<uint32_t *>(red_i + 4 * G);                // [G][words]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // Tail bits of the group's heads: the route's (fused path) or kb < t and not selected (op).
  for (int g = 0; g < G; ++g) {
    const int h = kvh * G + g;
    if (kMode == kMeanMergeInPlace) {
      const uint32_t *src = p.route.tail + p.route.row(b, h, t, p.H) * p.route.words;
      for (int w = tid; w < words; w += 128) bits[g * words + w] = src[w];
    } else {
      const int64_t col = ((int64_t)b * p.nb + t) * p.nb * p.H + h;
      for (int k0 = 0; k0 < 32 * words; k0 += 128) {
        const int kb = k0 + tid;
        const bool in = kb < t && p.mask[col + (int64_t)kb * p.H] == 0;
        const unsigned bal = __ballot_sync(0xffffffffu, in);
        if (lane == 0 && (kb >> 5) < words) bits[g * words + (kb >> 5)] = bal;
      }
    }
  }
  __syncthreads();
  {  // nothing to choose when no head of the group has a tail (every block selected)
    int any = 0;
    for (int i = tid; i < G * words; i += 128) any |= bits[i] != 0u;
    if (!__syncthreads_or(any)) return;
  }
  // Query means (kernels.py:278-279): sum over the valid rows in fp32, then divide.
  const int rows = min(kBlock, p.L - t * kBlock);
  for (int g = 0; g < G; ++g) {
    const int h = kvh * G + g;
    const __nv_bfloat16 *src = p.q + b * p.q_sb + (int64_t)t * kBlock * p.q_sl + h * p.q_sh + tid;
    float s = 0.f;
#pragma unroll 8
    for (int r = 0; r < rows; ++r) s += __bfloat162float(src[(int64_t)r * p.q_sl]);
    qm[g * kHeadDim + tid] = s / (float)rows;
  }
  __syncthreads();

  uint8_t *choice = p.choice;
  for (int kb = 0; kb < t; ++kb) {
    uint32_t any = 0;
    for (int g = 0; g < G; ++g) any |= bits[g * words + (kb >> 5)];
    if (!((any >> (kb & 31)) & 1u)) continue;  // uniform: no head has kb in its tail
    // Token tid's key row, in registers.
    uint32_t kr[64];
    const uint4 *row = reinterpret_cast<const uint4 *>(p.k + b * p.k_sb + ((int64_t)kb * kBlock + tid) * p.k_sl +
                                                       kvh * p.k_sh);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint4 u = row[i];
      kr[4 * i] = u.x; kr[4 * i + 1] = u.y; kr[4 * i + 2] = u.z; kr[4 * i + 3] = u.w;
    }
    for (int g = 0; g < G; ++g) {
      if (!((bits[g * words + (kb >> 5)] >> (kb & 31)) & 1u)) continue;  // uniform per head
      const float4 *m4 = reinterpret_cast<const float4 *>(qm + g * kHeadDim);
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float4 m = m4[i];
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&kr[2 * i]));
        const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&kr[2 * i + 1]));
        dot = fmaf(m.x, a.x, dot);
        dot = fmaf(m.y, a.y, dot);
        dot = fmaf(m.z, c.x, dot);
        dot = fmaf(m.w, c.y, dot);
      }
      // (value, index) maximum, the lower index on ties.
      float bv = dot;
      int bi = tid;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
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
      for (int w = 1; w < 4; ++w) {
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
  const size_t smem = (size_t)p.group * kHeadDim * 4 + 8 * p.group * 4 + (size_t)p.group * ((p.nb + 31) / 32) * 4;
  if (smem > 200 * 1024) return FPX_ERR_UNSUPPORTED;
  const dim3 grid(tiles, kv_count, B);
  if (mode == kMeanMergeInPlace) {
    cudaFuncSetAttribute(rescue_choice_kernel<kMeanMergeInPlace>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    rescue_choice_kernel<kMeanMergeInPlace><<<grid, 128, smem, s>>>(p);
  } else {
    cudaFuncSetAttribute(rescue_choice_kernel<kMeanStandalone>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    rescue_choice_kernel<kMeanStandalone><<<grid, 128, smem, s>>>(p);
  }
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

}  // namespace fpx
