// Routing kernels: block statistics, V1 proxy scores, the new selectors, the threshold +
// protected selection, and the conversions between compact lists and the reference's
// [B, nb, nb, H] layouts.
//
// Reference: upstream/flashprefill_native_forward.py:27-175, 357-417 (V1) and
// kernels.py:22-176 (descriptors, selectors, selection, index/mask conversion).
#include <algorithm>
#include <cstdint>

#include "attn.cuh"
#include "route.cuh"

namespace fpx {

// ----------------------------------------------------------------------------------------
// Block statistics. One CTA per (key block, KV head, batch); thread c owns dimension c and
// walks the block's valid rows in order, so the fp32 sums have a fixed sequential order
// (the bf16 V1 mean is bf16(sum / n), see upstream:58-68; the fp32 descriptors follow
// kernels.py:22-46).
// The statistics of one (block, KV head, batch) from its column sums (thread c: dimension c).
template <bool kBf16Mean, bool kDesc, int D>
__device__ __forceinline__ void block_stats_store(const StatsParams &p, int b, int blk, int kvh, int c, int n, float sk,
                                                  float sk2, float sv, float sv2) {
  const float fn = (float)n;
  const int64_t o = (((int64_t)b * p.nb + blk) * p.Hkv + kvh) * D + c;
  if (kBf16Mean) p.mean_bf16[o] = __float2bfloat16_rn(__fdiv_rn(sk, fn));
  if (kDesc) {
    __shared__ float red[D / 32];
    const float mk = __fdiv_rn(sk, fn);
    const float mv = __fdiv_rn(sv, fn);
    p.mean_k[o] = mk;
    const float vk = fmaxf(__fsub_rn(__fdiv_rn(sk2, fn), __fmul_rn(mk, mk)), 0.f);
    p.var_k[o] = vk;
    if (p.vk_hi) {
      const __nv_bfloat16 hi = __float2bfloat16_rn(vk);
      p.vk_hi[o] = hi;
      p.vk_lo[o] = __float2bfloat16_rn(__fsub_rn(vk, __bfloat162float(hi)));
    }
    p.mean_v[o] = mv;
    if (p.mk_hi) {  // mean_k = hi + lo exactly up to lo's rounding; the remainder is exact in fp32
      const __nv_bfloat16 hi = __float2bfloat16_rn(mk);
      p.mk_hi[o] = hi;
      p.mk_lo[o] = __float2bfloat16_rn(__fsub_rn(mk, __bfloat162float(hi)));
      p.mv_hi[o] = __float2bfloat16_rn(mv);
    }
    const float var_v = fmaxf(__fsub_rn(__fdiv_rn(sv2, fn), __fmul_rn(mv, mv)), 0.f);
    const float total = block_sum<D>(var_v, red);
    if (c == 0) p.sigma_v[((int64_t)b * p.nb + blk) * p.Hkv + kvh] = sqrtf(total);
    if (p.counts && c == 0 && b == 0 && kvh == p.kv_begin) p.counts[blk] = n;
  }
}

template <bool kBf16Mean, bool kDesc, int D = kHeadDim>
__global__ void __launch_bounds__(D) block_stats_kernel(StatsParams p) {
  const int blk = blockIdx.x, kvh = p.kv_begin + blockIdx.y, b = blockIdx.z;
  const int c = threadIdx.x;
  const int r0 = blk * kBlock;
  const int n = min(kBlock, p.L - r0);
  const __nv_bfloat16 *kp = p.k + b * p.k_sb + (int64_t)r0 * p.k_sl + kvh * p.k_sh + c;
  const __nv_bfloat16 *vp = p.v + b * p.v_sb + (int64_t)r0 * p.v_sl + kvh * p.v_sh + c;
  float sk = 0.f, sk2 = 0.f, sv = 0.f, sv2 = 0.f;
#pragma unroll 8
  for (int r = 0; r < n; ++r) {
    const float x = __bfloat162float(kp[(int64_t)r * p.k_sl]);
    sk = __fadd_rn(sk, x);
    if (kDesc) {
      sk2 = __fadd_rn(sk2, __fmul_rn(x, x));
      const float y = __bfloat162float(vp[(int64_t)r * p.v_sl]);
      sv = __fadd_rn(sv, y);
      sv2 = __fadd_rn(sv2, __fmul_rn(y, y));
    }
  }
  block_stats_store<kBf16Mean, kDesc, D>(p, b, blk, kvh, c, n, sk, sk2, sv, sv2);
}

// The same statistics with the block's rows staged through shared memory, kStageRows at a time:
// the whole stage is loaded at once by 16-byte coalesced loads, then thread c adds column c's
// rows in order, so every sum is the one the per-column walk above gives. For rows whose
// element strides are multiples of 8 and 16-byte aligned bases.
template <bool kBf16Mean, bool kDesc, int D = kHeadDim>
__global__ void __launch_bounds__(D) block_stats_staged_kernel(StatsParams p) {
  constexpr int kStageRows = D == 256 ? 32 : 64, kVecs = D / 8;  // 16-byte vectors per row
  __shared__ __align__(16) __nv_bfloat16 ks[kStageRows][D];
  __shared__ __align__(16) __nv_bfloat16 vs[kDesc ? kStageRows : 1][D];
  const int blk = blockIdx.x, kvh = p.kv_begin + blockIdx.y, b = blockIdx.z;
  const int c = threadIdx.x;
  const int r0 = blk * kBlock;
  const int n = min(kBlock, p.L - r0);
  const __nv_bfloat16 *kb = p.k + b * p.k_sb + (int64_t)r0 * p.k_sl + kvh * p.k_sh;
  const __nv_bfloat16 *vb = p.v + b * p.v_sb + (int64_t)r0 * p.v_sl + kvh * p.v_sh;
  float sk = 0.f, sk2 = 0.f, sv = 0.f, sv2 = 0.f;
  for (int base = 0; base < n; base += kStageRows) {
    const int rows = min(kStageRows, n - base);
#pragma unroll 4
    for (int e = c; e < rows * kVecs; e += D) {
      const int rr = e / kVecs, cv = e % kVecs;
      reinterpret_cast<uint4 *>(&ks[rr][0])[cv] =
          *reinterpret_cast<const uint4 *>(kb + (int64_t)(base + rr) * p.k_sl + 8 * cv);
      if (kDesc)
        reinterpret_cast<uint4 *>(&vs[rr][0])[cv] =
            *reinterpret_cast<const uint4 *>(vb + (int64_t)(base + rr) * p.v_sl + 8 * cv);
    }
    __syncthreads();
#pragma unroll 8
    for (int r = 0; r < rows; ++r) {
      const float x = __bfloat162float(ks[r][c]);
      sk = __fadd_rn(sk, x);
      if (kDesc) {
        sk2 = __fadd_rn(sk2, __fmul_rn(x, x));
        const float y = __bfloat162float(vs[r][c]);
        sv = __fadd_rn(sv, y);
        sv2 = __fadd_rn(sv2, __fmul_rn(y, y));
      }
    }
    __syncthreads();
  }
  block_stats_store<kBf16Mean, kDesc, D>(p, b, blk, kvh, c, n, sk, sk2, sv, sv2);
}

// 16-byte vector loads are legal for rows with element strides that are multiples of 8 from a
// 16-byte aligned base.
static bool rows_vectorizable(const void *base, int64_t sb, int64_t sl, int64_t sh) {
  return (reinterpret_cast<uintptr_t>(base) & 15u) == 0 && sb % 8 == 0 && sl % 8 == 0 && sh % 8 == 0;
}

template <int D>
static void launch_block_stats_d(const StatsParams &p, dim3 grid, bool bf16_mean, bool desc, bool staged,
                                 cudaStream_t s) {
  if (staged) {
    if (bf16_mean && desc)
      block_stats_staged_kernel<true, true, D><<<grid, D, 0, s>>>(p);
    else if (bf16_mean)
      block_stats_staged_kernel<true, false, D><<<grid, D, 0, s>>>(p);
    else if (desc)
      block_stats_staged_kernel<false, true, D><<<grid, D, 0, s>>>(p);
    return;
  }
  if (bf16_mean && desc)
    block_stats_kernel<true, true, D><<<grid, D, 0, s>>>(p);
  else if (bf16_mean)
    block_stats_kernel<true, false, D><<<grid, D, 0, s>>>(p);
  else if (desc)
    block_stats_kernel<false, true, D><<<grid, D, 0, s>>>(p);
}

int launch_block_stats(const StatsParams &p, int blocks, int kv_count, int B, bool bf16_mean,
                       bool desc, cudaStream_t s) {
  if (blocks <= 0 || kv_count <= 0) return FPX_OK;
  dim3 grid(blocks, kv_count, B);
  const bool staged = rows_vectorizable(p.k, p.k_sb, p.k_sl, p.k_sh) &&
                      (!desc || rows_vectorizable(p.v, p.v_sb, p.v_sl, p.v_sh));
  if (p.d == 256)  // head dim 256 (check_qwen35_math.py): one thread per dimension
    launch_block_stats_d<256>(p, grid, bf16_mean, desc, staged, s);
  else
    launch_block_stats_d<128>(p, grid, bf16_mean, desc, staged, s);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

// ----------------------------------------------------------------------------------------
// Selection epilogue shared by the routing kernels: from sc[0..nb) (normalised scores of
// query tile t, head h) build the active set, write the compact ascending list, its count
// and the tail bits (kb < t, not selected), and optionally the reference-layout scores.
// kRouted = true applies the new selectors' extra `score > 0` test (kernels.py:144);
// `all_causal` is the alpha == 0 rule of kernels.py:141-142.
template <int NT, bool kPositiveOnly>
__device__ void select_and_emit(const float *sc, float smax, const SelectArgs &a, int b, int h,
                                int t, int *scan_scratch) {
  const float thr = smax * a.alpha;
  const RouteView &r = a.route;
  const int64_t rrow = r.row(b, h, t, a.H);
  int32_t *list = r.lists + rrow * r.nb;
  uint32_t *tail = r.tail + rrow * r.words;
  int base = 0;
  for (int c0 = 0; c0 < a.nb; c0 += NT) {
    const int kb = c0 + threadIdx.x;
    bool active = false;
    if (kb < a.nb && kb <= t) {
      const float s = sc[kb];
      bool keep = a.all_causal || (s >= thr && (!kPositiveOnly || s > 0.f));
      active = keep || is_protected(t, kb, a.nb, a.sink, a.window, a.last_full);
    }
    int total;
    const int pos = block_exclusive_scan<NT>(active ? 1 : 0, scan_scratch, &total);
    if (active) list[base + pos] = kb;
    const unsigned tb = __ballot_sync(0xffffffffu, kb < a.nb && kb < t && !active);
    if ((threadIdx.x & 31) == 0 && kb < a.nb) tail[kb >> 5] = tb;
    base += total;
  }
  if (threadIdx.x == 0) r.counts[rrow] = base;
}

// ----------------------------------------------------------------------------------------
// V1 routing, fused: scores of one (b, h, query tile t) with mma.sync (bf16 products are
// exact in fp32), per-(tile, block) max / mass (upstream:147-175), normalisation
// (upstream:410-417), then the threshold + protected selection (upstream:366-385).
// 8 warps; warp w owns rows 16w..16w+15 of the tile. mean_k rows are staged 64 blocks at
// a time; rows are padded to 136 bf16 so fragment loads hit 32 distinct banks.
constexpr int kV1Chunk = 64;

template <int D>
__global__ void __launch_bounds__(256) v1_route_kernel(V1Params p) {
  constexpr int kPad = D + 8;
  constexpr int kChunks = D / 8;  // 16-byte pieces per row
  constexpr int kSteps = D / 16;  // mma K steps
  const int t = p.tile_begin + (gridDim.x - 1 - blockIdx.x);
  const int h = p.head_begin + blockIdx.y;
  const int b = blockIdx.z;
  const int kvh = h / p.group;
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16 *sq = reinterpret_cast<__nv_bfloat16 *>(smem);
  __nv_bfloat16 *smk = sq + kBlock * kPad;
  float *part_m = reinterpret_cast<float *>(smk + kV1Chunk * kPad);  // [8][64]
  float *part_s = part_m + 8 * kV1Chunk;                             // [8][64]
  float *bm = part_s + 8 * kV1Chunk;                                  // [nb] block max
  float *bs = bm + p.nb;                                              // [nb] block mass
  float *sc = bs + p.nb;                                              // [nb] scores
  int *scratch = reinterpret_cast<int *>(sc + p.nb);                  // [8]
  float *red = reinterpret_cast<float *>(scratch + 8);                // [8]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  // Stage the query tile (zero rows past L).
  for (int i = tid; i < kBlock * kChunks; i += 256) {
    const int row = i / kChunks, ch = i % kChunks;
    const int pos = t * kBlock + row;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (pos < p.L)
      val = *reinterpret_cast<const uint4 *>(p.q + b * p.q_sb + (int64_t)pos * p.q_sl +
                                             h * p.q_sh + ch * 8);
    *reinterpret_cast<uint4 *>(sq + row * kPad + ch * 8) = val;
  }
  __syncthreads();
  uint32_t af[kSteps][4];
#pragma unroll
  for (int kk = 0; kk < kSteps; ++kk) {
    const __nv_bfloat16 *r0 = sq + (16 * warp + g) * kPad + 16 * kk + 2 * tq;
    const __nv_bfloat16 *r1 = r0 + 8 * kPad;
    af[kk][0] = *reinterpret_cast<const uint32_t *>(r0);
    af[kk][1] = *reinterpret_cast<const uint32_t *>(r1);
    af[kk][2] = *reinterpret_cast<const uint32_t *>(r0 + 8);
    af[kk][3] = *reinterpret_cast<const uint32_t *>(r1 + 8);
  }
  const int row_a = t * kBlock + 16 * warp + g;
  const int row_b = row_a + 8;
  const int last_row = t * kBlock + kBlock - 1;
  const int nblk = t + 1;
  const __nv_bfloat16 *mk_base = p.mean_k + ((int64_t)b * p.nb * p.Hkv + kvh) * D;
  const int64_t mk_stride = (int64_t)p.Hkv * D;

  for (int c0 = 0; c0 < nblk; c0 += kV1Chunk) {
    const int cn = min(kV1Chunk, nblk - c0);
    const int cn8 = (cn + 7) & ~7;
    __syncthreads();
    for (int i = tid; i < cn8 * kChunks; i += 256) {
      const int j = i / kChunks, ch = i % kChunks;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (j < cn) val = *reinterpret_cast<const uint4 *>(mk_base + (c0 + j) * mk_stride + ch * 8);
      *reinterpret_cast<uint4 *>(smk + j * kPad + ch * 8) = val;
    }
    __syncthreads();
    for (int j0 = 0; j0 < cn8; j0 += 8) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < kSteps; ++kk) {
        const __nv_bfloat16 *bp = smk + (j0 + g) * kPad + 16 * kk + 2 * tq;
        mma_bf16_16816(acc, af[kk], *reinterpret_cast<const uint32_t *>(bp),
                       *reinterpret_cast<const uint32_t *>(bp + 8));
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kb = c0 + j0 + 2 * tq + e;
        // Row i sees block kb iff i >= 128 kb + 127 (upstream:149-160).
        const bool va = row_a < p.L && kb < nblk && (kb < t || row_a == last_row);
        const bool vb = row_b < p.L && kb < nblk && (kb < t || row_b == last_row);
        const float xa = va ? acc[e] * p.scale_log2 : -INFINITY;
        const float xb = vb ? acc[2 + e] * p.scale_log2 : -INFINITY;
        float m = fmaxf(xa, xb);
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 8));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
        float s = 0.f;
        if (m != -INFINITY) s = (va ? exp2f(xa - m) : 0.f) + (vb ? exp2f(xb - m) : 0.f);
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        s += __shfl_xor_sync(0xffffffffu, s, 8);
        s += __shfl_xor_sync(0xffffffffu, s, 16);
        if (g == 0) {
          part_m[warp * kV1Chunk + j0 + 2 * tq + e] = m;
          part_s[warp * kV1Chunk + j0 + 2 * tq + e] = s;
        }
      }
    }
    __syncthreads();
    for (int j = tid; j < cn; j += 256) {
      float m = -INFINITY;
#pragma unroll
      for (int w = 0; w < 8; ++w) m = fmaxf(m, part_m[w * kV1Chunk + j]);
      float s = 0.f;
      if (m != -INFINITY) {
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const float mw = part_m[w * kV1Chunk + j];
          if (mw != -INFINITY) s += part_s[w * kV1Chunk + j] * exp2f(mw - m);
        }
      }
      bm[c0 + j] = m;
      bs[c0 + j] = s;
    }
  }
  __syncthreads();
  // normalize_scores (upstream:410-417): rescale by exp2(M - max M), divide by (sum + 1e-9).
  float lmax = -INFINITY;
  for (int kb = tid; kb < nblk; kb += 256) lmax = fmaxf(lmax, bm[kb]);
  const float gmax = block_max<256>(lmax, red);
  float lsum = 0.f;
  for (int kb = tid; kb < nblk; kb += 256) {
    const float m = bm[kb];
    const float r = (m != -INFINITY) ? bs[kb] * exp2f(m - gmax) : 0.f;
    sc[kb] = r;
    lsum += r;
  }
  const float total = block_sum<256>(lsum, red) + 1e-9f;
  float lsmax = 0.f;
  for (int kb = tid; kb < p.nb; kb += 256) {
    const float s = kb < nblk ? sc[kb] / total : 0.f;
    sc[kb] = s;
    lsmax = fmaxf(lsmax, s);
    if (p.scores) p.scores[(((int64_t)b * p.nb + t) * p.nb + kb) * p.H + h] = s;
  }
  const float smax = block_max<256>(lsmax, red);
  if (p.sel.route.lists) select_and_emit<256, false>(sc, smax, p.sel, b, h, t, scratch);
}

size_t v1_route_smem(int nb, int d) {
  return (size_t)(kBlock + kV1Chunk) * (d + 8) * 2 + 2 * 8 * kV1Chunk * 4 + 3 * (size_t)nb * 4 + 64;
}

int launch_v1_route_selected(const V1Params &p, int tiles, int heads, int B, cudaStream_t s) {
  // The tcgen05 routing kernel holds up to 2048 blocks at head dim 128 and 512 at 256 (its
  // score arrays live in shared memory); longer head-dim-256 layers take the mma.sync kernel.
  const int d = p.d == 256 ? 256 : kHeadDim;
  return (get_option(kOptRouteKernel) == kRouteKernelMmaSync || !v1_route_tc_supports(d, p.nb))
             ? launch_v1_route(p, tiles, heads, B, s)
             : launch_v1_route_tc(p, B, tiles, heads, s);
}

int launch_v1_route(const V1Params &p, int tiles, int heads, int B, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  const int d = p.d == 256 ? 256 : kHeadDim;
  const size_t smem = v1_route_smem(p.nb, d);
  if (smem > 200 * 1024) return FPX_ERR_UNSUPPORTED;
  if (d == 256) {
    cudaFuncSetAttribute(v1_route_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    v1_route_kernel<256><<<dim3(tiles, heads, B), 256, smem, s>>>(p);
  } else {
    cudaFuncSetAttribute(v1_route_kernel<kHeadDim>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    v1_route_kernel<kHeadDim><<<dim3(tiles, heads, B), 256, smem, s>>>(p);
  }
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

// ----------------------------------------------------------------------------------------
// New selectors (kernels.py:49-126), fused with their selection (kernels.py:129-151).
// One CTA per (b, h, t), thread r owns query row r of the tile. Logits of the visible
// blocks kb < t are computed in fp32 from the fp32 descriptors, staged 32 blocks at a time:
//   ell0 = (q . mean_k) * scale + ln n_kb;  u = max((q^2 . var_k) * scale^2, 0);
//   logit = ell0 (+ u / 2 for cgf / dispersion).
// Pass 1 takes the per-row log-sum-exp online, pass 2 recomputes the logits and adds
// each row's softmax weight (x sqrt(u) sigma_v for dispersion) into per-block tile sums,
// reduced across rows in a fixed order (warp shuffles, then the 4 warps in sequence).
constexpr int kSelChunk = 32;

template <int kSel, int D = kHeadDim>  // kSel: 0 mean_balanced, 1 cgf_mean, 2 dispersion_mean
__global__ void __launch_bounds__(128) selector_route_kernel(SelParams p) {
  const int t = p.tile_begin + (gridDim.x - 1 - blockIdx.x);
  const int h = p.head_begin + blockIdx.y;
  const int b = blockIdx.z;
  const int kvh = h / p.group;
  extern __shared__ __align__(16) uint8_t smem[];
  float *smk = reinterpret_cast<float *>(smem);          // [32][D]
  float *svk = smk + kSelChunk * D;                       // [32][D]
  float *part = svk + kSelChunk * D;                      // [4][32]
  float *sc = part + 4 * kSelChunk;                       // [nb]
  int *scratch = reinterpret_cast<int *>(sc + p.nb);      // [4]
  float *red = reinterpret_cast<float *>(scratch + 4);    // [4]
  float *sinfo = red + 4;                                 // [32] ln n, [32] sigma_v

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rows = min(kBlock, p.L - t * kBlock);
  const bool valid = tid < rows;
  const int pos = t * kBlock + min(tid, rows - 1);
  uint32_t qv[D / 2];
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(p.q + b * p.q_sb + (int64_t)pos * p.q_sl +
                                                       h * p.q_sh);
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      const uint4 u = src[i];
      qv[4 * i] = u.x; qv[4 * i + 1] = u.y; qv[4 * i + 2] = u.z; qv[4 * i + 3] = u.w;
    }
  }
  const float *mk_base = p.mean_k + ((int64_t)b * p.nb * p.Hkv + kvh) * D;
  const float *vk_base = p.var_k + ((int64_t)b * p.nb * p.Hkv + kvh) * D;
  const int64_t dstride = (int64_t)p.Hkv * D;
  for (int kb = tid; kb < p.nb; kb += 128) sc[kb] = 0.f;

  auto stage = [&](int c0, int cn) {
    __syncthreads();
    for (int i = tid; i < cn * (D / 4); i += 128) {
      const int j = i / (D / 4), q4 = i % (D / 4);
      reinterpret_cast<float4 *>(smk + j * D)[q4] =
          reinterpret_cast<const float4 *>(mk_base + (c0 + j) * dstride)[q4];
      if (kSel > 0)
        reinterpret_cast<float4 *>(svk + j * D)[q4] =
            reinterpret_cast<const float4 *>(vk_base + (c0 + j) * dstride)[q4];
    }
    if (tid < cn) {
      const int n = min(kBlock, p.L - (c0 + tid) * kBlock);
      sinfo[tid] = logf((float)n);
      sinfo[kSelChunk + tid] = kSel == 2 ? p.sigma_v[((int64_t)b * p.nb + c0 + tid) * p.Hkv + kvh] : 0.f;
    }
    __syncthreads();
  };
  // Logit of block j of the staged chunk (and sqrt(u) for dispersion).
  auto logit = [&](int j, float &disp) -> float {
    const float4 *m4 = reinterpret_cast<const float4 *>(smk + j * D);
    const float4 *v4 = reinterpret_cast<const float4 *>(svk + j * D);
    float dot = 0.f, udot = 0.f;
#pragma unroll
    for (int i = 0; i < D / 4; ++i) {
      const float2 qa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&qv[2 * i]));
      const float2 qb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&qv[2 * i + 1]));
      const float4 m = m4[i];
      dot = fmaf(qa.x, m.x, dot); dot = fmaf(qa.y, m.y, dot);
      dot = fmaf(qb.x, m.z, dot); dot = fmaf(qb.y, m.w, dot);
      if (kSel > 0) {
        const float4 vv = v4[i];
        udot = fmaf(qa.x * qa.x, vv.x, udot); udot = fmaf(qa.y * qa.y, vv.y, udot);
        udot = fmaf(qb.x * qb.x, vv.z, udot); udot = fmaf(qb.y * qb.y, vv.w, udot);
      }
    }
    float l = __fadd_rn(__fmul_rn(dot, p.scale), sinfo[j]);
    if (kSel > 0) {
      const float u = fmaxf(__fmul_rn(udot, p.scale2), 0.f);
      l = __fadd_rn(l, 0.5f * u);
      disp = sqrtf(u);
    }
    return l;
  };

  const int nvis = t;  // blocks kb < t
  float m = -INFINITY, ssum = 0.f;
  for (int c0 = 0; c0 < nvis; c0 += kSelChunk) {
    const int cn = min(kSelChunk, nvis - c0);
    stage(c0, cn);
    for (int j = 0; j < cn; ++j) {
      float disp;
      const float l = logit(j, disp);
      const float mn = fmaxf(m, l);
      ssum = ssum * expf(m - mn) + expf(l - mn);
      m = mn;
    }
  }
  const float lse = m + logf(ssum);
  const float inv_rows = 1.f / (float)rows;
  for (int c0 = 0; c0 < nvis; c0 += kSelChunk) {
    const int cn = min(kSelChunk, nvis - c0);
    stage(c0, cn);
    for (int j = 0; j < cn; ++j) {
      float disp = 0.f;
      const float l = logit(j, disp);
      float w = valid ? expf(l - lse) : 0.f;
      if (kSel == 2) w = w * disp * sinfo[kSelChunk + j];
      w = warp_sum(w);
      if (lane == 0) part[warp * kSelChunk + j] = w;
    }
    __syncthreads();
    if (tid < cn) {
      const float s = ((part[tid] + part[kSelChunk + tid]) + part[2 * kSelChunk + tid]) +
                      part[3 * kSelChunk + tid];
      sc[c0 + tid] = s / (float)rows;
    }
  }
  (void)inv_rows;
  __syncthreads();
  float lsmax = 0.f;
  for (int kb = tid; kb < p.nb; kb += 128) {
    lsmax = fmaxf(lsmax, sc[kb]);
    if (p.scores) p.scores[(((int64_t)b * p.nb + t) * p.nb + kb) * p.H + h] = sc[kb];
  }
  const float smax = block_max<128>(lsmax, red);
  if (p.sel.route.lists) select_and_emit<128, true>(sc, smax, p.sel, b, h, t, scratch);
}

size_t selector_route_smem(int nb, int d) {
  return (size_t)2 * kSelChunk * d * 4 + 4 * kSelChunk * 4 + (size_t)nb * 4 + 32 + 2 * kSelChunk * 4 + 64;
}

int launch_selector_route(const SelParams &p, int selector, int tiles, int heads, int B,
                          cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  const int d = p.d == 256 ? 256 : kHeadDim;
  const size_t smem = selector_route_smem(p.nb, d);
  if (smem > 200 * 1024) return FPX_ERR_UNSUPPORTED;
  dim3 grid(tiles, heads, B);
#define FPX_SEL_LAUNCH(K, DD)                                                                    \
  do {                                                                                           \
    cudaFuncSetAttribute(selector_route_kernel<K, DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                         (int)smem);                                                             \
    selector_route_kernel<K, DD><<<grid, 128, smem, s>>>(p);                                     \
  } while (0)
  if (selector == FPX_METHOD_MEAN_BALANCED) {
    if (d == 256) FPX_SEL_LAUNCH(0, 256); else FPX_SEL_LAUNCH(0, kHeadDim);
  } else if (selector == FPX_METHOD_CGF_MEAN) {
    if (d == 256) FPX_SEL_LAUNCH(1, 256); else FPX_SEL_LAUNCH(1, kHeadDim);
  } else if (selector == FPX_METHOD_DISPERSION_MEAN) {
    if (d == 256) FPX_SEL_LAUNCH(2, 256); else FPX_SEL_LAUNCH(2, kHeadDim);
  } else {
    return FPX_ERR_INVALID;
  }
#undef FPX_SEL_LAUNCH
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

// ----------------------------------------------------------------------------------------
// All-causal routing (method "dense", and alpha == 0 for the new selectors,
// kernels.py:141-142): list = 0..t, no tail.
__global__ void __launch_bounds__(128) causal_route_kernel(RouteView r, int H, int head_begin,
                                                           int tile_begin) {
  const int t = tile_begin + blockIdx.x, h = head_begin + blockIdx.y, b = blockIdx.z;
  const int64_t rrow = r.row(b, h, t, H);
  for (int kb = threadIdx.x; kb <= t; kb += blockDim.x) r.lists[rrow * r.nb + kb] = kb;
  for (int w = threadIdx.x; w < r.words; w += blockDim.x) r.tail[rrow * r.words + w] = 0u;
  if (threadIdx.x == 0) r.counts[rrow] = t + 1;
}

int launch_causal_route(const RouteView &r, int H, int head_begin, int heads, int tile_begin,
                        int tiles, int B, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  causal_route_kernel<<<dim3(tiles, heads, B), 128, 0, s>>>(r, H, head_begin, tile_begin);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

// ----------------------------------------------------------------------------------------
// Reference-layout selection: one CTA per (b, t, h) column of [B, nb, nb, H] scores.
// mode 0: deal_output_score (upstream:366-385) -> int64 indices (sentinel nb) + counts;
// mode 1: protected_selection (kernels.py:137-151) -> uint8 mask.
// For min_budget > 0 an entry is in the top-k when fewer than k entries beat it, a tie
// going to the lower block id.
__global__ void __launch_bounds__(256) column_select_kernel(ColumnSelectParams p) {
  const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  extern __shared__ __align__(16) uint8_t smem[];
  float *sc = reinterpret_cast<float *>(smem);
  int *scratch = reinterpret_cast<int *>(sc + p.nb);
  float *red = reinterpret_cast<float *>(scratch + 8);
  const int tid = threadIdx.x;
  const int64_t col = ((int64_t)b * p.nb + t) * p.nb * p.H + h;
  float lmax = -INFINITY;
  for (int kb = tid; kb < p.nb; kb += 256) {
    const float s = p.scores[col + (int64_t)kb * p.H];
    sc[kb] = s;
    lmax = fmaxf(lmax, s);
  }
  const float smax = block_max<256>(lmax, red);
  const float thr = smax * p.alpha;
  int base = 0;
  for (int c0 = 0; c0 < p.nb; c0 += 256) {
    const int kb = c0 + tid;
    bool active = false;
    if (kb < p.nb) {
      const float s = sc[kb];
      bool keep;
      if (p.mode == 1) {
        keep = p.all_causal || (s > 0.f && s >= thr);
      } else if (p.min_budget > 0) {
        int rank = 0;
        for (int j = 0; j < p.nb; ++j) {
          const float o = sc[j];
          rank += (o > s || (o == s && j < kb)) ? 1 : 0;
        }
        keep = s >= thr || rank < p.min_budget;
      } else {
        keep = s >= thr;
      }
      active = kb <= t && (keep || (!p.all_causal && is_protected(t, kb, p.nb, p.sink, p.window,
                                                                  p.last_full)));
      if (p.mode == 1) p.mask[col + (int64_t)kb * p.H] = active ? 1 : 0;
    }
    int total;
    const int pos = block_exclusive_scan<256>(active ? 1 : 0, scratch, &total);
    if (p.mode == 0 && active) p.indices[col + (int64_t)(base + pos) * p.H] = kb;
    base += total;
  }
  if (p.mode == 0) {
    for (int j = base + tid; j < p.nb; j += 256) p.indices[col + (int64_t)j * p.H] = p.nb;
    if (tid == 0) p.counts[((int64_t)b * p.nb + t) * p.H + h] = base;
  }
}

int launch_column_select(const ColumnSelectParams &p, int B, cudaStream_t s) {
  const size_t smem = (size_t)p.nb * 4 + 64;
  if (smem > 200 * 1024) return FPX_ERR_UNSUPPORTED;
  cudaFuncSetAttribute(column_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  column_select_kernel<<<dim3(p.nb, p.H, B), 256, smem, s>>>(p);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

// indices_from_mask (kernels.py:154-160): one CTA per (b, t, h) column.
__global__ void __launch_bounds__(256) mask_to_indices_kernel(const uint8_t *mask, int nb, int H,
                                                              int64_t *indices, int32_t *counts) {
  const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  __shared__ int scratch[8];
  const int64_t col = ((int64_t)b * nb + t) * nb * H + h;
  int base = 0;
  for (int c0 = 0; c0 < nb; c0 += 256) {
    const int kb = c0 + threadIdx.x;
    const bool active = kb < nb && mask[col + (int64_t)kb * H] != 0;
    int total;
    const int pos = block_exclusive_scan<256>(active ? 1 : 0, scratch, &total);
    if (active) indices[col + (int64_t)(base + pos) * H] = kb;
    base += total;
  }
  for (int j = base + threadIdx.x; j < nb; j += 256) indices[col + (int64_t)j * H] = nb;
  if (threadIdx.x == 0) counts[((int64_t)b * nb + t) * H + h] = base;
}

// mask_from_indices (kernels.py:163-176): entries past the count never set a bit.
__global__ void mask_from_indices_kernel(const int64_t *indices, const int32_t *counts, int nb,
                                         int H, int64_t total, uint8_t *mask) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int h = (int)(i % H);
    const int64_t rest = i / H;
    const int pos = (int)(rest % nb);
    const int64_t bt = rest / nb;  // b * nb + t
    if (pos < counts[bt * H + h]) {
      const int64_t kb = indices[i];
      if (kb >= 0 && kb < nb) mask[(bt * nb + kb) * H + h] = 1;
    }
  }
}

// Internal lists -> reference layouts, for the heads / tiles the last prefill routed.
__global__ void __launch_bounds__(128) export_routing_kernel(RouteView r, int H, uint8_t *mask,
                                                             int64_t *indices, int32_t *counts) {
  const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int64_t rrow = r.row(b, h, t, H);
  // Clamped: a workspace whose routing was cut short by a failed launch holds stale values.
  const int cnt = min(max(r.counts[rrow], 0), r.nb);
  const int64_t col = ((int64_t)b * r.nb + t) * r.nb * H + h;
  const int32_t *list = r.lists + rrow * r.nb;
  for (int j = threadIdx.x; j < r.nb; j += blockDim.x) {
    const int kb = j < cnt ? list[j] : r.nb;
    const bool valid = kb >= 0 && kb < r.nb;
    if (indices) indices[col + (int64_t)j * H] = valid ? kb : r.nb;
    if (mask && valid) mask[col + (int64_t)kb * H] = 1;
  }
  if (counts && threadIdx.x == 0) counts[((int64_t)b * r.nb + t) * H + h] = cnt;
}

int launch_export_routing(const RouteView &r, int H, int B, uint8_t *mask, int64_t *indices,
                          int32_t *counts, cudaStream_t s) {
  export_routing_kernel<<<dim3(r.nb, H, B), 128, 0, s>>>(r, H, mask, indices, counts);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

// selection_accounting (kernels.py:328-407) integer counters over a [B, nb, nb, H] mask.
__global__ void accounting_kernel(const uint8_t *mask, int nb, int H, int L, int64_t total,
                                  unsigned long long *counters) {
  unsigned long long pairs = 0, blocks = 0, proxy = 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t rest = i / H;
    const int kb = (int)(rest % nb);
    const int t = (int)((rest / nb) % nb);
    const long long nq = min(kBlock, L - t * kBlock), nk = min(kBlock, L - kb * kBlock);
    if (mask[i]) {
      blocks += 1;
      if (kb < t) pairs += nq * nk;
      else if (kb == t) pairs += nq * (nq + 1) / 2;
    } else if (kb < t) {
      proxy += nq;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    pairs += __shfl_xor_sync(0xffffffffu, pairs, o);
    blocks += __shfl_xor_sync(0xffffffffu, blocks, o);
    proxy += __shfl_xor_sync(0xffffffffu, proxy, o);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(counters + 0, pairs);
    atomicAdd(counters + 1, blocks);
    atomicAdd(counters + 2, proxy);
  }
}

}  // namespace fpx

// ---------------------------------------------------------------------------------------------
// C ABI wrappers for the standalone routing ops.
using namespace fpx;

static bool stride_ok(int64_t sb, int64_t sl, int64_t sh) {
  return sb % 8 == 0 && sl % 8 == 0 && sh % 8 == 0;
}
static bool ptr_ok(const void *p) { return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int fpx_block_mean_k(const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh, int B,
                                int L, int Hkv, int d, int block, void *mean_k,
                                fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!k || !mean_k || B <= 0 || L <= 0 || Hkv <= 0) return FPX_ERR_INVALID;
  if ((d != kHeadDim && d != 256) || block != kBlock) return FPX_ERR_UNSUPPORTED;
  StatsParams p{};
  p.d = d;
  p.k = static_cast<const __nv_bfloat16 *>(k);
  p.k_sb = k_sb; p.k_sl = k_sl; p.k_sh = k_sh;
  p.v = p.k; p.v_sb = k_sb; p.v_sl = k_sl; p.v_sh = k_sh;
  p.L = L; p.nb = (L + kBlock - 1) / kBlock; p.Hkv = Hkv; p.kv_begin = 0;
  p.mean_bf16 = static_cast<__nv_bfloat16 *>(mean_k);
  return launch_block_stats(p, p.nb, Hkv, B, true, false, stream);
}

extern "C" int fpx_block_descriptors(const void *k, int64_t k_sb, int64_t k_sl, int64_t k_sh,
                                     const void *v, int64_t v_sb, int64_t v_sl, int64_t v_sh,
                                     int B, int L, int Hkv, int d, int block, float *mean_k,
                                     float *mean_v, float *var_k, float *sigma_v, int32_t *counts,
                                     fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!k || !v || !mean_k || !mean_v || !var_k || !sigma_v || B <= 0 || L <= 0 || Hkv <= 0)
    return FPX_ERR_INVALID;
  if ((d != kHeadDim && d != 256) || block != kBlock) return FPX_ERR_UNSUPPORTED;
  StatsParams p{};
  p.d = d;
  p.k = static_cast<const __nv_bfloat16 *>(k);
  p.k_sb = k_sb; p.k_sl = k_sl; p.k_sh = k_sh;
  p.v = static_cast<const __nv_bfloat16 *>(v);
  p.v_sb = v_sb; p.v_sl = v_sl; p.v_sh = v_sh;
  p.L = L; p.nb = (L + kBlock - 1) / kBlock; p.Hkv = Hkv; p.kv_begin = 0;
  p.mean_k = mean_k; p.mean_v = mean_v; p.var_k = var_k; p.sigma_v = sigma_v; p.counts = counts;
  return launch_block_stats(p, p.nb, Hkv, B, false, true, stream);
}

extern "C" int fpx_v1_scores(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                             const void *mean_k, int B, int L, int H, int Hkv, int d, int block,
                             double scale, float *scores, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!ptr_ok(q) || !ptr_ok(mean_k) || !scores || B <= 0 || L <= 0 || H <= 0 || Hkv <= 0)
    return FPX_ERR_INVALID;
  if ((d != kHeadDim && d != 256) || block != kBlock) return FPX_ERR_UNSUPPORTED;
  if (H % Hkv || !stride_ok(q_sb, q_sl, q_sh)) return FPX_ERR_SHAPE;
  V1Params p{};
  p.d = d;
  p.q = static_cast<const __nv_bfloat16 *>(q);
  p.q_sb = q_sb; p.q_sl = q_sl; p.q_sh = q_sh;
  p.mean_k = static_cast<const __nv_bfloat16 *>(mean_k);
  p.L = L; p.nb = (L + kBlock - 1) / kBlock; p.H = H; p.Hkv = Hkv; p.group = H / Hkv;
  p.scale_log2 = (float)scale * kLog2e;
  p.scores = scores;
  return launch_v1_route_selected(p, p.nb, H, B, stream);
}

extern "C" int fpx_selector_scores(const void *q, int64_t q_sb, int64_t q_sl, int64_t q_sh,
                                   const float *mean_k, const float *var_k, const float *sigma_v,
                                   const int32_t *counts, int B, int L, int H, int Hkv, int d,
                                   int block, int selector, double scale, float *scores,
                                   fpx_stream_t stream) {
  FPX_BIND(stream);
  (void)counts;  // n_kb follows from L; the reference's counts hold the same values
  if (!ptr_ok(q) || !mean_k || !var_k || !sigma_v || !scores || B <= 0 || L <= 0 || H <= 0 ||
      Hkv <= 0)
    return FPX_ERR_INVALID;
  if ((d != kHeadDim && d != 256) || block != kBlock) return FPX_ERR_UNSUPPORTED;
  if (selector < FPX_METHOD_MEAN_BALANCED || selector > FPX_METHOD_DISPERSION_MEAN)
    return FPX_ERR_INVALID;
  if (H % Hkv || !stride_ok(q_sb, q_sl, q_sh)) return FPX_ERR_SHAPE;
  SelParams p{};
  p.q = static_cast<const __nv_bfloat16 *>(q);
  p.q_sb = q_sb; p.q_sl = q_sl; p.q_sh = q_sh;
  p.mean_k = mean_k; p.var_k = var_k; p.sigma_v = sigma_v;
  p.L = L; p.nb = (L + kBlock - 1) / kBlock; p.H = H; p.Hkv = Hkv; p.group = H / Hkv;
  p.scale = (float)scale; p.scale2 = (float)(scale * scale);
  p.scores = scores;
  p.d = d;
  return launch_selector_route(p, selector, p.nb, H, B, stream);
}

extern "C" int fpx_deal_output_score(const float *scores, int B, int nb, int H, int sink,
                                     int window, double alpha, int last_full, int min_budget,
                                     int64_t *indices, int32_t *counts, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!scores || !indices || !counts || B <= 0 || nb <= 0 || H <= 0 || min_budget < 0)
    return FPX_ERR_INVALID;
  if (min_budget > nb) return FPX_ERR_SHAPE;
  ColumnSelectParams p{};
  p.scores = scores; p.nb = nb; p.H = H; p.sink = sink; p.window = window;
  p.last_full = last_full; p.alpha = (float)alpha; p.min_budget = min_budget;
  p.mode = 0; p.indices = indices; p.counts = counts;
  return launch_column_select(p, B, stream);
}

extern "C" int fpx_protected_selection(const float *scores, int B, int nb, int H, double alpha,
                                       int sink, int window, int last_full, uint8_t *selected,
                                       fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!scores || !selected || B <= 0 || nb <= 0 || H <= 0) return FPX_ERR_INVALID;
  ColumnSelectParams p{};
  p.scores = scores; p.nb = nb; p.H = H; p.sink = sink; p.window = window;
  p.last_full = last_full; p.alpha = (float)alpha; p.all_causal = alpha == 0.0;
  p.mode = 1; p.mask = selected;
  return launch_column_select(p, B, stream);
}

extern "C" int fpx_indices_from_mask(const uint8_t *selected, int B, int nb, int H,
                                     int64_t *indices, int32_t *counts, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!selected || !indices || !counts || B <= 0 || nb <= 0 || H <= 0) return FPX_ERR_INVALID;
  mask_to_indices_kernel<<<dim3(nb, H, B), 256, 0, stream>>>(selected, nb, H, indices, counts);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

extern "C" int fpx_mask_from_indices(const int64_t *indices, const int32_t *counts, int B, int nb,
                                     int H, uint8_t *selected, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!indices || !counts || !selected || B <= 0 || nb <= 0 || H <= 0) return FPX_ERR_INVALID;
  const int64_t total = (int64_t)B * nb * nb * H;
  if (cudaMemsetAsync(selected, 0, (size_t)total, stream) != cudaSuccess) return FPX_ERR_CUDA;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
  mask_from_indices_kernel<<<grid, 256, 0, stream>>>(indices, counts, nb, H, total, selected);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

extern "C" int fpx_selection_accounting(const uint8_t *selected, int B, int nb, int H, int L,
                                        int block, int64_t *counters, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!selected || !counters || B <= 0 || nb <= 0 || H <= 0 || L <= 0) return FPX_ERR_INVALID;
  if (block != kBlock) return FPX_ERR_UNSUPPORTED;
  if ((L + kBlock - 1) / kBlock != nb) return FPX_ERR_SHAPE;
  if (cudaMemsetAsync(counters, 0, 3 * sizeof(int64_t), stream) != cudaSuccess) return FPX_ERR_CUDA;
  const int64_t total = (int64_t)B * nb * nb * H;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
  accounting_kernel<<<grid, 256, 0, stream>>>(selected, nb, H, L, total,
                                              reinterpret_cast<unsigned long long *>(counters));
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}
