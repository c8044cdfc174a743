// Rescue tails of fp_v1_rescue / fp_v1_rescue_v2 on the tcgen05 tensor core, merged into the
// exact output in place (the fused path).
//
// Reference: kernels.py:233-309 (rescue_tail) and kernels.py:312-325 (merge_exact_mean). For
// query tile t of head h every tail block kb < t (unselected) contributes its rescue token,
// the key row chosen by rescue_choice_kernel (rescue.cu), with weight 1; fp_v1_rescue_v2 also
// adds the block's other 127 tokens through their mean, K_rest = (sum K - k_rescue) / 127
// (likewise V), with logit offset ln 127. Tail blocks are full, so sum K = 128 x mean_k exactly.
// The tail's softmax output and LSE are merged with the exact path's by logaddexp.
//
// One CTA of 128 threads per (b, h, t) with a tail; thread r owns query row r (TMEM lane r).
// The tail blocks are compacted into a list and processed as chunks of up to 128 key slots:
//   1. the 128 threads gather the chunk's keys into a 128-byte-swizzled K tile (slot j = row j):
//      rescue rows as bf16 (exact), or for the remainder pass K_rest as bf16 high + low
//      halves (hi = bf16(x), lo = bf16(x - hi)), and the values into a V tile (bf16 rows, or
//      bf16(V_rest));
//   2. one thread issues S = Q K^T (Q loaded once by TMA) into TMEM and commits to an
//      mbarrier; the remainder pass writes the low halves into the same tile afterwards and
//      accumulates Q K_lo^T, so one K tile serves both (96 KB: two CTAs per SM);
//   3. each thread reads its row of S, masks the empty slots, runs the online softmax in exp2
//      units and writes P (bf16) over S;
//   4. one thread issues O += P V and commits; the next chunk starts when it is done.
// Chunks run one after another (rescue chunks, then for _v2 the remainder chunks), each
// product tiny next to the gathers, so a serial protocol suffices. TMEM: S [0,128), O [128,256).
// Every wait is bounded (about 1 s); a wait that gives up sets the device error word and the
// CTA leaves the exact output as it was.
#include <cuda.h>

#include "attn.cuh"
#include "tc.cuh"

namespace fpx {
namespace {

using namespace tc;

constexpr uint32_t kHalfR = 128 * 128;   // 128 rows x 64 bf16: one SW128 atom column
constexpr uint32_t kTileR = 2 * kHalfR;  // 128 x 128 bf16
constexpr uint32_t kIdescQKR = idesc_bf16(128, 128, false);
constexpr uint32_t kIdescPVR = idesc_bf16(128, 128, true);
constexpr int kMaxBlocksR = 2048;
constexpr float kLog2Of127 = 6.988684686772166f;

template <int kKeys>
struct alignas(1024) SmemR {
  uint8_t q[kTileR];
  uint8_t k[kTileR];  // keys: rescue rows, or K_rest's high then low halves
  uint8_t v[kTileR];
  uint64_t q_full, mma;
  uint32_t tmem_base;
  int abort, ntail;
  int scratch[8];
  uint16_t list[kMaxBlocksR];
};

FPX_INLINE uint64_t desc_kmR(const uint8_t *tile, int kk) {
  return smem_desc_sw128(smem_u32(tile) + (kk >> 2) * kHalfR + (kk & 3) * 32, 16, 1024);
}
FPX_INLINE uint64_t desc_vR(const uint8_t *tile, int kk) {
  return smem_desc_sw128(smem_u32(tile) + kk * 2048, kHalfR, 1024);
}
// Byte offset of the 16-byte chunk ch (columns 8 ch .. 8 ch + 7) of row j in a SW128 tile.
FPX_INLINE uint32_t chunk_offset(int j, int ch) {
  return (ch >> 3) * kHalfR + j * 128 + (((ch & 7) ^ (j & 7)) << 4);
}

}  // namespace

template <int kKeys>
__global__ void __launch_bounds__(128) rescue_tail_tc_kernel(const __grid_constant__ CUtensorMap tm_q, MeanParams p,
                                                             float scale_log2, int *err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  SmemR<kKeys> &sh = *reinterpret_cast<SmemR<kKeys> *>(smem_raw + pad);
  volatile int *abort = &sh.abort;
  const int t = p.tile_begin + (gridDim.x - 1 - blockIdx.x);
  const int h = p.head_begin + blockIdx.y;
  const int b = blockIdx.z;
  const int kvh = h / p.group;
  const int tid = threadIdx.x, warp = tid >> 5;
  if (err && *reinterpret_cast<volatile int *>(err) != 0) return;

  // Ascending list of the tail blocks of (b, h, t).
  {
    const uint32_t *bits = p.route.tail + p.route.row(b, h, t, p.H) * p.route.words;
    int n = 0;
    for (int w0 = 0; w0 < p.route.words; w0 += 128) {
      const int w = w0 + tid;
      const uint32_t word = w < p.route.words ? bits[w] : 0u;
      int total;
      int pos = block_exclusive_scan<128>(__popc(word), sh.scratch, &total);
      for (uint32_t x = word; x; x &= x - 1) {
        const int kb = 32 * w + __ffs(x) - 1;
        if (n + pos < kMaxBlocksR) sh.list[n + pos] = (uint16_t)kb;
        ++pos;
      }
      n += total;
    }
    if (tid == 0) sh.ntail = min(n, kMaxBlocksR);
  }
  __syncthreads();
  const int ntail = sh.ntail;
  if (ntail == 0) return;  // nothing to merge (uniform across the CTA)

  if (tid == 0) {
    mbar_init(&sh.q_full, 1);
    mbar_init(&sh.mma, 1);
    sh.abort = 0;
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&sh.tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  if (tid == 0) {
    mbar_expect_tx(&sh.q_full, kTileR);
    tma_load_4d(sh.q, &tm_q, &sh.q_full, 0, h, t * 128, b);
    tma_load_4d(sh.q + kHalfR, &tm_q, &sh.q_full, 64, h, t * 128, b);
  }

  const int r = tid;
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  const uint32_t s_addr = tmem + lane_off, o_addr = tmem + lane_off + 128;
  const uint8_t *choice = p.choice + (((int64_t)b * p.H + h) * p.nb + t) * p.nb;
  const int64_t dstride = (int64_t)p.Hkv * kHeadDim;
  const float *mk_base = p.mean_k + ((int64_t)b * p.nb * p.Hkv + kvh) * kHeadDim;
  const float *mv_base = p.mean_v + ((int64_t)b * p.nb * p.Hkv + kvh) * kHeadDim;
  const int per_pass = (ntail + 127) / 128;
  const int chunks = kKeys == 2 ? 2 * per_pass : per_pass;
  float m = -INFINITY, l = 0.f;
  bool ok = mbar_wait(&sh.q_full, 0, abort);
  int phase = 0;
  for (int c = 0; c < chunks && ok; ++c) {
    const bool rest = kKeys == 2 && c >= per_pass;
    const int c0 = (rest ? c - per_pass : c) * 128;
    const int nc = min(128, ntail - c0);
    // 1-2. gather, then S = Q K^T. The remainder pass runs it twice through the one K tile:
    // part 0 writes K_rest's high halves (and V_rest), part 1 its low halves, accumulated into
    // S; thread j keeps its slot's low halves in registers from part 0.
    const int parts = rest ? 2 : 1;
    uint32_t klo[64];  // the remainder pass: K_rest's low halves, kept from part 0 for part 1
    for (int part = 0; part < parts && ok; ++part) {
      const int j = tid;
      if (j < nc) {
        const int kb = sh.list[c0 + j];
        const int64_t tok = (int64_t)kb * kBlock + (choice[kb] & (kBlock - 1));
        const uint4 *krow = reinterpret_cast<const uint4 *>(p.k + b * p.k_sb + tok * p.k_sl + kvh * p.k_sh);
        const uint4 *vrow = reinterpret_cast<const uint4 *>(p.v + b * p.v_sb + tok * p.v_sl + kvh * p.v_sh);
        if (rest && part == 1) {
#pragma unroll
          for (int ch = 0; ch < 16; ++ch)
            *reinterpret_cast<uint4 *>(sh.k + chunk_offset(j, ch)) =
                make_uint4(klo[4 * ch], klo[4 * ch + 1], klo[4 * ch + 2], klo[4 * ch + 3]);
        } else if (rest) {
          // (sum - rescue) / 127 with sum = 128 x mean (exact): the remainder's mean K / V
          const float4 *mk4 = reinterpret_cast<const float4 *>(mk_base + kb * dstride);
          const float4 *mv4 = reinterpret_cast<const float4 *>(mv_base + kb * dstride);
          auto rest_of = [](float mean, float x) { return __fdiv_rn(__fsub_rn(__fmul_rn(mean, 128.f), x), 127.f); };
#pragma unroll
          for (int ch = 0; ch < 16; ++ch) {
            const uint4 ku = krow[ch];
            const float4 ma = mk4[2 * ch], mb = mk4[2 * ch + 1];
            const uint32_t kw[4] = {ku.x, ku.y, ku.z, ku.w};
            const float mkv[8] = {ma.x, ma.y, ma.z, ma.w, mb.x, mb.y, mb.z, mb.w};
            uint32_t kout[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 kx = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&kw[e]));
              const float r0 = rest_of(mkv[2 * e], kx.x), r1 = rest_of(mkv[2 * e + 1], kx.y);
              const float h0 = __bfloat162float(__float2bfloat16_rn(r0)), h1 = __bfloat162float(__float2bfloat16_rn(r1));
              kout[e] = pack_bf16(h0, h1);
              klo[4 * ch + e] = pack_bf16(__fsub_rn(r0, h0), __fsub_rn(r1, h1));
            }
            *reinterpret_cast<uint4 *>(sh.k + chunk_offset(j, ch)) = make_uint4(kout[0], kout[1], kout[2], kout[3]);
            {
              const uint4 vu = vrow[ch];
              const float4 va = mv4[2 * ch], vb = mv4[2 * ch + 1];
              const uint32_t vw[4] = {vu.x, vu.y, vu.z, vu.w};
              const float mvv[8] = {va.x, va.y, va.z, va.w, vb.x, vb.y, vb.z, vb.w};
              uint32_t vo[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 vx = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&vw[e]));
                vo[e] = pack_bf16(rest_of(mvv[2 * e], vx.x), rest_of(mvv[2 * e + 1], vx.y));
              }
              *reinterpret_cast<uint4 *>(sh.v + chunk_offset(j, ch)) = make_uint4(vo[0], vo[1], vo[2], vo[3]);
            }
          }
        } else {
          uint4 kv[16], vv[16];
#pragma unroll
          for (int ch = 0; ch < 16; ++ch) {
            kv[ch] = krow[ch];
            vv[ch] = vrow[ch];
          }
#pragma unroll
          for (int ch = 0; ch < 16; ++ch) {
            *reinterpret_cast<uint4 *>(sh.k + chunk_offset(j, ch)) = kv[ch];
            *reinterpret_cast<uint4 *>(sh.v + chunk_offset(j, ch)) = vv[ch];
          }
        }
      } else {
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          *reinterpret_cast<uint4 *>(sh.k + chunk_offset(j, ch)) = z;
          if (part == 0) *reinterpret_cast<uint4 *>(sh.v + chunk_offset(j, ch)) = z;
        }
      }
      fence_proxy_async();  // the tensor core reads what the threads wrote
      tc_fence_before();
      __syncthreads();
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          mma_ss(tmem, desc_kmR(sh.q, kk), desc_kmR(sh.k, kk), kIdescQKR, (part > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&sh.mma);
      }
      __syncwarp();
      if (!(ok = mbar_wait_warp(&sh.mma, phase & 1, abort))) break;
      ++phase;
      tc_fence_after();
    }
    if (!ok) break;
    // 3. online softmax of row r over the chunk's slots; P (bf16) over S
    {
      float sv[128];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) tmem_ld32(s_addr + 32 * cc, *reinterpret_cast<float(*)[32]>(&sv[32 * cc]));
      tmem_wait_ld();
      const float off = rest ? kLog2Of127 : 0.f;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 128; ++j) {
        sv[j] = j < nc ? fmaf(sv[j], scale_log2, off) : -INFINITY;
        mx = fmaxf(mx, sv[j]);
      }
      const float mn = fmaxf(m, mx);
      const float corr = (m == -INFINITY) ? 0.f : ex2(m - mn);
      l *= corr;
      m = mn;
      float sum = 0.f;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float a = ex2(sv[32 * q4 + 2 * e] - m), d = ex2(sv[32 * q4 + 2 * e + 1] - m);
          sum += a + d;
          pk[e] = pack_bf16(a, d);
        }
        tmem_st16u(s_addr + 16 * q4, pk);
      }
      l += sum;
      if (c > 0 && __any_sync(0xffffffffu, corr != 1.f)) {  // O holds the earlier chunks
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          float o[32];
          tmem_ld32(o_addr + 32 * cc, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] *= corr;
          tmem_st32(o_addr + 32 * cc, o);
        }
      }
      tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    // 4. O += P V
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        mma_ts(tmem + 128, tmem + 8 * kk, desc_vR(sh.v, kk), kIdescPVR, (c > 0 || kk > 0) ? 1u : 0u);
      tc_commit(&sh.mma);
    }
    __syncwarp();
    if (!(ok = mbar_wait_warp(&sh.mma, phase & 1, abort))) break;
    ++phase;
    tc_fence_after();
  }
  // Merge with the exact output row (kernels.py:318-325), in place.
  ok = __syncthreads_and(ok);
  const int rows = min(kBlock, p.L - t * kBlock);
  if (ok && r < rows) {
    float o[128];
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) tmem_ld32(o_addr + 32 * cc, *reinterpret_cast<float(*)[32]>(&o[32 * cc]));
    tmem_wait_ld();
    const int pos = t * kBlock + r;
    const int64_t lrow = ((int64_t)b * p.L + pos) * p.H + h;
    const float lse_m = m * kLn2 + logf(l);
    const float inv = 1.f / l;
    const float lse_e = p.lse[lrow];
    const float total = logaddexp(lse_e, lse_m);
    const float we = expf(lse_e - total), wm = expf(lse_m - total);
    uint4 *dst = reinterpret_cast<uint4 *>(p.out + b * p.o_sb + (int64_t)pos * p.o_sl + h * p.o_sh);
#pragma unroll
    for (int ch = 0; ch < 16; ++ch) {
      const uint4 u = dst[ch];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      uint32_t res[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[e]));
        res[e] = pack_bf16(x.x * we + o[8 * ch + 2 * e] * inv * wm, x.y * we + o[8 * ch + 2 * e + 1] * inv * wm);
      }
      dst[ch] = make_uint4(res[0], res[1], res[2], res[3]);
    }
    p.lse[lrow] = total;
  } else if (r < rows) {
    // nothing: the exact output stays as it was
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && sh.abort && err) atomicExch(err, 1);
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

int launch_rescue_tail_tc(const MeanParams &p, int keys, int B, int L, int tiles, int heads, cudaStream_t s) {
  if (tiles <= 0 || heads <= 0) return FPX_OK;
  if ((keys != 1 && keys != 2) || !p.choice || !p.k || !p.v || !p.mean_k || !p.mean_v || !p.lse)
    return FPX_ERR_INVALID;
  if (p.nb > kMaxBlocksR) return FPX_ERR_UNSUPPORTED;
  CUtensorMap tq;
  if (!encode_4d(&tq, p.q, kHeadDim, p.H, L, B, p.q_sh, p.q_sl, p.q_sb)) return FPX_ERR_INVALID;
  const dim3 grid(tiles, heads, B);
  int *err = device_error_word();
  const float sl2 = p.scale * kLog2e;
  if (keys == 1) {
    const size_t smem = sizeof(SmemR<1>) + 1024;
    cudaFuncSetAttribute(rescue_tail_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    rescue_tail_tc_kernel<1><<<grid, 128, smem, s>>>(tq, p, sl2, err);
  } else {
    const size_t smem = sizeof(SmemR<2>) + 1024;
    cudaFuncSetAttribute(rescue_tail_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    rescue_tail_tc_kernel<2><<<grid, 128, smem, s>>>(tq, p, sl2, err);
  }
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

}  // namespace fpx
