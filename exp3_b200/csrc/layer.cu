// Elementwise pieces of the Qwen2 decoder layer around the attention path: residual add +
// RMSNorm, NeoX rotary embedding, and the SwiGLU activation. They follow the rounding points of
// HF transformers' Qwen2 modules (the model exp3 drives, evaluate.py:610-617), so the prefill
// matches an HF model with the same weights to bf16 noise:
//   Qwen2RMSNorm: fp32 mean of squares, x * rsqrt(var + eps), cast to bf16, times the weight;
//   apply_rotary_pos_emb: cos / sin cast to bf16, q * cos + rotate_half(q) * sin in bf16;
//   Qwen2MLP: silu(gate) in bf16, times up in bf16.
#include <algorithm>

#include "common.cuh"

namespace fpx {

// One CTA per row; hidden <= 8192, a multiple of 8.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16 *x, const __nv_bfloat16 *residual,
                                                      const __nv_bfloat16 *weight, float eps, int hidden,
                                                      __nv_bfloat16 *out, __nv_bfloat16 *residual_out) {
  extern __shared__ __align__(16) uint8_t smem[];
  __nv_bfloat16 *row = reinterpret_cast<__nv_bfloat16 *>(smem);
  __shared__ float red[8];
  const int64_t base = (int64_t)blockIdx.x * hidden;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < hidden; c += 256 * 8) {
    uint4 xv = *reinterpret_cast<const uint4 *>(x + base + c);
    __nv_bfloat16 *xe = reinterpret_cast<__nv_bfloat16 *>(&xv);
    if (residual) {
      const uint4 rv = *reinterpret_cast<const uint4 *>(residual + base + c);
      const __nv_bfloat16 *re = reinterpret_cast<const __nv_bfloat16 *>(&rv);
#pragma unroll
      for (int e = 0; e < 8; ++e) xe[e] = __float2bfloat16_rn(__bfloat162float(re[e]) + __bfloat162float(xe[e]));
      if (residual_out) *reinterpret_cast<uint4 *>(residual_out + base + c) = xv;
    }
    *reinterpret_cast<uint4 *>(row + c) = xv;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float f = __bfloat162float(xe[e]);
      ss = fmaf(f, f, ss);
    }
  }
  const float total = block_sum<256>(ss, red);
  const float inv = rsqrtf(total / (float)hidden + eps);
  for (int c = threadIdx.x * 8; c < hidden; c += 256 * 8) {
    const uint4 xv = *reinterpret_cast<const uint4 *>(row + c);
    const uint4 wv = *reinterpret_cast<const uint4 *>(weight + c);
    const __nv_bfloat16 *xe = reinterpret_cast<const __nv_bfloat16 *>(&xv);
    const __nv_bfloat16 *we = reinterpret_cast<const __nv_bfloat16 *>(&wv);
    uint4 ov;
    __nv_bfloat16 *oe = reinterpret_cast<__nv_bfloat16 *>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const __nv_bfloat16 normed = __float2bfloat16_rn(__bfloat162float(xe[e]) * inv);
      oe[e] = __float2bfloat16_rn(__bfloat162float(we[e]) * __bfloat162float(normed));
    }
    *reinterpret_cast<uint4 *>(out + base + c) = ov;
  }
}

// In place on a strided [B, L, heads, 128] view; position of row l = pos0 + l.
// inv_freq[i] = theta^(-2i/128) is precomputed in fp32 on the host (as HF does).
struct RopeParams {
  __nv_bfloat16 *x;
  int64_t sb, sl, sh;
  int64_t n;  // B * L * heads * 64 threads of work
  int L, heads;
  int pos0;
  const int32_t *pos_dev;  // if set, the position of row 0 is read here (CUDA-graph replays)
  float inv_freq[64];
};

__global__ void __launch_bounds__(256) rope_kernel(RopeParams p) {
  // thread = (row l, head, frequency i); pairs (i, i + 64) rotate together
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= p.n) return;
  const int i = idx & 63;
  const int64_t rest = idx >> 6;
  const int h = (int)(rest % p.heads);
  const int64_t bl = rest / p.heads;
  const int l = (int)(bl % p.L);
  const int b = (int)(bl / p.L);
  const float ang = (float)((p.pos_dev ? *p.pos_dev : p.pos0) + l) * p.inv_freq[i];
  const float c = __bfloat162float(__float2bfloat16_rn(cosf(ang)));
  const float s = __bfloat162float(__float2bfloat16_rn(sinf(ang)));
  __nv_bfloat16 *v = p.x + b * p.sb + (int64_t)l * p.sl + (int64_t)h * p.sh;
  const float x1 = __bfloat162float(v[i]), x2 = __bfloat162float(v[i + 64]);
  // rotate_half(x) = [-x2, x1]
  const float y1 = __bfloat162float(__float2bfloat16_rn(x1 * c)) + __bfloat162float(__float2bfloat16_rn(-x2 * s));
  const float y2 = __bfloat162float(__float2bfloat16_rn(x2 * c)) + __bfloat162float(__float2bfloat16_rn(x1 * s));
  v[i] = __float2bfloat16_rn(y1);
  v[i + 64] = __float2bfloat16_rn(y2);
}

// out[r, j] = silu(gu[r, j]) * gu[r, inter + j], bf16 rounding after silu and after the product.
__global__ void silu_mul_kernel(const __nv_bfloat16 *gu, int64_t rows, int inter, __nv_bfloat16 *out) {
  const int64_t n = rows * (int64_t)(inter / 8);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (inter / 8);
    const int j = (int)(i % (inter / 8)) * 8;
    const uint4 gv = *reinterpret_cast<const uint4 *>(gu + r * 2 * inter + j);
    const uint4 uv = *reinterpret_cast<const uint4 *>(gu + r * 2 * inter + inter + j);
    const __nv_bfloat16 *ge = reinterpret_cast<const __nv_bfloat16 *>(&gv);
    const __nv_bfloat16 *ue = reinterpret_cast<const __nv_bfloat16 *>(&uv);
    uint4 ov;
    __nv_bfloat16 *oe = reinterpret_cast<__nv_bfloat16 *>(&ov);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float g = __bfloat162float(ge[e]);
      const float act = __bfloat162float(__float2bfloat16_rn(g / (1.f + expf(-g))));
      oe[e] = __float2bfloat16_rn(act * __bfloat162float(ue[e]));
    }
    *reinterpret_cast<uint4 *>(out + r * inter + j) = ov;
  }
}

}  // namespace fpx

using namespace fpx;

extern "C" int fpx_rmsnorm(const void *x, const void *residual, const void *weight, double eps, int64_t rows,
                           int hidden, void *out, void *residual_out, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!x || !weight || !out || rows <= 0 || hidden <= 0) return FPX_ERR_INVALID;
  if (hidden % 8 || hidden > 16384) return FPX_ERR_SHAPE;
  if (rows > 0x7fffffff) return FPX_ERR_SHAPE;
  rmsnorm_kernel<<<(unsigned)rows, 256, hidden * 2, stream>>>(
      static_cast<const __nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(residual),
      static_cast<const __nv_bfloat16 *>(weight), (float)eps, hidden, static_cast<__nv_bfloat16 *>(out),
      static_cast<__nv_bfloat16 *>(residual_out));
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

static int rope_launch(void *x, int64_t x_sb, int64_t x_sl, int64_t x_sh, int B, int L, int heads, int d,
                       int pos0, const int32_t *pos_dev, double theta, cudaStream_t stream) {
  if (!x || B <= 0 || L <= 0 || heads <= 0) return FPX_ERR_INVALID;
  if (d != kHeadDim) return FPX_ERR_UNSUPPORTED;
  RopeParams p{};
  p.x = static_cast<__nv_bfloat16 *>(x);
  p.sb = x_sb; p.sl = x_sl; p.sh = x_sh; p.L = L; p.heads = heads; p.pos0 = pos0; p.pos_dev = pos_dev;
  for (int i = 0; i < 64; ++i) {
    // HF: 1 / theta ** (arange(0, d, 2) / d), evaluated in fp32.
    const float expo = (float)(2 * i) / (float)d;
    p.inv_freq[i] = 1.0f / powf((float)theta, expo);
  }
  const int64_t n = (int64_t)B * L * heads * 64;
  p.n = n;
  rope_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(p);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

extern "C" int fpx_rope_neox(void *x, int64_t x_sb, int64_t x_sl, int64_t x_sh, int B, int L, int heads, int d,
                             int pos0, double theta, fpx_stream_t stream) {
  FPX_BIND(stream);
  return rope_launch(x, x_sb, x_sl, x_sh, B, L, heads, d, pos0, nullptr, theta, stream);
}

extern "C" int fpx_rope_neox_at(void *x, int64_t x_sb, int64_t x_sl, int64_t x_sh, int B, int L, int heads,
                                int d, const int32_t *pos0, double theta, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!pos0) return FPX_ERR_INVALID;
  return rope_launch(x, x_sb, x_sl, x_sh, B, L, heads, d, 0, pos0, theta, stream);
}

extern "C" int fpx_silu_mul(const void *gate_up, int64_t rows, int inter, void *out, fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!gate_up || !out || rows <= 0 || inter <= 0) return FPX_ERR_INVALID;
  if (inter % 8) return FPX_ERR_SHAPE;
  const int64_t n = rows * (inter / 8);
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 32);
  silu_mul_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(gate_up), rows, inter,
                                           static_cast<__nv_bfloat16 *>(out));
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}
