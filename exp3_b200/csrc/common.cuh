// Shared device helpers for libfpx (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/fpx.h"

#define FPX_INLINE __device__ __forceinline__

namespace fpx {

constexpr int kBlock = 128;     // routing block (tokens) == query tile rows
constexpr int kHeadDim = 128;   // compiled head dimension
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Internal routing state for (b, h, query tile t), written by the routing kernels and
// read by the exact and mean kernels. All arrays live in the prefill workspace.
struct RouteView {
  int32_t *lists;    // [B][H][nb][nb] selected key blocks of (b, h, t), ascending
  int32_t *counts;   // [B][H][nb]     number of valid entries in lists
  uint32_t *tail;    // [B][H][nb][words] bit kb set: kb < t and kb not selected
  int nb, words;
  FPX_INLINE int64_t row(int b, int h, int t, int H) const {
    return ((int64_t)b * H + h) * nb + t;
  }
};

FPX_INLINE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
FPX_INLINE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions for blockDim.x = NT (multiple of 32); `red` holds >= NT/32 floats.
template <int NT>
FPX_INLINE float block_max(float v, float *red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < NT / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}
template <int NT>
FPX_INLINE float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) r += red[i];
  return r;
}
// Exclusive prefix sum of per-thread ints over the block; returns the exclusive prefix
// and writes the total to *total. `scratch` holds >= NT/32 ints.
template <int NT>
FPX_INLINE int block_exclusive_scan(int v, int *scratch, int *total) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (l >= o) incl += n;
  }
  __syncthreads();
  if (l == 31) scratch[w] = incl;
  __syncthreads();
  int base = 0, all = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; ++i) {
    const int s = scratch[i];
    if (i < w) base += s;
    all += s;
  }
  *total = all;
  return base + incl - v;
}

// Protected regions of upstream:374-381 / kernels.py:145-150.
FPX_INLINE bool is_protected(int t, int kb, int nb, int sink, int window, int last_full) {
  const int dist = t - kb;
  return kb < sink || (dist >= 0 && dist < window) || t >= nb - last_full;
}

FPX_INLINE uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

FPX_INLINE void cp_async16(void *smem, const void *gmem, bool pred) {
  const int n = pred ? 16 : 0;  // src-size 0 zero-fills the 16 bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(n));
}
FPX_INLINE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
FPX_INLINE void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

FPX_INLINE void ldmatrix_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
FPX_INLINE void ldmatrix_x4_trans(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3,
                                  uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
FPX_INLINE void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

FPX_INLINE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// torch.logaddexp for fp32 (max + log1p(exp(-|a - b|)), equal infinities kept).
FPX_INLINE float logaddexp(float a, float b) {
  if (a == b && isinf(a)) return a;
  const float m = fmaxf(a, b);
  return m + log1pf(expf(-fabsf(a - b)));
}

}  // namespace fpx

// Host-side helpers.

// The library carries its own (static) CUDA runtime; make the device that owns the caller's
// stream current before launching, so multi-GPU callers need no extra set-up.
static inline int fpx_bind_stream_device(cudaStream_t s) {
  if (!s) return FPX_OK;
  // While a stream is being captured into a CUDA graph, device queries on it are not allowed
  // (they would invalidate the capture); the capturing thread is already on the stream's device.
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &capture) == cudaSuccess && capture != cudaStreamCaptureStatusNone) return FPX_OK;
  int dev = -1, cur = -1;
  if (cudaStreamGetDevice(s, &dev) != cudaSuccess) return FPX_ERR_INVALID;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != dev) {
    if (cudaSetDevice(dev) != cudaSuccess) return FPX_ERR_CUDA;
  }
  return FPX_OK;
}
#define FPX_BIND(stream)                                   \
  do {                                                     \
    const int fpx_bind_rc_ = fpx_bind_stream_device(stream); \
    if (fpx_bind_rc_) return fpx_bind_rc_;                 \
  } while (0)

#define FPX_CHECK_LAUNCH()                               \
  do {                                                   \
    if (cudaPeekAtLastError() != cudaSuccess) return FPX_ERR_CUDA; \
  } while (0)
