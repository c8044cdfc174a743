// Measures how fast tcgen05.mma (kind::f16, bf16 in, fp32 accumulate, M = 128) can be issued
// and executed on one SM, by shape and by the number of issuing warps. With the descriptors
// rebuilt before each product, one thread issues a 128 x 128 x 16 product about every 95 cycles
// whatever N is, while the tensor core needs 64 cycles for it; with the descriptors computed
// before the loop (rate_pre_kernel) one thread issues at the tensor core's rate. The exact
// attention kernel (csrc/attn_tc.cu) issues the second way.
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -I include -o mma_issue_rate mma_issue_rate.cu
//   ./mma_issue_rate
//
// One CTA per SM (the dynamic shared memory forces it), 128 threads; lane 0 of each issuing
// warp issues `n` products into its own accumulator from operands already in shared memory
// (SS: both from shared memory; TS: A from TMEM, as P.V reads P), then commits and waits. The
// time per product is the issuing loop's clock64 span over n, median over the SMs. Every
// access stays inside the buffers it allocates and every wait is bounded.
#include <algorithm>
#include <cstdio>
#include <vector>

#include "exp3_b200/csrc/tc.cuh"

using namespace fpx;
using namespace fpx::tc;

namespace {

constexpr int kABytes = 32768;  // A: 128 x 128 bf16
constexpr int kBBytes = 65536;  // B: up to 256 x 128 bf16

__device__ __forceinline__ uint64_t desc_k(uint32_t base, int kk, uint32_t half_bytes) {
  return smem_desc_sw128(base + (kk >> 2) * half_bytes + (kk & 3) * 32, 16, 1024);
}

// issuers: warps 0..issuers-1 each issue n products; ts: A operand from TMEM columns 448..511.
// Accumulators: warp w writes TMEM columns [128 w, 128 w + N) (N <= 128) or [256 w, 256 w + 256).
__global__ void __launch_bounds__(128, 1) rate_kernel(int n, int N, int issuers, int ts, long long *out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  __shared__ uint64_t bar[4];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  for (int i = threadIdx.x; i < (kABytes + kBBytes) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t *>(base)[i] = 0x3c003c00u ^ ((uint32_t)i * 2654435761u & 0x00ff00ffu);
  if (threadIdx.x == 0) {
    for (int w = 0; w < 4; ++w) mbar_init(&bar[w], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < issuers && lane == 0) {
    const uint32_t idesc = idesc_bf16(128, N, false);
    const uint32_t sa = smem_u32(base), sb = smem_u32(base + kABytes), bhalf = (uint32_t)N * 128;
    const uint32_t d = tmem + (uint32_t)(N <= 128 ? 128 : 256) * warp;
    const long long t0 = clock64();
    for (int i = 0; i < n; ++i) {
      const int kk = i & 7;
      if (ts)
        mma_ts(d, tmem + 448 + 8 * kk, desc_k(sb, kk, bhalf), idesc, i > 0 ? 1u : 0u);
      else
        mma_ss(d, desc_k(sa, kk, 16384), desc_k(sb, kk, bhalf), idesc, i > 0 ? 1u : 0u);
    }
    tc_commit(&bar[warp]);
    mbar_wait(&bar[warp], 0, &abort_flag);
    out[blockIdx.x * 4 + warp] = clock64() - t0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem, 512);
}

// The same products with every descriptor computed before the timed loop and the loop unrolled,
// so the issuing thread runs little more than the tcgen05.mma instructions themselves.
// kChains accumulators take consecutive products in turn (TMEM columns [128 c, 128 c + N));
// kMode 0: all SS; 1: all TS; 2: SS and TS alternate (Q.K^T and P.V of two tiles).
template <int kChains, int kMode>
__global__ void __launch_bounds__(128, 1) rate_pre_kernel(int n, int N, long long *out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  for (int i = threadIdx.x; i < (kABytes + kBBytes) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t *>(base)[i] = 0x3c003c00u ^ ((uint32_t)i * 2654435761u & 0x00ff00ffu);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(&tmem_base, 512);
    tmem_relinquish();
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  if (threadIdx.x == 0) {
    const uint32_t idesc = idesc_bf16(128, N, false);
    const uint32_t sa = smem_u32(base), sb = smem_u32(base + kABytes), bhalf = (uint32_t)N * 128;
    uint64_t da[8], db[8];
    uint32_t ta[8];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      da[kk] = desc_k(sa, kk, 16384);
      db[kk] = desc_k(sb, kk, bhalf);
      ta[kk] = tmem + 448 + 8 * kk;
    }
    const long long t0 = clock64();
    for (int i = 0; i < n; i += 8 * kChains) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
#pragma unroll
        for (int c = 0; c < kChains; ++c) {
          const uint32_t d = tmem + 128 * c;
          const bool ts = kMode == 1 || (kMode == 2 && (c & 1));
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          if (ts)
            mma_ts(d, ta[kk], db[kk], idesc, acc);
          else
            mma_ss(d, da[kk], db[kk], idesc, acc);
        }
    }
    tc_commit(&bar);
    mbar_wait(&bar, 0, &abort_flag);
    out[blockIdx.x * 4] = clock64() - t0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem, 512);
}

}  // namespace

int main() {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  long long *d_out = nullptr;
  if (cudaMalloc(&d_out, sms * 4 * sizeof(long long)) != cudaSuccess) return 1;
  const int smem = kABytes + kBBytes + 1024 + 100000;  // more than half an SM's shared memory
  cudaFuncSetAttribute(rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  struct Case {
    int N, issuers, ts;
  };
  // TS reads A from columns 448..511, so it runs with at most 3 issuers of N = 128 (D below 384).
  const Case cases[] = {{32, 1, 0},  {64, 1, 0},  {128, 1, 0}, {256, 1, 0}, {128, 1, 1}, {128, 2, 0}, {128, 3, 0},
                        {128, 4, 0}, {64, 2, 0},  {64, 4, 0},  {256, 2, 0}, {128, 2, 1}, {128, 3, 1}};
  const int n = 512;
  printf("%-4s %5s %8s %18s %16s\n", "op", "N", "issuers", "cycles per product", "FLOP/cycle/SM");
  for (const Case &c : cases) {
    std::vector<long long> h(sms * 4);
    for (int rep = 0; rep < 2; ++rep) {
      rate_kernel<<<sms, 128, smem>>>(n, c.N, c.issuers, c.ts, d_out);
      const cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) {
        printf("error: %s\n", cudaGetErrorString(e));
        return 1;
      }
    }
    cudaMemcpy(h.data(), d_out, h.size() * sizeof(long long), cudaMemcpyDeviceToHost);
    std::vector<double> per;
    for (int i = 0; i < sms; ++i) {
      long long slowest = 0;
      for (int w = 0; w < c.issuers; ++w) slowest = std::max(slowest, h[i * 4 + w]);
      per.push_back(slowest / (double)(n * c.issuers));
    }
    std::sort(per.begin(), per.end());
    const double cyc = per[sms / 2];
    printf("%-4s %5d %8d %18.1f %16.0f\n", c.ts ? "TS" : "SS", c.N, c.issuers, cyc, 2.0 * 128 * c.N * 16 / cyc);
  }
  // Precomputed descriptors, one issuing thread.
  struct PreCase {
    const char *name;
    int N, chains, mode;
    void (*kernel)(int, int, long long *);
  };
  const PreCase pre[] = {{"SS pre", 128, 1, 0, rate_pre_kernel<1, 0>}, {"SS pre", 64, 1, 0, rate_pre_kernel<1, 0>},
                         {"SS pre", 256, 1, 0, rate_pre_kernel<1, 0>}, {"TS pre", 128, 1, 1, rate_pre_kernel<1, 1>},
                         {"SS pre", 128, 2, 0, rate_pre_kernel<2, 0>}, {"SS/TS pre", 128, 2, 2, rate_pre_kernel<2, 2>},
                         {"TS pre", 128, 2, 1, rate_pre_kernel<2, 1>}};
  printf("%-10s %5s %7s %18s %16s\n", "op", "N", "chains", "cycles per product", "FLOP/cycle/SM");
  for (const PreCase &c : pre) {
    cudaFuncSetAttribute(c.kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    std::vector<long long> h(sms * 4);
    for (int rep = 0; rep < 2; ++rep) {
      c.kernel<<<sms, 128, smem>>>(n, c.N, d_out);
      const cudaError_t e = cudaDeviceSynchronize();
      if (e != cudaSuccess) {
        printf("error: %s\n", cudaGetErrorString(e));
        return 1;
      }
    }
    cudaMemcpy(h.data(), d_out, h.size() * sizeof(long long), cudaMemcpyDeviceToHost);
    std::vector<double> per;
    for (int i = 0; i < sms; ++i) per.push_back(h[i * 4] / (double)n);
    std::sort(per.begin(), per.end());
    const double cyc = per[sms / 2];
    printf("%-10s %5d %7d %18.1f %16.0f\n", c.name, c.N, c.chains, cyc, 2.0 * 128 * c.N * 16 / cyc);
  }
  cudaFree(d_out);
  return 0;
}
