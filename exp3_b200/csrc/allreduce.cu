// One-shot all-reduce of a small bf16 vector across the tensor-parallel ranks of one node over
// NVLink peer memory (plain loads and stores: no TMA, no multicast, no library kernel), for the
// decode step, where a collective library's per-call latency dominates 7 KB messages.
//
// Every rank owns one buffer, mapped into every peer's address space through CUDA IPC:
//   [0]    error (i32): set when a wait gave up
//   [64]   epoch (u32): this rank's call counter (device memory, so CUDA-graph replays advance it)
//   [256 + 64 q]  flag of rank q (u32): the last call whose input rank q has pushed here
//   [768]  slots [2][kArMaxRanks][max_elems] bf16: rank q's input of calls with parity e & 1
// Call e = epoch + 1 on rank r (a push: every remote access is a store):
//   1. store the input into slot [e & 1][r] of every rank's buffer (its own included), fence at
//      system scope, then store flag e into flag r of every rank's buffer (release);
//   2. wait until every flag in this rank's own buffer is >= e (acquire, local polling);
//   3. sum the ranks' slots [e & 1][q] in rank order in fp32 (the same order everywhere, so
//      every rank gets the same bits) and write the bf16 result over the input.
// Slot [e & 1][r] of rank p is free when r writes it: r finished call e - 1, so it saw p's
// flag e - 1, which p stored after finishing call e - 2, the last reader of that slot.
// Every wait is bounded (about 1 s of clock64); a wait that gives up sets the error word and the
// kernel returns, so a missing rank ends the call instead of hanging the GPU.
#include <cstring>

#include "common.cuh"

namespace fpx {

constexpr int kArMaxRanks = 8;
constexpr int kArThreads = 512;
constexpr long long kArWaitCycles = 1ll << 31;
constexpr size_t kArFlags = 256, kArSlots = 768;

struct ArPeers {
  uint8_t *base[kArMaxRanks];
};

FPX_INLINE uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
FPX_INLINE void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
FPX_INLINE uint4 ld_relaxed_sys_v4(const uint4 *p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
// Wraparound-safe "flag has reached target" (epochs are u32 counters).
FPX_INLINE bool ar_wait(const uint32_t *flag, uint32_t target) {
  const long long start = clock64();
  while ((int32_t)(ld_acquire_sys(flag) - target) < 0) {
    if (clock64() - start > kArWaitCycles) return false;
  }
  return true;
}

__global__ void __launch_bounds__(kArThreads) allreduce_oneshot_kernel(__nv_bfloat16 *inout, int n, ArPeers peers,
                                                                        int rank, int world, int max_elems) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_fail;
  uint8_t *own = peers.base[rank];
  int *error = reinterpret_cast<int *>(own);
  uint32_t *epoch = reinterpret_cast<uint32_t *>(own + 64);
  if (threadIdx.x == 0) {
    s_epoch = *epoch + 1;
    s_fail = *reinterpret_cast<volatile int *>(error);
  }
  __syncthreads();
  if (s_fail) return;  // an earlier call already failed: the buffers are out of step
  const uint32_t e = s_epoch;
  auto flag = [&](int buf, int q) { return reinterpret_cast<uint32_t *>(peers.base[buf] + kArFlags + 64 * q); };
  auto slot = [&](int buf, int q) {
    return reinterpret_cast<uint4 *>(peers.base[buf] + kArSlots +
                                     ((size_t)(e & 1u) * kArMaxRanks + q) * (size_t)max_elems * 2);
  };
  // 1. push this rank's input into every rank's slot, then the flags
  const int n8 = n / 8;  // 16-byte pieces (n % 8 == 0 is checked on the host)
  const uint4 *src = reinterpret_cast<const uint4 *>(inout);
  for (int i = threadIdx.x; i < n8; i += kArThreads) {
    const uint4 v = src[i];
    for (int p = 0; p < world; ++p) slot(p, rank)[i] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) st_release_sys(flag(threadIdx.x, rank), e);
  // 2. every rank's input of call e has arrived here
  if (threadIdx.x < world && !ar_wait(flag(rank, threadIdx.x), e)) atomicExch(&s_fail, 1);
  __syncthreads();
  if (s_fail) {
    if (threadIdx.x == 0) atomicExch(error, 1);
    return;
  }
  // 3. sum in rank order (local slots; relaxed system-scope loads bypass stale L1 lines)
  uint4 *dst = reinterpret_cast<uint4 *>(inout);
  for (int i = threadIdx.x; i < n8; i += kArThreads) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < world; ++q) {
      const uint4 v = ld_relaxed_sys_v4(slot(rank, q) + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[k]));
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
    dst[i] = make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]),
                        pack_bf16(acc[6], acc[7]));
  }
  if (threadIdx.x == 0) *epoch = e;
}

}  // namespace fpx

using namespace fpx;

extern "C" size_t fpx_ar_buffer_bytes(int max_elems) {
  if (max_elems <= 0 || max_elems % 8) return 0;
  return kArSlots + (size_t)2 * kArMaxRanks * max_elems * 2;
}

extern "C" int fpx_ar_create(size_t bytes, void **base, void *ipc_handle) {
  if (!base || !ipc_handle || bytes < kArSlots) return FPX_ERR_INVALID;
  void *p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return FPX_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess ||
      cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(ipc_handle), p) != cudaSuccess) {
    cudaFree(p);
    return FPX_ERR_CUDA;
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return FPX_ERR_CUDA;  // zeroed before any peer reads it
  *base = p;
  return FPX_OK;
}

extern "C" int fpx_ar_open(const void *ipc_handle, void **peer_base) {
  if (!ipc_handle || !peer_base) return FPX_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(peer_base, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? FPX_OK : FPX_ERR_CUDA;
}

extern "C" int fpx_ar_close(void *peer_base) {
  return cudaIpcCloseMemHandle(peer_base) == cudaSuccess ? FPX_OK : FPX_ERR_CUDA;
}

extern "C" int fpx_ar_destroy(void *base) { return cudaFree(base) == cudaSuccess ? FPX_OK : FPX_ERR_CUDA; }

extern "C" int fpx_allreduce_bf16(void *inout, int64_t n, void *const *bases, int rank, int world, int max_elems,
                                  fpx_stream_t stream) {
  FPX_BIND(stream);
  if (!inout || !bases || world < 1 || world > kArMaxRanks || rank < 0 || rank >= world) return FPX_ERR_INVALID;
  if (n <= 0 || n > max_elems || n % 8 || (reinterpret_cast<uintptr_t>(inout) & 15)) return FPX_ERR_SHAPE;
  ArPeers peers{};
  for (int r = 0; r < world; ++r) {
    if (!bases[r]) return FPX_ERR_INVALID;
    peers.base[r] = static_cast<uint8_t *>(bases[r]);
  }
  allreduce_oneshot_kernel<<<1, kArThreads, 0, stream>>>(static_cast<__nv_bfloat16 *>(inout), (int)n, peers, rank,
                                                          world, max_elems);
  FPX_CHECK_LAUNCH();
  return FPX_OK;
}

extern "C" int fpx_ar_error(const void *base, int *code) {
  if (!base || !code) return FPX_ERR_INVALID;
  return cudaMemcpy(code, static_cast<const uint8_t *>(base), sizeof(int), cudaMemcpyDeviceToHost) ==
                 cudaSuccess
             ? FPX_OK
             : FPX_ERR_CUDA;
}
