// sm_100a building blocks: mbarriers with bounded waits, TMA tensor copies, tcgen05 MMA /
// TMEM access, and the shared-memory matrix descriptors of the 5th-generation tensor core.
//
// Descriptor formats (PTX ISA, tcgen05 "shared memory descriptor" and "instruction
// descriptor"): a 128-byte-swizzled tile stores rows of 64 bf16 (128 B) in 1024-byte atoms of
// 8 rows. K-major operands (Q, K, P) advance 32 B per K=16 step inside an atom, 8-row groups
// sit SBO = 1024 B apart. The MN-major V operand keeps 64-element MN atoms LBO apart and
// 8-row K groups SBO = 1024 B apart.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace fpx {
namespace tc {

constexpr long long kWaitCycles = 1ll << 31;  // ~1 s at 2 GHz: every wait gives up after this

FPX_INLINE void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
FPX_INLINE void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
FPX_INLINE void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
FPX_INLINE bool mbar_test(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking probe (test_wait never suspends the thread, unlike try_wait).
FPX_INLINE bool mbar_probe(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase with the given parity to complete. Gives up (returns false) when
// *abort is set by another role or after kWaitCycles, setting *abort itself then.
FPX_INLINE bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort) {
  if (mbar_test(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_test(bar, parity)) {
    if (*abort) return false;
    if (clock64() - start > kWaitCycles) {
      *abort = 1;
      return false;
    }
  }
  return true;
}
// Warp-uniform form: every lane of the warp agrees on the outcome, so warp-collective
// tcgen05 instructions that follow are never reached by part of a warp.
FPX_INLINE bool mbar_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}
FPX_INLINE void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
FPX_INLINE void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 4-D tiled TMA load into shared memory, completing bytes on `bar`.
FPX_INLINE void tma_load_4d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
// 4-D tiled TMA store from shared memory (rows past the tensor's extent are not written).
FPX_INLINE void tma_store_4d(const CUtensorMap *map, const void *src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(map),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
               : "memory");
}
FPX_INLINE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
FPX_INLINE void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
FPX_INLINE void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Named barrier among `count` threads.
FPX_INLINE void named_sync(int id, int count) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory"); }

// Register reallocation between warpgroups (all four warps of a warpgroup execute it).
template <int N>
FPX_INLINE void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
FPX_INLINE void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }

// ---- tcgen05 / TMEM ----------------------------------------------------------------------
FPX_INLINE void tmem_alloc(uint32_t *dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(cols)
               : "memory");
}
FPX_INLINE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;"); }
FPX_INLINE void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
FPX_INLINE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FPX_INLINE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
FPX_INLINE void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (bf16 in, fp32 accumulate).
FPX_INLINE void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem desc): A is M x K bf16 in TMEM, one row per lane, two
// consecutive K elements per 32-bit column (K = 16 spans 8 columns).
FPX_INLINE void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 2^x on the special-function unit (the hardware's approximate exp2, flush-to-zero).
// Maximum of three floats in one instruction (the three-input max.f32 of sm_100).
FPX_INLINE float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
FPX_INLINE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two lanes of work).
FPX_INLINE uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
FPX_INLINE void up2(uint64_t v, float &a, float &b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
FPX_INLINE uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
FPX_INLINE uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
FPX_INLINE uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// 2^x for a pair on the FMA pipe, to offload the special-function unit. Range reduction
// x = j + f with j = round(x) (the 1.5 * 2^23 magic-number add) and |f| <= 1/2, a cubic
// for 2^f fitted here by a relative-error weighted least-squares fit on Chebyshev nodes
// (max relative error 7.5e-5, 26x below bf16's rounding step), and 2^j added into the
// exponent bits. x is clamped to >= -126 so the exponent never underflows.
FPX_INLINE uint64_t exp2_poly2(uint64_t x2) {
  float a, b;
  up2(x2, a, b);
  x2 = pk2(fmaxf(a, -126.f), fmaxf(b, -126.f));
  const uint64_t magic = pk2(12582912.f, 12582912.f), nmagic = pk2(-12582912.f, -12582912.f);
  const uint64_t minus1 = pk2(-1.f, -1.f);
  const uint64_t t = fadd2(x2, magic);
  const uint64_t f = ffma2(fadd2(t, nmagic), minus1, x2);
  uint64_t poly = ffma2(f, pk2(0.05517113208770752f, 0.05517113208770752f), pk2(0.2426110804080963f, 0.2426110804080963f));
  poly = ffma2(poly, f, pk2(0.6932610869407654f, 0.6932610869407654f));
  poly = ffma2(poly, f, pk2(0.9999280571937561f, 0.9999280571937561f));
  float pa, pb, ta, tb;
  up2(poly, pa, pb);
  up2(t, ta, tb);
  return pk2(__uint_as_float(__float_as_uint(pa) + (__float_as_uint(ta) << 23)),
             __uint_as_float(__float_as_uint(pb) + (__float_as_uint(tb) << 23)));
}
FPX_INLINE uint32_t cvt_bf16x2(uint64_t v) {
  float a, b;
  up2(v, a, b);
  return pack_bf16(a, b);
}
FPX_INLINE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
FPX_INLINE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
FPX_INLINE void tmem_ld32(uint32_t taddr, float (&r)[32]) {
  uint32_t *u = reinterpret_cast<uint32_t *>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
        "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15]),
        "=r"(u[16]), "=r"(u[17]), "=r"(u[18]), "=r"(u[19]), "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]),
        "=r"(u[24]), "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]), "=r"(u[31])
      : "r"(taddr));
}
FPX_INLINE void tmem_st32(uint32_t taddr, const float (&r)[32]) {
  const uint32_t *u = reinterpret_cast<const uint32_t *>(r);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]), "r"(u[8]),
      "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15]), "r"(u[16]),
      "r"(u[17]), "r"(u[18]), "r"(u[19]), "r"(u[20]), "r"(u[21]), "r"(u[22]), "r"(u[23]), "r"(u[24]),
      "r"(u[25]), "r"(u[26]), "r"(u[27]), "r"(u[28]), "r"(u[29]), "r"(u[30]), "r"(u[31])
      : "memory");
}

FPX_INLINE void tmem_st32u(uint32_t taddr, const uint32_t *u) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]), "r"(u[8]),
      "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15]), "r"(u[16]),
      "r"(u[17]), "r"(u[18]), "r"(u[19]), "r"(u[20]), "r"(u[21]), "r"(u[22]), "r"(u[23]), "r"(u[24]),
      "r"(u[25]), "r"(u[26]), "r"(u[27]), "r"(u[28]), "r"(u[29]), "r"(u[30]), "r"(u[31])
      : "memory");
}

FPX_INLINE void tmem_st16u(uint32_t taddr, const uint32_t *u) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]), "r"(u[8]),
      "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15])
      : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), version 1 (sm_100).
FPX_INLINE uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// A shared-memory operand descriptor keeps the operand's address / 16 in its low 14 bits. Every
// operand lies below 2^18 bytes, so moving one by a byte offset (a multiple of 16) adds offset /
// 16 to the low word and leaves the other fields alone. An MMA issuer keeps one low word per
// buffer and adds each K-step's constant: one integer add per operand in front of a product
// instead of rebuilding the descriptor, which measured is what held one thread to a product
// every ~95 cycles (65 with the descriptors ready, the tensor core's own rate).
FPX_INLINE uint64_t desc_join(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}
FPX_INLINE uint32_t desc_lo(uint64_t d) { return (uint32_t)d; }
FPX_INLINE uint32_t desc_hi(uint64_t d) { return (uint32_t)(d >> 32); }
// Instruction descriptor, kind::f16: bf16 A and B, fp32 D, M x N, A K-major, B K- or MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

}  // namespace tc

// [B, rows, heads, d] bf16 with element strides -> 4-D TMA map (d, head, row, batch), box
// 64 x 1 x box_rows x 1, 128-byte swizzle, zero fill outside the tensor (attn_tc.cu).
bool encode_4d(CUtensorMap *map, const void *base, int64_t d, int64_t heads, int64_t rows, int64_t batch,
               int64_t sh, int64_t sl, int64_t sb, int box_rows = 128);

// Device address of the library's error word (fpx_device_error) on the current device, for
// kernels in other translation units; null if the runtime cannot resolve it.
int *device_error_word();

}  // namespace fpx
