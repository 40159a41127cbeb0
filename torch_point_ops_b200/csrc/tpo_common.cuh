// Shared device helpers for the tpo_b200 kernels (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tpo_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "tpo_b200 kernels are written for sm_100a (B200) only"
#endif

namespace tpo {

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100: one instruction drives two FP32 lanes, so
// the FP32 pipe can be saturated with half the issue slots).  Explicit .rn
// rounding: IEEE per element, never contracted by ptxas.
// ---------------------------------------------------------------------------
typedef unsigned long long u64;

__device__ __forceinline__ u64 pk(float lo, float hi) {
  u64 r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk(u64 v, float& lo, float& hi) {
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ u64 sub2(u64 a, u64 b) {
  u64 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 mul2(u64 a, u64 b) {
  u64 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 add2(u64 a, u64 b) {
  u64 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 fma2(u64 a, u64 b, u64 c) {
  u64 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// Squared distance of two packed lanes, in the reference's operation order.
// MODE 0 (TPO_ROUND_FMA): fma(dz,dz, fma(dx,dx, dy*dy)) -- bit-identical to the
// reference CUDA chamfer kernel as nvcc contracts it (measured on B200);
// MODE 1 (TPO_ROUND_EXACT): (dx*dx + dy*dy) + dz*dz, every operation rounded.
template <int MODE>
__device__ __forceinline__ u64 dist2x2(u64 dx, u64 dy, u64 dz) {
  if (MODE == TPO_ROUND_FMA) {
    u64 t = mul2(dy, dy);
    t = fma2(dx, dx, t);
    return fma2(dz, dz, t);
  } else {
    // Scalar .rn mul/add: PTX guarantees these are never fused.  (Measured on
    // B200: ptxas may fuse a mul.rn.f32x2 + add.rn.f32x2 pair into an FMA, which
    // would silently turn this mode into the FMA rounding.)
    float x0, x1, y0, y1, z0, z1;
    upk(dx, x0, x1);
    upk(dy, y0, y1);
    upk(dz, z0, z1);
    const float r0 = __fadd_rn(__fadd_rn(__fmul_rn(x0, x0), __fmul_rn(y0, y0)), __fmul_rn(z0, z0));
    const float r1 = __fadd_rn(__fadd_rn(__fmul_rn(x1, x1), __fmul_rn(y1, y1)), __fmul_rn(z1, z1));
    return pk(r0, r1);
  }
}

// Scalar forms with the same rounding (used by the finalize rescans).
template <int MODE>
__device__ __forceinline__ float dist1f(float dx, float dy, float dz) {
  if (MODE == TPO_ROUND_FMA) {
    return __fmaf_rn(dz, dz, __fmaf_rn(dx, dx, __fmul_rn(dy, dy)));
  } else {
    return __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
  }
}
template <int MODE>
__device__ __forceinline__ double dist1d(double dx, double dy, double dz) {
  if (MODE == TPO_ROUND_FMA) {
    return __fma_rn(dz, dz, __fma_rn(dx, dx, __dmul_rn(dy, dy)));
  } else {
    return __dadd_rn(__dadd_rn(__dmul_rn(dx, dx), __dmul_rn(dy, dy)), __dmul_rn(dz, dz));
  }
}

// fp16 with c10::Half semantics: every operation rounds to half (RN), nothing fused.
__device__ __forceinline__ __half hsub_rn(__half a, __half b) {
  __half r;
  asm("sub.rn.f16 %0, %1, %2;" : "=h"(*reinterpret_cast<unsigned short*>(&r))
      : "h"(*reinterpret_cast<unsigned short*>(&a)), "h"(*reinterpret_cast<unsigned short*>(&b)));
  return r;
}
__device__ __forceinline__ __half hmul_rn(__half a, __half b) {
  __half r;
  asm("mul.rn.f16 %0, %1, %2;" : "=h"(*reinterpret_cast<unsigned short*>(&r))
      : "h"(*reinterpret_cast<unsigned short*>(&a)), "h"(*reinterpret_cast<unsigned short*>(&b)));
  return r;
}
__device__ __forceinline__ __half hadd_rn(__half a, __half b) {
  __half r;
  asm("add.rn.f16 %0, %1, %2;" : "=h"(*reinterpret_cast<unsigned short*>(&r))
      : "h"(*reinterpret_cast<unsigned short*>(&a)), "h"(*reinterpret_cast<unsigned short*>(&b)));
  return r;
}
// (dx*dx + dy*dy) + dz*dz, each op rounded to half; chamfer.cu:64-67 with c10::Half.
__device__ __forceinline__ __half dist1h(__half dx, __half dy, __half dz) {
  return hadd_rn(hadd_rn(hmul_rn(dx, dx), hmul_rn(dy, dy)), hmul_rn(dz, dz));
}

// Packed f16x2 (two rows in one 32-bit register), every operation rounded (.rn).
typedef unsigned h2;  // raw f16x2 bits
__device__ __forceinline__ h2 hsub2r(h2 a, h2 b) {
  h2 r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ h2 hmul2r(h2 a, h2 b) {
  h2 r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ h2 hadd2r(h2 a, h2 b) {
  h2 r;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ h2 hmin2r(h2 a, h2 b) {
  h2 r;
  asm("min.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ h2 hpk(unsigned short lo, unsigned short hi) {
  return (h2)lo | ((h2)hi << 16);
}
// c10::Half distance (dx*dx + dy*dy) + dz*dz on two lanes at once.
__device__ __forceinline__ h2 hdist2(h2 dx, h2 dy, h2 dz) {
  return hadd2r(hadd2r(hmul2r(dx, dx), hmul2r(dy, dy)), hmul2r(dz, dz));
}

__device__ __forceinline__ float min3f(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ unsigned redux_min_u32(unsigned v) {
  unsigned r;
  asm volatile("redux.sync.min.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

// Fire-and-forget global atomic min on a packed 64-bit key.
__device__ __forceinline__ void red_min_u64(u64* addr, u64 v) {
  asm volatile("red.relaxed.gpu.global.min.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}

// 128-bit key {lo = chunk index, hi = distance bits} for fp64: lexicographic min
// via a 16-byte compare-and-swap loop (atom.cas.b128, sm_90+).
struct alignas(16) Key128 {
  u64 lo, hi;
};
__device__ __forceinline__ bool key128_less(u64 ahi, u64 alo, u64 bhi, u64 blo) {
  return ahi < bhi || (ahi == bhi && alo < blo);
}
__device__ __forceinline__ void cas128(Key128* addr, u64 cmp_lo, u64 cmp_hi, u64 new_lo,
                                       u64 new_hi, u64& old_lo, u64& old_hi) {
  asm volatile(
      "{\n\t.reg .b128 c, n, o;\n\t"
      "mov.b128 c, {%2, %3};\n\t"
      "mov.b128 n, {%4, %5};\n\t"
      "atom.relaxed.gpu.global.cas.b128 o, [%6], c, n;\n\t"
      "mov.b128 {%0, %1}, o;\n\t}"
      : "=l"(old_lo), "=l"(old_hi)
      : "l"(cmp_lo), "l"(cmp_hi), "l"(new_lo), "l"(new_hi), "l"(addr)
      : "memory");
}
__device__ __forceinline__ void key128_min(Key128* addr, u64 hi, u64 lo) {
  u64 cur_lo = addr->lo, cur_hi = addr->hi;  // a torn read only costs an extra CAS round
  // Bounded: every failed CAS means another thread stored a strictly smaller key,
  // which can happen at most once per competing writer.
  for (int it = 0; it < (1 << 20); ++it) {
    if (!key128_less(hi, lo, cur_hi, cur_lo)) return;
    u64 o_lo, o_hi;
    cas128(addr, cur_lo, cur_hi, lo, hi, o_lo, o_hi);
    if (o_lo == cur_lo && o_hi == cur_hi) return;
    cur_lo = o_lo;
    cur_hi = o_hi;
  }
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__host__ __device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// ---- 1-D bulk copies global -> shared (the TMA unit's non-tensor form) ----
// One thread issues a copy of `bytes` (multiple of 16; both addresses 16-byte
// aligned) that completes on an mbarrier as transaction bytes.  The wait is
// bounded: after kBulkWaitLimit polls it ORs kErrBulkTimeout into *err and
// returns false instead of spinning forever.
constexpr unsigned kBulkWaitLimit = 1u << 24;
constexpr unsigned kErrBulkTimeout = 1u;

__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes,
                                         unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, unsigned parity, unsigned* err) {
  for (unsigned it = 0; it < kBulkWaitLimit; ++it) {
    unsigned done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  atomicOr(err, kErrBulkTimeout);
  return false;
}

// Atomic add of a 3-vector of floats at p (4-byte aligned, as in an (n,3) array):
// one 8-byte vector reduction for the aligned pair plus one scalar, instead of
// three scalar reductions.  Each component is added (and rounded) on its own.
__device__ __forceinline__ void red_add_v2f(float* p, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void red_add3f(float* p, float x, float y, float z) {
  if ((reinterpret_cast<uintptr_t>(p) & 7) == 0) {
    red_add_v2f(p, x, y);
    atomicAdd(p + 2, z);
  } else {
    atomicAdd(p, x);
    red_add_v2f(p + 1, y, z);
  }
}

// The same for a 3-vector of halves (2-byte aligned): one packed half2 atomic for
// the 4-byte aligned pair plus one scalar.
__device__ __forceinline__ void red_add3h(__half* p, __half x, __half y, __half z) {
  if ((reinterpret_cast<uintptr_t>(p) & 3) == 0) {
    atomicAdd(reinterpret_cast<__half2*>(p), __halves2half2(x, y));
    atomicAdd(p + 2, z);
  } else {
    atomicAdd(p, x);
    atomicAdd(reinterpret_cast<__half2*>(p + 1), __halves2half2(y, z));
  }
}

// Programmatic dependent launch.  A kernel launched with launch_pdl may start
// while the previous kernel in the stream is still running; it must call
// pdl_wait() before touching global memory (that returns once the previous
// grid has completed and its writes are visible).  pdl_trigger() lets the next
// kernel's CTAs be scheduled early; both are no-ops without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ unsigned lane_id() {
  unsigned r;
  asm("mov.u32 %0, %%laneid;" : "=r"(r));
  return r;
}

}  // namespace tpo
