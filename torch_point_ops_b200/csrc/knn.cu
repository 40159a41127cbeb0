// K nearest neighbours (forward + backward) and knn_gather for sm_100a.
//
// Forward replaces knn_cuda_forward + KNearestNeighborKernelV0..V3
// (torch_point_ops/knn/csrc/cuda/knn.cu:16-227,295-398) and the host-side sort
// of knn_points (knn/__init__.py:110-131).  A warp serves KQ queries of one
// batch; its 32 lanes evaluate 32 consecutive target points per step (staged in
// shared memory, shared by the CTA's warps).  Each query's running top-K list is
// distributed across the warp (lane k holds the k-th best), so:
//   * filtering is one compare + ballot per query per step against the K-th
//     distance (kept uniform in a register);
//   * a surviving candidate is inserted with one shuffle-up shift of the list.
// Candidates are inserted in increasing index order and a candidate equal to an
// existing distance lands after it, and one equal to the K-th is rejected, so
// the list is exactly "K smallest by (dist, idx), ascending": the reference CPU
// priority_queue result (knn.cpp:61-95).  Output is sorted in the kernel; the
// torch.sort + mask pass of the reference disappears.
//
// Backward replaces KNearestNeighborBackwardKernel (knn.cu:401-466): one thread
// per query row sums its K terms in k order (deterministic, no atomics for
// grad_p1) and scatters the negated terms into grad_p2 with atomics.
#include <cstdlib>
#include <type_traits>

#include "tpo_internal.h"

namespace tpo {

#ifndef TPO_KQ
#define TPO_KQ 4
#endif
constexpr int KQ = TPO_KQ;   // queries per warp
#ifndef TPO_KW
#define TPO_KW 8
#endif
constexpr int KW = TPO_KW;   // warps per CTA
constexpr int KSTEP = 32;    // targets per step (one per lane)
#ifndef TPO_KTILE
#define TPO_KTILE 2048
#endif
constexpr int KTILE = TPO_KTILE;  // targets per shared-memory tile
constexpr int KDMAX = 8;     // the fast kernel's largest D

template <typename T>
struct KnnArith;
template <>
struct KnnArith<float> {
  using V = float;
  template <int MODE>
  __device__ static float sq_first(float a, float b) {
    const float d = __fsub_rn(a, b);
    return __fmul_rn(d, d);
  }
  template <int MODE>
  __device__ static float sq_acc(float t, float a, float b) {
    const float d = __fsub_rn(a, b);
    return MODE == TPO_ROUND_FMA ? __fmaf_rn(d, d, t) : __fadd_rn(t, __fmul_rn(d, d));
  }
  __device__ static float abs_first(float a, float b) { return fabsf(__fsub_rn(a, b)); }
  __device__ static float abs_acc(float t, float a, float b) { return __fadd_rn(t, fabsf(__fsub_rn(a, b))); }
  __device__ static V val(float x) { return x; }
  __device__ static float from(V v) { return v; }
  __device__ static float nan_() { return __int_as_float(0x7fffffff); }
};
template <>
struct KnnArith<double> {
  using V = double;
  template <int MODE>
  __device__ static double sq_first(double a, double b) {
    const double d = __dsub_rn(a, b);
    return __dmul_rn(d, d);
  }
  template <int MODE>
  __device__ static double sq_acc(double t, double a, double b) {
    const double d = __dsub_rn(a, b);
    return MODE == TPO_ROUND_FMA ? __fma_rn(d, d, t) : __dadd_rn(t, __dmul_rn(d, d));
  }
  __device__ static double abs_first(double a, double b) { return fabs(__dsub_rn(a, b)); }
  __device__ static double abs_acc(double t, double a, double b) { return __dadd_rn(t, fabs(__dsub_rn(a, b))); }
  __device__ static V val(double x) { return x; }
  __device__ static double from(V v) { return v; }
  __device__ static double nan_() { return __longlong_as_double(0x7fffffffffffffffll); }
};
template <>
struct KnnArith<__half> {
  using V = float;  // exact float image of the half result
  template <int MODE>
  __device__ static __half sq_first(__half a, __half b) {
    const __half d = hsub_rn(a, b);
    return hmul_rn(d, d);
  }
  template <int MODE>
  __device__ static __half sq_acc(__half t, __half a, __half b) {
    const __half d = hsub_rn(a, b);
    return hadd_rn(t, hmul_rn(d, d));
  }
  __device__ static __half abs_first(__half a, __half b) { return __habs(hsub_rn(a, b)); }
  __device__ static __half abs_acc(__half t, __half a, __half b) { return hadd_rn(t, __habs(hsub_rn(a, b))); }
  __device__ static V val(__half x) { return __half2float(x); }
  __device__ static __half from(V v) { return __float2half_rn(v); }
  __device__ static __half nan_() { return __ushort_as_half((unsigned short)0x7fff); }
};

template <typename T, int DT, int NORM, int MODE>
__device__ __forceinline__ typename KnnArith<T>::V knn_dist(const T* q, const T* c, int D) {
  using A = KnnArith<T>;
  const int Dn = DT > 0 ? DT : D;
  T t = NORM == 2 ? A::template sq_first<MODE>(q[0], c[0]) : A::abs_first(q[0], c[0]);
#pragma unroll
  for (int d = 1; d < (DT > 0 ? DT : KDMAX); ++d) {
    if (d < Dn) t = NORM == 2 ? A::template sq_acc<MODE>(t, q[d], c[d]) : A::abs_acc(t, q[d], c[d]);
  }
  return A::val(t);
}

template <typename T, int DT, int NORM, int MODE>
__global__ void __launch_bounds__(KW * 32)
    knn_fwd_kernel(const T* __restrict__ p1, const T* __restrict__ p2,
                   const int64_t* __restrict__ len1, const int64_t* __restrict__ len2, int64_t N,
                   int64_t P1, int64_t P2, int D, int K, int qblocks, T* __restrict__ dists,
                   int64_t* __restrict__ idxs) {
  using A = KnnArith<T>;
  using V = typename A::V;
  constexpr int DC = DT > 0 ? DT : KDMAX;
  // D=3 uses long tiles (fewer block barriers); general D keeps 256 targets
  constexpr int TILE = DT == 3 ? KTILE : 256;
  __shared__ T s_c[TILE][DC];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n = blockIdx.x / qblocks;
  const int64_t q0 = (int64_t)(blockIdx.x % qblocks) * (KW * KQ) + warp * KQ;
  const int64_t L1 = len1 ? min64(max64(len1[n], 0), P1) : P1;
  const int64_t L2 = len2 ? min64(max64(len2[n], 0), P2) : P2;
  const int Dn = DT > 0 ? DT : D;

  T q[KQ][DC];
  bool qv[KQ];
#pragma unroll
  for (int i = 0; i < KQ; ++i) {
    qv[i] = q0 + i < L1;
#pragma unroll
    for (int d = 0; d < DC; ++d)
      q[i][d] = (qv[i] && d < Dn) ? p1[(n * P1 + q0 + i) * Dn + d] : T(0.0f);
  }
  // fp32, D=3, squared L2: queries also kept as packed pairs {q_2i, q_2i+1}
  constexpr bool kPacked = std::is_same<T, float>::value && DT == 3 && NORM == 2 && (KQ % 2 == 0);
  u64 QP[kPacked ? KQ / 2 : 1][3];
  if constexpr (kPacked) {
#pragma unroll
    for (int ip = 0; ip < KQ / 2; ++ip)
#pragma unroll
      for (int d = 0; d < 3; ++d) QP[ip][d] = pk((float)q[2 * ip][d], (float)q[2 * ip + 1][d]);
  }
  V Ld[KQ], thr[KQ];
  int Li[KQ];
#pragma unroll
  for (int i = 0; i < KQ; ++i) {
    Ld[i] = (V)INFINITY;
    Li[i] = -1;
    thr[i] = (V)INFINITY;
  }
  const bool any_q = q0 < L1;
  const int64_t blk_q0 = (int64_t)(blockIdx.x % qblocks) * (KW * KQ);
  const bool blk_active = blk_q0 < L1;

  if (blk_active) {
    for (int64_t t0 = 0; t0 < L2; t0 += TILE) {
      const int nt = (int)min64(TILE, L2 - t0);
      __syncthreads();
      {
        const T* src = p2 + (n * P2 + t0) * Dn;
        for (int e = threadIdx.x; e < nt * Dn; e += blockDim.x) {
          const int c = e / Dn, d = e - c * Dn;
          s_c[c][d] = src[e];
        }
      }
      __syncthreads();
      if (any_q) {
        const int nsteps = (nt + KSTEP - 1) / KSTEP;
#pragma unroll 1
        for (int s = 0; s < nsteps; ++s) {
          const int c = s * KSTEP + lane;
          const bool cv = c < nt;
          T cc[DC];
#pragma unroll
          for (int d = 0; d < DC; ++d) cc[d] = (cv && d < Dn) ? s_c[c][d] : T(0.0f);
          const int cidx = (int)(t0 + c);
          // all distances and filters of the step first; one branch decides
          // whether any query of this warp has a candidate at all
          V dv[KQ];
          unsigned bal[KQ];
          if constexpr (kPacked) {
            // two queries per packed fp32x2 sub/mul; the sums stay scalar .rn adds
            // (never fused), giving ((dx*dx + dy*dy) + dz*dz) exactly
            const u64 CX = pk(cc[0], cc[0]), CY = pk(cc[1], cc[1]), CZ = pk(cc[2], cc[2]);
#pragma unroll
            for (int ip = 0; ip < KQ / 2; ++ip) {
              const u64 dx = sub2(QP[ip][0], CX), dy = sub2(QP[ip][1], CY), dz = sub2(QP[ip][2], CZ);
              float x0, x1, y0, y1, z0, z1;
              upk(mul2(dx, dx), x0, x1);
              upk(mul2(dy, dy), y0, y1);
              upk(mul2(dz, dz), z0, z1);
              dv[2 * ip] = __fadd_rn(__fadd_rn(x0, y0), z0);
              dv[2 * ip + 1] = __fadd_rn(__fadd_rn(x1, y1), z1);
            }
          } else {
#pragma unroll
            for (int i = 0; i < KQ; ++i) dv[i] = knn_dist<T, DT, NORM, MODE>(q[i], cc, Dn);
          }
          // one vote for the whole step; the per-query ballots only when some
          // lane holds a candidate
          bool pr[KQ];
          bool anyp = false;
#pragma unroll
          for (int i = 0; i < KQ; ++i) {
            pr[i] = qv[i] && cv && dv[i] < thr[i];
            anyp |= pr[i];
          }
          if (__any_sync(0xffffffffu, anyp)) {
#pragma unroll
            for (int i = 0; i < KQ; ++i) bal[i] = __ballot_sync(0xffffffffu, pr[i]);
#pragma unroll
            for (int i = 0; i < KQ; ++i) {
              while (bal[i]) {
                const int src = __ffs(bal[i]) - 1;
                bal[i] &= bal[i] - 1;
                const V cd = __shfl_sync(0xffffffffu, dv[i], src);
                if (cd < thr[i]) {
                  const int ci = cidx - lane + src;
                  const V upd = __shfl_up_sync(0xffffffffu, Ld[i], 1);
                  const int upi = __shfl_up_sync(0xffffffffu, Li[i], 1);
                  if (cd < Ld[i]) {
                    const bool take_prev = lane > 0 && cd < upd;
                    Ld[i] = take_prev ? upd : cd;
                    Li[i] = take_prev ? upi : ci;
                  }
                  thr[i] = __shfl_sync(0xffffffffu, Ld[i], K - 1);
                }
              }
            }
          }
        }
      }
    }
  }
  // write-out: every row of this warp's range, valid or padding
  if (lane < K) {
#pragma unroll
    for (int i = 0; i < KQ; ++i) {
      const int64_t row = q0 + i;
      if (row >= P1) break;
      const int64_t o = (n * P1 + row) * K + lane;
      const bool ok = qv[i] && Li[i] >= 0;
      dists[o] = ok ? A::from(Ld[i]) : T(0.0f);
      idxs[o] = ok ? (int64_t)Li[i] : -1;
    }
  }
}

// fp32, D=3, squared L2 (the benchmark's knn case): the same warp-distributed
// top-K lists, with the per-target work cut to the arithmetic plus one packed
// op of filtering:
//   * target tiles land by 1-D bulk copies (TMA) into two shared buffers (the
//     copy of tile t+2 runs while tile t is scanned) and are rewritten once per
//     tile into one structure-of-arrays tile, NaN padded to whole steps;
//   * a step covers 64 targets, two per lane: one 64-bit shared load gives the
//     lane's {x_a, x_b} (likewise y, z), and every query is held as {q, q}, so
//     each packed fp32x2 sub/mul serves the lane's two targets; the adds are
//     scalar .rn (the reference's ((dx*dx + dy*dy) + dz*dz), every operation
//     rounded, never fused);
//   * the filter is ONE packed subtraction per query, d - thr: for floats
//     fl(d - thr) is negative exactly when d < thr (distinct floats never
//     subtract to zero), +inf thresholds pass everything, the -inf threshold of
//     an invalid query slot and the NaN padding pass nothing -- so the pass
//     bits are sign bits, OR-ed across queries with logic ops, and one warp
//     vote per step decides whether any insertion runs;
//   * insertions run per query in increasing target index (lane-major, the
//     lane's first target before its second), which with "land after equal
//     entries" keeps the list "K smallest by (dist, idx)"; a candidate that
//     passed a stale threshold lands at a lane >= K and never reaches the output.
// SEED: the threshold starts at an upper bound of the query's K-th distance
// (knn_seed_kernel below) instead of +inf.
static __device__ unsigned g_knn_device_error = 0;
constexpr int KT3 = 1024;  // targets per tile (two bulk-copy buffers + one scan tile)
constexpr int KP3 = 64;    // targets per step (two per lane)
#ifndef TPO_KW3
#define TPO_KW3 8
#endif
constexpr int KW3 = TPO_KW3;  // warps per CTA of the fp32 D=3 kernel

__device__ __forceinline__ void knn_list_insert(float& L, int& I, float cd, int ci, int lane) {
  const float upd = __shfl_up_sync(0xffffffffu, L, 1);
  const int upi = __shfl_up_sync(0xffffffffu, I, 1);
  if (cd < L) {
    const bool take_prev = lane > 0 && cd < upd;
    L = take_prev ? upd : cd;
    I = take_prev ? upi : ci;
  }
}

template <int KQF, bool SEED>
__global__ void __launch_bounds__(KW3 * 32)
    knn_fwd_f32x3_kernel(const float* __restrict__ p1, const float* __restrict__ p2,
                         const int64_t* __restrict__ len1, const int64_t* __restrict__ len2,
                         int64_t N, int64_t P1, int64_t P2, int K, int qblocks,
                         float* __restrict__ dists, int64_t* __restrict__ idxs) {
  static_assert(KT3 % KP3 == 0, "tile/step shape");
  __shared__ __align__(16) float s_raw[2][KT3 * 3];
  __shared__ __align__(16) float s_soa[3][KT3];
  __shared__ __align__(8) unsigned long long s_bar[2];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t n = blockIdx.x / qblocks;
  const int64_t blk_q0 = (int64_t)(blockIdx.x % qblocks) * (KW3 * KQF);
  const int64_t q0 = blk_q0 + warp * KQF;
  const int64_t L1 = len1 ? min64(max64(len1[n], 0), P1) : P1;
  const int64_t L2 = len2 ? min64(max64(len2[n], 0), P2) : P2;
  const float qnan = __int_as_float(0x7fffffff);
  const float pinf = __int_as_float(0x7f800000);
  // Seeded launches follow knn_seed_kernel with programmatic serialisation:
  // until pdl_wait() only the inputs are read (queries, the first target
  // tiles) -- the seeds in dists and the seed kernel's scratch in idxs are
  // touched after it.
  if (blk_q0 >= L1) {  // no valid query in this CTA: padding rows only
    pdl_wait();
    if (lane < K)
      for (int i = 0; i < KQF; ++i) {
        const int64_t row = q0 + i;
        if (row >= P1) break;
        dists[(n * P1 + row) * K + lane] = 0.f;
        idxs[(n * P1 + row) * K + lane] = -1;
      }
    return;
  }

  u64 QQ[KQF][3], THR[KQF];
  float cap[KQF], Ld[KQF];
  int Li[KQF];
  bool qv[KQF];
#pragma unroll
  for (int i = 0; i < KQF; ++i) {
    qv[i] = q0 + i < L1;
    Ld[i] = pinf;
    Li[i] = -1;
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      const float a = qv[i] ? p1[(n * P1 + q0 + i) * 3 + d] : 0.f;
      QQ[i][d] = pk(a, a);
    }
  }
  const bool any_q = q0 < L1;
  const int ntiles = (int)((L2 + KT3 - 1) / KT3);
  if (threadIdx.x == 0) {
    mbar_init(&s_bar[0], 1);
    mbar_init(&s_bar[1], 1);
  }
  __syncthreads();
  // start tile t's copy into buffer t & 1: the 16-byte aligned body by one bulk
  // copy, the rest by plain loads
  auto issue = [&](int t) {
    const int64_t t0 = (int64_t)t * KT3;
    const int nt = (int)min64(KT3, L2 - t0);
    const float* src = p2 + (n * P2 + t0) * 3;
    float* dst = s_raw[t & 1];
    const int nfl = nt * 3;
    const int bulk = (((uintptr_t)src & 15) == 0) ? (nfl & ~3) : 0;
    if (threadIdx.x == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect_tx(&s_bar[t & 1], (unsigned)bulk * 4u);
      if (bulk) bulk_g2s(dst, src, (unsigned)bulk * 4u, &s_bar[t & 1]);
    }
    for (int e = bulk + threadIdx.x; e < nfl; e += blockDim.x) dst[e] = __ldg(src + e);
  };
  unsigned phase[2] = {0u, 0u};
  issue(0);
  if (ntiles > 1) issue(1);
  pdl_wait();
#pragma unroll
  for (int i = 0; i < KQF; ++i) {
    // cap: an upper bound on the query's K-th distance, raised by one ulp so a
    // candidate equal to it still passes (the seed is the K-th smallest distance
    // over a subset of the targets: at least K targets lie at or below it)
    cap[i] = pinf;
    if (SEED && qv[i]) {
      const float T = dists[(n * P1 + q0 + i) * K];  // written by knn_seed_kernel
      if (T < pinf) cap[i] = __uint_as_float(__float_as_uint(T) + 1u);
    }
    const float th = qv[i] ? cap[i] : -pinf;
    THR[i] = pk(th, th);
  }
  for (int t = 0; t < ntiles; ++t) {
    const int b = t & 1;
    const int t0 = t * KT3;
    const int nt = (int)min64(KT3, L2 - t0);
    const int nsteps = (nt + KP3 - 1) / KP3;
    mbar_wait(&s_bar[b], phase[b], &g_knn_device_error);
    phase[b] ^= 1u;
    __syncthreads();  // tile t complete in s_raw[b]; the previous scan is done with s_soa
    {
      const float* raw = s_raw[b];
      for (int e = threadIdx.x; e < nsteps * KP3; e += blockDim.x) {
        const bool ok = e < nt;
        s_soa[0][e] = ok ? raw[e * 3] : qnan;
        s_soa[1][e] = ok ? raw[e * 3 + 1] : qnan;
        s_soa[2][e] = ok ? raw[e * 3 + 2] : qnan;
      }
    }
    __syncthreads();  // s_soa ready, s_raw[b] free
    if (t + 2 < ntiles) issue(t + 2);
    if (any_q) {
#pragma unroll 1
      for (int s = 0; s < nsteps; ++s) {
        const int e = s * KP3 + 2 * lane;
        const u64 X = *reinterpret_cast<const u64*>(&s_soa[0][e]);
        const u64 Y = *reinterpret_cast<const u64*>(&s_soa[1][e]);
        const u64 Z = *reinterpret_cast<const u64*>(&s_soa[2][e]);
        u64 dv[KQF], sg[KQF];
        unsigned acc = 0;
#pragma unroll
        for (int i = 0; i < KQF; ++i) {
          const u64 dx = sub2(QQ[i][0], X), dy = sub2(QQ[i][1], Y), dz = sub2(QQ[i][2], Z);
          float x0, x1, y0, y1, z0, z1;
          upk(mul2(dx, dx), x0, x1);
          upk(mul2(dy, dy), y0, y1);
          upk(mul2(dz, dz), z0, z1);
          dv[i] = pk(__fadd_rn(__fadd_rn(x0, y0), z0), __fadd_rn(__fadd_rn(x1, y1), z1));
          sg[i] = sub2(dv[i], THR[i]);
          acc |= (unsigned)sg[i] | (unsigned)(sg[i] >> 32);
        }
        if (__any_sync(0xffffffffu, (int)acc < 0)) {
          const int cbase = t0 + s * KP3;
          // the lane's pass bits (two per query, from the sign bits) and, by one
          // redux, the warp's set of queries with candidates
          unsigned m = 0;
#pragma unroll
          for (int i = 0; i < KQF; ++i)
            m |= (((unsigned)sg[i] >> 31) | (((unsigned)(sg[i] >> 32) >> 31) << 1)) << (2 * i);
          const unsigned qm = __reduce_or_sync(0xffffffffu, m);
#pragma unroll
          for (int i = 0; i < KQF; ++i) {
            if (!((qm >> (2 * i)) & 3u)) continue;
            const unsigned mine = (m >> (2 * i)) & 3u;
            unsigned bal = __ballot_sync(0xffffffffu, mine != 0u);
            float va, vb;
            upk(dv[i], va, vb);
            while (bal) {
              const int src = __ffs(bal) - 1;
              bal &= bal - 1;
              const unsigned pb = __shfl_sync(0xffffffffu, mine, src);
              if (pb & 1u) knn_list_insert(Ld[i], Li[i], __shfl_sync(0xffffffffu, va, src), cbase + 2 * src, lane);
              if (pb & 2u) knn_list_insert(Ld[i], Li[i], __shfl_sync(0xffffffffu, vb, src), cbase + 2 * src + 1, lane);
            }
            float th = __shfl_sync(0xffffffffu, Ld[i], K - 1);
            if constexpr (SEED) th = fminf(th, cap[i]);
            THR[i] = pk(th, th);
          }
        }
      }
    }
  }
  if (lane < K) {
#pragma unroll
    for (int i = 0; i < KQF; ++i) {
      const int64_t row = q0 + i;
      if (row >= P1) break;
      const int64_t o = (n * P1 + row) * K + lane;
      const bool ok = qv[i] && Li[i] >= 0;
      dists[o] = ok ? Ld[i] : 0.f;
      idxs[o] = ok ? (int64_t)Li[i] : -1;
    }
  }
}

// ---- threshold seeds for the fp32 D=3 kernel ----
// The scan of the kernel above accepts a candidate whenever it beats the K-th
// entry of the query's list so far; over targets in index order that is about
// K(1 + ln(L2/K)) insertions per query (~110 for config 4), and the insertions,
// not the distances, dominate the kernel's instructions.  A seed T -- the K-th
// smallest distance of the query to some subset of the targets, computed with
// the kernel's own arithmetic -- is an upper bound on the true K-th distance,
// so capping the threshold at T from the start changes no result (every target
// of the final list lies at or below T) but rejects almost every candidate that
// would be evicted later.  The subset is the 128 targets around the query's
// position in a Morton order of the targets (a counting sort over 16^3 cells of
// the batch's bounding box), and T is the K-th smallest of the 32 lane minima of
// those 128 distances (K <= 32 lanes each holding a distinct target): ~30
// accepted candidates per query on uniform clouds instead of ~110.  The scan
// order, the acceptance rule and the output are unchanged.
constexpr int KC_AXIS_BITS = 4;
constexpr int KC_CELLS = 1 << (3 * KC_AXIS_BITS);  // 4096 Morton cells
constexpr int KC_THREADS = 1024;
constexpr int KC_PPT = 8;        // targets per thread held in registers (larger clouds loop)
constexpr int KSD_WINDOW = 128;  // targets per seed window (4 per lane)
constexpr int KSD_WARPS = 8;
constexpr int KSD_QPW = 4;  // queries per warp, processed together
constexpr int KSD_QPB = KSD_WARPS * KSD_QPW;
constexpr int64_t kSeedMinTargets = 1024;  // below this the plain scan is short anyway

struct KnnCells {
  float* hdr;    // per batch: lo[3], inv[3] (cell = (x - lo) * inv), 8 floats
  int* cstart;   // per batch: KC_CELLS + 1 cell starts into `order`
  void* order;   // per batch, the L2 valid targets in cell order: float4 {x, y, z, 0}
                 // copies (COORDS) or int32 indices (when the copies do not fit)
};

static size_t align16(size_t v) { return (v + 15) & ~(size_t)15; }

static size_t knn_seed_scratch_bytes(int64_t N, int64_t P2, bool coords) {
  return align16((size_t)N * 8 * sizeof(float)) + align16((size_t)N * (KC_CELLS + 1) * sizeof(int)) +
         (size_t)N * P2 * (coords ? sizeof(float4) : sizeof(int));
}

static KnnCells knn_cells_layout(void* base, int64_t N) {
  char* p = (char*)base;
  KnnCells c;
  c.hdr = (float*)p;
  p += align16((size_t)N * 8 * sizeof(float));
  c.cstart = (int*)p;
  p += align16((size_t)N * (KC_CELLS + 1) * sizeof(int));
  c.order = p;
  return c;
}

static bool knn_seed_enabled() {
  static const int on = [] {
    const char* e = getenv("TPO_KNN_SEED");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on != 0;
}

__device__ __forceinline__ unsigned kc_spread4(unsigned v) {
  return (v & 1u) | ((v & 2u) << 2) | ((v & 4u) << 4) | ((v & 8u) << 6);
}

__device__ __forceinline__ int kc_cell(float x, float y, float z, const float* h) {
  const float lim = (float)((1 << KC_AXIS_BITS) - 1);
  const unsigned cx = (unsigned)fminf(fmaxf((x - h[0]) * h[3], 0.f), lim);
  const unsigned cy = (unsigned)fminf(fmaxf((y - h[1]) * h[4], 0.f), lim);
  const unsigned cz = (unsigned)fminf(fmaxf((z - h[2]) * h[5], 0.f), lim);
  return (int)(kc_spread4(cx) | (kc_spread4(cy) << 1) | (kc_spread4(cz) << 2));
}

// One CTA per batch: bounding box, cell histogram, scan, scatter of the target
// indices.  Up to KC_THREADS * KC_PPT targets stay in registers between the
// passes (one round of loads); larger clouds re-read them.
template <bool COORDS>
__global__ void __launch_bounds__(KC_THREADS)
    knn_cells_kernel(const float* __restrict__ p2, const int64_t* __restrict__ len2, int64_t N,
                     int64_t P2, float* __restrict__ hdr, int* __restrict__ cstart,
                     void* __restrict__ order) {
  __shared__ int s_cnt[KC_CELLS];
  __shared__ float s_red[6][KC_THREADS / 32];
  __shared__ int s_wsum[KC_THREADS / 32];
  __shared__ float s_h[6];
  pdl_trigger();  // the seed kernel may start loading its queries
  const int64_t n = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int L2 = (int)(len2 ? min64(max64(len2[n], 0), P2) : P2);
  const float* src = p2 + n * P2 * 3;
  const bool regs = L2 <= KC_THREADS * KC_PPT;
  const float pinf = __int_as_float(0x7f800000);
  float px[KC_PPT], py[KC_PPT], pz[KC_PPT];
  float mn[3] = {pinf, pinf, pinf};
  float mx[3] = {-pinf, -pinf, -pinf};
  auto fold = [&](float x, float y, float z) {
    mn[0] = fminf(mn[0], x); mx[0] = fmaxf(mx[0], x);
    mn[1] = fminf(mn[1], y); mx[1] = fmaxf(mx[1], y);
    mn[2] = fminf(mn[2], z); mx[2] = fmaxf(mx[2], z);
  };
  if (regs) {
#pragma unroll
    for (int j = 0; j < KC_PPT; ++j) {
      const int i = tid + j * KC_THREADS;
      const bool ok = i < L2;
      px[j] = ok ? src[i * 3] : 0.f;
      py[j] = ok ? src[i * 3 + 1] : 0.f;
      pz[j] = ok ? src[i * 3 + 2] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < KC_PPT; ++j)
      if (tid + j * KC_THREADS < L2) fold(px[j], py[j], pz[j]);
  } else {
    for (int i = tid; i < L2; i += KC_THREADS) fold(src[i * 3], src[i * 3 + 1], src[i * 3 + 2]);
  }
#pragma unroll
  for (int d = 0; d < 3; ++d)
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      mn[d] = fminf(mn[d], __shfl_xor_sync(0xffffffffu, mn[d], o));
      mx[d] = fmaxf(mx[d], __shfl_xor_sync(0xffffffffu, mx[d], o));
    }
  if (lane == 0)
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      s_red[d][warp] = mn[d];
      s_red[3 + d][warp] = mx[d];
    }
  for (int c = tid; c < KC_CELLS; c += KC_THREADS) s_cnt[c] = 0;
  __syncthreads();
  if (tid < 3) {
    float lo = s_red[tid][0], hi = s_red[3 + tid][0];
    for (int w = 1; w < KC_THREADS / 32; ++w) {
      lo = fminf(lo, s_red[tid][w]);
      hi = fmaxf(hi, s_red[3 + tid][w]);
    }
    const float ext = hi - lo;
    // cells per axis / extent; 0 for a flat (or empty / non-finite) axis
    const float inv = (ext > 0.f && ext < pinf) ? (float)(1 << KC_AXIS_BITS) / ext : 0.f;
    s_h[tid] = (lo > -pinf && lo < pinf) ? lo : 0.f;
    s_h[3 + tid] = inv;
  }
  __syncthreads();
  int cell[KC_PPT];
  if (regs) {
#pragma unroll
    for (int j = 0; j < KC_PPT; ++j) {
      cell[j] = kc_cell(px[j], py[j], pz[j], s_h);
      if (tid + j * KC_THREADS < L2) atomicAdd(&s_cnt[cell[j]], 1);
    }
  } else {
    for (int i = tid; i < L2; i += KC_THREADS)
      atomicAdd(&s_cnt[kc_cell(src[i * 3], src[i * 3 + 1], src[i * 3 + 2], s_h)], 1);
  }
  __syncthreads();
  // exclusive scan of the 4096 counts: 4 per thread, then over the block
  constexpr int PER = KC_CELLS / KC_THREADS;
  int v[PER], sum = 0;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    v[j] = s_cnt[tid * PER + j];
    sum += v[j];
  }
  int incl = sum;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) s_wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int w = s_wsum[lane];
    int wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    s_wsum[lane] = wi - w;
  }
  __syncthreads();
  int run = s_wsum[warp] + incl - sum;
  int* cs = cstart + n * (KC_CELLS + 1);
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    cs[tid * PER + j] = run;
    s_cnt[tid * PER + j] = run;  // becomes the scatter cursor
    run += v[j];
  }
  if (tid == 0) {
    cs[KC_CELLS] = L2;
#pragma unroll
    for (int d = 0; d < 6; ++d) hdr[n * 8 + d] = s_h[d];
  }
  __syncthreads();
  auto put = [&](int pos, int i, float x, float y, float z) {
    if constexpr (COORDS) ((float4*)order)[n * P2 + pos] = make_float4(x, y, z, 0.f);
    else ((int*)order)[n * P2 + pos] = i;
  };
  if (regs) {
#pragma unroll
    for (int j = 0; j < KC_PPT; ++j) {
      const int i = tid + j * KC_THREADS;
      if (i < L2) put(atomicAdd(&s_cnt[cell[j]], 1), i, px[j], py[j], pz[j]);
    }
  } else {
    for (int i = tid; i < L2; i += KC_THREADS) {
      const float x = src[i * 3], y = src[i * 3 + 1], z = src[i * 3 + 2];
      put(atomicAdd(&s_cnt[kc_cell(x, y, z, s_h)], 1), i, x, y, z);
    }
  }
}

// One warp per KSD_QPW queries, processed together so that their loads and
// shuffle chains overlap: the seed T (see above) into dists[row, 0].
template <bool COORDS>
__global__ void __launch_bounds__(KSD_WARPS * 32)
    knn_seed_kernel(const float* __restrict__ p1, const float* __restrict__ p2,
                    const int64_t* __restrict__ len1, const int64_t* __restrict__ len2, int64_t N,
                    int64_t P1, int64_t P2, int K, int sblocks, const float* __restrict__ hdr,
                    const int* __restrict__ cstart, const void* __restrict__ order,
                    float* __restrict__ seeds) {
  pdl_trigger();  // the scan may start loading its queries and first tiles
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t n = blockIdx.x / sblocks;
  const int64_t qb = (int64_t)(blockIdx.x % sblocks) * KSD_QPB + warp * KSD_QPW;
  const int64_t L1 = len1 ? min64(max64(len1[n], 0), P1) : P1;
  if (qb >= L1) return;
  const int L2 = (int)(len2 ? min64(max64(len2[n], 0), P2) : P2);
  const float* h = hdr + n * 8;
  const int* cs = cstart + n * (KC_CELLS + 1);
  const int* od = (const int*)order + n * P2;
  const float4* oc = (const float4*)order + n * P2;
  const float* tp = p2 + n * P2 * 3;
  constexpr int J = KSD_WINDOW / 32;
  float qx[KSD_QPW], qy[KSD_QPW], qz[KSD_QPW], m[KSD_QPW];
  int a[KSD_QPW];
  float4 tc[KSD_QPW][J];
#pragma unroll
  for (int u = 0; u < KSD_QPW; ++u) {
    const int64_t q = min64(qb + u, L1 - 1);  // past L1: a duplicate, not stored
    qx[u] = p1[(n * P1 + q) * 3];
    qy[u] = p1[(n * P1 + q) * 3 + 1];
    qz[u] = p1[(n * P1 + q) * 3 + 2];
  }
  // launched after knn_cells_kernel with programmatic serialisation: the
  // queries above are inputs; the cell table is read after this wait
  pdl_wait();
#pragma unroll
  for (int u = 0; u < KSD_QPW; ++u) {
    const int c = kc_cell(qx[u], qy[u], qz[u], h);
    const int mid = (cs[c] + cs[c + 1]) >> 1;
    a[u] = max(0, min(mid - KSD_WINDOW / 2, L2 - KSD_WINDOW));
  }
  // the window's targets (NaN past L2: a NaN distance never wins a min)
  const float qnan = __int_as_float(0x7fffffff);
#pragma unroll
  for (int u = 0; u < KSD_QPW; ++u)
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int t = a[u] + j * 32 + lane;
      if (t >= L2) {
        tc[u][j] = make_float4(qnan, qnan, qnan, 0.f);
      } else if constexpr (COORDS) {
        tc[u][j] = oc[t];
      } else {
        const float* c = tp + (int64_t)od[t] * 3;
        tc[u][j] = make_float4(c[0], c[1], c[2], 0.f);
      }
    }
#pragma unroll
  for (int u = 0; u < KSD_QPW; ++u) {
    m[u] = __int_as_float(0x7f800000);
#pragma unroll
    for (int j = 0; j < J; ++j) {
      // the fp32 D=3 kernel's arithmetic: ((dx*dx + dy*dy) + dz*dz), dx = q - t,
      // every operation rounded
      const float4 c = tc[u][j];
      const float dx = __fsub_rn(qx[u], c.x), dy = __fsub_rn(qy[u], c.y), dz = __fsub_rn(qz[u], c.z);
      const float d = __fadd_rn(__fadd_rn(__fmul_rn(dx, dx), __fmul_rn(dy, dy)), __fmul_rn(dz, dz));
      m[u] = fminf(m[u], d);
    }
  }
  // K-th smallest of the 32 lane minima (each lane's targets are distinct):
  // bitonic sort over the warp
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const bool lo = ((lane & j) == 0) == ((lane & k) == 0);
#pragma unroll
      for (int u = 0; u < KSD_QPW; ++u) {
        const float p = __shfl_xor_sync(0xffffffffu, m[u], j);
        m[u] = lo ? fminf(m[u], p) : fmaxf(m[u], p);
      }
    }
#pragma unroll
  for (int u = 0; u < KSD_QPW; ++u) {
    const float T = __shfl_sync(0xffffffffu, m[u], K - 1);
    if (lane == 0 && qb + u < L1) seeds[(n * P1 + qb + u) * K] = T;
  }
}

#ifndef TPO_KQF
#define TPO_KQF 4
#endif

template <int Q>
static int launch_knn_f32x3_q(const float* p1, const float* p2, const int64_t* l1, const int64_t* l2,
                              int64_t N, int64_t P1, int64_t P2, int K, float* dists, int64_t* idxs,
                              cudaStream_t st) {
  const int qblocks = (int)((P1 + KW3 * Q - 1) / (KW3 * Q));
  const int64_t ctas = N * qblocks;
  if (ctas <= 0) return TPO_OK;
  const size_t room = (size_t)N * P1 * K * sizeof(int64_t);
  const bool coords = room >= knn_seed_scratch_bytes(N, P2, true);
  const bool seed = knn_seed_enabled() && P2 >= kSeedMinTargets &&
                    (coords || room >= knn_seed_scratch_bytes(N, P2, false));
  if (seed) {
    // the cell order of the targets lives in the idxs buffer until the main
    // kernel overwrites it; the seeds in dists[row, 0]
    const KnnCells c = knn_cells_layout(idxs, N);
    if (coords)
      knn_cells_kernel<true><<<(unsigned)N, KC_THREADS, 0, st>>>(p2, l2, N, P2, c.hdr, c.cstart, c.order);
    else
      knn_cells_kernel<false><<<(unsigned)N, KC_THREADS, 0, st>>>(p2, l2, N, P2, c.hdr, c.cstart, c.order);
    int s = check_launch();
    if (s) return s;
    const int64_t sblocks = (P1 + KSD_QPB - 1) / KSD_QPB;
    s = launch_pdl(coords ? knn_seed_kernel<true> : knn_seed_kernel<false>, dim3((unsigned)(N * sblocks)),
                   dim3(KSD_WARPS * 32), 0, st, p1, p2, l1, l2, N, P1, P2, K, (int)sblocks,
                   (const float*)c.hdr, (const int*)c.cstart, (const void*)c.order, dists);
    if (s) return s;
    return launch_pdl(knn_fwd_f32x3_kernel<Q, true>, dim3((unsigned)ctas), dim3(KW3 * 32), 0, st, p1, p2,
                      l1, l2, N, P1, P2, K, qblocks, dists, idxs);
  } else {
    knn_fwd_f32x3_kernel<Q, false><<<(unsigned)ctas, KW3 * 32, 0, st>>>(
        p1, p2, l1, l2, N, P1, P2, K, qblocks, dists, idxs);
  }
  return check_launch();
}

// TPO_KQF queries per warp; 2 when that leaves fewer CTAs than about two per SM
// (small problems, e.g. one rank's share of a split batch), so every SM has work.
static int launch_knn_f32x3(const float* p1, const float* p2, const int64_t* l1, const int64_t* l2,
                            int64_t N, int64_t P1, int64_t P2, int K, float* dists, int64_t* idxs,
                            cudaStream_t st) {
  constexpr int Q = TPO_KQF;
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!sms[dev & 63]) cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev);
  const int64_t ctas = N * ((P1 + KW3 * Q - 1) / (KW3 * Q));
  if (Q > 2 && ctas < 2LL * sms[dev & 63])
    return launch_knn_f32x3_q<2>(p1, p2, l1, l2, N, P1, P2, K, dists, idxs, st);
  return launch_knn_f32x3_q<Q>(p1, p2, l1, l2, N, P1, P2, K, dists, idxs, st);
}

template <typename T, int DT, int NORM, int MODE>
static int launch_knn_fwd(const T* p1, const T* p2, const int64_t* l1, const int64_t* l2, int64_t N,
                          int64_t P1, int64_t P2, int D, int K, T* dists, int64_t* idxs,
                          cudaStream_t st) {
  const int qblocks = (int)((P1 + KW * KQ - 1) / (KW * KQ));
  const int64_t ctas = N * qblocks;
  if (ctas <= 0) return TPO_OK;
  knn_fwd_kernel<T, DT, NORM, MODE><<<(unsigned)ctas, KW * 32, 0, st>>>(p1, p2, l1, l2, N, P1, P2, D,
                                                                       K, qblocks, dists, idxs);
  return check_launch();
}

template <typename T, int MODE>
static int dispatch_knn_fwd(const void* p1, const void* p2, const int64_t* l1, const int64_t* l2,
                            int64_t N, int64_t P1, int64_t P2, int64_t D, int64_t norm, int64_t K,
                            void* dists, int64_t* idxs, cudaStream_t st) {
  const T* a = (const T*)p1;
  const T* b = (const T*)p2;
  T* o = (T*)dists;
  if constexpr (std::is_same<T, float>::value) {
    if (D == 3 && norm == 2)
      return launch_knn_f32x3(a, b, l1, l2, N, P1, P2, (int)K, o, idxs, st);
  }
  if (D == 3)
    return norm == 2 ? launch_knn_fwd<T, 3, 2, MODE>(a, b, l1, l2, N, P1, P2, 3, (int)K, o, idxs, st)
                     : launch_knn_fwd<T, 3, 1, MODE>(a, b, l1, l2, N, P1, P2, 3, (int)K, o, idxs, st);
  return norm == 2 ? launch_knn_fwd<T, 0, 2, MODE>(a, b, l1, l2, N, P1, P2, (int)D, (int)K, o, idxs, st)
                   : launch_knn_fwd<T, 0, 1, MODE>(a, b, l1, l2, N, P1, P2, (int)D, (int)K, o, idxs, st);
}

// ---- any D, K up to 32*KR: the general path (the reference's V0/V1 range) ----
// One warp per query; the CTA's warps share nothing but L1 (targets are read
// straight from global memory, lane c of a step taking target t0 + c, so every
// D works without a shared-memory tile).  The running top-K list is spread over
// the warp in KR rows: position p = r*32 + lane.  A candidate is accepted when
// it beats the K-th entry and inserted by shifting every later position by one
// (shuffle-up within a row, lane 31 of the row before feeding lane 0).  Same
// acceptance/tie rule as the fast kernel: "K smallest by (dist, idx)".
constexpr int KGW = 8;  // warps (queries) per CTA in the general kernel

template <typename T, int NORM, int KR>
__global__ void __launch_bounds__(KGW * 32)
    knn_fwd_general_kernel(const T* __restrict__ p1, const T* __restrict__ p2,
                           const int64_t* __restrict__ len1, const int64_t* __restrict__ len2,
                           int64_t N, int64_t P1, int64_t P2, int D, int K, int64_t qblocks,
                           T* __restrict__ dists, int64_t* __restrict__ idxs) {
  using A = KnnArith<T>;
  using V = typename A::V;
  extern __shared__ __align__(16) unsigned char knn_gsmem[];
  T* sq = reinterpret_cast<T*>(knn_gsmem) + (threadIdx.x >> 5) * D;  // this warp's query
  const int lane = threadIdx.x & 31;
  const int64_t n = blockIdx.x / qblocks;
  const int64_t row = (blockIdx.x % qblocks) * KGW + (threadIdx.x >> 5);
  if (row >= P1) return;  // whole warp: nothing to write
  const int64_t L1 = len1 ? min64(max64(len1[n], 0), P1) : P1;
  const int64_t L2 = len2 ? min64(max64(len2[n], 0), P2) : P2;
  const bool qv = row < L1;
  for (int d = lane; d < D; d += 32) sq[d] = p1[(n * P1 + row) * D + d];
  __syncwarp();
  V Ld[KR];
  int Li[KR];
#pragma unroll
  for (int r = 0; r < KR; ++r) {
    Ld[r] = (V)INFINITY;
    Li[r] = -1;
  }
  V thr = (V)INFINITY;
  const int kr_last = (K - 1) >> 5, kl_last = (K - 1) & 31;
  if (qv) {
    for (int64_t t0 = 0; t0 < L2; t0 += 32) {
      const int64_t c = t0 + lane;
      const bool cv = c < L2;
      V dv = (V)INFINITY;
      if (cv) {
        const T* pc = p2 + (n * P2 + c) * D;
        T t = NORM == 2 ? A::template sq_first<TPO_ROUND_EXACT>(sq[0], pc[0]) : A::abs_first(sq[0], pc[0]);
        for (int d = 1; d < D; ++d)
          t = NORM == 2 ? A::template sq_acc<TPO_ROUND_EXACT>(t, sq[d], pc[d]) : A::abs_acc(t, sq[d], pc[d]);
        dv = A::val(t);
      }
      unsigned bal = __ballot_sync(0xffffffffu, cv && dv < thr);
      while (bal) {
        const int src = __ffs(bal) - 1;
        bal &= bal - 1;
        const V cd = __shfl_sync(0xffffffffu, dv, src);
        if (!(cd < thr)) continue;
        const int ci = (int)(t0 + src);
        // shift every position holding a larger distance down by one, from the
        // last row up (each row's lane 0 takes the previous row's lane 31 value
        // before that row moves)
#pragma unroll
        for (int r = KR - 1; r >= 0; --r) {
          V upd = __shfl_up_sync(0xffffffffu, Ld[r], 1);
          int upi = __shfl_up_sync(0xffffffffu, Li[r], 1);
          if (r > 0) {
            const V pd = __shfl_sync(0xffffffffu, Ld[r - 1], 31);
            const int pi = __shfl_sync(0xffffffffu, Li[r - 1], 31);
            if (lane == 0) {
              upd = pd;
              upi = pi;
            }
          }
          if (cd < Ld[r]) {
            const bool take_prev = (lane > 0 || r > 0) && cd < upd;
            Ld[r] = take_prev ? upd : cd;
            Li[r] = take_prev ? upi : ci;
          }
        }
        V kth = Ld[0];
#pragma unroll
        for (int r = 1; r < KR; ++r)
          if (r == kr_last) kth = Ld[r];
        thr = __shfl_sync(0xffffffffu, kth, kl_last);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < KR; ++r) {
    const int k = r * 32 + lane;
    if (k < K) {
      const int64_t o = (n * P1 + row) * K + k;
      const bool ok = qv && Li[r] >= 0;
      dists[o] = ok ? A::from(Ld[r]) : T(0.0f);
      idxs[o] = ok ? (int64_t)Li[r] : -1;
    }
  }
}

template <typename T, int NORM, int KR>
static int launch_knn_general(const void* p1, const void* p2, const int64_t* l1, const int64_t* l2,
                              int64_t N, int64_t P1, int64_t P2, int64_t D, int64_t K, void* dists,
                              int64_t* idxs, cudaStream_t st) {
  const int64_t qblocks = (P1 + KGW - 1) / KGW;
  const int64_t ctas = N * qblocks;
  if (ctas <= 0) return TPO_OK;
  const size_t smem = (size_t)KGW * D * sizeof(T);
  auto fn = knn_fwd_general_kernel<T, NORM, KR>;
  if (smem > 48 * 1024)
    if (int s = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)))
      return s;
  fn<<<(unsigned)ctas, KGW * 32, smem, st>>>((const T*)p1, (const T*)p2, l1, l2, N, P1, P2, (int)D,
                                             (int)K, qblocks, (T*)dists, idxs);
  return check_launch();
}

template <typename T, int NORM>
static int dispatch_knn_general(const void* p1, const void* p2, const int64_t* l1, const int64_t* l2,
                                int64_t N, int64_t P1, int64_t P2, int64_t D, int64_t K,
                                void* dists, int64_t* idxs, cudaStream_t st) {
  if (K <= 32) return launch_knn_general<T, NORM, 1>(p1, p2, l1, l2, N, P1, P2, D, K, dists, idxs, st);
  if (K <= 64) return launch_knn_general<T, NORM, 2>(p1, p2, l1, l2, N, P1, P2, D, K, dists, idxs, st);
  if (K <= 128) return launch_knn_general<T, NORM, 4>(p1, p2, l1, l2, N, P1, P2, D, K, dists, idxs, st);
  if (K <= 256) return launch_knn_general<T, NORM, 8>(p1, p2, l1, l2, N, P1, P2, D, K, dists, idxs, st);
  if (K <= 512) return launch_knn_general<T, NORM, 16>(p1, p2, l1, l2, N, P1, P2, D, K, dists, idxs, st);
  return launch_knn_general<T, NORM, 32>(p1, p2, l1, l2, N, P1, P2, D, K, dists, idxs, st);
}

template <typename T>
static int knn_general(const void* p1, const void* p2, const int64_t* l1, const int64_t* l2,
                       int64_t N, int64_t P1, int64_t P2, int64_t D, int64_t norm, int64_t K,
                       void* dists, int64_t* idxs, cudaStream_t st) {
  return norm == 2 ? dispatch_knn_general<T, 2>(p1, p2, l1, l2, N, P1, P2, D, K, dists, idxs, st)
                   : dispatch_knn_general<T, 1>(p1, p2, l1, l2, N, P1, P2, D, K, dists, idxs, st);
}

int knn_forward(int dtype, int flags, const void* p1, const void* p2, const int64_t* l1,
                const int64_t* l2, int64_t N, int64_t P1, int64_t P2, int64_t D, int64_t norm,
                int64_t K, void* dists, int64_t* idxs, cudaStream_t st) {
  if (K > kKnnMaxK) return TPO_ERR_UNSUPPORTED;
  if (D > KDMAX || K > 32) {
    switch (dtype) {
      case TPO_F32: return knn_general<float>(p1, p2, l1, l2, N, P1, P2, D, norm, K, dists, idxs, st);
      case TPO_F16: return knn_general<__half>(p1, p2, l1, l2, N, P1, P2, D, norm, K, dists, idxs, st);
      case TPO_F64: return knn_general<double>(p1, p2, l1, l2, N, P1, P2, D, norm, K, dists, idxs, st);
    }
    return TPO_ERR_INVALID_ARGUMENT;
  }
  // The reference knn kernels are compiled without contraction of
  // `dist += diff * diff` (measured on B200: bit-identical to the uncontracted
  // CPU path), so knn has a single rounding and ignores the flag.
  (void)flags;
  const bool exact = true;
  switch (dtype) {
    case TPO_F32:
      return exact ? dispatch_knn_fwd<float, TPO_ROUND_EXACT>(p1, p2, l1, l2, N, P1, P2, D, norm, K, dists, idxs, st)
                   : dispatch_knn_fwd<float, TPO_ROUND_FMA>(p1, p2, l1, l2, N, P1, P2, D, norm, K, dists, idxs, st);
    case TPO_F16:
      return dispatch_knn_fwd<__half, TPO_ROUND_EXACT>(p1, p2, l1, l2, N, P1, P2, D, norm, K, dists, idxs, st);
    case TPO_F64:
      return exact ? dispatch_knn_fwd<double, TPO_ROUND_EXACT>(p1, p2, l1, l2, N, P1, P2, D, norm, K, dists, idxs, st)
                   : dispatch_knn_fwd<double, TPO_ROUND_FMA>(p1, p2, l1, l2, N, P1, P2, D, norm, K, dists, idxs, st);
  }
  return TPO_ERR_INVALID_ARGUMENT;
}

// ------------------------------- backward -------------------------------
template <typename T>
struct KbOps;
template <>
struct KbOps<float> {
  __device__ static float l2(float g, float a, float b) { return __fmul_rn(__fmul_rn(g, 2.0f), __fsub_rn(a, b)); }
  __device__ static float l1(float g, float a, float b) { return a > b ? g : (a == b ? 0.0f : -g); }
  __device__ static float add(float a, float b) { return __fadd_rn(a, b); }
  __device__ static void atomic_sub(float* p, float v) { atomicAdd(p, -v); }
  __device__ static void atomic_sub3(float* p, const float* v) { red_add3f(p, -v[0], -v[1], -v[2]); }
  __device__ static float zero() { return 0.0f; }
};
template <>
struct KbOps<double> {
  __device__ static double l2(double g, double a, double b) { return __dmul_rn(__dmul_rn(g, 2.0), __dsub_rn(a, b)); }
  __device__ static double l1(double g, double a, double b) { return a > b ? g : (a == b ? 0.0 : -g); }
  __device__ static double add(double a, double b) { return __dadd_rn(a, b); }
  __device__ static void atomic_sub(double* p, double v) { atomicAdd(p, -v); }
  __device__ static void atomic_sub3(double* p, const double* v) {
    atomicAdd(p, -v[0]);
    atomicAdd(p + 1, -v[1]);
    atomicAdd(p + 2, -v[2]);
  }
  __device__ static double zero() { return 0.0; }
};
template <>
struct KbOps<__half> {
  __device__ static __half l2(__half g, __half a, __half b) {
    return hmul_rn(hmul_rn(g, __float2half_rn(2.0f)), hsub_rn(a, b));
  }
  __device__ static __half l1(__half g, __half a, __half b) {
    const float fa = __half2float(a), fb = __half2float(b);
    return fa > fb ? g : (fa == fb ? __float2half_rn(0.0f) : __hneg(g));
  }
  __device__ static __half add(__half a, __half b) { return hadd_rn(a, b); }
  __device__ static void atomic_sub(__half* p, __half v) { atomicAdd(p, __hneg(v)); }
  __device__ static void atomic_sub3(__half* p, const __half* v) {
    red_add3h(p, __hneg(v[0]), __hneg(v[1]), __hneg(v[2]));
  }
  __device__ static __half zero() { return __float2half_rn(0.0f); }
};

template <typename T>
__global__ void knn_bwd_kernel(const T* __restrict__ p1, const T* __restrict__ p2,
                               const int64_t* __restrict__ len1, const int64_t* __restrict__ len2,
                               const int64_t* __restrict__ idxs, int64_t N, int64_t P1, int64_t P2,
                               int D, int K, int norm, const T* __restrict__ gd,
                               T* __restrict__ g1, T* __restrict__ g2) {
  using O = KbOps<T>;
  const int64_t total = N * P1;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = t / P1, i = t % P1;
    const int64_t L1 = len1 ? len1[n] : P1;
    const int64_t L2 = len2 ? len2[n] : P2;
    const int kk = (int)min64(K, max64(L2, 0));
    if (D > KDMAX) {  // general D: one coordinate at a time, same k order per coordinate
      for (int d = 0; d < D; ++d) {
        T acc = O::zero();
        if (i < L1) {
          for (int k = 0; k < kk; ++k) {
            const int64_t j = idxs[t * K + k];
            if (j < 0 || j >= P2) continue;
            const T g = gd[t * K + k];
            const T a = p1[t * D + d], b = p2[(n * P2 + j) * D + d];
            const T v = norm == 1 ? O::l1(g, a, b) : O::l2(g, a, b);
            acc = O::add(acc, v);
            O::atomic_sub(g2 + (n * P2 + j) * D + d, v);
          }
        }
        g1[t * D + d] = acc;
      }
      continue;
    }
    if (D == 3) {
      // Neighbours in batches of KB: all indices and grads of a batch are loaded
      // first, then all their coordinates, so a query costs two dependent memory
      // round trips per KB neighbours instead of two per neighbour.  The query's
      // own gradient still sums the terms in k order; the neighbour's 3-vector
      // goes out as one vector reduction plus one scalar.
      constexpr int KB = 8;
      T acc3[3] = {O::zero(), O::zero(), O::zero()};
      if (i < L1) {
        const T a[3] = {p1[t * 3], p1[t * 3 + 1], p1[t * 3 + 2]};
        for (int k0 = 0; k0 < kk; k0 += KB) {
          int64_t jj[KB];
          T gg[KB];
#pragma unroll
          for (int u = 0; u < KB; ++u) {
            const bool in = k0 + u < kk;
            jj[u] = in ? idxs[t * K + k0 + u] : -1;
            gg[u] = in ? gd[t * K + k0 + u] : O::zero();
          }
          T bb[KB][3];
#pragma unroll
          for (int u = 0; u < KB; ++u) {
            const bool ok = jj[u] >= 0 && jj[u] < P2;
            const T* q = p2 + (n * P2 + (ok ? jj[u] : 0)) * 3;
#pragma unroll
            for (int d = 0; d < 3; ++d) bb[u][d] = ok ? q[d] : O::zero();
          }
#pragma unroll
          for (int u = 0; u < KB; ++u) {
            if (jj[u] < 0 || jj[u] >= P2) continue;
            T v[3];
#pragma unroll
            for (int d = 0; d < 3; ++d) {
              v[d] = norm == 1 ? O::l1(gg[u], a[d], bb[u][d]) : O::l2(gg[u], a[d], bb[u][d]);
              acc3[d] = O::add(acc3[d], v[d]);
            }
            O::atomic_sub3(g2 + (n * P2 + jj[u]) * 3, v);
          }
        }
      }
#pragma unroll
      for (int d = 0; d < 3; ++d) g1[t * 3 + d] = acc3[d];
      continue;
    }
    T acc[KDMAX];
#pragma unroll
    for (int d = 0; d < KDMAX; ++d) acc[d] = O::zero();
    if (i < L1) {
      for (int k = 0; k < kk; ++k) {
        const int64_t j = idxs[t * K + k];
        if (j < 0 || j >= P2) continue;
        const T g = gd[t * K + k];
#pragma unroll
        for (int d = 0; d < KDMAX; ++d) {
          if (d < D) {
            const T a = p1[t * D + d], b = p2[(n * P2 + j) * D + d];
            const T v = norm == 1 ? O::l1(g, a, b) : O::l2(g, a, b);
            acc[d] = O::add(acc[d], v);
            O::atomic_sub(g2 + (n * P2 + j) * D + d, v);
          }
        }
      }
    }
#pragma unroll
    for (int d = 0; d < KDMAX; ++d)
      if (d < D) g1[t * D + d] = acc[d];
  }
}

int knn_backward(int dtype, const void* p1, const void* p2, const int64_t* l1, const int64_t* l2,
                 const int64_t* idxs, int64_t N, int64_t P1, int64_t P2, int64_t D, int64_t K,
                 int64_t norm, const void* gd, void* g1, void* g2, cudaStream_t st) {
  const int64_t total = N * P1;
  if (total <= 0) return TPO_OK;
  // one thread per query, a latency chain each: small blocks spread the
  // queries evenly over the SMs
  const int threads = 64;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + threads - 1) / threads, 148 * 64);
#define TPO_KB(T)                                                                              \
  knn_bwd_kernel<T><<<blocks, threads, 0, st>>>((const T*)p1, (const T*)p2, l1, l2, idxs, N, P1, \
                                                P2, (int)D, (int)K, (int)norm, (const T*)gd,    \
                                                (T*)g1, (T*)g2)
  switch (dtype) {
    case TPO_F32: TPO_KB(float); break;
    case TPO_F16: TPO_KB(__half); break;
    case TPO_F64: TPO_KB(double); break;
    default: return TPO_ERR_INVALID_ARGUMENT;
  }
#undef TPO_KB
  return check_launch();
}

// ------------------------------- knn_gather -------------------------------
// out[n,l,k,u] = x[n, idx[n,l,k], u]; zero when k >= lengths[n] or idx invalid.
// One thread per (n, l, k) slot, all U features of it; index math in IdxT
// (32-bit whenever N*L*K and the element offsets fit).
template <typename T, typename IdxT>
__global__ void knn_gather_fwd_kernel(const T* __restrict__ x, const int64_t* __restrict__ idx,
                                      const int64_t* __restrict__ lengths, IdxT N, IdxT M, IdxT U,
                                      IdxT L, IdxT K, T* __restrict__ out) {
  const IdxT slots = N * L * K;
  for (IdxT e = blockIdx.x * (IdxT)blockDim.x + threadIdx.x; e < slots;
       e += (IdxT)gridDim.x * blockDim.x) {
    const IdxT k = e % K;
    const IdxT n = e / (L * K);
    const int64_t len = lengths ? lengths[n] : (int64_t)M;
    const int64_t j = idx[e];
    const bool ok = k < len && j >= 0 && j < (int64_t)M;
    const T* src = x + ((int64_t)n * M + (ok ? j : 0)) * U;
    T* dst = out + (int64_t)e * U;
    for (IdxT u = 0; u < U; ++u) dst[u] = ok ? src[u] : T(0.0f);
  }
}

template <typename T>
__device__ __forceinline__ void gather_add3(T* p, const T* v);
template <>
__device__ __forceinline__ void gather_add3<float>(float* p, const float* v) { red_add3f(p, v[0], v[1], v[2]); }
template <>
__device__ __forceinline__ void gather_add3<__half>(__half* p, const __half* v) { red_add3h(p, v[0], v[1], v[2]); }
template <>
__device__ __forceinline__ void gather_add3<double>(double* p, const double* v) {
  atomicAdd(p, v[0]);
  atomicAdd(p + 1, v[1]);
  atomicAdd(p + 2, v[2]);
}

template <typename T, typename IdxT>
__global__ void knn_gather_bwd_kernel(const T* __restrict__ gout, const int64_t* __restrict__ idx,
                                      const int64_t* __restrict__ lengths, IdxT N, IdxT M, IdxT U,
                                      IdxT L, IdxT K, T* __restrict__ gx) {
  const IdxT slots = N * L * K;
  for (IdxT e = blockIdx.x * (IdxT)blockDim.x + threadIdx.x; e < slots;
       e += (IdxT)gridDim.x * blockDim.x) {
    const IdxT k = e % K;
    const IdxT n = e / (L * K);
    const int64_t len = lengths ? lengths[n] : (int64_t)M;
    const int64_t j = idx[e];
    if (!(k < len && j >= 0 && j < (int64_t)M)) continue;
    T* dst = gx + ((int64_t)n * M + j) * U;
    const T* src = gout + (int64_t)e * U;
    if (U == 3) {
      const T v[3] = {src[0], src[1], src[2]};
      gather_add3<T>(dst, v);
    } else {
      for (IdxT u = 0; u < U; ++u) atomicAdd(dst + u, src[u]);
    }
  }
}

template <typename T, typename IdxT>
static void launch_gather(bool bwd, const void* a, const int64_t* idx, const int64_t* lengths,
                          int64_t N, int64_t M, int64_t U, int64_t L, int64_t K, void* out,
                          cudaStream_t st) {
  const int64_t slots = N * L * K;
  const int threads = 256;
  const unsigned blocks = (unsigned)std::min<int64_t>((slots + threads - 1) / threads, 148 * 16);
  if (bwd)
    knn_gather_bwd_kernel<T, IdxT><<<blocks, threads, 0, st>>>((const T*)a, idx, lengths, (IdxT)N, (IdxT)M,
                                                               (IdxT)U, (IdxT)L, (IdxT)K, (T*)out);
  else
    knn_gather_fwd_kernel<T, IdxT><<<blocks, threads, 0, st>>>((const T*)a, idx, lengths, (IdxT)N, (IdxT)M,
                                                               (IdxT)U, (IdxT)L, (IdxT)K, (T*)out);
}

static int gather_dispatch(bool bwd, int dtype, const void* a, const int64_t* idx,
                           const int64_t* lengths, int64_t N, int64_t M, int64_t U, int64_t L,
                           int64_t K, void* out, cudaStream_t st) {
  if (N * L * K <= 0 || U <= 0) return TPO_OK;
  // 32-bit index math when every slot index and slot-count product fits
  const bool small = N * L * K < (int64_t(1) << 31) && N * M < (int64_t(1) << 31);
  switch (dtype) {
    case TPO_F32:
      small ? launch_gather<float, int>(bwd, a, idx, lengths, N, M, U, L, K, out, st)
            : launch_gather<float, int64_t>(bwd, a, idx, lengths, N, M, U, L, K, out, st);
      break;
    case TPO_F16:
      small ? launch_gather<__half, int>(bwd, a, idx, lengths, N, M, U, L, K, out, st)
            : launch_gather<__half, int64_t>(bwd, a, idx, lengths, N, M, U, L, K, out, st);
      break;
    case TPO_F64:
      small ? launch_gather<double, int>(bwd, a, idx, lengths, N, M, U, L, K, out, st)
            : launch_gather<double, int64_t>(bwd, a, idx, lengths, N, M, U, L, K, out, st);
      break;
    default: return TPO_ERR_INVALID_ARGUMENT;
  }
  return check_launch();
}

int knn_gather_forward(int dtype, const void* x, const int64_t* idx, const int64_t* lengths,
                       int64_t N, int64_t M, int64_t U, int64_t L, int64_t K, void* out,
                       cudaStream_t st) {
  return gather_dispatch(false, dtype, x, idx, lengths, N, M, U, L, K, out, st);
}

int knn_gather_backward(int dtype, const void* gout, const int64_t* idx, const int64_t* lengths,
                        int64_t N, int64_t M, int64_t U, int64_t L, int64_t K, void* gx,
                        cudaStream_t st) {
  return gather_dispatch(true, dtype, gout, idx, lengths, N, M, U, L, K, gx, st);
}

int knn_device_error_flags(unsigned* out, bool clear) {
  int s = cuda_status(cudaMemcpyFromSymbol(out, g_knn_device_error, sizeof(unsigned)));
  if (s || !clear) return s;
  const unsigned zero = 0;
  return cuda_status(cudaMemcpyToSymbol(g_knn_device_error, &zero, sizeof(unsigned)));
}

}  // namespace tpo
