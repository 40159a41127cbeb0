// Furthest point sampling (FPS), reference CUDA semantics.
//
// Replaces furthest_point_sampling_kernel and its launcher
// (torch_point_ops/fps/csrc/cuda/fps.cu:108-316).  The reference runs one CTA of
// up to 512 threads per cloud and, for every one of the nsamples-1 steps, re-reads
// every point and its running distance from global memory and reduces through
// nine __syncthreads.  Here a cloud is spread over a GROUP of CTAs whose threads
// hold their points and running distances in REGISTERS for the whole kernel;
// a step is then: update PT points per thread (packed f32x2 / f16x2), one
// redux.sync per warp, and an exchange of the warps' candidates -- through
// shared memory and one CTA barrier (one CTA per cloud); in a thread-block
// cluster, the same CTA stage and then one st.async push of each CTA's winner
// into every CTA of the cluster, each CTA waiting on its own mbarrier (no
// cluster barrier); or through global memory and a grid barrier (cooperative
// grid, for clouds larger than a cluster holds).  Work per step is O(P / (group threads)), latency a few
// hundred cycles.
//
// Bit-exact parity with the reference:
//  * distance d = fma(dz,dz, fma(dx,dx, dy*dy)) (nvcc's contraction of fps.cu:142,
//    same as chamfer.cu:67); fp16 rounds every operation (c10::Half); fp64 like
//    fp32 in double.  A point with x*x+y*y+z*z <= 1e-3 (fps.cu:139-140,
//    contracted the same way) keeps the distance -1 and never wins.
//  * temp starts at 1e10 (1e4 for fp16, fps.cu:291) and becomes min(d, temp).
//  * ties: reference thread t (of bs = min(512, 2^floor(log2 P)), fps.cu:56-59)
//    scans k = t, t+bs, ... and keeps its first maximum (strict '>'); the
//    halving tree (:152-205) merges slot i with i+s for s = bs/2 .. 1 and keeps
//    slot i on ties, which decides bit 0 of the winning thread last -- so among
//    equal maxima the winner has the smallest bit-reversed thread number, then
//    the smallest k.  Here the points are laid out in exactly that RANK order
//    (virtual rank r = c*Q + j with Q = ceil(P/bs): class c holds thread
//    t = bitrev(c)'s points k = t + j*bs, slots with k >= P are padding); CTA g,
//    thread t owns ranks [(g*NT + t)*PT, +PT), and every reduction level keeps
//    the lowest rank among equal keys.
//  * if no point is valid the step selects 0 (besti's initial value, fps.cu:131).
#include <cooperative_groups.h>

#include <map>
#include <mutex>
#include <tuple>

#include <type_traits>

#include "tpo_internal.h"

namespace tpo {
namespace cg = cooperative_groups;

static __device__ unsigned g_fps_device_error = 0;

// Point record in shared memory (indexed by local rank): coordinates and index.
struct FpsPtF {
  float x, y, z;
  int k;
};
struct FpsPtD {
  double x, y, z;
  long long k;
};
// A warp's candidate for the step: its maximum key and that point's coordinates.
// (The point index never travels: the owning lane writes it out if it wins.)
struct __align__(16) FpsSlotF {
  int key;
  float x, y, z;
};
struct __align__(16) FpsSlotD {
  long long key;
  double x, y, z;
};
__device__ __forceinline__ int warp_max_s32(int v) {
  int r;
  asm volatile("redux.sync.max.s32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}
__device__ __forceinline__ long long warp_max_s64(long long v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

// ---- per-dtype arithmetic on two points at a time ----
struct FpsF32 {
  using S = float;    // storage type of the input
  using C = float;    // coordinate type of the selected point
  using Key = int;    // order-preserving key of a running distance (>= -1)
  using Pt = FpsPtF;
  using Slot = FpsSlotF;
  static constexpr float kLarge = 1e10f;
  struct Pair {
    u64 x, y, z, t;
  };
  struct Sel {
    u64 x, y, z;
  };
  __device__ static Sel sel(C x, C y, C z) { return {pk(x, x), pk(y, y), pk(z, z)}; }
  __device__ static C coord(S v) { return v; }
  __device__ static bool valid(S x, S y, S z) {
    return __fmaf_rn(z, z, __fmaf_rn(x, x, __fmul_rn(y, y))) > 1e-3f;
  }
  __device__ static Pair make(const Pt& a, const Pt& b, bool va, bool vb) {
    return {pk(a.x, b.x), pk(a.y, b.y), pk(a.z, b.z), pk(va ? kLarge : -1.0f, vb ? kLarge : -1.0f)};
  }
  __device__ static Key update(Pair& p, const Sel& s) {
    const u64 dx = sub2(p.x, s.x), dy = sub2(p.y, s.y), dz = sub2(p.z, s.z);
    const u64 d = fma2(dz, dz, fma2(dx, dx, mul2(dy, dy)));
    float d0, d1, t0, t1;
    upk(d, d0, d1);
    upk(p.t, t0, t1);
    t0 = fminf(d0, t0);
    t1 = fminf(d1, t1);
    p.t = pk(t0, t1);
    return __float_as_int(fmaxf(t0, t1));
  }
  __device__ static Key key_lo(const Pair& p) { float a, b; upk(p.t, a, b); return __float_as_int(a); }
  __device__ static Key key_hi(const Pair& p) { float a, b; upk(p.t, a, b); return __float_as_int(b); }
  __device__ static Key warp_max(Key k) { return warp_max_s32(k); }
  static constexpr Key kNone = (Key)0xBF800000;  // key of -1.0f
  static constexpr Key kMin = INT_MIN;
};

struct FpsF16 {
  using S = __half;
  using C = float;
  using Key = int;
  using Pt = FpsPtF;
  using Slot = FpsSlotF;
  struct Pair {
    h2 x, y, z, t;
  };
  struct Sel {
    h2 x, y, z;
  };
  __device__ static unsigned short hb(float v) { return __half_as_ushort(__float2half_rn(v)); }
  __device__ static Sel sel(C x, C y, C z) {
    return {hpk(hb(x), hb(x)), hpk(hb(y), hb(y)), hpk(hb(z), hb(z))};
  }
  __device__ static C coord(S v) { return __half2float(v); }
  __device__ static bool valid(S x, S y, S z) {
    const __half m = hadd_rn(hadd_rn(hmul_rn(x, x), hmul_rn(y, y)), hmul_rn(z, z));
    return __half2float(m) > __half2float(__float2half_rn(1e-3f));
  }
  __device__ static Pair make(const Pt& a, const Pt& b, bool va, bool vb) {
    const unsigned short big = 0x70E2, neg1 = 0xBC00;  // 1e4 and -1 in fp16
    return {hpk(hb(a.x), hb(b.x)), hpk(hb(a.y), hb(b.y)), hpk(hb(a.z), hb(b.z)),
            hpk(va ? big : neg1, vb ? big : neg1)};
  }
  __device__ static Key update(Pair& p, const Sel& s) {
    const h2 dx = hsub2r(p.x, s.x), dy = hsub2r(p.y, s.y), dz = hsub2r(p.z, s.z);
    p.t = hmin2r(hdist2(dx, dy, dz), p.t);
    const int lo = (int)(short)(p.t & 0xffffu), hi = (int)(short)(p.t >> 16);
    return max(lo, hi);
  }
  // fp16 bits of a value >= -1, sign-extended: ordered like the values
  __device__ static Key key_lo(const Pair& p) { return (int)(short)(p.t & 0xffffu); }
  __device__ static Key key_hi(const Pair& p) { return (int)(short)(p.t >> 16); }
  __device__ static Key warp_max(Key k) { return warp_max_s32(k); }
  static constexpr Key kNone = (Key)(short)0xBC00;
  static constexpr Key kMin = INT_MIN;
};

struct FpsF64 {
  using S = double;
  using C = double;
  using Key = long long;
  using Pt = FpsPtD;
  using Slot = FpsSlotD;
  struct Pair {
    double x0, y0, z0, t0, x1, y1, z1, t1;
  };
  struct Sel {
    double x, y, z;
  };
  __device__ static Sel sel(C x, C y, C z) { return {x, y, z}; }
  __device__ static C coord(S v) { return v; }
  __device__ static bool valid(S x, S y, S z) {
    return __fma_rn(z, z, __fma_rn(x, x, __dmul_rn(y, y))) > 1e-3;
  }
  __device__ static Pair make(const Pt& a, const Pt& b, bool va, bool vb) {
    return {a.x, a.y, a.z, va ? 1e10 : -1.0, b.x, b.y, b.z, vb ? 1e10 : -1.0};
  }
  __device__ static double d(double x, double y, double z, const Sel& s) {
    const double dx = __dsub_rn(x, s.x), dy = __dsub_rn(y, s.y), dz = __dsub_rn(z, s.z);
    return __fma_rn(dz, dz, __fma_rn(dx, dx, __dmul_rn(dy, dy)));
  }
  __device__ static Key update(Pair& p, const Sel& s) {
    p.t0 = fmin(d(p.x0, p.y0, p.z0, s), p.t0);
    p.t1 = fmin(d(p.x1, p.y1, p.z1, s), p.t1);
    return __double_as_longlong(fmax(p.t0, p.t1));
  }
  __device__ static Key key_lo(const Pair& p) { return __double_as_longlong(p.t0); }
  __device__ static Key key_hi(const Pair& p) { return __double_as_longlong(p.t1); }
  __device__ static Key warp_max(Key k) { return warp_max_s64(k); }
  static constexpr Key kNone = (Key)0xBFF0000000000000ull;
  static constexpr Key kMin = LLONG_MIN;
};

// Shared-memory candidate slots of one CTA (double-buffered).
__host__ __device__ constexpr int fps_slot_count(int mode, int G, int NW) {
  return mode == 2 ? 0 : mode == 1 ? 2 * (NW + G) : 2 * NW;
}

// Point index of virtual rank r (see the tie rule above); -1 for padding.
__device__ __forceinline__ int fps_rank_to_index(int r, int P, int bs, int lbs, int Q) {
  const int c = r / Q, j = r - c * Q;
  const int t = lbs ? (int)(__brev((unsigned)c) >> (32 - lbs)) : 0;
  const int64_t k = t + (int64_t)bs * j;
  return k < P ? (int)k : -1;
}

constexpr unsigned kFpsWaitLimit = 1u << 22;
constexpr int kFpsMaxThreads = 256;
constexpr int kFpsMaxCluster = 16;
constexpr int kFpsSmemCap = 200 * 1024;  // dynamic shared memory limit of every plan

enum FpsMode { kFpsCta = 0, kFpsCluster = 1, kFpsGrid = 2 };

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned mapa_u32(unsigned local, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
// 16 bytes into (possibly another CTA's) shared memory, completing on that CTA's
// mbarrier as 16 transaction bytes.
__device__ __forceinline__ void st_async16(unsigned raddr, uint4 v, unsigned rbar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(raddr),
      "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(rbar)
      : "memory");
}
__device__ __forceinline__ bool mbar_try(unsigned bar, unsigned parity) {
  unsigned done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

template <class Slot>
__device__ __forceinline__ void slot_store_global(Slot* dst, const Slot& v) {
#pragma unroll
  for (int i = 0; i < (int)(sizeof(Slot) / 16); ++i)
    __stcg(reinterpret_cast<int4*>(dst) + i, *(reinterpret_cast<const int4*>(&v) + i));
}
template <class Slot>
__device__ __forceinline__ Slot slot_load_global(const Slot* src) {
  Slot v;
#pragma unroll
  for (int i = 0; i < (int)(sizeof(Slot) / 16); ++i)
    *(reinterpret_cast<int4*>(&v) + i) = __ldcg(reinterpret_cast<const int4*>(src) + i);
  return v;
}

// One group of G CTAs (a cluster, G consecutive CTAs of a cooperative grid, or
// G == 1) samples one cloud.  Dynamic shared memory: 2 mbarriers (16 B), slots
// [2][nslots], points [NT*PT].
template <class Tr, int PT, int MODE>
__global__ void __launch_bounds__(kFpsMaxThreads, 1)
fps_kernel(const typename Tr::S* __restrict__ pts, int P, int S, int G, int bs, int lbs, int Q,
           int64_t b0, int64_t* __restrict__ out, typename Tr::Slot* __restrict__ gslots,
           unsigned* __restrict__ gcount) {
  using Pt = typename Tr::Pt;
  using Slot = typename Tr::Slot;
  using Key = typename Tr::Key;
  using C = typename Tr::C;
  extern __shared__ __align__(16) unsigned char fps_smem[];
  const int NT = blockDim.x, NW = NT >> 5;
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(fps_smem);
  Slot* sslots = reinterpret_cast<Slot*>(fps_smem + 16);
  // CTA mode: slots [2][NW]; cluster mode: [2][NW] for the CTA stage, then [2][G]
  Pt* spts = reinterpret_cast<Pt*>(fps_smem + 16 + fps_slot_count(MODE, G, NW) * sizeof(Slot));
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int g = 0;
  int64_t b;
  if (MODE == kFpsCluster) {
    g = (int)cg::this_cluster().block_rank();
    b = blockIdx.x / G;
  } else if (MODE == kFpsGrid) {
    g = blockIdx.x % G;
    b = blockIdx.x / G;
  } else {
    b = blockIdx.x;
  }
  b += b0;
  const typename Tr::S* bp = pts + b * (int64_t)P * 3;
  int64_t* bo = out + b * (int64_t)S;

  // Load this thread's PT points in rank order (registers + shared copy).
  typename Tr::Pair R[PT / 2];
#pragma unroll
  for (int q = 0; q < PT / 2; ++q) {
    Pt e[2];
    bool v[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t r = ((int64_t)g * NT + tid) * PT + 2 * q + h;
      const int k = r < (int64_t)bs * Q ? fps_rank_to_index((int)r, P, bs, lbs, Q) : -1;
      if (k >= 0) {
        const typename Tr::S x = bp[3 * (int64_t)k], y = bp[3 * (int64_t)k + 1], z = bp[3 * (int64_t)k + 2];
        e[h].x = Tr::coord(x);
        e[h].y = Tr::coord(y);
        e[h].z = Tr::coord(z);
        e[h].k = k;
        v[h] = Tr::valid(x, y, z);
      } else {
        e[h].x = e[h].y = e[h].z = C(0);
        e[h].k = 0;
        v[h] = false;
      }
      spts[tid * PT + 2 * q + h] = e[h];
    }
    R[q] = Tr::make(e[0], e[1], v[0], v[1]);
  }
  const C p0x = Tr::coord(bp[0]), p0y = Tr::coord(bp[1]), p0z = Tr::coord(bp[2]);
  C sx = p0x, sy = p0y, sz = p0z;
  if (g == 0 && tid == 0) bo[0] = 0;
  if (tid == 0) {
    s_abort = 0;
    if (MODE == kFpsCluster) {
      mbar_init(&bars[0], 1);
      mbar_init(&bars[1], 1);
    }
  }
  if (MODE == kFpsCluster)
    cg::this_cluster().sync();  // every CTA's mbarriers exist before the first push
  else
    __syncthreads();

  const int per = (G + 31) >> 5;  // grid mode: CTA slots per lane
  bool abort = false;
  for (int j = 1; j < S; ++j) {
    const int buf = j & 1;
    if (MODE == kFpsCluster && tid == 0)
      mbar_expect_tx(&bars[buf], (unsigned)(G * sizeof(Slot)));
    // 1. fold the newest sample into this thread's running distances
    const typename Tr::Sel s = Tr::sel(sx, sy, sz);
    Key tk = Tr::update(R[0], s);
#pragma unroll
    for (int q = 1; q < PT / 2; ++q) {
      const Key u = Tr::update(R[q], s);
      tk = u > tk ? u : tk;
    }
    // 2. warp candidate: max key, lowest lane, first point of that lane
    const Key wk = Tr::warp_max(tk);
    const int L = __ffs(__ballot_sync(0xffffffffu, tk == wk)) - 1;
    int mk = -1;  // the point index this lane proposed (lane L only)
    C ex = C(0), ey = C(0), ez = C(0);
    const int my_slot = g * NW + warp;
    if (lane == L) {
      int p = 0;
#pragma unroll
      for (int q = PT / 2 - 1; q >= 0; --q) {
        if (Tr::key_hi(R[q]) == wk) p = 2 * q + 1;
        if (Tr::key_lo(R[q]) == wk) p = 2 * q;
      }
      const Pt e = spts[tid * PT + p];
      mk = e.k;
      ex = e.x;
      ey = e.y;
      ez = e.z;
      Slot sl;
      sl.key = wk;
      sl.x = e.x;
      sl.y = e.y;
      sl.z = e.z;
      sslots[buf * NW + warp] = sl;  // the CTA's warp slots [2][NW]
    }
    int cw = 0;  // cluster / grid mode: the CTA's winning warp
    if (MODE != kFpsCta) {
      // CTA stage: every warp reduces the CTA's warp slots (no second barrier)
      __syncthreads();
      Slot cv;
      if (lane < NW) cv = sslots[buf * NW + lane]; else cv.key = Tr::kMin;
      const Key ck = Tr::warp_max(cv.key);
      cw = __ffs(__ballot_sync(0xffffffffu, cv.key == ck)) - 1;
      Slot sl;
      sl.key = ck;
      sl.x = __shfl_sync(0xffffffffu, cv.x, cw);
      sl.y = __shfl_sync(0xffffffffu, cv.y, cw);
      sl.z = __shfl_sync(0xffffffffu, cv.z, cw);
      if (MODE == kFpsGrid && tid == 0) slot_store_global(gslots + (b * 2 + buf) * G + g, sl);
      if (MODE == kFpsCluster && warp == 0 && lane < G) {
        // lane c pushes the CTA's winner into CTA c's slot [buf][g]
        Slot* cl = sslots + 2 * NW;
        const unsigned ra = mapa_u32(smem_addr(cl + buf * G + g), lane);
        const unsigned rb = mapa_u32(smem_addr(&bars[buf]), lane);
#pragma unroll
        for (int i = 0; i < (int)(sizeof(Slot) / 16); ++i)
          st_async16(ra + 16 * i, *(reinterpret_cast<const uint4*>(&sl) + i), rb);
      }
    }
    // 3. wait until every candidate of the group is visible
    if (MODE == kFpsCta) {
      __syncthreads();
    } else if (MODE == kFpsCluster) {
      if (!abort) {
        // buffer (j & 1) serves steps j, j+2, ...: its phase for step j is (j-1)/2
        const unsigned bar = smem_addr(&bars[buf]), parity = (unsigned)((j - 1) >> 1) & 1u;
        unsigned it = 0;
        while (!mbar_try(bar, parity)) {
          if (++it == kFpsWaitLimit) {
            atomicOr(&g_fps_device_error, (unsigned)TPO_DEVERR_GRID_TIMEOUT);
            abort = true;  // skip later waits; the output is garbage, the kernel ends
            break;
          }
        }
      }
    } else {
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        atomicAdd(gcount + b, 1u);
        const unsigned target = (unsigned)G * (unsigned)j;
        unsigned it = 0;
        while (ld_acquire_u32(gcount + b) < target) {
          if (++it == kFpsWaitLimit) {
            atomicOr(&g_fps_device_error, (unsigned)TPO_DEVERR_GRID_TIMEOUT);
            s_abort = 1;
            break;
          }
        }
        __threadfence();
      }
      __syncthreads();
      if (s_abort) return;
    }
    // 4. group winner over the slots (warps in CTA mode, CTAs otherwise); lanes
    // take contiguous runs, so the lowest slot wins ties
    Key bk = Tr::kMin;
    int bslot = 0;
    C bx = C(0), by = C(0), bz = C(0);
    if (MODE == kFpsGrid) {
      for (int i = 0; i < per; ++i) {
        const int si = lane * per + i;
        if (si < G) {
          const Slot v = slot_load_global(gslots + (b * 2 + buf) * G + si);
          if (v.key > bk) {
            bk = v.key;
            bslot = si;
            bx = v.x;
            by = v.y;
            bz = v.z;
          }
        }
      }
    } else {
      const int n2 = MODE == kFpsCluster ? G : NW;
      const Slot* base = MODE == kFpsCluster ? sslots + 2 * NW + buf * G : sslots + buf * NW;
      if (lane < n2) {
        const Slot v = base[lane];
        bk = v.key;
        bslot = lane;
        bx = v.x;
        by = v.y;
        bz = v.z;
      }
    }
    const Key gk = Tr::warp_max(bk);
    const int W = __ffs(__ballot_sync(0xffffffffu, bk == gk)) - 1;
    const int wslot = __shfl_sync(0xffffffffu, bslot, W);
    sx = __shfl_sync(0xffffffffu, bx, W);
    sy = __shfl_sync(0xffffffffu, by, W);
    sz = __shfl_sync(0xffffffffu, bz, W);
    if (gk == Tr::kNone) {  // no valid point anywhere: the reference selects 0
      sx = p0x;
      sy = p0y;
      sz = p0z;
      if (g == 0 && tid == 0) bo[j] = 0;
    } else if (lane == L && (MODE == kFpsCta ? wslot == warp : (wslot == g && cw == warp))) {
      bo[j] = mk;
    }
  }
  // no CTA of the cluster leaves while a peer may still push into it
  if (MODE == kFpsCluster) cg::this_cluster().sync();
}

// ---------------------------------------------------------------------------
// Host side: plan (group size G, threads NT, points per thread PT), launch.
// ---------------------------------------------------------------------------
struct FpsPlan {
  int mode, G, NT, PT;
  int64_t batches_per_launch;  // grid mode: clouds per cooperative launch
};

static int fps_block_size(int64_t P) {
  int bs = 1;
  while ((int64_t)bs * 2 <= P && bs < 512) bs *= 2;
  return bs;
}
static int fps_log2(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}
// Virtual rank count bs * ceil(P / bs) (P plus at most bs - 1 padding slots).
static int64_t fps_virtual_points(int64_t P) {
  const int64_t bs = fps_block_size(P);
  return bs * ((P + bs - 1) / bs);
}

template <class Tr>
static size_t fps_smem_bytes(int mode, int G, int NT, int PT) {
  return 16 + fps_slot_count(mode, G, NT / 32) * sizeof(typename Tr::Slot) +
         (size_t)NT * PT * sizeof(typename Tr::Pt);
}

template <class Tr, int PT, int MODE>
static void* fps_kernel_ptr() {
  return reinterpret_cast<void*>(&fps_kernel<Tr, PT, MODE>);
}

template <class Tr, int MODE>
static void* fps_kernel_for(int PT) {
  switch (PT) {
    case 2: return fps_kernel_ptr<Tr, 2, MODE>();
    case 4: return fps_kernel_ptr<Tr, 4, MODE>();
    case 8: return fps_kernel_ptr<Tr, 8, MODE>();
    case 16: return fps_kernel_ptr<Tr, 16, MODE>();
    case 32:  // fp64 stops at 16 points per thread (32 would spill)
      if constexpr (!std::is_same<Tr, FpsF64>::value) return fps_kernel_ptr<Tr, 32, MODE>();
      return nullptr;
  }
  return nullptr;
}

template <class Tr>
static void* fps_kernel_for(int mode, int PT) {
  if (mode == kFpsCta) return fps_kernel_for<Tr, kFpsCta>(PT);
  if (mode == kFpsCluster) return fps_kernel_for<Tr, kFpsCluster>(PT);
  return fps_kernel_for<Tr, kFpsGrid>(PT);
}

static int g_num_sms = 0;

// How many clusters of G CTAs (NT threads, PT points each) can run at once.
template <class Tr>
static int fps_cluster_capacity(int G, int NT, int PT, int* out) {
  void* fn = fps_kernel_for<Tr>(kFpsCluster, PT);
  if (!fn) return TPO_ERR_UNSUPPORTED;
  const size_t smem = fps_smem_bytes<Tr>(kFpsCluster, G, NT, PT);
  if (int s = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kFpsSmemCap)))
    return s;
  if (G > 8)
    if (int s = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)))
      return s;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = G;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaOccupancyMaxActiveClusters(out, fn, &cfg));
}

// Estimated cycles of one sampling step for a group shape: the running-distance
// update (about 9 cycles per point per resident warp of a scheduler; fp64
// twice that) plus the exchange's fixed latency (warp reduce, candidate pick,
// barrier or push + wait, final reduce), measured on B200 for each mode.
static double fps_step_cycles(int dtype, int mode, int G, int NT, int PT) {
  const double per_pt = dtype == TPO_F64 ? 18.0 : 9.0;
  const int NW = NT / 32;
  double c = per_pt * PT * ((NW + 3) / 4);  // 4 schedulers per SM
  if (mode == kFpsCta) c += NW > 1 ? 650.0 : 550.0;
  if (mode == kFpsCluster) c += 950.0 + 5.0 * G;
  if (mode == kFpsGrid) c += 7000.0 + 30.0 * ((G + 31) / 32);
  return c;
}

template <class Tr>
static int fps_plan_uncached(int dtype, int64_t B, int64_t P, FpsPlan* plan);

// Plans are cached per (device, dtype, B, P): planning queries the occupancy
// calculator and sets kernel attributes, which costs more than a small launch.
template <class Tr>
static int fps_plan(int dtype, int64_t B, int64_t P, FpsPlan* plan) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int64_t, int64_t>, FpsPlan> cache;
  int dev = 0;
  if (int s = cuda_status(cudaGetDevice(&dev))) return s;
  const auto key = std::make_tuple(dev, dtype, B, P);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *plan = it->second;
      return TPO_OK;
    }
  }
  if (int s = fps_plan_uncached<Tr>(dtype, B, P, plan)) return s;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache[key] = *plan;
  return TPO_OK;
}

template <class Tr>
static int fps_plan_uncached(int dtype, int64_t B, int64_t P, FpsPlan* plan) {
  if (!g_num_sms) {
    int dev = 0;
    if (int s = cuda_status(cudaGetDevice(&dev))) return s;
    if (int s = cuda_status(cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev))) return s;
  }
  const int sms = g_num_sms;
  const int maxPT = dtype == TPO_F64 ? 16 : 32;
  const int64_t Pv = fps_virtual_points(P);
  double best = 1e300;
  bool found = false;
  for (int mode = 0; mode < 3; ++mode)
    for (int G = 1; G <= (mode == kFpsCta ? 1 : mode == kFpsCluster ? kFpsMaxCluster : sms); G *= 2) {
      if (mode != kFpsCta && G == 1) continue;
      for (int NT = 32; NT <= kFpsMaxThreads; NT *= 2)
        for (int PT = 2; PT <= maxPT; PT *= 2) {
          if ((int64_t)G * NT * PT < Pv) continue;
          // smallest PT that covers the cloud for this (G, NT)
          if (PT > 2 && (int64_t)G * NT * (PT / 2) >= Pv) continue;
          if (fps_smem_bytes<Tr>(mode, G, NT, PT) > (size_t)kFpsSmemCap) continue;
          // concurrent groups (one CTA per SM assumed for G > 1)
          int64_t per_wave = mode == kFpsCta ? (int64_t)sms * std::max(1, 1024 / NT) : sms / G;
          if (per_wave < 1) continue;
          if (mode == kFpsGrid && B > per_wave * 64) continue;  // too many launches
          int64_t waves = (B + per_wave - 1) / per_wave;
          double cost = waves * fps_step_cycles(dtype, mode, G, NT, PT);
          if (cost < best && mode == kFpsCluster) {
            // clusters must fit a GPC: ask the occupancy calculator
            int ncl = 0;
            if (fps_cluster_capacity<Tr>(G, NT, PT, &ncl) || ncl < 1) continue;
            per_wave = std::min<int64_t>(per_wave, ncl);
            waves = (B + per_wave - 1) / per_wave;
            cost = waves * fps_step_cycles(dtype, mode, G, NT, PT);
          }
          if (cost < best) {
            best = cost;
            *plan = {mode, G, NT, PT, mode == kFpsGrid ? per_wave : B};
            found = true;
          }
        }
    }
  // P beyond every shape (larger than the grid can hold): not supported
  if (!found) return set_error(TPO_ERR_UNSUPPORTED, "fps: point cloud too large for one GPU's registers");
  return TPO_OK;
}

static size_t fps_ws_bytes_for(int dtype, int64_t B, const FpsPlan& p) {
  if (p.mode != kFpsGrid) return 0;
  const size_t slot = dtype == TPO_F64 ? sizeof(FpsSlotD) : sizeof(FpsSlotF);
  // counters, then slots [B][2][G]
  const size_t cnt = ((size_t)B * 4 + 255) & ~(size_t)255;
  return cnt + (size_t)B * 2 * p.G * slot;
}

template <class Tr>
static int fps_run(int dtype, const void* pts, int64_t B, int64_t P, int64_t S, int64_t* idx,
                   void* ws, size_t ws_bytes, cudaStream_t st) {
  FpsPlan p;
  if (int s = fps_plan<Tr>(dtype, B, P, &p)) return s;
  const size_t need = fps_ws_bytes_for(dtype, B, p);
  if (need > ws_bytes) return set_error(TPO_ERR_WORKSPACE, "fps: workspace too small");
  void* fn = fps_kernel_for<Tr>(p.mode, p.PT);
  const size_t smem = fps_smem_bytes<Tr>(p.mode, p.G, p.NT, p.PT);
  // one fixed cap for every plan (plans need at most kFpsSmemCap): concurrent
  // callers with different plans never lower each other's limit
  if (int s = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kFpsSmemCap)))
    return s;
  unsigned* gcount = nullptr;
  typename Tr::Slot* gslots = nullptr;
  if (p.mode == kFpsGrid) {
    gcount = static_cast<unsigned*>(ws);
    gslots = reinterpret_cast<typename Tr::Slot*>(static_cast<char*>(ws) + (((size_t)B * 4 + 255) & ~(size_t)255));
    if (int s = cuda_status(cudaMemsetAsync(gcount, 0, (size_t)B * 4, st))) return s;
  }
  if (p.mode == kFpsCluster && p.G > 8)
    if (int s = cuda_status(cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)))
      return s;
  const int bs = fps_block_size(P), lbs = fps_log2(bs), Q = (int)((P + bs - 1) / bs);
  const typename Tr::S* tp = static_cast<const typename Tr::S*>(pts);
  int Pi = (int)P, Si = (int)S, Gi = p.G;
  for (int64_t b0 = 0; b0 < B; b0 += p.batches_per_launch) {
    const int64_t nb = std::min<int64_t>(p.batches_per_launch, B - b0);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(nb * (p.mode == kFpsCta ? 1 : p.G)));
    cfg.blockDim = dim3(p.NT);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (p.mode == kFpsCluster) {
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = p.G;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
    } else if (p.mode == kFpsGrid) {
      attr[0].id = cudaLaunchAttributeCooperative;
      attr[0].val.cooperative = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
    }
    int64_t b0v = b0;
    int bsi = bs, lbsi = lbs, Qi = Q;
    void* args[] = {(void*)&tp, &Pi, &Si, &Gi, &bsi, &lbsi, &Qi, &b0v, &idx, &gslots, &gcount};
    if (int s = cuda_status(cudaLaunchKernelExC(&cfg, fn, args))) return s;
  }
  return TPO_OK;
}

size_t fps_workspace_size(int dtype, int64_t B, int64_t P) {
  FpsPlan p;
  int s;
  switch (dtype) {
    case TPO_F32: s = fps_plan<FpsF32>(dtype, B, P, &p); break;
    case TPO_F16: s = fps_plan<FpsF16>(dtype, B, P, &p); break;
    case TPO_F64: s = fps_plan<FpsF64>(dtype, B, P, &p); break;
    default: return 0;
  }
  return s ? 0 : fps_ws_bytes_for(dtype, B, p);
}

int fps_forward(int dtype, const void* pts, int64_t B, int64_t P, int64_t S, int64_t* idx,
                void* ws, size_t ws_bytes, cudaStream_t st) {
  if (B == 0 || S == 0) return TPO_OK;
  switch (dtype) {
    case TPO_F32: return fps_run<FpsF32>(dtype, pts, B, P, S, idx, ws, ws_bytes, st);
    case TPO_F16: return fps_run<FpsF16>(dtype, pts, B, P, S, idx, ws, ws_bytes, st);
    case TPO_F64: return fps_run<FpsF64>(dtype, pts, B, P, S, idx, ws, ws_bytes, st);
  }
  return TPO_ERR_INVALID_ARGUMENT;
}

int fps_device_error_flags(unsigned* out, bool clear) {
  int s = cuda_status(cudaMemcpyFromSymbol(out, g_fps_device_error, sizeof(unsigned)));
  if (s || !clear) return s;
  const unsigned zero = 0;
  return cuda_status(cudaMemcpyToSymbol(g_fps_device_error, &zero, sizeof(unsigned)));
}

}  // namespace tpo
