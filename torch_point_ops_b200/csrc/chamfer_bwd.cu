// Chamfer backward: gradient scatter through the argmin indices.
//
// Replaces chamfer_dist_grad_kernel (torch_point_ops/chamfer/csrc/cuda/
// chamfer.cu:200-234), which is launched twice on 16 CTAs.  Here both directions
// run in ONE grid-stride launch sized to the whole GPU; each point gathers its
// nearest neighbour, forms v = (2*grad) * (p - nn) with the reference's
// per-operation rounding (g = grad*2, :222; g*(x1-x2), :226-231), adds v to its
// own gradient and subtracts it from its neighbour's with fire-and-forget
// atomics.  HBM-bound: per point it reads its coordinates, index and grad, the
// neighbour's coordinates, and issues 6 reductions.
#include "tpo_internal.h"

namespace tpo {

template <typename T>
struct BwdOps;
template <>
struct BwdOps<float> {
  __device__ static float two_g(float g) { return __fmul_rn(g, 2.0f); }
  __device__ static float term(float g2, float a, float b) { return __fmul_rn(g2, __fsub_rn(a, b)); }
  __device__ static void add(float* p, float v) { atomicAdd(p, v); }
  __device__ static void add3(float* p, const float* v) { red_add3f(p, v[0], v[1], v[2]); }
  __device__ static float neg(float v) { return -v; }
  __device__ static float div(float g, int64_t n) { return __fdiv_rn(g, (float)n); }
};
template <>
struct BwdOps<double> {
  __device__ static double two_g(double g) { return __dmul_rn(g, 2.0); }
  __device__ static double term(double g2, double a, double b) { return __dmul_rn(g2, __dsub_rn(a, b)); }
  __device__ static void add(double* p, double v) { atomicAdd(p, v); }
  __device__ static void add3(double* p, const double* v) {
    atomicAdd(p, v[0]);
    atomicAdd(p + 1, v[1]);
    atomicAdd(p + 2, v[2]);
  }
  __device__ static double neg(double v) { return -v; }
  __device__ static double div(double g, int64_t n) { return __ddiv_rn(g, (double)n); }
};
template <>
struct BwdOps<__half> {
  __device__ static __half two_g(__half g) { return hmul_rn(g, __float2half_rn(2.0f)); }
  __device__ static __half term(__half g2, __half a, __half b) { return hmul_rn(g2, hsub_rn(a, b)); }
  __device__ static void add(__half* p, __half v) { atomicAdd(p, v); }
  __device__ static void add3(__half* p, const __half* v) { red_add3h(p, v[0], v[1], v[2]); }
  __device__ static __half neg(__half v) { return __hneg(v); }
  __device__ static __half div(__half g, int64_t n) { return __float2half_rn(__half2float(g) / (float)n); }
};

template <typename T>
__global__ void chamfer_bwd_kernel(const T* __restrict__ x1, const T* __restrict__ x2, int64_t B,
                                   int64_t N, int64_t M, int64_t r0, int64_t r1, int64_t c0,
                                   int64_t c1, const int32_t* __restrict__ i1,
                                   const int32_t* __restrict__ i2, const T* __restrict__ g1,
                                   const T* __restrict__ g2, const T* __restrict__ gs,
                                   int scalar_mode, T* __restrict__ gx1, T* __restrict__ gx2) {
  using O = BwdOps<T>;
  // scalar_mode: 0 per-point grads g1/g2; 1 loss = mean(d1)+mean(d2) (grad gs/(B*N),
  // gs/(B*M), as torch's MeanBackward divides); 2 loss = sum(d1)+sum(d2) (grad gs)
  T gs1 = T(0.0f), gs2 = T(0.0f);
  if (scalar_mode) {
    const T g = *gs;
    gs1 = scalar_mode == 1 ? O::div(g, B * N) : g;
    gs2 = scalar_mode == 1 ? O::div(g, B * M) : g;
  }
  const int64_t nr = ((g1 || scalar_mode) && M > 0) ? r1 - r0 : 0;
  const int64_t nc = ((g2 || scalar_mode) && N > 0) ? c1 - c0 : 0;
  const int64_t n1 = B * nr;
  const int64_t total = n1 + B * nc;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const T *pa, *pb;
    T *ga, *gb;
    T g;
    if (t < n1) {
      const int64_t b = t / nr, i = r0 + t % nr;
      const int64_t o = b * N + i;
      const int64_t j = i1[o];
      pa = x1 + o * 3;
      pb = x2 + (b * M + j) * 3;
      ga = gx1 + o * 3;
      gb = gx2 + (b * M + j) * 3;
      g = scalar_mode ? gs1 : g1[o];
    } else {
      const int64_t u = t - n1;
      const int64_t b = u / nc, j = c0 + u % nc;
      const int64_t o = b * M + j;
      const int64_t i = i2[o];
      pa = x2 + o * 3;
      pb = x1 + (b * N + i) * 3;
      ga = gx2 + o * 3;
      gb = gx1 + (b * N + i) * 3;
      g = scalar_mode ? gs2 : g2[o];
    }
    const T gg = O::two_g(g);
    T v[3], nv[3];
#pragma unroll
    for (int d = 0; d < 3; ++d) {
      v[d] = O::term(gg, pa[d], pb[d]);
      nv[d] = O::neg(v[d]);
    }
    O::add3(ga, v);
    O::add3(gb, nv);
  }
}

template <typename T>
static int launch_bwd(const T* x1, const T* x2, int64_t B, int64_t N, int64_t M, int64_t r0,
                      int64_t r1, int64_t c0, int64_t c1, const int32_t* i1, const int32_t* i2,
                      const T* g1, const T* g2, const T* gs, int sm, T* gx1, T* gx2,
                      cudaStream_t st) {
  const int64_t total = B * (((g1 || sm) && M > 0) ? r1 - r0 : 0) + B * (((g2 || sm) && N > 0) ? c1 - c0 : 0);
  if (total <= 0) return TPO_OK;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, 148 * 16);
  chamfer_bwd_kernel<T><<<(unsigned)blocks, threads, 0, st>>>(x1, x2, B, N, M, r0, r1, c0, c1, i1,
                                                               i2, g1, g2, gs, sm, gx1, gx2);
  return check_launch();
}

int chamfer_bwd_accumulate(int dtype, const void* x1, const void* x2, int64_t B, int64_t N,
                           int64_t M, int64_t r0, int64_t r1, int64_t c0, int64_t c1,
                           const int32_t* i1, const int32_t* i2, const void* g1, const void* g2,
                           const void* gs, int sm, void* gx1, void* gx2, cudaStream_t st) {
  switch (dtype) {
    case TPO_F32:
      return launch_bwd<float>((const float*)x1, (const float*)x2, B, N, M, r0, r1, c0, c1, i1, i2,
                               (const float*)g1, (const float*)g2, (const float*)gs, sm, (float*)gx1, (float*)gx2, st);
    case TPO_F16:
      return launch_bwd<__half>((const __half*)x1, (const __half*)x2, B, N, M, r0, r1, c0, c1, i1,
                                i2, (const __half*)g1, (const __half*)g2, (const __half*)gs, sm, (__half*)gx1,
                                (__half*)gx2, st);
    case TPO_F64:
      return launch_bwd<double>((const double*)x1, (const double*)x2, B, N, M, r0, r1, c0, c1, i1,
                                i2, (const double*)g1, (const double*)g2, (const double*)gs, sm, (double*)gx1,
                                (double*)gx2, st);
  }
  return TPO_ERR_INVALID_ARGUMENT;
}

}  // namespace tpo

namespace tpo {

// Workspace / gradient initialisation as one kernel: fills up to two byte ranges
// (16-byte stores where aligned) and, meanwhile, asks L2 to fetch up to two
// input arrays (prefetch.global.L2: no register result, nothing waits on it) so
// that the next kernel's first touches of its inputs hit L2.
__global__ void fill_prefetch_kernel(unsigned char* d0, size_t n0, unsigned char* d1, size_t n1,
                                     unsigned v32a, unsigned v32b, const char* p0, size_t m0,
                                     const char* p1, size_t m1) {
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t nth = (size_t)gridDim.x * blockDim.x;
  pdl_trigger();  // the (PDL-launched) consumer may be scheduled; it waits for this grid
  for (int r = 0; r < 2; ++r) {
    unsigned char* d = r ? d1 : d0;
    const size_t n = r ? n1 : n0;
    const unsigned v32 = r ? v32b : v32a;
    const uint4 v = make_uint4(v32, v32, v32, v32);
    if (!d || !n) continue;
    size_t head = (16 - ((uintptr_t)d & 15)) & 15;
    if (head > n) head = n;
    for (size_t i = tid; i < head; i += nth) d[i] = (unsigned char)v32;
    const size_t nv = (n - head) / 16;
    uint4* dv = reinterpret_cast<uint4*>(d + head);
    for (size_t i = tid; i < nv; i += nth) dv[i] = v;
    for (size_t i = head + nv * 16 + tid; i < n; i += nth) d[i] = (unsigned char)v32;
  }
  for (int r = 0; r < 2; ++r) {
    const char* p = r ? p1 : p0;
    const size_t m = r ? m1 : m0;
    if (!p) continue;
    for (size_t i = tid * 128; i < m; i += nth * 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p + i));
  }
}

int fill_prefetch(void* d0, size_t n0, void* d1, size_t n1, unsigned char value, const void* p0,
                  size_t m0, const void* p1, size_t m1, cudaStream_t st, int value1) {
  const size_t work = std::max(n0 + n1, (m0 + m1) / 8);
  if (work == 0) return TPO_OK;
  const int threads = 256;
  const unsigned blocks = (unsigned)std::min<size_t>((work / 16 + threads - 1) / threads + 1, 148 * 4);
  const unsigned v32 = value * 0x01010101u;
  const unsigned v32b = (value1 < 0 ? value : (unsigned char)value1) * 0x01010101u;
  fill_prefetch_kernel<<<blocks, threads, 0, st>>>((unsigned char*)d0, n0, (unsigned char*)d1, n1,
                                                   v32, v32b, (const char*)p0, m0, (const char*)p1, m1);
  return check_launch();
}

}  // namespace tpo
