// gather_points forward / backward (channel-first point features).
//
// Replaces gather_points_kernel / gather_points_grad_kernel
// (torch_point_ops/fps/csrc/cuda/fps.cu:63-97, launched at :318-401), the gather that follows
// furthest-point sampling: out[n,c,j] = points[n,c,idx[n,j]] for points (N,C,P),
// idx (N,M) int64, out (N,C,M).  One thread per output element, consecutive
// threads on consecutive j (coalesced stores, idx row reused from L1 across c).
// Backward scatters with atomics (like the reference); indices outside [0,P)
// read as zero / are skipped instead of faulting.
#include "tpo_internal.h"

namespace tpo {

template <typename T>
__global__ void gather_points_fwd_kernel(const T* __restrict__ pts, const int64_t* __restrict__ idx,
                                         int64_t N, int64_t C, int64_t P, int64_t M,
                                         T* __restrict__ out) {
  const int64_t total = N * C * M;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = t % M;
    const int64_t nc = t / M;
    const int64_t n = nc / C;
    const int64_t a = __ldg(idx + n * M + j);
    out[t] = (a >= 0 && a < P) ? pts[nc * P + a] : T(0.0f);
  }
}

template <typename T>
__global__ void gather_points_bwd_kernel(const T* __restrict__ gout, const int64_t* __restrict__ idx,
                                         int64_t N, int64_t C, int64_t P, int64_t M,
                                         T* __restrict__ gpts) {
  const int64_t total = N * C * M;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = t % M;
    const int64_t nc = t / M;
    const int64_t n = nc / C;
    const int64_t a = __ldg(idx + n * M + j);
    if (a >= 0 && a < P) atomicAdd(gpts + nc * P + a, gout[t]);
  }
}

int gather_points_forward(int dtype, const void* pts, const int64_t* idx, int64_t N, int64_t C,
                          int64_t P, int64_t M, void* out, cudaStream_t st) {
  const int64_t total = N * C * M;
  if (total <= 0) return TPO_OK;
  const int threads = 256;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + threads - 1) / threads, 148 * 16);
  switch (dtype) {
    case TPO_F32: gather_points_fwd_kernel<float><<<blocks, threads, 0, st>>>((const float*)pts, idx, N, C, P, M, (float*)out); break;
    case TPO_F16: gather_points_fwd_kernel<__half><<<blocks, threads, 0, st>>>((const __half*)pts, idx, N, C, P, M, (__half*)out); break;
    case TPO_F64: gather_points_fwd_kernel<double><<<blocks, threads, 0, st>>>((const double*)pts, idx, N, C, P, M, (double*)out); break;
    default: return TPO_ERR_INVALID_ARGUMENT;
  }
  return check_launch();
}

int gather_points_backward(int dtype, const void* gout, const int64_t* idx, int64_t N, int64_t C,
                           int64_t P, int64_t M, void* gpts, cudaStream_t st) {
  const int64_t total = N * C * M;
  if (total <= 0) return TPO_OK;
  const int threads = 256;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + threads - 1) / threads, 148 * 16);
  switch (dtype) {
    case TPO_F32: gather_points_bwd_kernel<float><<<blocks, threads, 0, st>>>((const float*)gout, idx, N, C, P, M, (float*)gpts); break;
    case TPO_F16: gather_points_bwd_kernel<__half><<<blocks, threads, 0, st>>>((const __half*)gout, idx, N, C, P, M, (__half*)gpts); break;
    case TPO_F64: gather_points_bwd_kernel<double><<<blocks, threads, 0, st>>>((const double*)gout, idx, N, C, P, M, (double*)gpts); break;
    default: return TPO_ERR_INVALID_ARGUMENT;
  }
  return check_launch();
}

}  // namespace tpo
