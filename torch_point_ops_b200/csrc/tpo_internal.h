// Internal declarations shared by the tpo_b200 translation units.
#pragma once

#include <algorithm>
#include <climits>
#include <cstdint>

#include "tpo_common.cuh"

namespace tpo {

// Records the CUDA error text for tpo_status_string and maps it to TPO_ERR_CUDA.
int cuda_status(cudaError_t e);
// cudaGetLastError() after a launch.
int check_launch();
// Records `msg` for tpo_status_string and returns `code`.
int set_error(int code, const char* msg);
int pipe_probe(int kind, double* lane_ops_per_s, double* sm_mhz);

int chamfer_fwd_keys(int dtype, int flags, const void* x1, const void* x2, int64_t B, int64_t N,
                     int64_t M, int64_t rb0, int64_t rb1, void* k1, void* k2, cudaStream_t st);
// Finalize keys into (dist, idx).  do_cols: also the column side.  loss != null:
// fused reduction (0 = mean(d1)+mean(d2), 1 = sums) using loss_ws
// (kFinLossWorkspace bytes, the counter word at kFinPartialBytes set to 0xffffffff).
constexpr int kFinMaxBlocks = 148 * 32;
constexpr size_t kFinPartialBytes = (size_t)kFinMaxBlocks * 2 * sizeof(double);
constexpr size_t kFinLossWorkspace = kFinPartialBytes + 256;
int chamfer_finalize(int dtype, int flags, const void* x1, const void* x2, int64_t B, int64_t N,
                     int64_t M, int64_t rb0, int64_t rb1, const void* k1, const void* k2, void* d1,
                     int32_t* i1, void* d2, int32_t* i2, bool do_cols, void* loss, int reduction,
                     void* loss_ws, cudaStream_t st);
int chamfer_bwd_accumulate(int dtype, const void* x1, const void* x2, int64_t B, int64_t N,
                           int64_t M, int64_t r0, int64_t r1, int64_t c0, int64_t c1,
                           const int32_t* i1, const int32_t* i2, const void* g1, const void* g2,
                           const void* gscalar, int scalar_mode, void* gx1, void* gx2,
                           cudaStream_t st);
// Largest K of knn_forward (the list lives in registers, 8 rows of 32 lanes).
constexpr int64_t kKnnMaxK = 1024;
int knn_forward(int dtype, int flags, const void* p1, const void* p2, const int64_t* l1,
                const int64_t* l2, int64_t N, int64_t P1, int64_t P2, int64_t D, int64_t norm,
                int64_t K, void* dists, int64_t* idxs, cudaStream_t st);
int knn_backward(int dtype, const void* p1, const void* p2, const int64_t* l1, const int64_t* l2,
                 const int64_t* idxs, int64_t N, int64_t P1, int64_t P2, int64_t D, int64_t K,
                 int64_t norm, const void* gd, void* g1, void* g2, cudaStream_t st);
int knn_gather_forward(int dtype, const void* x, const int64_t* idx, const int64_t* lengths,
                       int64_t N, int64_t M, int64_t U, int64_t L, int64_t K, void* out,
                       cudaStream_t st);
int knn_gather_backward(int dtype, const void* gout, const int64_t* idx, const int64_t* lengths,
                        int64_t N, int64_t M, int64_t U, int64_t L, int64_t K, void* gx,
                        cudaStream_t st);

// Fused-loss forward: keys kernel (rows 0..N, all columns) + keys reduction.
// lossws: keys_loss_bytes(B) bytes whose first keys_loss_counter_bytes(B) are
// 0xff-filled (word B is the reduction's counter); partials: >= 296*16 bytes.
inline size_t keys_loss_counter_bytes(int64_t B) { return ((size_t)(B + 1) * 4 + 255) & ~(size_t)255; }
inline size_t keys_loss_bytes(int64_t B) { return keys_loss_counter_bytes(B) + (((size_t)B * 16 + 255) & ~(size_t)255); }
int chamfer_loss_keys(int dtype, int flags, const void* x1, const void* x2, int64_t B, int64_t N,
                      int64_t M, int reduction, void* k1, void* k2, void* lossws, void* loss,
                      void* partials, cudaStream_t st);
int chamfer_bwd_from_keys(int dtype, int flags, const void* x1, const void* x2, int64_t B, int64_t N,
                              int64_t M, const void* k1, const void* k2, const void* grad_loss,
                              int reduction, void* gx1, void* gx2, cudaStream_t st);

// Fills [d0, d0+n0) with `value` and [d1, d1+n1) with `value1` (default: the
// same) and prefetches the byte ranges [p0, p0+m0), [p1, p1+m1) into L2, in one
// launch (null / zero-size parts skipped).
int fill_prefetch(void* d0, size_t n0, void* d1, size_t n1, unsigned char value, const void* p0,
                  size_t m0, const void* p1, size_t m1, cudaStream_t st, int value1 = -1);

// Reads (and optionally clears) the device-side error flags of this device.
int device_error_flags(unsigned* out, bool clear);

size_t fps_workspace_size(int dtype, int64_t B, int64_t P);
int fps_forward(int dtype, const void* pts, int64_t B, int64_t P, int64_t S, int64_t* idx,
                void* ws, size_t ws_bytes, cudaStream_t st);
int fps_device_error_flags(unsigned* out, bool clear);
int knn_device_error_flags(unsigned* out, bool clear);
int gather_points_forward(int dtype, const void* pts, const int64_t* idx, int64_t N, int64_t C,
                          int64_t P, int64_t M, void* out, cudaStream_t st);
int gather_points_backward(int dtype, const void* gout, const int64_t* idx, int64_t N, int64_t C,
                           int64_t P, int64_t M, void* gpts, cudaStream_t st);

// Launches `kern` with programmatic stream serialisation allowed (see pdl_wait).
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                      Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
}

inline int dtype_size(int dtype) {
  return dtype == TPO_F32 ? 4 : dtype == TPO_F16 ? 2 : dtype == TPO_F64 ? 8 : 0;
}

}  // namespace tpo
