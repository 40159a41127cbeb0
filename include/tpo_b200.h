/*
 * tpo_b200 -- C ABI of the B200-native chamfer / knn nearest-neighbour path.
 *
 * Plain pointers and sizes only; no torch types.  Every pointer argument is a
 * DEVICE pointer on the current CUDA device unless stated otherwise, all point
 * clouds are contiguous (B, P, D) arrays in the dtype given by `dtype`, and every
 * call is asynchronous on `stream` (a cudaStream_t passed as void*; NULL = the
 * legacy default stream).  Calls never abort the process: each returns a
 * tpo_status (0 = success).  The library keeps no state between calls except
 * per-device launch tuning, so calls are re-entrant.
 *
 * Each entry point names the reference function it replaces (paths relative to
 * satyajitghana/torch-point-ops v0.1.0).
 */
#ifndef TPO_B200_H
#define TPO_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TPO_API __attribute__((visibility("default")))
#else
#define TPO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TPO_B200_ABI_VERSION 1

/* element types (match torch's float32 / float16 / float64) */
enum tpo_dtype { TPO_F32 = 0, TPO_F16 = 1, TPO_F64 = 2 };

/* flags for the chamfer distance arithmetic.
 * TPO_ROUND_FMA (default, 0): d = fma(dz,dz, fma(dx,dx, dy*dy)) -- bit-identical to
 *   the reference CUDA chamfer kernel (nvcc's contraction of chamfer.cu:67,
 *   measured on B200).
 * TPO_ROUND_EXACT: d = (dx*dx + dy*dy) + dz*dz with every operation rounded --
 *   the rounding of the reference CPU path (knn.cpp:64-72).
 * knn ignores the flag: the reference knn CUDA kernels are not contracted
 *   (measured), so both reference knn paths round like TPO_ROUND_EXACT.
 * fp16 always rounds every operation (c10::Half semantics). */
enum tpo_flags { TPO_ROUND_FMA = 0, TPO_ROUND_EXACT = 1 };

enum tpo_status {
  TPO_OK = 0,
  TPO_ERR_INVALID_ARGUMENT = 1, /* bad shape / dtype / K / norm / null pointer   */
  TPO_ERR_UNSUPPORTED = 2,      /* valid request this build does not implement  */
  TPO_ERR_WORKSPACE = 3,        /* workspace missing or smaller than required   */
  TPO_ERR_CUDA = 4,             /* a CUDA runtime call failed (see message)     */
  TPO_ERR_DEVICE = 5            /* no usable sm_100 device                      */
};

/* Human-readable text for a status, including the last CUDA error text for
 * TPO_ERR_CUDA on the calling thread. */
TPO_API const char* tpo_status_string(int status);
TPO_API int tpo_abi_version(void);

/* Device-side error flags of the current device (no counterpart in the
 * reference, which has no bounded waits): kernels never spin forever; a wait for
 * a bulk copy into shared memory that gives up sets bit 0
 * (TPO_DEVERR_BULK_TIMEOUT) and the kernel continues.  Reads the flags into
 * *flags (synchronous) and clears them if `clear` is non-zero. */
enum tpo_device_errors {
  TPO_DEVERR_BULK_TIMEOUT = 1, /* a bulk copy's mbarrier wait gave up           */
  TPO_DEVERR_GRID_TIMEOUT = 2  /* fps: a grid-wide step barrier wait gave up     */
};
TPO_API int tpo_device_error_flags(unsigned* flags, int clear);

/* ------------------------------------------------------------------------- */
/* Chamfer distance forward.  Replaces chamfer_cuda_forward
 * (torch_point_ops/chamfer/csrc/cuda/chamfer.cu:169-198) behind the
 * torch_point_ops_chamfer::chamfer_forward schema (chamfer/csrc/chamfer.cpp:34-39).
 *   xyz1 (B,N,3), xyz2 (B,M,3)                       dtype
 *   dist1 (B,N), dist2 (B,M)                         dtype   (squared distance)
 *   idx1 (B,N), idx2 (B,M)                           int32   (argmin, lowest index on ties)
 * Both directions are produced from ONE evaluation of each (i,j) pair.
 * Empty clouds give zeros, like the reference's torch::zeros outputs.
 * `workspace` must hold tpo_chamfer_fwd_workspace_size() bytes (256-byte aligned);
 * its contents on entry are ignored. */
TPO_API size_t tpo_chamfer_fwd_workspace_size(int dtype, int64_t B, int64_t N, int64_t M);
TPO_API int tpo_chamfer_fwd(int dtype, int flags, const void* xyz1, const void* xyz2, int64_t B,
                    int64_t N, int64_t M, void* dist1, void* dist2, int32_t* idx1,
                    int32_t* idx2, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free chamfer forward.  No counterpart in the reference.
 * For callers that cannot allocate device memory (no cudaMalloc, no allocator
 * they may call: code inside an allocator or memory pool, services that forbid
 * device allocation after start-up, hosts that only receive buffers).  Same
 * arguments and results as tpo_chamfer_fwd minus the workspace: the keys live
 * in a device array of 16 MiB (+512 bytes of alignment padding) owned by the
 * library, which every GPU that loads the library holds until process exit.
 * Limit: B*(N+M) <= 2,097,152 points for f32/f16 (1,048,576 for f64), whatever
 * the split between N and M; larger problems return TPO_ERR_WORKSPACE.  The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress) -- make that first call
 * before any stream capture.  Calls share the array: calls that overlap on the
 * GPU (other streams or threads on the same device) race and must be
 * serialised by the caller.  Allocates nothing. */
TPO_API int tpo_chamfer_fwd_noalloc(int dtype, int flags, const void* xyz1, const void* xyz2,
                                    int64_t B, int64_t N, int64_t M, void* dist1, void* dist2,
                                    int32_t* idx1, int32_t* idx2, void* stream);

/* Split form of tpo_chamfer_fwd for row-sharded multi-GPU runs (one rank owns rows
 * [row_begin,row_end) of xyz1 and all of xyz2).  Keys are packed (distance bits,
 * candidate-chunk) words; their minimum over ranks is the global answer, so an
 * element-wise MIN all-reduce of keys2 (as int64 for f32/f16) merges ranks.
 *   key bytes per point: tpo_chamfer_key_bytes(dtype) (8 for f32/f16, 16 for f64)
 *   keys_init:  set n keys to the empty value.
 *   fwd_keys:   fold pairs (rows [row_begin,row_end) x all M) into keys1/keys2.
 *   finalize:   turn keys into (dist, idx) for rows [row_begin,row_end) of cloud 1
 *               (dist1/idx1 point at row 0 of each batch as usual) and for all of
 *               cloud 2 when dist2 != NULL. */
TPO_API int tpo_chamfer_key_bytes(int dtype);
TPO_API int tpo_chamfer_keys_init(int dtype, void* keys, int64_t n, void* stream);
TPO_API int tpo_chamfer_fwd_keys(int dtype, int flags, const void* xyz1, const void* xyz2, int64_t B,
                         int64_t N, int64_t M, int64_t row_begin, int64_t row_end,
                         void* keys1, void* keys2, void* stream);
TPO_API int tpo_chamfer_finalize(int dtype, int flags, const void* xyz1, const void* xyz2, int64_t B,
                         int64_t N, int64_t M, int64_t row_begin, int64_t row_end,
                         const void* keys1, const void* keys2, void* dist1, int32_t* idx1,
                         void* dist2, int32_t* idx2, void* stream);

/* Chamfer distance backward.  Replaces chamfer_cuda_backward (chamfer.cu:236-271):
 *   grad_xyz1[i]      += 2*g1[i]*(xyz1[i] - xyz2[idx1[i]])
 *   grad_xyz2[idx1[i]] -= the same, and symmetrically for direction 2.
 * grad_xyz1 / grad_xyz2 are fully written (no need to zero them).
 * Either grad_dist pointer may be NULL (treated as zeros). */
TPO_API int tpo_chamfer_bwd(int dtype, const void* xyz1, const void* xyz2, int64_t B, int64_t N,
                    int64_t M, const int32_t* idx1, const int32_t* idx2,
                    const void* grad_dist1, const void* grad_dist2, void* grad_xyz1,
                    void* grad_xyz2, void* stream);
/* Row-sharded backward: only rows [row_begin,row_end) of cloud 1 and columns
 * [col_begin,col_end) of cloud 2 contribute; grads are ACCUMULATED (caller zeroes
 * them) so that a SUM all-reduce over ranks gives the full gradient. */
TPO_API int tpo_chamfer_bwd_partial(int dtype, const void* xyz1, const void* xyz2, int64_t B,
                            int64_t N, int64_t M, int64_t row_begin, int64_t row_end,
                            int64_t col_begin, int64_t col_end, const int32_t* idx1,
                            const int32_t* idx2, const void* grad_dist1,
                            const void* grad_dist2, void* grad_xyz1, void* grad_xyz2,
                            void* stream);

/* Fused ChamferDistance loss (chamfer/chamfer.py:18-23: reduction "mean" ->
 * mean(dist1) + mean(dist2), "sum" -> sum(dist1) + sum(dist2)).  Replaces the
 * reference's chamfer_forward + two torch reductions + the expanded per-point
 * gradients of its backward.  The forward writes the scalar `loss` (1 element,
 * dtype); for fp32 the reduction runs inside the distance kernel itself
 * (deterministic, fixed order).  Everything the backward needs stays in
 * `workspace` (tpo_chamfer_loss_workspace_size() bytes, 256-byte aligned): pass
 * the same, unmodified workspace and the same inputs/flags to the backward,
 * which reads the scalar grad_loss from device memory and applies the
 * reduction's scaling inside the scatter kernel. */
enum tpo_reduction { TPO_REDUCE_MEAN = 0, TPO_REDUCE_SUM = 1 };
TPO_API size_t tpo_chamfer_loss_workspace_size(int dtype, int64_t B, int64_t N, int64_t M);
TPO_API int tpo_chamfer_loss_fwd(int dtype, int flags, const void* xyz1, const void* xyz2,
                                 int64_t B, int64_t N, int64_t M, int reduction, void* loss,
                                 void* workspace, size_t workspace_bytes, void* stream);
TPO_API int tpo_chamfer_loss_bwd(int dtype, int flags, const void* xyz1, const void* xyz2,
                                 int64_t B, int64_t N, int64_t M, int reduction,
                                 const void* workspace, const void* grad_loss, void* grad_xyz1,
                                 void* grad_xyz2, void* stream);

/* Backward of the fused loss without a gradient fill: tpo_chamfer_loss_fwd also
 * zero-fills a gradient region inside the workspace (in the launch that resets
 * the keys), and this call scatters the gradients there -- grad_xyz1 (B,N,3) at
 * byte offset tpo_chamfer_loss_grad_offset(...,1) of the workspace, grad_xyz2
 * (B,M,3) at offset tpo_chamfer_loss_grad_offset(...,2), both 256-byte
 * aligned.  Valid once per forward (a second backward of the same forward must
 * use tpo_chamfer_loss_bwd, which fills caller buffers). */
TPO_API size_t tpo_chamfer_loss_grad_offset(int dtype, int64_t B, int64_t N, int64_t M, int which);
TPO_API int tpo_chamfer_loss_bwd_workspace(int dtype, int flags, const void* xyz1, const void* xyz2,
                                           int64_t B, int64_t N, int64_t M, int reduction,
                                           void* workspace, const void* grad_loss, void* stream);

/* ------------------------------------------------------------------------- */
/* K nearest neighbours forward.  Replaces knn_cuda_forward
 * (torch_point_ops/knn/csrc/cuda/knn.cu:295-398) behind
 * torch_point_ops_knn::knn_forward (knn/csrc/knn.cpp:167-169), with the sort of
 * knn_points (knn/__init__.py:110-131) done in the kernel:
 *   p1 (N,P1,D), p2 (N,P2,D) dtype; lengths1/lengths2 (N,) int64 (NULL = full)
 *   dists (N,P1,K) dtype, idxs (N,P1,K) int64
 * For each valid query (p < lengths1[n]) the K smallest (dist, idx) pairs over
 * the first lengths2[n] points, ascending by (dist, idx).  Slots k >= lengths2[n]
 * and rows p >= lengths1[n] hold idx -1 / dist 0 (the reference CPU padding,
 * knn.cpp:44-45).  norm: 2 = squared L2, 1 = L1.  1 <= K <= 1024 (larger K returns
 * TPO_ERR_UNSUPPORTED), any D >= 1; D <= 8 with K <= 32 takes the fast kernel.
 * fp32, D=3, L2, P2 >= 1024: the call also uses the idxs and dists buffers as
 * its scratch (a cell order of p2 and per-query thresholds) before the final
 * results overwrite them, so both must be distinct, writable and not read by
 * anyone until the call completes on `stream`; no other memory is allocated.
 * The environment variable TPO_KNN_SEED=0 (read once) turns the threshold seeds
 * off; results are identical either way. */
TPO_API int tpo_knn_fwd(int dtype, int flags, const void* p1, const void* p2,
                const int64_t* lengths1, const int64_t* lengths2, int64_t N, int64_t P1,
                int64_t P2, int64_t D, int64_t norm, int64_t K, void* dists, int64_t* idxs,
                void* stream);

/* knn backward.  Replaces knn_cuda_backward (knn.cu:469-534):
 *   L2: v = 2*g*(p1-p2); L1: v = g*sign(p1-p2) (0 at equality, knn.cu:447-449)
 *   grad_p1[row] += v; grad_p2[idx] -= v; rows >= lengths1 and idx -1 skipped.
 * grad_p1 / grad_p2 are fully written. */
TPO_API int tpo_knn_bwd(int dtype, const void* p1, const void* p2, const int64_t* lengths1,
                const int64_t* lengths2, const int64_t* idxs, int64_t N, int64_t P1,
                int64_t P2, int64_t D, int64_t K, int64_t norm, const void* grad_dists,
                void* grad_p1, void* grad_p2, void* stream);

/* knn_gather forward (knn/__init__.py:136-183): out[n,l,k,:] = x[n, idx[n,l,k], :],
 * zero where k >= lengths[n] or idx == -1.  x (N,M,U), idx (N,L,K) int64,
 * lengths (N,) int64 or NULL, out (N,L,K,U). */
TPO_API int tpo_knn_gather_fwd(int dtype, const void* x, const int64_t* idx, const int64_t* lengths,
                       int64_t N, int64_t M, int64_t U, int64_t L, int64_t K, void* out,
                       void* stream);
/* Its backward: grad_x (N,M,U) fully written with the scatter-add of grad_out. */
TPO_API int tpo_knn_gather_bwd(int dtype, const void* grad_out, const int64_t* idx,
                       const int64_t* lengths, int64_t N, int64_t M, int64_t U, int64_t L,
                       int64_t K, void* grad_x, void* stream);

/* ------------------------------------------------------------------------- */
/* gather_points (the gather that follows furthest-point sampling).  Replaces
 * gather_points_cuda_forward / _backward (torch_point_ops/fps/csrc/cuda/fps.cu:
 * 63-97, 318-401) behind torch_point_ops_fps::gather_points_forward /
 * gather_points_backward (fps/csrc/fps.cpp:160-161):
 *   points (N,C,P) dtype, idx (N,M) int64, out (N,C,M): out[n,c,j] = points[n,c,idx[n,j]]
 * Indices outside [0,P) give 0 (the reference does not check them).  The
 * backward fully writes grad_points (N,C,P) with the scatter-add of grad_out. */
/* Furthest point sampling.  Replaces fps_cuda_forward (torch_point_ops/fps/csrc/
 * cuda/fps.cu:261-316, kernel :108-213) behind torch_point_ops_fps::fps_forward
 * (fps/csrc/fps.cpp:159):
 *   points (B,P,3) dtype, idx (B,S) int64; 0 < S <= P (else TPO_ERR_INVALID_ARGUMENT).
 * Same indices as the reference CUDA kernel, ties included (see fps.cu here).
 * Clouds larger than the GPU's register file can hold (about 4.7M fp32 points)
 * return TPO_ERR_UNSUPPORTED.  Large clouds run as a cooperative grid that
 * needs tpo_fps_workspace_size() bytes of workspace (0 otherwise). */
TPO_API size_t tpo_fps_workspace_size(int dtype, int64_t B, int64_t P);
TPO_API int tpo_fps_fwd(int dtype, const void* points, int64_t B, int64_t P, int64_t S,
                        int64_t* idx, void* workspace, size_t workspace_bytes, void* stream);

TPO_API int tpo_gather_points_fwd(int dtype, const void* points, const int64_t* idx, int64_t N,
                                  int64_t C, int64_t P, int64_t M, void* out, void* stream);
TPO_API int tpo_gather_points_bwd(int dtype, const void* grad_out, const int64_t* idx, int64_t N,
                                  int64_t C, int64_t P, int64_t M, void* grad_points, void* stream);

/* Measurement aid (no counterpart in the reference): the sustained issue rate of
 * one arithmetic instruction kind on the current device, for quoting the CUDA-core
 * kernels' rooflines against a measured peak.  kind: 0 fma.rn.f32, 1 fma.rn.f32x2,
 * 2 fma.rn.f16x2, 3 fma.rn.f64.  *lane_ops_per_s = element results per second
 * over the whole GPU (a packed x2 instruction counts 2 per lane); *sm_mhz = the SM
 * clock seen during the run.  Synchronous (own stream, ~0.1-0.5 s); allocates
 * 32 bytes of device memory. */
TPO_API int tpo_probe_pipe_peak(int kind, double* lane_ops_per_s, double* sm_mhz);

#ifdef __cplusplus
}
#endif
#endif /* TPO_B200_H */
