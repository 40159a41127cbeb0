// extern "C" boundary of libtpo_b200 (declared in include/tpo_b200.h).
// Validates arguments, never aborts, returns tpo_status codes.
#include <cstdio>
#include <cstring>

#include "tpo_internal.h"

namespace tpo {

static thread_local char g_msg[256] = "";

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return TPO_OK;
  snprintf(g_msg, sizeof(g_msg), "CUDA error: %s", cudaGetErrorString(e));
  return TPO_ERR_CUDA;
}
int check_launch() { return cuda_status(cudaGetLastError()); }

static bool valid_dtype(int dt) { return dt == TPO_F32 || dt == TPO_F16 || dt == TPO_F64; }

static int fail(int code, const char* what) {
  snprintf(g_msg, sizeof(g_msg), "%s", what);
  return code;
}

int set_error(int code, const char* msg) { return fail(code, msg); }

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace tpo

using namespace tpo;

extern "C" {

int tpo_abi_version(void) { return TPO_B200_ABI_VERSION; }

const char* tpo_status_string(int status) {
  switch (status) {
    case TPO_OK: return "ok";
    case TPO_ERR_INVALID_ARGUMENT: return g_msg[0] ? g_msg : "invalid argument";
    case TPO_ERR_UNSUPPORTED: return g_msg[0] ? g_msg : "unsupported";
    case TPO_ERR_WORKSPACE: return g_msg[0] ? g_msg : "workspace too small";
    case TPO_ERR_CUDA: return g_msg[0] ? g_msg : "CUDA error";
    case TPO_ERR_DEVICE: return g_msg[0] ? g_msg : "no usable device";
  }
  return "unknown status";
}

int tpo_device_error_flags(unsigned* flags, int clear) {
  if (!flags) return fail(TPO_ERR_INVALID_ARGUMENT, "device_error_flags: null output");
  unsigned a = 0, b = 0, c = 0;
  int s = device_error_flags(&a, clear != 0);
  if (!s) s = fps_device_error_flags(&b, clear != 0);
  if (!s) s = knn_device_error_flags(&c, clear != 0);
  *flags = a | b | c;
  return s;
}

int tpo_chamfer_key_bytes(int dtype) {
  if (!valid_dtype(dtype)) return 0;
  return dtype == TPO_F64 ? 16 : 8;
}

size_t tpo_chamfer_fwd_workspace_size(int dtype, int64_t B, int64_t N, int64_t M) {
  if (!valid_dtype(dtype) || B < 0 || N < 0 || M < 0) return 0;
  const size_t kb = (size_t)tpo_chamfer_key_bytes(dtype);
  return align256(kb * (size_t)B * (size_t)N) + align256(kb * (size_t)B * (size_t)M);
}

int tpo_chamfer_keys_init(int dtype, void* keys, int64_t n, void* stream) {
  if (!valid_dtype(dtype) || n < 0) return fail(TPO_ERR_INVALID_ARGUMENT, "keys_init: bad dtype or size");
  if (n == 0) return TPO_OK;
  if (!keys) return fail(TPO_ERR_INVALID_ARGUMENT, "keys_init: null keys");
  return cuda_status(cudaMemsetAsync(keys, 0xff, (size_t)n * tpo_chamfer_key_bytes(dtype),
                                     (cudaStream_t)stream));
}

static int check_chamfer_shape(int dtype, const void* x1, const void* x2, int64_t B, int64_t N,
                               int64_t M) {
  if (!valid_dtype(dtype)) return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: dtype must be f32, f16 or f64");
  if (B < 0 || N < 0 || M < 0) return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: negative size");
  if (N >= (int64_t(1) << 31) || M >= (int64_t(1) << 31))
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: clouds are limited to 2^31-1 points (int32 indices)");
  if ((B * N > 0 && !x1) || (B * M > 0 && !x2)) return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: null input");
  return TPO_OK;
}

int tpo_chamfer_fwd_keys(int dtype, int flags, const void* xyz1, const void* xyz2, int64_t B,
                         int64_t N, int64_t M, int64_t row_begin, int64_t row_end, void* keys1,
                         void* keys2, void* stream) {
  int s = check_chamfer_shape(dtype, xyz1, xyz2, B, N, M);
  if (s) return s;
  if (row_begin < 0 || row_end > N || row_begin > row_end)
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: bad row range");
  if (B * (row_end - row_begin) > 0 && M > 0 && (!keys1 || !keys2))
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: null keys");
  return chamfer_fwd_keys(dtype, flags, xyz1, xyz2, B, N, M, row_begin, row_end, keys1, keys2,
                          (cudaStream_t)stream);
}

int tpo_chamfer_finalize(int dtype, int flags, const void* xyz1, const void* xyz2, int64_t B,
                         int64_t N, int64_t M, int64_t row_begin, int64_t row_end,
                         const void* keys1, const void* keys2, void* dist1, int32_t* idx1,
                         void* dist2, int32_t* idx2, void* stream) {
  int s = check_chamfer_shape(dtype, xyz1, xyz2, B, N, M);
  if (s) return s;
  if (row_begin < 0 || row_end > N || row_begin > row_end)
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: bad row range");
  if (B * (row_end - row_begin) > 0 && (!dist1 || !idx1 || (M > 0 && !keys1)))
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: null row outputs");
  if (dist2 && B * M > 0 && (!idx2 || (N > 0 && !keys2)))
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: null column outputs");
  return chamfer_finalize(dtype, flags, xyz1, xyz2, B, N, M, row_begin, row_end, keys1, keys2,
                          dist1, idx1, dist2, idx2, dist2 != nullptr, nullptr, 0, nullptr,
                          (cudaStream_t)stream);
}

int tpo_chamfer_fwd(int dtype, int flags, const void* xyz1, const void* xyz2, int64_t B,
                    int64_t N, int64_t M, void* dist1, void* dist2, int32_t* idx1, int32_t* idx2,
                    void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_chamfer_shape(dtype, xyz1, xyz2, B, N, M);
  if (s) return s;
  if ((B * N > 0 && (!dist1 || !idx1)) || (B * M > 0 && (!dist2 || !idx2)))
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer: null output");
  const size_t need = tpo_chamfer_fwd_workspace_size(dtype, B, N, M);
  if (need > 0 && (!workspace || workspace_bytes < need))
    return fail(TPO_ERR_WORKSPACE, "chamfer: workspace missing or smaller than tpo_chamfer_fwd_workspace_size()");
  if ((uintptr_t)workspace % 256) return fail(TPO_ERR_WORKSPACE, "chamfer: workspace must be 256-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const size_t kb = (size_t)tpo_chamfer_key_bytes(dtype);
  char* k1 = (char*)workspace;
  char* k2 = k1 + align256(kb * (size_t)B * (size_t)N);
  if (B > 0 && N > 0 && M > 0) {
    const size_t es = (size_t)dtype_size(dtype);
    if ((s = fill_prefetch(workspace, need, nullptr, 0, 0xff, xyz1, es * 3 * B * N, xyz2,
                           es * 3 * B * M, st)))
      return s;
    if ((s = chamfer_fwd_keys(dtype, flags, xyz1, xyz2, B, N, M, 0, N, k1, k2, st))) return s;
  }
  return chamfer_finalize(dtype, flags, xyz1, xyz2, B, N, M, 0, N, k1, k2, dist1, idx1, dist2, idx2,
                          true, nullptr, 0, nullptr, st);
}

int tpo_chamfer_bwd(int dtype, const void* xyz1, const void* xyz2, int64_t B, int64_t N,
                    int64_t M, const int32_t* idx1, const int32_t* idx2, const void* grad_dist1,
                    const void* grad_dist2, void* grad_xyz1, void* grad_xyz2, void* stream) {
  int s = check_chamfer_shape(dtype, xyz1, xyz2, B, N, M);
  if (s) return s;
  if ((B * N > 0 && !grad_xyz1) || (B * M > 0 && !grad_xyz2))
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_bwd: null gradient output");
  if ((grad_dist1 && B * N > 0 && !idx1) || (grad_dist2 && B * M > 0 && !idx2))
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_bwd: null index");
  cudaStream_t st = (cudaStream_t)stream;
  const size_t es = (size_t)dtype_size(dtype);
  if (B * N > 0 && (s = cuda_status(cudaMemsetAsync(grad_xyz1, 0, es * 3 * B * N, st)))) return s;
  if (B * M > 0 && (s = cuda_status(cudaMemsetAsync(grad_xyz2, 0, es * 3 * B * M, st)))) return s;
  return chamfer_bwd_accumulate(dtype, xyz1, xyz2, B, N, M, 0, N, 0, M, idx1, idx2, grad_dist1,
                                grad_dist2, nullptr, 0, grad_xyz1, grad_xyz2, st);
}

int tpo_chamfer_bwd_partial(int dtype, const void* xyz1, const void* xyz2, int64_t B, int64_t N,
                            int64_t M, int64_t row_begin, int64_t row_end, int64_t col_begin,
                            int64_t col_end, const int32_t* idx1, const int32_t* idx2,
                            const void* grad_dist1, const void* grad_dist2, void* grad_xyz1,
                            void* grad_xyz2, void* stream) {
  int s = check_chamfer_shape(dtype, xyz1, xyz2, B, N, M);
  if (s) return s;
  if (row_begin < 0 || row_end > N || row_begin > row_end || col_begin < 0 || col_end > M ||
      col_begin > col_end)
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_bwd_partial: bad range");
  if ((B * N > 0 && !grad_xyz1) || (B * M > 0 && !grad_xyz2))
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_bwd_partial: null gradient output");
  return chamfer_bwd_accumulate(dtype, xyz1, xyz2, B, N, M, row_begin, row_end, col_begin, col_end,
                                idx1, idx2, grad_dist1, grad_dist2, nullptr, 0, grad_xyz1,
                                grad_xyz2, (cudaStream_t)stream);
}

// Fused-loss workspace: everything the backward needs stays in it.
//   [keys1|keys2][keys-loss counters|batch partials][finalize partials|counter][idx1][idx2]
// fp32 with a non-empty problem uses the keys kernel's fused reduction and the
// backward re-derives the neighbours from the keys; other cases finalize into
// idx1/idx2 and reduce there.
struct LossLayout {
  size_t keys, kl, fin, idx1, idx2, g1, g2, total;
};
static LossLayout loss_layout(int dtype, int64_t B, int64_t N, int64_t M) {
  LossLayout L;
  L.keys = 0;
  L.kl = tpo_chamfer_fwd_workspace_size(dtype, B, N, M);
  L.fin = L.kl + keys_loss_bytes(B);
  L.idx1 = L.fin + align256(kFinLossWorkspace);
  L.idx2 = L.idx1 + align256(4 * (size_t)B * (size_t)N);
  // gradient region, zero-filled by the forward (tpo_chamfer_loss_bwd_workspace)
  const size_t es = (size_t)dtype_size(dtype);
  L.g1 = L.idx2 + align256(4 * (size_t)B * (size_t)M);
  L.g2 = L.g1 + align256(es * 3 * (size_t)B * (size_t)N);
  L.total = L.g2 + align256(es * 3 * (size_t)B * (size_t)M);
  return L;
}
static bool loss_uses_keys_kernel(int dtype, int64_t B, int64_t N, int64_t M) {
  return (dtype == TPO_F32 || dtype == TPO_F16) && B > 0 && N > 0 && M > 0;
}

size_t tpo_chamfer_loss_workspace_size(int dtype, int64_t B, int64_t N, int64_t M) {
  if (!valid_dtype(dtype) || B < 0 || N < 0 || M < 0) return 0;
  return loss_layout(dtype, B, N, M).total;
}

int tpo_chamfer_loss_fwd(int dtype, int flags, const void* xyz1, const void* xyz2, int64_t B,
                         int64_t N, int64_t M, int reduction, void* loss, void* workspace,
                         size_t workspace_bytes, void* stream) {
  int s = check_chamfer_shape(dtype, xyz1, xyz2, B, N, M);
  if (s) return s;
  if (reduction != TPO_REDUCE_MEAN && reduction != TPO_REDUCE_SUM)
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_loss: reduction must be TPO_REDUCE_MEAN or TPO_REDUCE_SUM");
  if (!loss) return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_loss: null loss");
  const LossLayout L = loss_layout(dtype, B, N, M);
  if (!workspace || workspace_bytes < L.total || (uintptr_t)workspace % 256)
    return fail(TPO_ERR_WORKSPACE, "chamfer_loss: workspace missing, unaligned or smaller than tpo_chamfer_loss_workspace_size()");
  cudaStream_t st = (cudaStream_t)stream;
  char* w = (char*)workspace;
  const size_t kb = (size_t)tpo_chamfer_key_bytes(dtype);
  char* k1 = w;
  char* k2 = k1 + align256(kb * (size_t)B * (size_t)N);
  if (loss_uses_keys_kernel(dtype, B, N, M)) {
    // keys to the empty key and the reduction counters to 0xffffffff: one fill
    const size_t es = (size_t)dtype_size(dtype);
    // ... and the gradient region to zero, in the same launch
    if ((s = fill_prefetch(w, L.kl + keys_loss_counter_bytes(B), w + L.g1, L.total - L.g1, 0xff,
                           xyz1, es * 3 * B * N, xyz2, es * 3 * B * M, st, 0)))
      return s;
    return chamfer_loss_keys(dtype, flags, xyz1, xyz2, B, N, M, reduction, k1, k2, w + L.kl, loss,
                             w + L.fin, st);
  }
  if (L.kl && (s = cuda_status(cudaMemsetAsync(w, 0xff, L.kl, st)))) return s;
  if ((s = cuda_status(cudaMemsetAsync(w + L.fin + kFinPartialBytes, 0xff, 256, st)))) return s;
  if (L.total > L.g1 && (s = cuda_status(cudaMemsetAsync(w + L.g1, 0, L.total - L.g1, st)))) return s;
  if (B > 0 && N > 0 && M > 0 &&
      (s = chamfer_fwd_keys(dtype, flags, xyz1, xyz2, B, N, M, 0, N, k1, k2, st)))
    return s;
  return chamfer_finalize(dtype, flags, xyz1, xyz2, B, N, M, 0, N, k1, k2, nullptr,
                          (int32_t*)(w + L.idx1), nullptr, (int32_t*)(w + L.idx2), true, loss,
                          reduction, w + L.fin, st);
}

// The gradient scatter of the fused loss into (already zeroed) gradient buffers.
static int loss_bwd_scatter(int dtype, int flags, const void* xyz1, const void* xyz2, int64_t B,
                            int64_t N, int64_t M, int reduction, const char* w,
                            const void* grad_loss, void* grad_xyz1, void* grad_xyz2, cudaStream_t st) {
  const LossLayout L = loss_layout(dtype, B, N, M);
  if (loss_uses_keys_kernel(dtype, B, N, M)) {
    const size_t kb = (size_t)tpo_chamfer_key_bytes(dtype);
    return chamfer_bwd_from_keys(dtype, flags, xyz1, xyz2, B, N, M, w,
                                 w + align256(kb * (size_t)B * (size_t)N), grad_loss, reduction,
                                 grad_xyz1, grad_xyz2, st);
  }
  return chamfer_bwd_accumulate(dtype, xyz1, xyz2, B, N, M, 0, N, 0, M,
                                (const int32_t*)(w + L.idx1), (const int32_t*)(w + L.idx2),
                                nullptr, nullptr, grad_loss,
                                reduction == TPO_REDUCE_MEAN ? 1 : 2, grad_xyz1, grad_xyz2, st);
}

int tpo_chamfer_loss_bwd(int dtype, int flags, const void* xyz1, const void* xyz2, int64_t B,
                         int64_t N, int64_t M, int reduction, const void* workspace,
                         const void* grad_loss, void* grad_xyz1, void* grad_xyz2, void* stream) {
  int s = check_chamfer_shape(dtype, xyz1, xyz2, B, N, M);
  if (s) return s;
  if (reduction != TPO_REDUCE_MEAN && reduction != TPO_REDUCE_SUM)
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_loss_bwd: bad reduction");
  if (!grad_loss || !workspace || (B * N > 0 && !grad_xyz1) || (B * M > 0 && !grad_xyz2))
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_loss_bwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const size_t es = (size_t)dtype_size(dtype);
  if ((s = fill_prefetch(grad_xyz1, es * 3 * B * N, grad_xyz2, es * 3 * B * M, 0, nullptr, 0,
                         nullptr, 0, st)))
    return s;
  return loss_bwd_scatter(dtype, flags, xyz1, xyz2, B, N, M, reduction, (const char*)workspace,
                          grad_loss, grad_xyz1, grad_xyz2, st);
}

size_t tpo_chamfer_loss_grad_offset(int dtype, int64_t B, int64_t N, int64_t M, int which) {
  if (!valid_dtype(dtype) || B < 0 || N < 0 || M < 0 || (which != 1 && which != 2)) return 0;
  const LossLayout L = loss_layout(dtype, B, N, M);
  return which == 1 ? L.g1 : L.g2;
}

int tpo_chamfer_loss_bwd_workspace(int dtype, int flags, const void* xyz1, const void* xyz2,
                                   int64_t B, int64_t N, int64_t M, int reduction,
                                   void* workspace, const void* grad_loss, void* stream) {
  int s = check_chamfer_shape(dtype, xyz1, xyz2, B, N, M);
  if (s) return s;
  if (reduction != TPO_REDUCE_MEAN && reduction != TPO_REDUCE_SUM)
    return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_loss_bwd_workspace: bad reduction");
  if (!grad_loss || !workspace) return fail(TPO_ERR_INVALID_ARGUMENT, "chamfer_loss_bwd_workspace: null pointer");
  const LossLayout L = loss_layout(dtype, B, N, M);
  char* w = (char*)workspace;
  return loss_bwd_scatter(dtype, flags, xyz1, xyz2, B, N, M, reduction, w, grad_loss, w + L.g1,
                          w + L.g2, (cudaStream_t)stream);
}

static int check_knn(int dtype, const void* p1, const void* p2, int64_t N, int64_t P1, int64_t P2,
                     int64_t D, int64_t norm, int64_t K) {
  if (!valid_dtype(dtype)) return fail(TPO_ERR_INVALID_ARGUMENT, "knn: dtype must be f32, f16 or f64");
  if (N < 0 || P1 < 0 || P2 < 0 || D < 1) return fail(TPO_ERR_INVALID_ARGUMENT, "knn: bad shape");
  if (norm != 1 && norm != 2) return fail(TPO_ERR_INVALID_ARGUMENT, "Norm must be 1 or 2.");
  if (K < 1) return fail(TPO_ERR_INVALID_ARGUMENT, "knn: K must be >= 1");
  if (K > kKnnMaxK) return fail(TPO_ERR_UNSUPPORTED, "knn: this build supports K <= 1024");
  if (P2 >= (int64_t(1) << 31)) return fail(TPO_ERR_INVALID_ARGUMENT, "knn: P2 limited to 2^31-1");
  if ((N * P1 > 0 && !p1) || (N * P2 > 0 && !p2)) return fail(TPO_ERR_INVALID_ARGUMENT, "knn: null input");
  return TPO_OK;
}

int tpo_knn_fwd(int dtype, int flags, const void* p1, const void* p2, const int64_t* lengths1,
                const int64_t* lengths2, int64_t N, int64_t P1, int64_t P2, int64_t D,
                int64_t norm, int64_t K, void* dists, int64_t* idxs, void* stream) {
  int s = check_knn(dtype, p1, p2, N, P1, P2, D, norm, K);
  if (s) return s;
  if (N * P1 > 0 && (!dists || !idxs)) return fail(TPO_ERR_INVALID_ARGUMENT, "knn: null output");
  return knn_forward(dtype, flags, p1, p2, lengths1, lengths2, N, P1, P2, D, norm, K, dists, idxs,
                     (cudaStream_t)stream);
}

int tpo_knn_bwd(int dtype, const void* p1, const void* p2, const int64_t* lengths1,
                const int64_t* lengths2, const int64_t* idxs, int64_t N, int64_t P1, int64_t P2,
                int64_t D, int64_t K, int64_t norm, const void* grad_dists, void* grad_p1,
                void* grad_p2, void* stream) {
  int s = check_knn(dtype, p1, p2, N, P1, P2, D, norm, K);
  if (s) return s;
  if ((N * P1 > 0 && (!grad_p1 || !idxs || !grad_dists)) || (N * P2 > 0 && !grad_p2))
    return fail(TPO_ERR_INVALID_ARGUMENT, "knn_bwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (N * P2 > 0 &&
      (s = cuda_status(cudaMemsetAsync(grad_p2, 0, (size_t)dtype_size(dtype) * N * P2 * D, st))))
    return s;
  return knn_backward(dtype, p1, p2, lengths1, lengths2, idxs, N, P1, P2, D, K, norm, grad_dists,
                      grad_p1, grad_p2, st);
}

int tpo_knn_gather_fwd(int dtype, const void* x, const int64_t* idx, const int64_t* lengths,
                       int64_t N, int64_t M, int64_t U, int64_t L, int64_t K, void* out,
                       void* stream) {
  if (!valid_dtype(dtype)) return fail(TPO_ERR_INVALID_ARGUMENT, "knn_gather: bad dtype");
  if (N < 0 || M < 0 || U < 0 || L < 0 || K < 0) return fail(TPO_ERR_INVALID_ARGUMENT, "knn_gather: bad shape");
  if (N * L * K * U > 0 && (!idx || !out || (M * U > 0 && !x)))
    return fail(TPO_ERR_INVALID_ARGUMENT, "knn_gather: null pointer");
  return knn_gather_forward(dtype, x, idx, lengths, N, M, U, L, K, out, (cudaStream_t)stream);
}

int tpo_knn_gather_bwd(int dtype, const void* grad_out, const int64_t* idx, const int64_t* lengths,
                       int64_t N, int64_t M, int64_t U, int64_t L, int64_t K, void* grad_x,
                       void* stream) {
  if (!valid_dtype(dtype)) return fail(TPO_ERR_INVALID_ARGUMENT, "knn_gather_bwd: bad dtype");
  if (N < 0 || M < 0 || U < 0 || L < 0 || K < 0) return fail(TPO_ERR_INVALID_ARGUMENT, "knn_gather_bwd: bad shape");
  if (N * M * U > 0 && !grad_x) return fail(TPO_ERR_INVALID_ARGUMENT, "knn_gather_bwd: null grad_x");
  if (N * L * K * U > 0 && (!idx || !grad_out)) return fail(TPO_ERR_INVALID_ARGUMENT, "knn_gather_bwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  int s;
  if (N * M * U > 0 &&
      (s = cuda_status(cudaMemsetAsync(grad_x, 0, (size_t)dtype_size(dtype) * N * M * U, st))))
    return s;
  return knn_gather_backward(dtype, grad_out, idx, lengths, N, M, U, L, K, grad_x, st);
}

size_t tpo_fps_workspace_size(int dtype, int64_t B, int64_t P) {
  if (!valid_dtype(dtype) || B < 0 || P <= 0) return 0;
  return fps_workspace_size(dtype, B, P);
}

int tpo_fps_fwd(int dtype, const void* points, int64_t B, int64_t P, int64_t S, int64_t* idx,
                void* workspace, size_t workspace_bytes, void* stream) {
  if (!valid_dtype(dtype)) return fail(TPO_ERR_INVALID_ARGUMENT, "fps: dtype must be f32, f16 or f64");
  if (B < 0 || P < 0 || P > INT32_MAX) return fail(TPO_ERR_INVALID_ARGUMENT, "fps: bad shape");
  if (S <= 0) return fail(TPO_ERR_INVALID_ARGUMENT, "fps: nsamples must be positive");
  if (S > P) return fail(TPO_ERR_INVALID_ARGUMENT, "fps: nsamples cannot exceed number of points");
  if (B > 0 && (!points || !idx)) return fail(TPO_ERR_INVALID_ARGUMENT, "fps: null pointer");
  return fps_forward(dtype, points, B, P, S, idx, workspace, workspace_bytes, (cudaStream_t)stream);
}

int tpo_gather_points_fwd(int dtype, const void* points, const int64_t* idx, int64_t N, int64_t C,
                          int64_t P, int64_t M, void* out, void* stream) {
  if (!valid_dtype(dtype)) return fail(TPO_ERR_INVALID_ARGUMENT, "gather_points: bad dtype");
  if (N < 0 || C < 0 || P < 0 || M < 0) return fail(TPO_ERR_INVALID_ARGUMENT, "gather_points: bad shape");
  if (N * C * M > 0 && (!points || !idx || !out)) return fail(TPO_ERR_INVALID_ARGUMENT, "gather_points: null pointer");
  return gather_points_forward(dtype, points, idx, N, C, P, M, out, (cudaStream_t)stream);
}

int tpo_gather_points_bwd(int dtype, const void* grad_out, const int64_t* idx, int64_t N, int64_t C,
                          int64_t P, int64_t M, void* grad_points, void* stream) {
  if (!valid_dtype(dtype)) return fail(TPO_ERR_INVALID_ARGUMENT, "gather_points_bwd: bad dtype");
  if (N < 0 || C < 0 || P < 0 || M < 0) return fail(TPO_ERR_INVALID_ARGUMENT, "gather_points_bwd: bad shape");
  if ((N * C * P > 0 && !grad_points) || (N * C * M > 0 && (!grad_out || !idx)))
    return fail(TPO_ERR_INVALID_ARGUMENT, "gather_points_bwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  int s;
  if (N * C * P > 0 &&
      (s = cuda_status(cudaMemsetAsync(grad_points, 0, (size_t)dtype_size(dtype) * N * C * P, st))))
    return s;
  return gather_points_backward(dtype, grad_out, idx, N, C, P, M, grad_points, st);
}

}  // extern "C"
