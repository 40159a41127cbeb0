// torch.library binding over the tpo_b200 C ABI.
//
// Same schemas as the reference's operator libraries
//   torch_point_ops_chamfer  (torch_point_ops/chamfer/csrc/chamfer.cpp:34-39)
//   torch_point_ops_knn      (torch_point_ops/knn/csrc/knn.cpp:167-172)
//   torch_point_ops_fps      (torch_point_ops/fps/csrc/fps.cpp:158-162; fps_forward,
//                             gather_points_forward / _backward)
// registered under the namespaces torch_point_ops_b200_chamfer /
// torch_point_ops_b200_knn / torch_point_ops_b200_fps so both libraries can live
// in one process.  Extra ops:
// *_ex variants taking the rounding flags, the row-sharded split of the chamfer
// forward, and knn_gather forward/backward (a torch expand+gather in the
// reference, knn/__init__.py:136-183).  Only CUDA implementations are
// registered: there is no CPU fallback, a CPU tensor raises.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>
#include <torch/all.h>
#include <torch/autograd.h>

#include "../../include/tpo_b200.h"

namespace {

int to_dtype(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return TPO_F32;
    case at::kHalf: return TPO_F16;
    case at::kDouble: return TPO_F64;
    default: TORCH_CHECK(false, "tpo_b200: expected float32, float16 or float64, got ", t.scalar_type());
  }
  return -1;
}

void ok(int status, const char* where) {
  TORCH_CHECK(status == TPO_OK, where, ": ", tpo_status_string(status));
}

void check_cloud(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == 3, name, " must have shape (B, P, D)");
}

void* stream_of(const at::Tensor& t) {
  return (void*)at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> chamfer_forward_ex(
    const at::Tensor& xyz1_, const at::Tensor& xyz2_, int64_t flags) {
  check_cloud(xyz1_, "xyz1");
  check_cloud(xyz2_, "xyz2");
  TORCH_CHECK(xyz1_.size(2) == 3 && xyz2_.size(2) == 3, "chamfer: points must be 3-D");
  TORCH_CHECK(xyz1_.size(0) == xyz2_.size(0), "chamfer: batch sizes differ");
  TORCH_CHECK(xyz1_.scalar_type() == xyz2_.scalar_type(), "chamfer: dtypes differ");
  TORCH_CHECK(xyz1_.device() == xyz2_.device(), "chamfer: devices differ");
  const c10::cuda::CUDAGuard g(xyz1_.device());
  const at::Tensor xyz1 = xyz1_.contiguous(), xyz2 = xyz2_.contiguous();
  const int64_t B = xyz1.size(0), N = xyz1.size(1), M = xyz2.size(1);
  const int dt = to_dtype(xyz1);
  auto dist1 = at::empty({B, N}, xyz1.options());
  auto dist2 = at::empty({B, M}, xyz1.options());
  auto idx1 = at::empty({B, N}, xyz1.options().dtype(at::kInt));
  auto idx2 = at::empty({B, M}, xyz1.options().dtype(at::kInt));
  const size_t ws_bytes = tpo_chamfer_fwd_workspace_size(dt, B, N, M);
  at::Tensor ws;
  if (ws_bytes) ws = at::empty({(int64_t)ws_bytes}, xyz1.options().dtype(at::kByte));
  ok(tpo_chamfer_fwd(dt, (int)flags, xyz1.data_ptr(), xyz2.data_ptr(), B, N, M, dist1.data_ptr(),
                     dist2.data_ptr(), idx1.data_ptr<int32_t>(), idx2.data_ptr<int32_t>(),
                     ws_bytes ? ws.data_ptr() : nullptr, ws_bytes, stream_of(xyz1)),
     "chamfer_forward");
  return {dist1, dist2, idx1, idx2};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> chamfer_forward(const at::Tensor& a,
                                                                           const at::Tensor& b) {
  return chamfer_forward_ex(a, b, TPO_ROUND_FMA);
}

std::tuple<at::Tensor, at::Tensor> chamfer_backward(const at::Tensor& xyz1_, const at::Tensor& xyz2_,
                                                    const at::Tensor& idx1_, const at::Tensor& idx2_,
                                                    const at::Tensor& g1_, const at::Tensor& g2_) {
  check_cloud(xyz1_, "xyz1");
  check_cloud(xyz2_, "xyz2");
  const c10::cuda::CUDAGuard g(xyz1_.device());
  const at::Tensor xyz1 = xyz1_.contiguous(), xyz2 = xyz2_.contiguous();
  const int64_t B = xyz1.size(0), N = xyz1.size(1), M = xyz2.size(1);
  const at::Tensor idx1 = idx1_.to(at::kInt).contiguous(), idx2 = idx2_.to(at::kInt).contiguous();
  const at::Tensor g1 = g1_.to(xyz1.scalar_type()).contiguous().expand({B, N}).contiguous();
  const at::Tensor g2 = g2_.to(xyz1.scalar_type()).contiguous().expand({B, M}).contiguous();
  TORCH_CHECK(idx1.numel() == B * N && idx2.numel() == B * M, "chamfer_backward: index shape");
  auto gx1 = at::empty_like(xyz1);
  auto gx2 = at::empty_like(xyz2);
  ok(tpo_chamfer_bwd(to_dtype(xyz1), xyz1.data_ptr(), xyz2.data_ptr(), B, N, M,
                     idx1.data_ptr<int32_t>(), idx2.data_ptr<int32_t>(), g1.data_ptr(), g2.data_ptr(),
                     gx1.data_ptr(), gx2.data_ptr(), stream_of(xyz1)),
     "chamfer_backward");
  return {gx1, gx2};
}

// ---- fused ChamferDistance loss (reduction 0 = mean, 1 = sum) ----
// Returns (loss, state): `state` is the byte workspace the backward consumes.
std::tuple<at::Tensor, at::Tensor> chamfer_loss(const at::Tensor& xyz1_, const at::Tensor& xyz2_,
                                                int64_t reduction, int64_t flags) {
  check_cloud(xyz1_, "xyz1");
  check_cloud(xyz2_, "xyz2");
  TORCH_CHECK(xyz1_.size(2) == 3 && xyz2_.size(2) == 3, "chamfer: points must be 3-D");
  TORCH_CHECK(xyz1_.size(0) == xyz2_.size(0), "chamfer: batch sizes differ");
  TORCH_CHECK(xyz1_.scalar_type() == xyz2_.scalar_type(), "chamfer: dtypes differ");
  const c10::cuda::CUDAGuard g(xyz1_.device());
  const at::Tensor xyz1 = xyz1_.contiguous(), xyz2 = xyz2_.contiguous();
  const int64_t B = xyz1.size(0), N = xyz1.size(1), M = xyz2.size(1);
  const int dt = to_dtype(xyz1);
  auto loss = at::empty({}, xyz1.options());
  const size_t ws_bytes = tpo_chamfer_loss_workspace_size(dt, B, N, M);
  auto ws = at::empty({(int64_t)ws_bytes}, xyz1.options().dtype(at::kByte));
  ok(tpo_chamfer_loss_fwd(dt, (int)flags, xyz1.data_ptr(), xyz2.data_ptr(), B, N, M, (int)reduction,
                          loss.data_ptr(), ws.data_ptr(), ws_bytes, stream_of(xyz1)),
     "chamfer_loss");
  return {loss, ws};
}

std::tuple<at::Tensor, at::Tensor> chamfer_loss_backward(const at::Tensor& xyz1_,
                                                         const at::Tensor& xyz2_,
                                                         const at::Tensor& state,
                                                         const at::Tensor& grad_loss,
                                                         int64_t reduction, int64_t flags) {
  const c10::cuda::CUDAGuard g(xyz1_.device());
  const at::Tensor xyz1 = xyz1_.contiguous(), xyz2 = xyz2_.contiguous();
  const int64_t B = xyz1.size(0), N = xyz1.size(1), M = xyz2.size(1);
  const int dt = to_dtype(xyz1);
  TORCH_CHECK(state.numel() >= (int64_t)tpo_chamfer_loss_workspace_size(dt, B, N, M),
              "chamfer_loss_backward: state does not belong to these inputs");
  const at::Tensor gl = grad_loss.to(xyz1.scalar_type()).reshape({1}).contiguous();
  auto gx1 = at::empty_like(xyz1);
  auto gx2 = at::empty_like(xyz2);
  ok(tpo_chamfer_loss_bwd(dt, (int)flags, xyz1.data_ptr(), xyz2.data_ptr(), B, N, M, (int)reduction,
                          state.data_ptr(), gl.data_ptr(), gx1.data_ptr(), gx2.data_ptr(),
                          stream_of(xyz1)),
     "chamfer_loss_backward");
  return {gx1, gx2};
}

// First backward of a fused-loss forward: the gradients land in the zeroed region
// of the forward's workspace and are returned as views of it (no fill launch).
std::tuple<at::Tensor, at::Tensor> chamfer_loss_backward_in_state(const at::Tensor& xyz1_,
                                                                  const at::Tensor& xyz2_,
                                                                  const at::Tensor& state,
                                                                  const at::Tensor& grad_loss,
                                                                  int64_t reduction, int64_t flags) {
  const c10::cuda::CUDAGuard g(xyz1_.device());
  const at::Tensor xyz1 = xyz1_.contiguous(), xyz2 = xyz2_.contiguous();
  const int64_t B = xyz1.size(0), N = xyz1.size(1), M = xyz2.size(1);
  const int dt = to_dtype(xyz1);
  TORCH_CHECK(state.numel() >= (int64_t)tpo_chamfer_loss_workspace_size(dt, B, N, M),
              "chamfer_loss_backward: state does not belong to these inputs");
  const at::Tensor gl = grad_loss.to(xyz1.scalar_type()).reshape({1}).contiguous();
  ok(tpo_chamfer_loss_bwd_workspace(dt, (int)flags, xyz1.data_ptr(), xyz2.data_ptr(), B, N, M,
                                    (int)reduction, state.data_ptr(), gl.data_ptr(), stream_of(xyz1)),
     "chamfer_loss_backward");
  const int64_t es = xyz1.element_size();
  const int64_t o1 = (int64_t)tpo_chamfer_loss_grad_offset(dt, B, N, M, 1);
  const int64_t o2 = (int64_t)tpo_chamfer_loss_grad_offset(dt, B, N, M, 2);
  auto gx1 = state.narrow(0, o1, es * 3 * B * N).view(xyz1.scalar_type()).view({B, N, 3});
  auto gx2 = state.narrow(0, o2, es * 3 * B * M).view(xyz1.scalar_type()).view({B, M, 3});
  return {gx1, gx2};
}

// Autograd for the fused loss in C++ (no Python on the training-step path).
class ChamferLossFn : public torch::autograd::Function<ChamferLossFn> {
 public:
  static torch::autograd::variable_list forward(torch::autograd::AutogradContext* ctx,
                                                const at::Tensor& xyz1, const at::Tensor& xyz2,
                                                int64_t reduction, int64_t flags) {
    at::AutoDispatchBelowADInplaceOrView guard;
    auto out = chamfer_loss(xyz1, xyz2, reduction, flags);
    ctx->save_for_backward({xyz1, xyz2, std::get<1>(out)});
    ctx->saved_data["reduction"] = reduction;
    ctx->saved_data["flags"] = flags;
    ctx->saved_data["grads_in_state"] = true;  // the state's gradient region is still zero
    ctx->mark_non_differentiable({std::get<1>(out)});
    ctx->set_materialize_grads(false);  // no zero-filled grad for the state output
    return {std::get<0>(out), std::get<1>(out)};
  }
  static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                 torch::autograd::variable_list grads) {
    auto saved = ctx->get_saved_variables();
    if (!grads[0].defined()) return {at::Tensor(), at::Tensor(), at::Tensor(), at::Tensor()};
    const bool first = ctx->saved_data["grads_in_state"].toBool();
    ctx->saved_data["grads_in_state"] = false;
    auto g = first ? chamfer_loss_backward_in_state(saved[0], saved[1], saved[2], grads[0],
                                                    ctx->saved_data["reduction"].toInt(),
                                                    ctx->saved_data["flags"].toInt())
                   : chamfer_loss_backward(saved[0], saved[1], saved[2], grads[0],
                                           ctx->saved_data["reduction"].toInt(),
                                           ctx->saved_data["flags"].toInt());
    return {std::get<0>(g), std::get<1>(g), at::Tensor(), at::Tensor()};
  }
};

std::tuple<at::Tensor, at::Tensor> chamfer_loss_autograd(const at::Tensor& xyz1,
                                                         const at::Tensor& xyz2,
                                                         int64_t reduction, int64_t flags) {
  auto r = ChamferLossFn::apply(xyz1, xyz2, reduction, flags);
  return {r[0], r[1]};
}

// ---- row-sharded split (multi-GPU): keys live in int64 tensors ----
at::Tensor chamfer_keys_empty(const at::Tensor& like, int64_t n) {
  const int dt = to_dtype(like);
  const int64_t words = n * tpo_chamfer_key_bytes(dt) / 8;
  auto k = at::empty({words}, like.options().dtype(at::kLong));
  ok(tpo_chamfer_keys_init(dt, k.data_ptr(), n, stream_of(like)), "chamfer_keys_empty");
  return k;
}

void chamfer_fwd_keys(const at::Tensor& xyz1, const at::Tensor& xyz2, int64_t row_begin,
                      int64_t row_end, int64_t flags, at::Tensor keys1, at::Tensor keys2) {
  check_cloud(xyz1, "xyz1");
  check_cloud(xyz2, "xyz2");
  TORCH_CHECK(xyz1.is_contiguous() && xyz2.is_contiguous(), "chamfer_fwd_keys: contiguous inputs");
  const c10::cuda::CUDAGuard g(xyz1.device());
  const int dt = to_dtype(xyz1);
  const int64_t B = xyz1.size(0), N = xyz1.size(1), M = xyz2.size(1);
  const int kb = tpo_chamfer_key_bytes(dt);
  TORCH_CHECK(keys1.numel() * 8 >= B * N * kb && keys2.numel() * 8 >= B * M * kb, "keys too small");
  ok(tpo_chamfer_fwd_keys(dt, (int)flags, xyz1.data_ptr(), xyz2.data_ptr(), B, N, M, row_begin,
                          row_end, keys1.data_ptr(), keys2.data_ptr(), stream_of(xyz1)),
     "chamfer_fwd_keys");
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor> chamfer_finalize(
    const at::Tensor& xyz1, const at::Tensor& xyz2, int64_t row_begin, int64_t row_end,
    int64_t flags, const at::Tensor& keys1, const at::Tensor& keys2) {
  const c10::cuda::CUDAGuard g(xyz1.device());
  const int dt = to_dtype(xyz1);
  const int64_t B = xyz1.size(0), N = xyz1.size(1), M = xyz2.size(1);
  auto dist1 = at::zeros({B, N}, xyz1.options());
  auto dist2 = at::empty({B, M}, xyz1.options());
  auto idx1 = at::zeros({B, N}, xyz1.options().dtype(at::kInt));
  auto idx2 = at::empty({B, M}, xyz1.options().dtype(at::kInt));
  ok(tpo_chamfer_finalize(dt, (int)flags, xyz1.data_ptr(), xyz2.data_ptr(), B, N, M, row_begin,
                          row_end, keys1.data_ptr(), keys2.data_ptr(), dist1.data_ptr(),
                          idx1.data_ptr<int32_t>(), dist2.data_ptr(), idx2.data_ptr<int32_t>(),
                          stream_of(xyz1)),
     "chamfer_finalize");
  return {dist1, dist2, idx1, idx2};
}

void chamfer_bwd_partial(const at::Tensor& xyz1, const at::Tensor& xyz2, int64_t r0, int64_t r1,
                         int64_t c0, int64_t c1, const at::Tensor& idx1, const at::Tensor& idx2,
                         const at::Tensor& g1, const at::Tensor& g2, at::Tensor gx1, at::Tensor gx2) {
  const c10::cuda::CUDAGuard g(xyz1.device());
  const int64_t B = xyz1.size(0), N = xyz1.size(1), M = xyz2.size(1);
  TORCH_CHECK(gx1.is_contiguous() && gx2.is_contiguous() && g1.is_contiguous() && g2.is_contiguous() &&
                  idx1.is_contiguous() && idx2.is_contiguous(),
              "chamfer_bwd_partial: contiguous tensors required");
  ok(tpo_chamfer_bwd_partial(to_dtype(xyz1), xyz1.data_ptr(), xyz2.data_ptr(), B, N, M, r0, r1, c0,
                             c1, idx1.data_ptr<int32_t>(), idx2.data_ptr<int32_t>(), g1.data_ptr(),
                             g2.data_ptr(), gx1.data_ptr(), gx2.data_ptr(), stream_of(xyz1)),
     "chamfer_bwd_partial");
}

// ------------------------------------ knn ------------------------------------
at::Tensor lengths_or_full(const c10::optional<at::Tensor>& l, int64_t N, int64_t P,
                           const at::Tensor& like) {
  if (l.has_value() && l->defined()) {
    TORCH_CHECK(l->numel() == N, "knn: lengths must have shape (N,)");
    return l->to(like.device(), at::kLong).contiguous();
  }
  return at::full({N}, P, like.options().dtype(at::kLong));
}

std::tuple<at::Tensor, at::Tensor> knn_forward_ex(const at::Tensor& p1_, const at::Tensor& p2_,
                                                  const at::Tensor& lengths1,
                                                  const at::Tensor& lengths2, int64_t norm,
                                                  int64_t K, int64_t version, int64_t flags) {
  (void)version;  // one kernel family: accepted for schema compatibility, ignored
  check_cloud(p1_, "p1");
  check_cloud(p2_, "p2");
  TORCH_CHECK(p1_.size(0) == p2_.size(0), "p1 and p2 must have the same batch dimension.");
  TORCH_CHECK(p1_.size(2) == p2_.size(2), "Point sets must have the same last dimension");
  TORCH_CHECK(p1_.scalar_type() == p2_.scalar_type(), "knn: dtypes differ");
  TORCH_CHECK((norm == 1) || (norm == 2), "Norm must be 1 or 2.");
  const c10::cuda::CUDAGuard g(p1_.device());
  const at::Tensor p1 = p1_.contiguous(), p2 = p2_.contiguous();
  const int64_t N = p1.size(0), P1 = p1.size(1), P2 = p2.size(1), D = p1.size(2);
  const at::Tensor l1 = lengths1.to(p1.device(), at::kLong).contiguous();
  const at::Tensor l2 = lengths2.to(p1.device(), at::kLong).contiguous();
  TORCH_CHECK(l1.numel() == N && l2.numel() == N, "knn: lengths must have shape (N,)");
  auto idxs = at::empty({N, P1, K}, p1.options().dtype(at::kLong));
  auto dists = at::empty({N, P1, K}, p1.options());
  ok(tpo_knn_fwd(to_dtype(p1), (int)flags, p1.data_ptr(), p2.data_ptr(), l1.data_ptr<int64_t>(),
                 l2.data_ptr<int64_t>(), N, P1, P2, D, norm, K, dists.data_ptr(),
                 idxs.data_ptr<int64_t>(), stream_of(p1)),
     "knn_forward");
  return {idxs, dists};
}

std::tuple<at::Tensor, at::Tensor> knn_forward(const at::Tensor& p1, const at::Tensor& p2,
                                               const at::Tensor& l1, const at::Tensor& l2,
                                               int64_t norm, int64_t K, int64_t version) {
  return knn_forward_ex(p1, p2, l1, l2, norm, K, version, TPO_ROUND_FMA);
}

std::tuple<at::Tensor, at::Tensor> knn_backward(const at::Tensor& p1_, const at::Tensor& p2_,
                                                const at::Tensor& lengths1,
                                                const at::Tensor& lengths2,
                                                const at::Tensor& idxs_, int64_t norm,
                                                const at::Tensor& grad_dists_) {
  check_cloud(p1_, "p1");
  check_cloud(p2_, "p2");
  const c10::cuda::CUDAGuard g(p1_.device());
  const at::Tensor p1 = p1_.contiguous(), p2 = p2_.contiguous();
  const int64_t N = p1.size(0), P1 = p1.size(1), P2 = p2.size(1), D = p1.size(2);
  const at::Tensor idxs = idxs_.to(at::kLong).contiguous();
  TORCH_CHECK(idxs.dim() == 3 && idxs.size(0) == N && idxs.size(1) == P1,
              "KNN idxs must have shape (N, P1, K)");
  const int64_t K = idxs.size(2);
  const at::Tensor gd = grad_dists_.to(p1.scalar_type()).contiguous();
  TORCH_CHECK(gd.sizes() == idxs.sizes(), "grad_dists must have shape (N, P1, K)");
  const at::Tensor l1 = lengths1.to(p1.device(), at::kLong).contiguous();
  const at::Tensor l2 = lengths2.to(p1.device(), at::kLong).contiguous();
  auto g1 = at::empty_like(p1);
  auto g2 = at::empty_like(p2);
  ok(tpo_knn_bwd(to_dtype(p1), p1.data_ptr(), p2.data_ptr(), l1.data_ptr<int64_t>(),
                 l2.data_ptr<int64_t>(), idxs.data_ptr<int64_t>(), N, P1, P2, D, K, norm,
                 gd.data_ptr(), g1.data_ptr(), g2.data_ptr(), stream_of(p1)),
     "knn_backward");
  return {g1, g2};
}

at::Tensor knn_gather_forward(const at::Tensor& x_, const at::Tensor& idx_,
                              const c10::optional<at::Tensor>& lengths) {
  check_cloud(x_, "x");
  TORCH_CHECK(idx_.dim() == 3 && idx_.size(0) == x_.size(0), "x and idx must have same batch dimension.");
  const c10::cuda::CUDAGuard g(x_.device());
  const at::Tensor x = x_.contiguous(), idx = idx_.to(at::kLong).contiguous();
  const int64_t N = x.size(0), M = x.size(1), U = x.size(2), L = idx.size(1), K = idx.size(2);
  const at::Tensor len = lengths_or_full(lengths, N, M, x);
  auto out = at::empty({N, L, K, U}, x.options());
  ok(tpo_knn_gather_fwd(to_dtype(x), x.data_ptr(), idx.data_ptr<int64_t>(), len.data_ptr<int64_t>(),
                        N, M, U, L, K, out.data_ptr(), stream_of(x)),
     "knn_gather");
  return out;
}

at::Tensor knn_gather_backward(const at::Tensor& grad_out_, const at::Tensor& idx_,
                               const c10::optional<at::Tensor>& lengths, int64_t M) {
  const c10::cuda::CUDAGuard g(grad_out_.device());
  const at::Tensor go = grad_out_.contiguous(), idx = idx_.to(at::kLong).contiguous();
  TORCH_CHECK(go.dim() == 4, "knn_gather_backward: grad must be (N, L, K, U)");
  const int64_t N = go.size(0), L = go.size(1), K = go.size(2), U = go.size(3);
  const at::Tensor len = lengths_or_full(lengths, N, M, go);
  auto gx = at::empty({N, M, U}, go.options());
  ok(tpo_knn_gather_bwd(to_dtype(go), go.data_ptr(), idx.data_ptr<int64_t>(), len.data_ptr<int64_t>(),
                        N, M, U, L, K, gx.data_ptr(), stream_of(go)),
     "knn_gather_backward");
  return gx;
}

// fps_forward: points (N,P,3) -> idx (N,nsamples) int64.  Mirrors fps_cuda_forward
// (torch_point_ops/fps/csrc/cuda/fps.cu:273-316) and its checks.
at::Tensor fps_forward(const at::Tensor& points_, int64_t nsamples) {
  TORCH_CHECK(points_.is_cuda(), "fps: points must be a CUDA tensor");
  TORCH_CHECK(points_.dim() == 3, "fps: points must be (N, P, 3)");
  TORCH_CHECK(points_.size(2) == 3, "FPS only supports 3D points, but got dimension ", points_.size(2));
  TORCH_CHECK(nsamples > 0, "nsamples must be positive, but got ", nsamples);
  TORCH_CHECK(nsamples <= points_.size(1), "nsamples (", nsamples,
              ") cannot exceed number of points (", points_.size(1), ")");
  const c10::cuda::CUDAGuard g(points_.device());
  const at::Tensor pts = points_.contiguous();
  const int64_t N = pts.size(0), P = pts.size(1);
  auto idx = at::empty({N, nsamples}, pts.options().dtype(at::kLong));
  const int dt = to_dtype(pts);
  const size_t wsb = tpo_fps_workspace_size(dt, N, P);
  at::Tensor ws;
  if (wsb) ws = at::empty({(int64_t)wsb}, pts.options().dtype(at::kByte));
  ok(tpo_fps_fwd(dt, pts.data_ptr(), N, P, nsamples, idx.data_ptr<int64_t>(),
                 wsb ? ws.data_ptr() : nullptr, wsb, stream_of(pts)),
     "fps_forward");
  return idx;
}

// gather_points: points (N,C,P), idx (N,M) int64 -> (N,C,M).  Mirrors
// gather_points_cuda_forward / _backward (torch_point_ops/fps/csrc/cuda/fps.cu:318-401).
at::Tensor gather_points_forward(const at::Tensor& points_, const at::Tensor& idx_) {
  TORCH_CHECK(points_.is_cuda() && idx_.device() == points_.device(),
              "points and idx must be on the same CUDA device");
  TORCH_CHECK(points_.dim() == 3 && idx_.dim() == 2 && idx_.size(0) == points_.size(0),
              "gather_points: points must be (N, C, P) and idx (N, M)");
  const c10::cuda::CUDAGuard g(points_.device());
  const at::Tensor pts = points_.contiguous(), idx = idx_.to(at::kLong).contiguous();
  const int64_t N = pts.size(0), C = pts.size(1), P = pts.size(2), M = idx.size(1);
  auto out = at::empty({N, C, M}, pts.options());
  ok(tpo_gather_points_fwd(to_dtype(pts), pts.data_ptr(), idx.data_ptr<int64_t>(), N, C, P, M,
                           out.data_ptr(), stream_of(pts)),
     "gather_points_forward");
  return out;
}

at::Tensor gather_points_backward(const at::Tensor& grad_out_, const at::Tensor& idx_, int64_t n) {
  TORCH_CHECK(grad_out_.is_cuda() && idx_.device() == grad_out_.device(),
              "grad_out and idx must be on the same CUDA device");
  TORCH_CHECK(grad_out_.dim() == 3 && idx_.dim() == 2 && idx_.size(0) == grad_out_.size(0) &&
                  idx_.size(1) == grad_out_.size(2) && n >= 0,
              "gather_points_backward: grad_out must be (N, C, M), idx (N, M), n >= 0");
  const c10::cuda::CUDAGuard g(grad_out_.device());
  const at::Tensor go = grad_out_.contiguous(), idx = idx_.to(at::kLong).contiguous();
  const int64_t N = go.size(0), C = go.size(1), M = go.size(2);
  auto gp = at::empty({N, C, n}, go.options());
  ok(tpo_gather_points_bwd(to_dtype(go), go.data_ptr(), idx.data_ptr<int64_t>(), N, C, n, M,
                           gp.data_ptr(), stream_of(go)),
     "gather_points_backward");
  return gp;
}

}  // namespace

TORCH_LIBRARY(torch_point_ops_b200_fps, m) {
  m.def("fps_forward(Tensor points, int nsamples) -> Tensor");
  m.def("gather_points_forward(Tensor points, Tensor idx) -> Tensor");
  m.def("gather_points_backward(Tensor grad_out, Tensor idx, int n) -> Tensor");
}

TORCH_LIBRARY_IMPL(torch_point_ops_b200_fps, CUDA, m) {
  m.impl("fps_forward", &fps_forward);
  m.impl("gather_points_forward", &gather_points_forward);
  m.impl("gather_points_backward", &gather_points_backward);
}

TORCH_LIBRARY(torch_point_ops_b200_chamfer, m) {
  m.def("chamfer_forward(Tensor xyz1, Tensor xyz2) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("chamfer_backward(Tensor xyz1, Tensor xyz2, Tensor idx1, Tensor idx2, "
        "Tensor grad_dist1, Tensor grad_dist2) -> (Tensor, Tensor)");
  m.def("chamfer_forward_ex(Tensor xyz1, Tensor xyz2, int flags) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("chamfer_loss(Tensor xyz1, Tensor xyz2, int reduction, int flags) -> (Tensor, Tensor)");
  m.def("chamfer_loss_backward(Tensor xyz1, Tensor xyz2, Tensor state, Tensor grad_loss, "
        "int reduction, int flags) -> (Tensor, Tensor)");
  m.def("chamfer_keys_empty(Tensor like, int n) -> Tensor");
  m.def("chamfer_fwd_keys(Tensor xyz1, Tensor xyz2, int row_begin, int row_end, int flags, "
        "Tensor(a!) keys1, Tensor(b!) keys2) -> ()");
  m.def("chamfer_finalize(Tensor xyz1, Tensor xyz2, int row_begin, int row_end, int flags, "
        "Tensor keys1, Tensor keys2) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("chamfer_bwd_partial(Tensor xyz1, Tensor xyz2, int row_begin, int row_end, int col_begin, "
        "int col_end, Tensor idx1, Tensor idx2, Tensor grad_dist1, Tensor grad_dist2, "
        "Tensor(a!) grad_xyz1, Tensor(b!) grad_xyz2) -> ()");
}

TORCH_LIBRARY_IMPL(torch_point_ops_b200_chamfer, CUDA, m) {
  m.impl("chamfer_forward", &chamfer_forward);
  m.impl("chamfer_backward", &chamfer_backward);
  m.impl("chamfer_forward_ex", &chamfer_forward_ex);
  m.impl("chamfer_loss", &chamfer_loss);
  m.impl("chamfer_loss_backward", &chamfer_loss_backward);
  m.impl("chamfer_keys_empty", &chamfer_keys_empty);
  m.impl("chamfer_fwd_keys", &chamfer_fwd_keys);
  m.impl("chamfer_finalize", &chamfer_finalize);
  m.impl("chamfer_bwd_partial", &chamfer_bwd_partial);
}

TORCH_LIBRARY_IMPL(torch_point_ops_b200_chamfer, Autograd, m) {
  m.impl("chamfer_loss", &chamfer_loss_autograd);
}

TORCH_LIBRARY(torch_point_ops_b200_knn, m) {
  m.def("knn_forward(Tensor p1, Tensor p2, Tensor lengths1, Tensor lengths2, "
        "int norm, int K, int version) -> (Tensor, Tensor)");
  m.def("knn_backward(Tensor p1, Tensor p2, Tensor lengths1, Tensor lengths2, "
        "Tensor idxs, int norm, Tensor grad_dists) -> (Tensor, Tensor)");
  m.def("knn_forward_ex(Tensor p1, Tensor p2, Tensor lengths1, Tensor lengths2, "
        "int norm, int K, int version, int flags) -> (Tensor, Tensor)");
  m.def("knn_gather_forward(Tensor x, Tensor idx, Tensor? lengths) -> Tensor");
  m.def("knn_gather_backward(Tensor grad_out, Tensor idx, Tensor? lengths, int M) -> Tensor");
}

TORCH_LIBRARY_IMPL(torch_point_ops_b200_knn, CUDA, m) {
  m.impl("knn_forward", &knn_forward);
  m.impl("knn_backward", &knn_backward);
  m.impl("knn_forward_ex", &knn_forward_ex);
  m.impl("knn_gather_forward", &knn_gather_forward);
  m.impl("knn_gather_backward", &knn_gather_backward);
}
