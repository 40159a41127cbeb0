"""K nearest neighbours -- drop-in for torch_point_ops.knn
(torch_point_ops/knn/__init__.py:1-187)."""
import torch

from .. import _lib

_ops = _lib.knn_ops


def _knn_backward(ctx, grad_idxs, grad_dists):
    p1, p2, lengths1, lengths2, idxs = ctx.saved_tensors
    if grad_dists is None:
        return None, None, None, None, None, None, None
    grad_p1, grad_p2 = _ops.knn_backward(p1, p2, lengths1, lengths2, idxs, ctx.norm, grad_dists)
    return grad_p1, grad_p2, None, None, None, None, None


def _knn_setup_context(ctx, inputs, output):
    p1, p2, lengths1, lengths2, norm = inputs[:5]
    idxs, _ = output
    ctx.save_for_backward(p1, p2, lengths1, lengths2, idxs)
    ctx.norm = norm
    ctx.set_materialize_grads(False)


def _knn_backward_ex(ctx, gi, gd):
    return _knn_backward(ctx, gi, gd) + (None,)


torch.library.register_autograd(
    "torch_point_ops_b200_knn::knn_forward", _knn_backward, setup_context=_knn_setup_context)
torch.library.register_autograd(
    "torch_point_ops_b200_knn::knn_forward_ex", _knn_backward_ex, setup_context=_knn_setup_context)


def _fake_knn(p1, p2, lengths1, lengths2, norm, K, version, flags=0):
    b, n, _ = p1.shape
    return p1.new_empty(b, n, K, dtype=torch.int64), p1.new_empty(b, n, K)


torch.library.register_fake("torch_point_ops_b200_knn::knn_forward")(
    lambda p1, p2, l1, l2, norm, K, version: _fake_knn(p1, p2, l1, l2, norm, K, version))
torch.library.register_fake("torch_point_ops_b200_knn::knn_forward_ex")(_fake_knn)


@torch.library.register_fake("torch_point_ops_b200_knn::knn_backward")
def _(p1, p2, lengths1, lengths2, idxs, norm, grad_dists):
    return torch.empty_like(p1), torch.empty_like(p2)


@torch.library.register_fake("torch_point_ops_b200_knn::knn_gather_forward")
def _(x, idx, lengths):
    return x.new_empty(x.shape[0], idx.shape[1], idx.shape[2], x.shape[2])


@torch.library.register_fake("torch_point_ops_b200_knn::knn_gather_backward")
def _(grad_out, idx, lengths, M):
    return grad_out.new_empty(grad_out.shape[0], M, grad_out.shape[3])


def _gather_setup(ctx, inputs, output):
    x, idx, lengths = inputs
    ctx.save_for_backward(idx, lengths if lengths is not None else torch.empty(0))
    ctx.has_len = lengths is not None
    ctx.M = x.shape[1]


def _gather_backward(ctx, grad_out):
    idx, lengths = ctx.saved_tensors
    gx = _ops.knn_gather_backward(grad_out, idx, lengths if ctx.has_len else None, ctx.M)
    return gx, None, None


torch.library.register_autograd(
    "torch_point_ops_b200_knn::knn_gather_forward", _gather_backward, setup_context=_gather_setup)


def knn_points(
    p1: torch.Tensor,
    p2: torch.Tensor,
    lengths1: torch.Tensor = None,
    lengths2: torch.Tensor = None,
    norm: int = 2,
    K: int = 1,
    version: int = -1,
    return_sorted: bool = True,
) -> tuple[torch.Tensor, torch.Tensor]:
    """K-nearest neighbours of each p1 point among the p2 points.

    Args:
        p1: (N, P1, D) queries; p2: (N, P2, D) targets (CUDA, same dtype)
        lengths1, lengths2: (N,) int64 valid sizes per cloud (None = full)
        norm: 2 (squared L2) or 1 (L1); K: neighbours; version: accepted, ignored
        return_sorted: results are always ascending by (dist, idx)
    Returns:
        idxs (N, P1, K) int64 and dists (N, P1, K); padding idx -1 / dist 0 for
        rows p >= lengths1[n] and slots k >= lengths2[n].
    """
    if p1.shape[0] != p2.shape[0]:
        raise ValueError("p1 and p2 must have the same batch dimension.")
    if p1.shape[2] != p2.shape[2]:
        raise ValueError("p1 and p2 must have the same point dimension.")
    N, P1, D = p1.shape
    P2 = p2.shape[1]
    if lengths1 is None:
        lengths1 = torch.full((N,), P1, dtype=torch.int64, device=p1.device)
    if lengths2 is None:
        lengths2 = torch.full((N,), P2, dtype=torch.int64, device=p1.device)
    flags = _lib.rounding_flags()
    if flags == _lib.ROUND_FMA:
        return _ops.knn_forward(p1.contiguous(), p2.contiguous(), lengths1, lengths2, norm, K, version)
    return _ops.knn_forward_ex(p1.contiguous(), p2.contiguous(), lengths1, lengths2, norm, K,
                               version, flags)


def knn_gather(x: torch.Tensor, idx: torch.Tensor, lengths: torch.Tensor = None) -> torch.Tensor:
    """x_out[n, l, k] = x[n, idx[n, l, k]]; zero where k >= lengths[n] or idx == -1.

    Args:
        x: (N, M, U) features; idx: (N, L, K) from knn_points; lengths: (N,) or None
    Returns:
        (N, L, K, U)
    """
    if x.shape[0] != idx.shape[0]:
        raise ValueError("x and idx must have same batch dimension.")
    return _ops.knn_gather_forward(x, idx, lengths)


from .knn import KNearestNeighbors, KNNFunction, knn_function  # noqa: E402

__all__ = ["knn_points", "knn_gather", "KNearestNeighbors", "KNNFunction", "knn_function"]
