"""Chamfer distance -- drop-in for torch_point_ops.chamfer
(torch_point_ops/chamfer/__init__.py:1-75)."""
import torch

from .. import _lib

_ops = _lib.chamfer_ops


def _chamfer_backward(ctx, grad_dist1, grad_dist2, grad_idx1, grad_idx2):
    xyz1, xyz2, idx1, idx2 = ctx.saved_tensors
    if grad_dist1 is None and grad_dist2 is None:
        return None, None
    if grad_dist1 is None:
        grad_dist1 = torch.zeros(idx1.shape, dtype=xyz1.dtype, device=xyz1.device)
    if grad_dist2 is None:
        grad_dist2 = torch.zeros(idx2.shape, dtype=xyz1.dtype, device=xyz1.device)
    grad_xyz1, grad_xyz2 = _ops.chamfer_backward(xyz1, xyz2, idx1, idx2, grad_dist1, grad_dist2)
    return grad_xyz1, grad_xyz2


def _setup(ctx, inputs, output):
    xyz1, xyz2 = inputs[0], inputs[1]
    _, _, idx1, idx2 = output
    ctx.save_for_backward(xyz1, xyz2, idx1, idx2)
    ctx.set_materialize_grads(False)


def _backward_ex(ctx, g1, g2, gi1, gi2):
    gx1, gx2 = _chamfer_backward(ctx, g1, g2, gi1, gi2)
    return gx1, gx2, None


torch.library.register_autograd(
    "torch_point_ops_b200_chamfer::chamfer_forward", _chamfer_backward, setup_context=_setup)
torch.library.register_autograd(
    "torch_point_ops_b200_chamfer::chamfer_forward_ex", _backward_ex, setup_context=_setup)


def _fake_fwd(xyz1, xyz2, flags=0):
    b, n, _ = xyz1.shape
    m = xyz2.shape[1]
    return (xyz1.new_empty(b, n), xyz1.new_empty(b, m),
            xyz1.new_empty(b, n, dtype=torch.int32), xyz1.new_empty(b, m, dtype=torch.int32))


torch.library.register_fake("torch_point_ops_b200_chamfer::chamfer_forward")(
    lambda xyz1, xyz2: _fake_fwd(xyz1, xyz2))
torch.library.register_fake("torch_point_ops_b200_chamfer::chamfer_forward_ex")(_fake_fwd)


@torch.library.register_fake("torch_point_ops_b200_chamfer::chamfer_backward")
def _(xyz1, xyz2, idx1, idx2, grad_dist1, grad_dist2):
    return torch.empty_like(xyz1), torch.empty_like(xyz2)


# chamfer_loss has its autograd formula registered in C++ (csrc/torch_ops.cpp).


@torch.library.register_fake("torch_point_ops_b200_chamfer::chamfer_loss")
def _(xyz1, xyz2, reduction, flags):
    ctx = torch.library.get_ctx()
    n = ctx.new_dynamic_size()
    return xyz1.new_empty(()), xyz1.new_empty(n, dtype=torch.uint8)


@torch.library.register_fake("torch_point_ops_b200_chamfer::chamfer_loss_backward")
def _(xyz1, xyz2, state, grad_loss, reduction, flags):
    return torch.empty_like(xyz1), torch.empty_like(xyz2)


def chamfer_loss(xyz1: torch.Tensor, xyz2: torch.Tensor, reduction: str = "mean") -> torch.Tensor:
    """Fused ChamferDistance loss: mean(dist1) + mean(dist2) ("mean") or
    sum(dist1) + sum(dist2) ("sum"), computed inside the forward kernels (no
    per-point distance tensors, no separate reduction launches); autograd-aware."""
    red = {"mean": 0, "sum": 1}[reduction]
    loss, _ = _ops.chamfer_loss(xyz1, xyz2, red, _lib.rounding_flags())
    return loss


def chamfer_distance(xyz1: torch.Tensor, xyz2: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Chamfer distance between two point clouds.

    Args:
        xyz1: (B, N, 3) point cloud 1 (CUDA; float32, float16 or float64)
        xyz2: (B, M, 3) point cloud 2
    Returns:
        dist1 (B, N): squared distance from each xyz1 point to its nearest xyz2 point
        dist2 (B, M): squared distance from each xyz2 point to its nearest xyz1 point
    Both directions come from one fused kernel that evaluates each pair once.
    """
    xyz1 = xyz1.contiguous()
    xyz2 = xyz2.contiguous()
    flags = _lib.rounding_flags()
    if flags == _lib.ROUND_FMA:
        dist1, dist2, _, _ = _ops.chamfer_forward(xyz1, xyz2)
    else:
        dist1, dist2, _, _ = _ops.chamfer_forward_ex(xyz1, xyz2, flags)
    return dist1, dist2


def chamfer_distance_with_idx(xyz1, xyz2):
    """As chamfer_distance but also returns the int32 argmin indices (idx1, idx2)."""
    return _ops.chamfer_forward_ex(xyz1.contiguous(), xyz2.contiguous(), _lib.rounding_flags())


from .chamfer import ChamferDistance  # noqa: E402

__all__ = ["chamfer_distance", "chamfer_distance_with_idx", "chamfer_loss", "ChamferDistance"]
