"""Furthest point sampling and gather_points -- drop-in for torch_point_ops.fps
(torch_point_ops/fps/__init__.py, fps/fps.py): same functions, modules, errors
and autograd.  The reference's approximate kd-tree sampler (quick_* names,
fps/csrc/cuda/quick_fps.cu) is not part of this package."""
import torch

from .. import _lib

_ops = _lib.fps_ops


def _gather_points_backward(ctx, grad_output):
    (idx,) = ctx.saved_tensors
    return _ops.gather_points_backward(grad_output, idx, ctx.n_points), None


def _gather_points_setup_context(ctx, inputs, output):
    points, idx = inputs
    ctx.save_for_backward(idx)
    ctx.n_points = points.shape[2]


torch.library.register_autograd(
    "torch_point_ops_b200_fps::gather_points_forward", _gather_points_backward,
    setup_context=_gather_points_setup_context)


@torch.library.register_fake("torch_point_ops_b200_fps::fps_forward")
def _(points, nsamples):
    return points.new_empty(points.shape[0], nsamples, dtype=torch.int64)


@torch.library.register_fake("torch_point_ops_b200_fps::gather_points_forward")
def _(points, idx):
    return points.new_empty(points.shape[0], points.shape[1], idx.shape[1])


@torch.library.register_fake("torch_point_ops_b200_fps::gather_points_backward")
def _(grad_output, idx, n_points):
    return grad_output.new_empty(grad_output.shape[0], grad_output.shape[1], n_points)


def furthest_point_sampling(points: torch.Tensor, nsamples: int) -> torch.Tensor:
    """Indices (N, nsamples) int64 of the furthest point sampling of (N, P, 3) points.

    The first index is 0; each next one is the point whose distance to the
    chosen set is largest, with the reference CUDA kernel's ties and its rule
    that points with |p|^2 <= 1e-3 are never chosen."""
    if points.dim() != 3 or points.shape[2] != 3:
        raise ValueError(f"Expected points to have shape (N, P, 3), but got {points.shape}")
    if nsamples <= 0:
        raise ValueError(f"nsamples must be positive, but got {nsamples}")
    if nsamples > points.shape[1]:
        raise ValueError(f"nsamples ({nsamples}) cannot exceed number of points ({points.shape[1]})")
    return _ops.fps_forward(points.contiguous(), nsamples)


def gather_points(points: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """out[n, c, m] = points[n, c, idx[n, m]]: (N, C, P), (N, M) -> (N, C, M).
    Differentiable in points (the backward scatter-adds)."""
    if points.dim() != 3:
        raise ValueError(f"Expected points to have 3 dimensions (N, C, P), but got {points.dim()}")
    if idx.dim() != 2:
        raise ValueError(f"Expected idx to have 2 dimensions (N, M), but got {idx.dim()}")
    if points.shape[0] != idx.shape[0]:
        raise ValueError(f"Batch dimensions must match: points {points.shape[0]} vs idx {idx.shape[0]}")
    return _ops.gather_points_forward(points.contiguous(), idx.contiguous())


def farthest_point_sample_and_gather(points: torch.Tensor, nsamples: int):
    """(indices (N, nsamples), sampled points (N, nsamples, 3))."""
    indices = furthest_point_sampling(points, nsamples)
    sampled = gather_points(points.transpose(1, 2), indices).transpose(1, 2)
    return indices, sampled


from .fps import FarthestPointSampling, FPSFunction, PointGatherer, fps_function  # noqa: E402

__all__ = [
    "furthest_point_sampling", "gather_points", "farthest_point_sample_and_gather",
    "FarthestPointSampling", "PointGatherer", "FPSFunction", "fps_function",
]
