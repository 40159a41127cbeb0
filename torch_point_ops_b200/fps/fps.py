"""Module wrappers of furthest point sampling / gather_points
(torch_point_ops/fps/fps.py: FarthestPointSampling, PointGatherer, FPSFunction)."""
import torch

from . import furthest_point_sampling, gather_points


def _sample(points, nsamples, return_gathered):
    indices = furthest_point_sampling(points, nsamples)
    if not return_gathered:
        return indices
    sampled = gather_points(points.transpose(1, 2), indices).transpose(1, 2)
    return indices, sampled


class FarthestPointSampling(torch.nn.Module):
    """FPS of (N, P, 3) clouds to `nsamples` points; returns indices, or
    (indices, sampled points (N, nsamples, 3)) when return_gathered."""

    def __init__(self, nsamples, return_gathered=False):
        super().__init__()
        if nsamples <= 0:
            raise ValueError(f"nsamples must be positive, but got {nsamples}")
        self.nsamples = nsamples
        self.return_gathered = return_gathered

    def forward(self, points):
        return _sample(points, self.nsamples, self.return_gathered)


class PointGatherer(torch.nn.Module):
    """gather_points as a module: (N, C, P), (N, M) -> (N, C, M)."""

    def forward(self, points, indices):
        return gather_points(points, indices)


class FPSFunction(torch.nn.Module):
    """Functional FPS: forward(points, nsamples, return_gathered=False)."""

    def forward(self, points, nsamples, return_gathered=False):
        return _sample(points, nsamples, return_gathered)


fps_function = FPSFunction()
