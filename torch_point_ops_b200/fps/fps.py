"""Module wrappers of furthest point sampling / gather_points
(torch_point_ops/fps/fps.py: FarthestPointSampling, PointGatherer, FPSFunction,
QuickFarthestPointSampling, QuickFPSFunction)."""
import torch

from . import furthest_point_sampling, gather_points, quick_furthest_point_sampling


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


def _quick(points, nsamples, kd_depth, return_gathered):
    indices = quick_furthest_point_sampling(points, nsamples, kd_depth)
    if not return_gathered:
        return indices
    sampled = gather_points(points.transpose(1, 2), indices).transpose(1, 2)
    return indices, sampled


class QuickFarthestPointSampling(torch.nn.Module):
    """The reference's quick-FPS module (same arguments and checks); samples with
    the exact FPS."""

    def __init__(self, nsamples, kd_depth=4, return_gathered=False):
        super().__init__()
        if nsamples <= 0:
            raise ValueError(f"nsamples must be positive, but got {nsamples}")
        if kd_depth <= 0 or kd_depth > 10:
            raise ValueError(f"kd_depth must be between 1 and 10, but got {kd_depth}")
        self.nsamples = nsamples
        self.kd_depth = kd_depth
        self.return_gathered = return_gathered

    def forward(self, points):
        return _quick(points, self.nsamples, self.kd_depth, self.return_gathered)


class QuickFPSFunction(torch.nn.Module):
    """Functional quick FPS: forward(points, nsamples, kd_depth=4, return_gathered=False)."""

    def forward(self, points, nsamples, kd_depth=4, return_gathered=False):
        return _quick(points, nsamples, kd_depth, return_gathered)


fps_function = FPSFunction()
quick_fps_function = QuickFPSFunction()
