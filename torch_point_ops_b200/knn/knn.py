"""KNearestNeighbors / KNNFunction modules -- drop-in for torch_point_ops/knn/knn.py:5-135."""
import torch

from . import knn_gather, knn_points


class KNearestNeighbors(torch.nn.Module):
    """K nearest neighbours between two point clouds, optionally gathering the
    neighbour points (return_nn)."""

    def __init__(self, K=1, norm=2, return_nn=False, return_sorted=True, version=-1):
        super().__init__()
        if K < 1:
            raise ValueError(f"K must be >= 1, but got {K}")
        if norm not in [1, 2]:
            raise ValueError(f"norm must be 1 or 2, but got {norm}")
        self.K = K
        self.norm = norm
        self.return_nn = return_nn
        self.return_sorted = return_sorted
        self.version = version

    def forward(self, p1, p2, lengths1=None, lengths2=None):
        idxs, dists = knn_points(p1, p2, lengths1=lengths1, lengths2=lengths2, norm=self.norm,
                                 K=self.K, version=self.version, return_sorted=self.return_sorted)
        if self.return_nn:
            return idxs, dists, knn_gather(p2, idxs, lengths2)
        return idxs, dists


class KNNFunction(torch.nn.Module):
    """Functional KNN interface (PyTorch3D style)."""

    def forward(self, p1, p2, lengths1=None, lengths2=None, norm=2, K=1, version=-1,
                return_nn=False, return_sorted=True):
        idxs, dists = knn_points(p1, p2, lengths1=lengths1, lengths2=lengths2, norm=norm, K=K,
                                 version=version, return_sorted=return_sorted)
        if return_nn:
            return idxs, dists, knn_gather(p2, idxs, lengths2)
        return idxs, dists


knn_function = KNNFunction()
