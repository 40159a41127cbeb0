"""torch_point_ops_b200 -- B200-native (sm_100a) chamfer / knn nearest-neighbour path
and the furthest-point-sampling / gather_points ops beside it.

Drop-in for the corresponding part of torch_point_ops (same function and module
names): ``import torch_point_ops_b200 as torch_point_ops``.
"""
from . import _lib
from ._lib import get_rounding, set_rounding
from .chamfer import ChamferDistance, chamfer_distance, chamfer_distance_with_idx, chamfer_loss
from .knn import KNearestNeighbors, KNNFunction, knn_function, knn_gather, knn_points
from .fps import (FarthestPointSampling, FPSFunction, PointGatherer, farthest_point_sample_and_gather,
                  furthest_point_sampling, gather_points)

__version__ = "0.1.0"
__all__ = [
    "chamfer_distance", "chamfer_distance_with_idx", "chamfer_loss", "ChamferDistance",
    "knn_points", "knn_gather", "KNearestNeighbors", "KNNFunction", "knn_function",
    "furthest_point_sampling", "gather_points", "farthest_point_sample_and_gather",
    "FarthestPointSampling", "PointGatherer", "FPSFunction",
    "set_rounding", "get_rounding",
]
