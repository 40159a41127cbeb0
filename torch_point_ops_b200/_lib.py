"""Loads the in-tree native libraries.  There is no fallback: if the sm_100a
build is missing, importing the package raises."""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(_HERE, "lib")
CAPI_PATH = os.path.join(LIB_DIR, "libtpo_b200.so")
TORCH_BINDING_PATH = os.path.join(LIB_DIR, "libtpo_b200_torch.so")

if not (os.path.exists(CAPI_PATH) and os.path.exists(TORCH_BINDING_PATH)):
    raise ImportError(
        "torch_point_ops_b200: native libraries not built; run "
        "`python torch_point_ops_b200/build.py` (needs nvcc for sm_100a)")

torch.ops.load_library(TORCH_BINDING_PATH)
chamfer_ops = torch.ops.torch_point_ops_b200_chamfer
knn_ops = torch.ops.torch_point_ops_b200_knn
fps_ops = torch.ops.torch_point_ops_b200_fps

_capi = None


def capi() -> ctypes.CDLL:
    """ctypes handle on the C ABI library (include/tpo_b200.h)."""
    global _capi
    if _capi is None:
        _capi = ctypes.CDLL(CAPI_PATH)
        _capi.tpo_status_string.restype = ctypes.c_char_p
        _capi.tpo_chamfer_fwd_workspace_size.restype = ctypes.c_size_t
    return _capi


# Rounding of the distance arithmetic (see include/tpo_b200.h, tpo_flags):
#   "fma"   -- the reference CUDA kernels' rounding (default)
#   "exact" -- the reference CPU path's rounding (every product/sum rounded)
ROUND_FMA, ROUND_EXACT = 0, 1
_rounding = ROUND_FMA


def set_rounding(mode: str) -> None:
    global _rounding
    if mode not in ("fma", "exact"):
        raise ValueError("rounding must be 'fma' or 'exact'")
    _rounding = ROUND_FMA if mode == "fma" else ROUND_EXACT


def get_rounding() -> str:
    return "fma" if _rounding == ROUND_FMA else "exact"


def rounding_flags() -> int:
    return _rounding
