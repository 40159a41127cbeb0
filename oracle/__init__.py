"""CPU oracle for the chamfer / knn path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this package, and only as the checker (or the timed CPU baseline).
The product package never imports it and has no CPU fallback.

The arithmetic lives in ``tpo_oracle.c`` (each function there cites the
reference file:line it restates); this module is a numpy/ctypes front end.
Rounding ``mode``: 0 = uncontracted (reference CPU path), 1 = nvcc-style FMA
contraction ``fma(dz,dz,fma(dy,dy,dx*dx))`` (reference CUDA build).

``ref_cpu()`` / ``ref_cuda()`` load the *unmodified reference sources* compiled by
``oracle/Makefile.ref`` into ``oracle/_ref`` (when present) so tests can pin this
restatement against the reference itself.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libtpo_oracle.so")
REF_DIR = os.path.join(HERE, "_ref")

_lib = None


def build(force: bool = False) -> str:
    """Compile the C oracle (gcc, seconds)."""
    if force or not os.path.exists(LIB_PATH) or (
        os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "tpo_oracle.c"))
    ):
        subprocess.check_call(["make", "-s", "-f", os.path.join(HERE, "Makefile")])
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(LIB_PATH)
    return _lib


_SUFFIX = {np.dtype(np.float32): "f32", np.dtype(np.float64): "f64", np.dtype(np.float16): "f16"}


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype=None):
    return np.ascontiguousarray(a if dtype is None else a.astype(dtype, copy=False))


def nn(a, b, mode: int = 0):
    """One chamfer direction: for each point of a (B,N,3), min/argmin over b (B,M,3)."""
    a = _c(a)
    b = _c(b, a.dtype)
    B, N, _ = a.shape
    M = b.shape[1]
    dist = np.zeros((B, N), a.dtype)
    idx = np.zeros((B, N), np.int32)
    fn = getattr(lib(), "oracle_nn_" + _SUFFIX[a.dtype])
    I = ctypes.c_int64
    fn(ctypes.c_int(mode), I(B), I(N), I(M), _p(a), _p(b), _p(dist), _p(idx))
    return dist, idx


def chamfer_fwd(x1, x2, mode: int = 0):
    d1, i1 = nn(x1, x2, mode)
    d2, i2 = nn(x2, x1, mode)
    return d1, d2, i1, i2


def chamfer_bwd(x1, x2, i1, i2, g1, g2):
    x1 = _c(x1)
    dt = x1.dtype
    x2, g1, g2 = _c(x2, dt), _c(g1, dt), _c(g2, dt)
    i1, i2 = _c(i1, np.int32), _c(i2, np.int32)
    B, N, _ = x1.shape
    M = x2.shape[1]
    gx1 = np.zeros_like(x1)
    gx2 = np.zeros_like(x2)
    fn = getattr(lib(), "oracle_chamfer_bwd_" + _SUFFIX[dt])
    I = ctypes.c_int64
    fn(I(B), I(N), I(M), _p(x1), _p(x2), _p(i1), _p(i2), _p(g1), _p(g2), _p(gx1), _p(gx2))
    return gx1, gx2


def knn_fwd(p1, p2, lengths1=None, lengths2=None, norm: int = 2, K: int = 1, mode: int = 0):
    """Reference CPU knn_forward semantics: (idxs int64 (-1 pad), dists (0 pad)), sorted."""
    p1 = _c(p1)
    dt = p1.dtype
    p2 = _c(p2, dt)
    Nb, P1, D = p1.shape
    P2 = p2.shape[1]
    l1 = _c(np.full(Nb, P1) if lengths1 is None else lengths1, np.int64)
    l2 = _c(np.full(Nb, P2) if lengths2 is None else lengths2, np.int64)
    dists = np.zeros((Nb, P1, K), dt)
    idxs = np.full((Nb, P1, K), -1, np.int64)
    fn = getattr(lib(), "oracle_knn_" + _SUFFIX[dt])
    I = ctypes.c_int64
    fn(ctypes.c_int(mode), I(Nb), I(P1), I(P2), I(D), _p(p1), _p(p2), _p(l1), _p(l2),
       I(norm), I(K), _p(dists), _p(idxs))
    return idxs, dists


def knn_bwd(p1, p2, lengths1, lengths2, idxs, norm, grad_dists, l1_zero_at_tie: bool = True):
    p1 = _c(p1)
    dt = p1.dtype
    p2, gd = _c(p2, dt), _c(grad_dists, dt)
    Nb, P1, D = p1.shape
    P2 = p2.shape[1]
    K = idxs.shape[2]
    l1 = _c(np.full(Nb, P1) if lengths1 is None else lengths1, np.int64)
    l2 = _c(np.full(Nb, P2) if lengths2 is None else lengths2, np.int64)
    idxs = _c(idxs, np.int64)
    g1 = np.zeros_like(p1)
    g2 = np.zeros_like(p2)
    fn = getattr(lib(), "oracle_knn_bwd_" + _SUFFIX[dt])
    I = ctypes.c_int64
    fn(I(Nb), I(P1), I(P2), I(D), _p(p1), _p(p2), _p(l1), _p(l2), _p(idxs), I(norm), I(K),
       _p(gd), ctypes.c_int(1 if l1_zero_at_tie else 0), _p(g1), _p(g2))
    return g1, g2


def knn_gather(x, idx, lengths=None):
    """x_out[n,l,k] = x[n, idx[n,l,k]]; zero where k >= lengths[n] or idx == -1
    (knn/__init__.py:136-183; -1 rows are zero instead of raising)."""
    x = np.asarray(x)
    Nb, M, U = x.shape
    _, L, K = idx.shape
    lengths = np.full(Nb, M) if lengths is None else np.asarray(lengths)
    out = np.zeros((Nb, L, K, U), x.dtype)
    for n in range(Nb):
        ii = idx[n]
        valid = (ii >= 0) & (np.arange(K)[None, :] < lengths[n])
        safe = np.where(valid, ii, 0)
        out[n] = np.where(valid[..., None], x[n][safe], 0)
    return out


def fps(points, nsamples: int):
    """Reference CUDA furthest_point_sampling semantics: (B,P,3) -> (B,nsamples) int64."""
    points = _c(points)
    B, P, _ = points.shape
    idx = np.zeros((B, nsamples), np.int64)
    fn = getattr(lib(), "oracle_fps_" + _SUFFIX[points.dtype])
    I = ctypes.c_int64
    fn(I(B), I(P), I(nsamples), _p(points), _p(idx))
    return idx


def gather_points(points, idx):
    """out[b,c,j] = points[b,c,idx[b,j]]: (B,C,P), (B,S) -> (B,C,S)."""
    points = _c(points)
    idx = _c(idx, np.int64)
    B, C, P = points.shape
    S = idx.shape[1]
    out = np.zeros((B, C, S), points.dtype)
    fn = getattr(lib(), "oracle_gather_points_" + _SUFFIX[points.dtype])
    I = ctypes.c_int64
    fn(I(B), I(C), I(P), I(S), _p(points), _p(idx), _p(out))
    return out


def gather_points_bwd(grad_out, idx, P: int):
    """Scatter-add of grad_out (B,C,S) into (B,C,P), in (b, c, j) order."""
    go = _c(grad_out)
    idx = _c(idx, np.int64)
    B, C, S = go.shape
    gp = np.zeros((B, C, P), go.dtype)
    fn = getattr(lib(), "oracle_gather_points_bwd_" + _SUFFIX[go.dtype])
    I = ctypes.c_int64
    fn(I(B), I(C), I(P), I(S), _p(go), _p(idx), _p(gp))
    return gp


# ---------------- the unmodified reference, built by oracle/Makefile.ref ----------------
_ref_loaded = {}


def _load_ref(name):
    import torch

    path = os.path.join(REF_DIR, name)
    if name in _ref_loaded:
        return _ref_loaded[name]
    if not os.path.exists(path):
        _ref_loaded[name] = None
        return None
    torch.ops.load_library(path)
    _ref_loaded[name] = path
    return path


def ref_knn():
    """Load the reference knn op library (CUDA build if present, else CPU build).
    Returns torch.ops.torch_point_ops_knn or None."""
    import torch

    if _load_ref("knn_cuda_ref.so") is None and _load_ref("knn_cpu_ref.so") is None:
        return None
    return torch.ops.torch_point_ops_knn


def ref_chamfer():
    """Reference chamfer op library (CUDA only; its CPU impl raises)."""
    import torch

    if _load_ref("chamfer_cuda_ref.so") is None:
        return None
    return torch.ops.torch_point_ops_chamfer


def ref_fps():
    """Reference fps op library (CPU and CUDA kernels of torch_point_ops.fps).
    Returns torch.ops.torch_point_ops_fps or None."""
    import torch

    if _load_ref("fps_cuda_ref.so") is None:
        return None
    return torch.ops.torch_point_ops_fps
