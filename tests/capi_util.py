"""ctypes helpers that drive include/tpo_b200.h directly with torch-owned device
buffers (torch is used only to allocate device memory and get the stream)."""
import ctypes
import os
import re

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tpo_b200.h")
LIB = os.path.join(ROOT, "torch_point_ops_b200", "lib", "libtpo_b200.so")

DT = {torch.float32: 0, torch.float16: 1, torch.float64: 2}
I64 = ctypes.c_int64
VP = ctypes.c_void_p


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"TPO_API\s+[\w\s\*]+?\b(tpo_\w+)\s*\(", src)))


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(LIB)
        _lib.tpo_status_string.restype = ctypes.c_char_p
        _lib.tpo_chamfer_fwd_workspace_size.restype = ctypes.c_size_t
        _lib.tpo_chamfer_fwd_workspace_size.argtypes = [ctypes.c_int, I64, I64, I64]
    return _lib


def p(t):
    return VP(t.data_ptr()) if t is not None else VP(0)


def stream():
    return VP(torch.cuda.current_stream().cuda_stream)


def check(rc):
    if rc != 0:
        raise RuntimeError(lib().tpo_status_string(rc).decode())


def chamfer_fwd(x1, x2, flags=0):
    B, N, _ = x1.shape
    M = x2.shape[1]
    dt = DT[x1.dtype]
    d1 = torch.empty(B, N, dtype=x1.dtype, device=x1.device)
    d2 = torch.empty(B, M, dtype=x1.dtype, device=x1.device)
    i1 = torch.empty(B, N, dtype=torch.int32, device=x1.device)
    i2 = torch.empty(B, M, dtype=torch.int32, device=x1.device)
    ws_n = lib().tpo_chamfer_fwd_workspace_size(dt, B, N, M)
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=x1.device)
    check(lib().tpo_chamfer_fwd(dt, flags, p(x1), p(x2), I64(B), I64(N), I64(M), p(d1), p(d2),
                                p(i1), p(i2), p(ws), ctypes.c_size_t(ws_n), stream()))
    return d1, d2, i1, i2


def chamfer_bwd(x1, x2, i1, i2, g1, g2):
    B, N, _ = x1.shape
    M = x2.shape[1]
    gx1 = torch.empty_like(x1)
    gx2 = torch.empty_like(x2)
    check(lib().tpo_chamfer_bwd(DT[x1.dtype], p(x1), p(x2), I64(B), I64(N), I64(M), p(i1), p(i2),
                                p(g1), p(g2), p(gx1), p(gx2), stream()))
    return gx1, gx2


def knn_fwd(p1, p2, l1, l2, norm, K, flags=0):
    N, P1, D = p1.shape
    P2 = p2.shape[1]
    d = torch.empty(N, P1, K, dtype=p1.dtype, device=p1.device)
    i = torch.empty(N, P1, K, dtype=torch.int64, device=p1.device)
    check(lib().tpo_knn_fwd(DT[p1.dtype], flags, p(p1), p(p2), p(l1), p(l2), I64(N), I64(P1),
                            I64(P2), I64(D), I64(norm), I64(K), p(d), p(i), stream()))
    return i, d


def knn_bwd(p1, p2, l1, l2, idx, norm, gd):
    N, P1, D = p1.shape
    P2 = p2.shape[1]
    K = idx.shape[2]
    g1 = torch.empty_like(p1)
    g2 = torch.empty_like(p2)
    check(lib().tpo_knn_bwd(DT[p1.dtype], p(p1), p(p2), p(l1), p(l2), p(idx), I64(N), I64(P1),
                            I64(P2), I64(D), I64(K), I64(norm), p(gd), p(g1), p(g2), stream()))
    return g1, g2


def gather_fwd(x, idx, lengths):
    N, M, U = x.shape
    L, K = idx.shape[1], idx.shape[2]
    out = torch.empty(N, L, K, U, dtype=x.dtype, device=x.device)
    check(lib().tpo_knn_gather_fwd(DT[x.dtype], p(x), p(idx), p(lengths), I64(N), I64(M), I64(U),
                                   I64(L), I64(K), p(out), stream()))
    return out


def gather_bwd(gout, idx, lengths, M):
    N, L, K, U = gout.shape
    gx = torch.empty(N, M, U, dtype=gout.dtype, device=gout.device)
    check(lib().tpo_knn_gather_bwd(DT[gout.dtype], p(gout), p(idx), p(lengths), I64(N), I64(M),
                                   I64(U), I64(L), I64(K), p(gx), stream()))
    return gx


def chamfer_loss_fwd(x1, x2, reduction=0, flags=0):
    """Returns (loss, state); state is the workspace the backward consumes."""
    B, N, _ = x1.shape
    M = x2.shape[1]
    dt = DT[x1.dtype]
    loss = torch.empty((), dtype=x1.dtype, device=x1.device)
    lib().tpo_chamfer_loss_workspace_size.restype = ctypes.c_size_t
    lib().tpo_chamfer_loss_workspace_size.argtypes = [ctypes.c_int, I64, I64, I64]
    n = lib().tpo_chamfer_loss_workspace_size(dt, B, N, M)
    ws = torch.empty(n, dtype=torch.uint8, device=x1.device)
    check(lib().tpo_chamfer_loss_fwd(dt, flags, p(x1), p(x2), I64(B), I64(N), I64(M),
                                     ctypes.c_int(reduction), p(loss), p(ws), ctypes.c_size_t(n),
                                     stream()))
    return loss, ws


def chamfer_loss_bwd(x1, x2, state, grad_loss, reduction=0, flags=0):
    B, N, _ = x1.shape
    M = x2.shape[1]
    gx1 = torch.empty_like(x1)
    gx2 = torch.empty_like(x2)
    check(lib().tpo_chamfer_loss_bwd(DT[x1.dtype], flags, p(x1), p(x2), I64(B), I64(N), I64(M),
                                     ctypes.c_int(reduction), p(state), p(grad_loss), p(gx1),
                                     p(gx2), stream()))
    return gx1, gx2


def fps_fwd(points, S):
    B, P, _ = points.shape
    dt = DT[points.dtype]
    idx = torch.empty(B, S, dtype=torch.int64, device=points.device)
    lib().tpo_fps_workspace_size.restype = ctypes.c_size_t
    ws_n = lib().tpo_fps_workspace_size(dt, I64(B), I64(P))
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=points.device)
    check(lib().tpo_fps_fwd(dt, p(points), I64(B), I64(P), I64(S), p(idx), p(ws),
                            ctypes.c_size_t(ws_n), stream()))
    return idx


def gather_points_fwd(points, idx):
    B, Cc, P = points.shape
    S = idx.shape[1]
    out = torch.empty(B, Cc, S, dtype=points.dtype, device=points.device)
    check(lib().tpo_gather_points_fwd(DT[points.dtype], p(points), p(idx), I64(B), I64(Cc), I64(P),
                                      I64(S), p(out), stream()))
    return out


def gather_points_bwd(gout, idx, P):
    B, Cc, S = gout.shape
    gp = torch.empty(B, Cc, P, dtype=gout.dtype, device=gout.device)
    check(lib().tpo_gather_points_bwd(DT[gout.dtype], p(gout), p(idx), I64(B), I64(Cc), I64(P),
                                      I64(S), p(gp), stream()))
    return gp


def chamfer_loss_bwd_in_state(x1, x2, state, grad_loss, reduction=0, flags=0):
    """tpo_chamfer_loss_bwd_workspace: gradients scattered into the forward's
    zeroed gradient region; returned as views of the workspace."""
    B, N, _ = x1.shape
    M = x2.shape[1]
    dt = DT[x1.dtype]
    check(lib().tpo_chamfer_loss_bwd_workspace(dt, flags, p(x1), p(x2), I64(B), I64(N), I64(M),
                                               ctypes.c_int(reduction), p(state), p(grad_loss),
                                               stream()))
    lib().tpo_chamfer_loss_grad_offset.restype = ctypes.c_size_t
    o1 = lib().tpo_chamfer_loss_grad_offset(dt, I64(B), I64(N), I64(M), 1)
    o2 = lib().tpo_chamfer_loss_grad_offset(dt, I64(B), I64(N), I64(M), 2)
    es = x1.element_size()
    g1 = state[o1:o1 + es * 3 * B * N].view(x1.dtype).view(B, N, 3)
    g2 = state[o2:o2 + es * 3 * B * M].view(x1.dtype).view(B, M, 3)
    return g1, g2
