"""Furthest point sampling and gather_points on the B200 against the CPU oracle
(a restatement of the reference CUDA kernels, torch_point_ops/fps/csrc/cuda/
fps.cu), through the C ABI and the torch API.  FPS indices are bit-exact; the
cases cover every group shape the planner picks (one CTA, a thread-block
cluster, a cooperative grid), ties, degenerate points and ragged sizes."""
import numpy as np
import pytest
import torch

import capi_util as C
import oracle
import torch_point_ops_b200 as tpo

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _cloud(B, P, dtype, seed, kind="normal"):
    g = torch.Generator().manual_seed(seed)
    if kind == "normal":
        x = torch.randn(B, P, 3, generator=g)
    elif kind == "lattice":  # integer grid: many exactly equal distances
        x = torch.randint(-4, 5, (B, P, 3), generator=g).float()
    elif kind == "degenerate":  # a third of the points inside |p|^2 <= 1e-3
        x = torch.randn(B, P, 3, generator=g)
        x[:, ::3] *= 1e-3
    elif kind == "duplicates":
        x = torch.randn(B, P, 3, generator=g)
        x[:, P // 2:] = x[:, : P - P // 2]
    return x.to(dtype)


CASES = [
    (3, 100, 20, "normal"),
    (2, 1000, 64, "normal"),
    (4, 37, 37, "normal"),       # nsamples == P
    (1, 1, 1, "normal"),
    (2, 513, 100, "lattice"),    # bs = 512, P not a multiple of it
    (2, 300, 300, "lattice"),    # bs = 256; runs out of distinct points
    (2, 2000, 200, "degenerate"),
    (2, 700, 400, "duplicates"),
    (2, 16384, 300, "normal"),   # cluster of CTAs
    (1, 20000, 200, "lattice"),
    (8, 4096, 128, "normal"),
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.float64])
@pytest.mark.parametrize("B,P,S,kind", CASES)
def test_fps_matches_oracle(B, P, S, kind, dtype):
    x = _cloud(B, P, dtype, seed=P + S, kind=kind)
    idx = C.fps_fwd(x.to(DEV), S)
    torch.cuda.synchronize()
    ref = oracle.fps(x.numpy(), S)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_fps_all_degenerate(dtype):
    x = torch.zeros(2, 50, 3, dtype=dtype)
    idx = tpo.furthest_point_sampling(x.to(DEV), 10)
    assert torch.equal(idx.cpu(), torch.zeros(2, 10, dtype=torch.int64))
    np.testing.assert_array_equal(idx.cpu().numpy(), oracle.fps(x.numpy(), 10))


@pytest.mark.parametrize("P,S", [(200_000, 48), (600_000, 24)])
def test_fps_large_cloud_grid(P, S):
    """Clouds beyond one cluster's registers run as a cooperative grid."""
    x = _cloud(1, P, torch.float32, seed=7, kind="normal")
    idx = C.fps_fwd(x.to(DEV), S)
    np.testing.assert_array_equal(idx.cpu().numpy(), oracle.fps(x.numpy(), S))
    flags = ctypes_flags()
    assert flags == 0


def ctypes_flags():
    import ctypes

    f = ctypes.c_uint(0)
    C.check(C.lib().tpo_device_error_flags(ctypes.byref(f), 1))
    return f.value


def test_fps_torch_api_and_errors():
    x = _cloud(2, 500, torch.float32, seed=3).to(DEV)
    idx = tpo.furthest_point_sampling(x, 32)
    assert idx.dtype == torch.int64 and idx.shape == (2, 32)
    assert torch.all(idx[:, 0] == 0)
    for n in range(2):
        assert len(torch.unique(idx[n])) == 32
    with pytest.raises(ValueError):
        tpo.furthest_point_sampling(x[0], 5)
    with pytest.raises(ValueError):
        tpo.furthest_point_sampling(x[..., :2], 5)
    with pytest.raises(ValueError):
        tpo.furthest_point_sampling(x, 0)
    with pytest.raises(ValueError):
        tpo.furthest_point_sampling(x, 501)
    # C ABI rejects the same
    import ctypes

    out = torch.empty(2, 600, dtype=torch.int64, device=DEV)
    rc = C.lib().tpo_fps_fwd(0, C.p(x), C.I64(2), C.I64(500), C.I64(600), C.p(out), C.VP(0),
                             ctypes.c_size_t(0), C.stream())
    assert rc == 1


def test_fps_modules():
    x = _cloud(2, 400, torch.float32, seed=4).to(DEV)
    m = tpo.FarthestPointSampling(16, return_gathered=True)
    idx, pts = m(x)
    assert torch.equal(pts, torch.stack([x[n, idx[n]] for n in range(2)]))
    idx2, pts2 = tpo.farthest_point_sample_and_gather(x, 16)
    assert torch.equal(idx, idx2) and torch.equal(pts, pts2)
    assert torch.equal(tpo.FPSFunction()(x, 16), idx)
    with pytest.raises(ValueError):
        tpo.FarthestPointSampling(0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.float64])
def test_gather_points_fwd_bwd(dtype):
    g = torch.Generator().manual_seed(11)
    B, Cc, P, S = 3, 6, 500, 77
    pts = torch.randn(B, Cc, P, generator=g).to(dtype)
    idx = torch.stack([torch.randperm(P, generator=g)[:S] for _ in range(B)])
    idx[:, 5] = idx[:, 9]  # repeated index: the backward must accumulate
    out = C.gather_points_fwd(pts.to(DEV), idx.to(DEV))
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.gather_points(pts.numpy(), idx.numpy()))
    go = torch.randn(B, Cc, S, generator=g).to(dtype)
    gp = C.gather_points_bwd(go.to(DEV), idx.to(DEV), P)
    ref = oracle.gather_points_bwd(go.numpy(), idx.numpy(), P)
    # at most two terms meet in one slot here: the sum is order-independent
    np.testing.assert_array_equal(gp.cpu().numpy(), ref)


def test_gather_points_autograd_and_errors():
    g = torch.Generator().manual_seed(12)
    pts = torch.randn(2, 4, 100, generator=g, dtype=torch.float64).to(DEV).requires_grad_()
    idx = torch.randint(0, 100, (2, 30), generator=g).to(DEV)
    out = tpo.gather_points(pts, idx)
    ref = torch.gather(pts, 2, idx[:, None, :].expand(-1, 4, -1))
    assert torch.equal(out, ref)
    w = torch.randn_like(out)
    (gp,) = torch.autograd.grad((out * w).sum(), pts)
    (gr,) = torch.autograd.grad((ref * w).sum(), pts)
    torch.testing.assert_close(gp, gr, rtol=0, atol=1e-12)
    assert torch.autograd.gradcheck(lambda p: tpo.gather_points(p, idx), (pts,))
    gath = tpo.PointGatherer()(pts, idx)
    assert torch.equal(gath, out)
    with pytest.raises(ValueError):
        tpo.gather_points(pts[0], idx)
    with pytest.raises(ValueError):
        tpo.gather_points(pts, idx[..., None])
    with pytest.raises(ValueError):
        tpo.gather_points(pts, idx[:1])
    # empty gathers
    e = tpo.gather_points(pts, idx[:, :0])
    assert e.shape == (2, 4, 0)


def test_fps_opcheck_and_compile():
    """torch.library.opcheck on the fps / gather_points operators and torch.compile
    of the public functions (the reference's tests/test_fps.py test_opcheck /
    test_compile)."""
    pts = torch.randn(1, 10, 3, device=DEV)
    feats = torch.randn(1, 4, 10, device=DEV)
    idx = torch.tensor([[0, 2, 4, 6]], device=DEV)
    torch.library.opcheck(torch.ops.torch_point_ops_b200_fps.fps_forward.default, (pts, 4),
                          raise_exception=True)
    torch.library.opcheck(torch.ops.torch_point_ops_b200_fps.gather_points_forward.default,
                          (feats, idx), raise_exception=True)
    gout = torch.randn(1, 4, 4, device=DEV)
    torch.library.opcheck(torch.ops.torch_point_ops_b200_fps.gather_points_backward.default,
                          (gout, idx, 10), raise_exception=True)
    p20 = torch.randn(1, 20, 3, device=DEV)
    eager = tpo.furthest_point_sampling(p20, 8)
    compiled = torch.compile(tpo.furthest_point_sampling)(p20, 8)
    assert torch.equal(eager, compiled)
    f20 = torch.randn(1, 6, 20, device=DEV)
    assert torch.equal(torch.compile(tpo.gather_points)(f20, eager), tpo.gather_points(f20, eager))


def test_fps_known_grid_and_degenerate():
    """A 5x5 grid in the z=0 plane (the reference's test_known_configurations): the
    centre point sits at the origin, so it is degenerate and never chosen; and
    points placed at 1e-4 (test_degenerate_points) are never chosen either."""
    x = torch.linspace(-1, 1, 5)
    xx, yy = torch.meshgrid(x, x, indexing="ij")
    grid = torch.stack([xx.flatten(), yy.flatten(), torch.zeros(25)], dim=-1)[None]
    idx = tpo.furthest_point_sampling(grid.to(DEV), 5).cpu()
    np.testing.assert_array_equal(idx.numpy(), oracle.fps(grid.numpy(), 5))
    assert idx[0, 0] == 0 and len(torch.unique(idx[0])) == 5 and 12 not in idx[0].tolist()
    g = torch.Generator().manual_seed(5)
    p = torch.randn(1, 10, 3, generator=g)
    p[0, 5:8] = 1e-4
    idx = tpo.furthest_point_sampling(p.to(DEV), 5).cpu()
    np.testing.assert_array_equal(idx.numpy(), oracle.fps(p.numpy(), 5))
    assert not set(idx[0].tolist()) & {5, 6, 7}


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.float64])
def test_fps_gather_multi_precision(dtype):
    """fps + gather_points keep the input dtype; gradients flow in every dtype
    (the reference's test_multi_precision)."""
    g = torch.Generator().manual_seed(6)
    pts = torch.randn(1, 50, 3, generator=g).to(dtype).to(DEV)
    feats = torch.randn(1, 4, 50, generator=g).to(dtype).to(DEV).requires_grad_()
    idx = tpo.furthest_point_sampling(pts, 8)
    np.testing.assert_array_equal(idx.cpu().numpy(), oracle.fps(pts.cpu().numpy(), 8))
    out = tpo.gather_points(feats, idx)
    assert out.dtype == dtype and out.shape == (1, 4, 8)
    out.sum().backward()
    assert feats.grad.dtype == dtype and float(feats.grad.float().sum()) == 4 * 8


def test_quick_fps_names_are_not_exported():
    """The approximate kd-tree sampler is out of scope: its names are absent
    rather than silently returning a different (exact) sampling."""
    assert not hasattr(tpo, "quick_furthest_point_sampling")
    assert not hasattr(tpo, "QuickFarthestPointSampling")
    from torch_point_ops_b200.fps import fps_function
    x = _cloud(2, 300, torch.float32, seed=9).to(DEV)
    assert torch.equal(fps_function(x, 16), tpo.furthest_point_sampling(x, 16))
