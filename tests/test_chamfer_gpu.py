"""Chamfer parity on the B200: the CUDA path (through the C ABI and through the
torch API) against the CPU oracle on the same seeded inputs.
Indices bit-exact; distances bit-exact (same rounding as the selected mode);
gradients within 1e-6 (fp32) / 1e-12 (fp64) / 1e-3 (fp16) of the summed term
magnitude (the reference itself scatters with atomics, so summation order is free)."""
import numpy as np
import pytest
import torch

import capi_util as C
import datagen
import oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"
from tolerances import tolerance


def _bits(t):
    a = t.detach().cpu().contiguous().numpy()
    return a.view(np.uint8)


def _check_fwd(x1, x2, flags=0):
    mode = 1 if flags == 0 else 0
    d1, d2, i1, i2 = C.chamfer_fwd(x1.to(DEV), x2.to(DEV), flags)
    torch.cuda.synchronize()
    od1, od2, oi1, oi2 = oracle.chamfer_fwd(x1.numpy(), x2.numpy(), mode)
    assert np.array_equal(i1.cpu().numpy(), oi1), "idx1 mismatch"
    assert np.array_equal(i2.cpu().numpy(), oi2), "idx2 mismatch"
    assert np.array_equal(_bits(d1), od1.view(np.uint8)), "dist1 bits"
    assert np.array_equal(_bits(d2), od2.view(np.uint8)), "dist2 bits"
    return d1, d2, i1, i2


def _term_scale(x1, x2, i1, i2, g1, g2):
    """Per-element sum of |terms| entering each gradient element (float64)."""
    a, b = x1.double().numpy(), x2.double().numpy()
    i1, i2 = i1.cpu().numpy().astype(np.int64), i2.cpu().numpy().astype(np.int64)
    s1, s2 = np.zeros_like(a), np.zeros_like(b)
    n1, n2 = np.ones_like(a), np.ones_like(b)
    for bi in range(a.shape[0]):
        t = np.abs(2 * g1[bi].double().numpy()[:, None] * (a[bi] - b[bi][i1[bi]]))
        s1[bi] += t
        np.add.at(s2[bi], i1[bi], t)
        np.add.at(n2[bi], i1[bi], 1.0)
        t = np.abs(2 * g2[bi].double().numpy()[:, None] * (b[bi] - a[bi][i2[bi]]))
        s2[bi] += t
        np.add.at(s1[bi], i2[bi], t)
        np.add.at(n1[bi], i2[bi], 1.0)
    return s1, s2, n1, n2


def _check_bwd(x1, x2, i1, i2, seed=0):
    B, N, _ = x1.shape
    M = x2.shape[1]
    g = torch.Generator().manual_seed(seed)
    g1 = torch.randn(B, N, generator=g).to(x1.dtype)
    g2 = torch.randn(B, M, generator=g).to(x1.dtype)
    gx1, gx2 = C.chamfer_bwd(x1.to(DEV), x2.to(DEV), i1, i2, g1.to(DEV), g2.to(DEV))
    torch.cuda.synchronize()
    o1, o2 = oracle.chamfer_bwd(x1.numpy(), x2.numpy(), i1.cpu().numpy(), i2.cpu().numpy(),
                                g1.numpy(), g2.numpy())
    s1, s2, n1, n2 = _term_scale(x1, x2, i1, i2, g1, g2)
    e1 = np.abs(gx1.cpu().double().numpy() - o1.astype(np.float64))
    e2 = np.abs(gx2.cpu().double().numpy() - o2.astype(np.float64))
    t1, t2 = tolerance(x1.dtype, s1, n1), tolerance(x1.dtype, s2, n2)
    assert np.all(e1 <= t1), float(np.max(e1 - t1))
    assert np.all(e2 <= t2), float(np.max(e2 - t2))


SIZES = [(1, 1, 1), (1, 3, 4), (2, 5, 7), (1, 8, 6), (2, 64, 128), (2, 511, 513), (3, 1000, 1500),
         (1, 2048, 64), (1, 64, 2048), (4, 1024, 1024), (1, 2049, 777)]


@pytest.mark.parametrize("B,N,M", SIZES)
@pytest.mark.parametrize("flags", [0, 1])
def test_fwd_bwd_f32_uniform(B, N, M, flags):
    x1 = datagen.uniform(B, N, seed=N * 31 + M)
    x2 = datagen.uniform(B, M, seed=N * 17 + M + 1)
    d1, d2, i1, i2 = _check_fwd(x1, x2, flags)
    _check_bwd(x1, x2, i1, i2)


@pytest.mark.parametrize("dtype", [torch.float64, torch.float16])
@pytest.mark.parametrize("B,N,M", [(1, 3, 4), (2, 300, 517), (3, 1000, 1500), (1, 2049, 777)])
def test_fwd_bwd_f64_f16(dtype, B, N, M):
    x1 = datagen.sphere_noise(B, N, seed=N, dtype=dtype)
    x2 = datagen.sphere_noise(B, M, seed=M + 7, dtype=dtype)
    d1, d2, i1, i2 = _check_fwd(x1, x2, 0)
    _check_bwd(x1, x2, i1, i2)
    if dtype == torch.float64:
        _check_fwd(x1, x2, 1)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16])
def test_ties_lowest_index(dtype):
    # integer grid points: many exactly equal distances; duplicates in both clouds
    g = torch.Generator().manual_seed(11)
    x1 = torch.randint(0, 5, (2, 700, 3), generator=g).to(dtype)
    x2 = torch.randint(0, 5, (2, 900, 3), generator=g).to(dtype)
    _check_fwd(x1, x2, 0)
    _check_fwd(x1, x2, 1)


def test_known_values():
    a = torch.zeros(1, 1, 3, device=DEV)
    b = torch.tensor([[[1.0, 2.0, 3.0]]], device=DEV)
    d1, d2, i1, i2 = C.chamfer_fwd(a, b)
    assert d1.item() == 14 and d2.item() == 14
    x = torch.rand(2, 100, 3, device=DEV)
    d1, d2, i1, i2 = C.chamfer_fwd(x, x)
    assert torch.all(d1 == 0) and torch.all(d2 == 0)


@pytest.mark.parametrize("N,M", [(0, 5), (5, 0), (0, 0)])
def test_empty_clouds(N, M):
    x1 = torch.rand(2, N, 3, device=DEV)
    x2 = torch.rand(2, M, 3, device=DEV)
    d1, d2, i1, i2 = C.chamfer_fwd(x1, x2)
    assert d1.shape == (2, N) and d2.shape == (2, M)
    assert torch.all(d1 == 0) and torch.all(i1 == 0) and torch.all(d2 == 0)


def test_torch_api_autograd_matches_capi():
    import torch_point_ops_b200 as tpo

    x1 = datagen.uniform(3, 700, seed=1).to(DEV).requires_grad_()
    x2 = datagen.uniform(3, 500, seed=2).to(DEV).requires_grad_()
    loss = tpo.ChamferDistance("mean")(x1, x2)
    loss.backward()
    d1, d2, i1, i2 = C.chamfer_fwd(x1.detach(), x2.detach())
    ref = d1.mean() + d2.mean()
    assert torch.allclose(loss.detach(), ref, rtol=1e-6)
    g1 = torch.full_like(d1, 1.0 / d1.numel())
    g2 = torch.full_like(d2, 1.0 / d2.numel())
    # autograd's gradients against the oracle's scatter at the contract's bound
    a, b = x1.detach().cpu(), x2.detach().cpu()
    o1, o2 = oracle.chamfer_bwd(a.numpy(), b.numpy(), i1.cpu().numpy(), i2.cpu().numpy(),
                                g1.cpu().numpy(), g2.cpu().numpy())
    s1, s2, n1, n2 = _term_scale(a, b, i1, i2, g1.cpu(), g2.cpu())
    assert np.all(np.abs(x1.grad.cpu().double().numpy() - o1) <= tolerance(torch.float32, s1, n1))
    assert np.all(np.abs(x2.grad.cpu().double().numpy() - o2) <= tolerance(torch.float32, s2, n2))
    for red in ("sum", None, "none"):
        out = tpo.ChamferDistance(red)(x1, x2)
    assert isinstance(out, tuple) and out[0].shape == (3, 700)
    with pytest.raises(ValueError):
        tpo.ChamferDistance("max")


def test_gradcheck_f64():
    import torch_point_ops_b200 as tpo

    g = torch.Generator().manual_seed(5)
    x1 = torch.rand(1, 8, 3, generator=g, dtype=torch.float64).to(DEV).requires_grad_()
    x2 = torch.rand(1, 6, 3, generator=g, dtype=torch.float64).to(DEV).requires_grad_()
    assert torch.autograd.gradcheck(lambda a, b: tpo.chamfer_distance(a, b), (x1, x2),
                                    nondet_tol=1e-12)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16])
@pytest.mark.parametrize("reduction", [0, 1])
@pytest.mark.parametrize("shape", [(3, 1111, 777), (1, 1, 1), (2, 3000, 5)])
def test_fused_loss_capi(dtype, reduction, shape):
    """tpo_chamfer_loss_fwd/bwd == chamfer_fwd + torch reduction + chamfer_bwd
    (the fused backward re-derives the same neighbours from the forward's state)."""
    B, N, M = shape
    x1 = datagen.sphere_noise(B, N, seed=8, dtype=dtype).to(DEV)
    x2 = datagen.sphere_noise(B, M, seed=9, dtype=dtype).to(DEV)
    loss, state = C.chamfer_loss_fwd(x1, x2, reduction)
    d1, d2, i1, i2 = C.chamfer_fwd(x1, x2)
    # the loss against the float64 reduction of the ORACLE's distances, at the
    # contract's tolerance (1e-6 fp32, 1e-3 fp16, 1e-12 fp64)
    od1, od2, _, _ = oracle.chamfer_fwd(x1.cpu().numpy(), x2.cpu().numpy(), 1)
    od1, od2 = od1.astype(np.float64), od2.astype(np.float64)
    ref = (od1.mean() + od2.mean()) if reduction == 0 else (od1.sum() + od2.sum())
    rtol = {torch.float32: 1e-6, torch.float64: 1e-12, torch.float16: 1e-3}[dtype]
    assert abs(float(loss) - ref) <= rtol * abs(ref), (float(loss), ref)
    gl = torch.tensor([0.75], dtype=dtype, device=DEV)
    gx1, gx2 = C.chamfer_loss_bwd(x1, x2, state, gl, reduction)
    if reduction == 0:
        g1 = (gl / d1.numel()).expand(d1.shape).contiguous()
        g2 = (gl / d2.numel()).expand(d2.shape).contiguous()
    else:
        g1 = gl.expand(d1.shape).contiguous()
        g2 = gl.expand(d2.shape).contiguous()
    rx1, rx2 = C.chamfer_bwd(x1, x2, i1, i2, g1, g2)
    s1, s2, n1, n2 = _term_scale(x1.cpu(), x2.cpu(), i1, i2, g1.cpu(), g2.cpu())
    e1 = np.abs(gx1.cpu().double().numpy() - rx1.cpu().double().numpy())
    e2 = np.abs(gx2.cpu().double().numpy() - rx2.cpu().double().numpy())
    # both sides scatter with atomics: twice the single-sum bound
    assert np.all(e1 <= 2 * tolerance(dtype, s1, n1))
    assert np.all(e2 <= 2 * tolerance(dtype, s2, n2))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16])
@pytest.mark.parametrize("shape", [(3, 1111, 777), (1, 1, 1), (2, 0, 5)])
def test_fused_loss_backward_in_workspace(dtype, shape):
    """The fill-free backward (gradients in the forward's zeroed workspace region)
    equals the backward into caller buffers."""
    B, N, M = shape
    x1 = datagen.sphere_noise(B, N, seed=18, dtype=dtype).to(DEV)
    x2 = datagen.sphere_noise(B, M, seed=19, dtype=dtype).to(DEV)
    loss, state = C.chamfer_loss_fwd(x1, x2, 0)
    gl = torch.tensor([1.25], dtype=dtype, device=DEV)
    r1, r2 = C.chamfer_loss_bwd(x1, x2, state, gl, 0)
    w1, w2 = C.chamfer_loss_bwd_in_state(x1, x2, state, gl, 0)
    tol = {torch.float32: 1e-6, torch.float64: 1e-12, torch.float16: 2e-3}[dtype]
    torch.testing.assert_close(w1, r1, rtol=tol, atol=tol)
    torch.testing.assert_close(w2, r2, rtol=tol, atol=tol)


def test_chamfer_distance_module_double_backward_call():
    """A second backward of the same forward (retain_graph) must not accumulate
    onto the first one's in-workspace gradients."""
    import torch_point_ops_b200 as tpo

    x1 = datagen.sphere_noise(2, 500, seed=21).to(DEV).requires_grad_()
    x2 = datagen.sphere_noise(2, 400, seed=22).to(DEV).requires_grad_()
    loss = tpo.ChamferDistance("mean")(x1, x2)
    a1, a2 = torch.autograd.grad(loss, [x1, x2], retain_graph=True)
    a1, a2 = a1.clone(), a2.clone()
    b1, b2 = torch.autograd.grad(loss, [x1, x2])
    torch.testing.assert_close(a1, b1, rtol=1e-6, atol=1e-9)
    torch.testing.assert_close(a2, b2, rtol=1e-6, atol=1e-9)
    # and a plain .backward() accumulates into .grad as usual
    loss2 = tpo.ChamferDistance("mean")(x1, x2)
    loss2.backward()
    torch.testing.assert_close(x1.grad, a1, rtol=1e-6, atol=1e-9)


def test_fused_loss_two_calls_deterministic():
    x1 = datagen.gmm(4, 3000, seed=3).to(DEV)
    x2 = datagen.gmm(4, 2000, seed=4).to(DEV)
    a = C.chamfer_loss_fwd(x1, x2)[0]
    b = C.chamfer_loss_fwd(x1, x2)[0]
    c = C.chamfer_loss_fwd(x1, x2, flags=1)[0]
    assert torch.allclose(a, c, rtol=1e-6)
    assert torch.equal(a, b)


def test_fused_loss_empty_is_nan_like_torch():
    x1 = torch.rand(2, 0, 3, device=DEV)
    x2 = torch.rand(2, 5, 3, device=DEV)
    loss, _ = C.chamfer_loss_fwd(x1, x2)
    ref = torch.zeros(2, 0, device=DEV).mean() + torch.zeros(2, 5, device=DEV).mean()
    assert torch.isnan(loss) and torch.isnan(ref)
