"""Parity at the benchmark configurations' full sizes, forward AND backward.

* Configs 2 and 3 (every point): indices and distances bit-exact against the
  oracle; gradients of chamfer_backward and of the fused ChamferDistance loss
  within the per-dtype bound of tolerances.py; the loss value within 1e-6 (fp32)
  / 1e-3 (fp16) relative of the float64 sum of the ORACLE's distances.
* Config 5 (B=1, N=M=2^20, fp32 and fp64): a full GPU run; the oracle re-derives
  2048 sampled rows per direction (a CPU pass over all 2^40 pairs takes hours);
  the backward is checked on every point against the oracle's scatter through
  the GPU's indices (the indices themselves are pinned on the samples), and the
  loss against the float64 sum of the checked distances.

Tolerances from the north-star contract: 1e-6 relative (fp32), 1e-3 (fp16),
1e-12 (fp64)."""
import numpy as np
import pytest
import torch

import capi_util as C
import datagen
import oracle
from tolerances import term_scale as _term_scale, tolerance

pytestmark = pytest.mark.gpu
DEV = "cuda"
LOSS_RTOL = {torch.float32: 1e-6, torch.float16: 1e-3, torch.float64: 1e-12}


def _bits(t):
    return t.detach().cpu().contiguous().numpy().view(np.uint8)


def _assert_grads(x1, x2, i1, i2, g1, g2, gx1, gx2, factor=1.0):
    """gx1/gx2 (device) against the oracle's sequential scatter through i1/i2."""
    o1, o2 = oracle.chamfer_bwd(x1.numpy(), x2.numpy(), i1.cpu().numpy(), i2.cpu().numpy(),
                                g1.numpy(), g2.numpy())
    s1, s2, n1, n2 = _term_scale(x1, x2, i1, i2, g1, g2)
    e1 = np.abs(gx1.detach().cpu().double().numpy() - o1.astype(np.float64))
    e2 = np.abs(gx2.detach().cpu().double().numpy() - o2.astype(np.float64))
    t1 = factor * tolerance(x1.dtype, s1, n1)
    t2 = factor * tolerance(x1.dtype, s2, n2)
    assert np.all(e1 <= t1), float(np.max(e1 - t1))
    assert np.all(e2 <= t2), float(np.max(e2 - t2))


def _loss_and_grads(x1, x2):
    """The public API step the benchmark times: ChamferDistance('mean') + backward."""
    import torch_point_ops_b200 as tpo

    a = x1.to(DEV).requires_grad_()
    b = x2.to(DEV).requires_grad_()
    loss = tpo.ChamferDistance("mean")(a, b)
    ga, gb = torch.autograd.grad(loss, [a, b])
    return loss.detach(), ga, gb


def _mean_grads(x1, x2):
    B, N, M = x1.shape[0], x1.shape[1], x2.shape[1]
    return (torch.full((B, N), 1.0 / (B * N), dtype=torch.float64).to(x1.dtype),
            torch.full((B, M), 1.0 / (B * M), dtype=torch.float64).to(x1.dtype))


def _full_check(x1, x2):
    """Every point: fwd bit-exact, bwd and fused loss within tolerance."""
    dt = x1.dtype
    d1, d2, i1, i2 = C.chamfer_fwd(x1.to(DEV), x2.to(DEV), 0)
    torch.cuda.synchronize()
    od1, od2, oi1, oi2 = oracle.chamfer_fwd(x1.numpy(), x2.numpy(), 1)
    assert np.array_equal(i1.cpu().numpy(), oi1) and np.array_equal(i2.cpu().numpy(), oi2)
    assert np.array_equal(_bits(d1), od1.view(np.uint8))
    assert np.array_equal(_bits(d2), od2.view(np.uint8))
    g = torch.Generator().manual_seed(7)
    g1 = torch.randn(d1.shape, generator=g).to(dt)
    g2 = torch.randn(d2.shape, generator=g).to(dt)
    gx1, gx2 = C.chamfer_bwd(x1.to(DEV), x2.to(DEV), i1, i2, g1.to(DEV), g2.to(DEV))
    _assert_grads(x1, x2, i1, i2, g1, g2, gx1, gx2)
    # the fused loss (the benchmark's step) against the oracle's distances
    loss, ga, gb = _loss_and_grads(x1, x2)
    want = od1.astype(np.float64).mean() + od2.astype(np.float64).mean()
    assert abs(float(loss) - want) <= LOSS_RTOL[dt] * abs(want), (float(loss), want)
    m1, m2 = _mean_grads(x1, x2)
    _assert_grads(x1, x2, i1, i2, m1, m2, ga, gb)


def test_config2_full_f32():
    _full_check(datagen.sphere_noise(32, 2048, seed=20), datagen.sphere_noise(32, 2048, seed=21))


def test_config2_full_f16():
    _full_check(datagen.sphere_noise(32, 2048, seed=20, dtype=torch.float16),
                datagen.sphere_noise(32, 2048, seed=21, dtype=torch.float16))


def test_config3_full_fwd_bwd():
    _full_check(datagen.gmm(16, 16384, seed=30), datagen.gmm(16, 8192, seed=31))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_config5_fwd_bwd(dtype):
    N = 1 << 20
    x1 = datagen.lidar(N, seed=50, dtype=dtype)
    x2 = datagen.lidar(N, seed=51, dtype=dtype)
    d1, d2, i1, i2 = C.chamfer_fwd(x1.to(DEV), x2.to(DEV), 0)
    torch.cuda.synchronize()
    # sampled rows of both directions, bit-exact against the oracle
    g = torch.Generator().manual_seed(int(dtype == torch.float64))
    for xa, xb, d, i in ((x1, x2, d1, i1), (x2, x1, d2, i2)):
        rows = torch.randint(0, N, (2048,), generator=g)
        od, oi = oracle.nn(xa[:, rows].numpy(), xb.numpy(), 1)
        assert np.array_equal(i[:, rows].cpu().numpy(), oi)
        assert np.array_equal(_bits(d[:, rows]), od.view(np.uint8))
    # every point: the reported distance is the distance to the reported neighbour
    for xa, xb, d, i in ((x1, x2, d1, i1), (x2, x1, d2, i2)):
        a, b = xa[0].to(DEV), xb[0].to(DEV)
        r = ((b[i[0].long()] - a) ** 2).sum(-1)
        eps = 1e-6 if dtype == torch.float32 else 1e-14
        assert torch.all((d[0] - r).abs() <= eps * r + 1e-30)
    # backward on every point through the GPU's indices
    g1 = torch.randn(d1.shape, generator=g).to(dtype)
    g2 = torch.randn(d2.shape, generator=g).to(dtype)
    gx1, gx2 = C.chamfer_bwd(x1.to(DEV), x2.to(DEV), i1, i2, g1.to(DEV), g2.to(DEV))
    _assert_grads(x1, x2, i1, i2, g1, g2, gx1, gx2)
    # the fused loss and its gradients
    loss, ga, gb = _loss_and_grads(x1, x2)
    want = d1.double().mean().item() + d2.double().mean().item()
    assert abs(float(loss) - want) <= LOSS_RTOL[dtype] * abs(want), (float(loss), want)
    m1, m2 = _mean_grads(x1, x2)
    _assert_grads(x1, x2, i1, i2, m1, m2, ga, gb)
