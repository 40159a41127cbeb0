"""Pins the rounding of the reference's own CUDA kernels on the B200.

oracle/_ref holds the reference chamfer/knn sources compiled unmodified with the
flags of the reference's setup.py (oracle/Makefile.ref).  On the GPU this checks
that (a) the reference CUDA chamfer distances equal the oracle's "fma" mode bit for
bit -- nvcc contracts x2*x2+y2*y2+z2*z2 into fma(dz,dz,fma(dx,dx,dy*dy)) -- and
the reference CUDA knn distances equal the uncontracted mode,
and (b) this library's default output equals the reference CUDA output.
Skipped when oracle/_ref was not built."""
import numpy as np
import pytest
import torch

import capi_util as C
import datagen
import oracle

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.detach().cpu().contiguous().numpy().view(np.uint8)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16])
def test_reference_chamfer_cuda_rounding(dtype):
    ops = oracle.ref_chamfer()
    if ops is None:
        pytest.skip("reference CUDA build not present in oracle/_ref")
    x1 = datagen.sphere_noise(4, 1500, seed=1, dtype=dtype)
    x2 = datagen.sphere_noise(4, 1300, seed=2, dtype=dtype)
    rd1, rd2, ri1, ri2 = ops.chamfer_forward(x1.cuda(), x2.cuda())
    od1, od2, oi1, oi2 = oracle.chamfer_fwd(x1.numpy(), x2.numpy(), 1)
    assert np.array_equal(_bits(rd1), od1.view(np.uint8)), "reference CUDA rounding != fma mode"
    assert np.array_equal(ri1.cpu().numpy(), oi1)
    assert np.array_equal(ri2.cpu().numpy(), oi2)
    d1, d2, i1, i2 = C.chamfer_fwd(x1.cuda(), x2.cuda(), 0)
    assert torch.equal(i1.cpu(), ri1.cpu()) and torch.equal(i2.cpu(), ri2.cpu())
    assert np.array_equal(_bits(d1), _bits(rd1)) and np.array_equal(_bits(d2), _bits(rd2))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_reference_knn_cuda_rounding(dtype):
    ops = oracle.ref_knn()
    if ops is None or not oracle._ref_loaded.get("knn_cuda_ref.so"):
        pytest.skip("reference CUDA knn build not present in oracle/_ref")
    g = torch.Generator().manual_seed(3)
    p1 = torch.randn(2, 500, 3, generator=g).to(dtype)
    p2 = torch.randn(2, 700, 3, generator=g).to(dtype)
    L1 = torch.full((2,), 500)
    L2 = torch.full((2,), 700)
    ri, rd = ops.knn_forward(p1.cuda(), p2.cuda(), L1.cuda(), L2.cuda(), 2, 16, -1)
    # the reference sorts in Python (knn/__init__.py:130-131)
    rd, order = rd.sort(dim=2)
    ri = ri.gather(2, order)
    oi, od = oracle.knn_fwd(p1.numpy(), p2.numpy(), L1.numpy(), L2.numpy(), 2, 16, 0)
    assert np.array_equal(_bits(rd), od.view(np.uint8))
    assert np.array_equal(ri.cpu().numpy(), oi)
    i, d = C.knn_fwd(p1.cuda(), p2.cuda(), L1.cuda(), L2.cuda(), 2, 16, 0)
    assert torch.equal(i.cpu(), ri.cpu())


FPS_PIN_CASES = [(2, 1000, 64, 0), (2, 300, 300, 1), (1, 5000, 200, 2), (2, 2048, 128, 3),
                 (3, 777, 100, 4)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16])
@pytest.mark.parametrize("B,P,S,kind", FPS_PIN_CASES)
def test_reference_fps_cuda(B, P, S, kind, dtype):
    """The reference CUDA FPS kernel, the oracle and this library agree index for
    index -- lattice clouds (kind 1, 3) force ties, kind 2 has degenerate points,
    kind 4 duplicates."""
    ops = oracle.ref_fps()
    if ops is None:
        pytest.skip("reference fps build not present in oracle/_ref")
    g = torch.Generator().manual_seed(P + kind)
    if kind in (1, 3):
        x = torch.randint(-3, 4, (B, P, 3), generator=g).float()
    else:
        x = torch.randn(B, P, 3, generator=g)
        if kind == 2:
            x[:, 1::4] *= 1e-2
        if kind == 4:
            x[:, P // 2:] = x[:, : P - P // 2]
    x = x.to(dtype)
    ri = ops.fps_forward(x.cuda(), S).cpu()
    np.testing.assert_array_equal(ri.numpy(), oracle.fps(x.numpy(), S))
    mine = C.fps_fwd(x.cuda(), S).cpu()
    assert torch.equal(mine, ri)


def test_reference_gather_points_cuda():
    ops = oracle.ref_fps()
    if ops is None:
        pytest.skip("reference fps build not present in oracle/_ref")
    g = torch.Generator().manual_seed(5)
    pts = torch.randn(2, 5, 300, generator=g)
    idx = torch.randint(0, 300, (2, 64), generator=g)
    ref = ops.gather_points_forward(pts.cuda(), idx.cuda()).cpu()
    assert torch.equal(C.gather_points_fwd(pts.cuda(), idx.cuda()).cpu(), ref)


@pytest.mark.parametrize("D,K", [(16, 40), (40, 8), (3, 100)])
def test_reference_knn_cuda_general(D, K):
    """The reference's V1 / V0 kernels (D > 8 or K > 32) against the general path."""
    ops = oracle.ref_knn()
    if ops is None or not oracle._ref_loaded.get("knn_cuda_ref.so"):
        pytest.skip("reference CUDA knn build not present in oracle/_ref")
    g = torch.Generator().manual_seed(D * K)
    p1 = torch.randn(2, 90, D, generator=g)
    p2 = torch.randn(2, 400, D, generator=g)
    L1 = torch.tensor([90, 61])
    L2 = torch.tensor([400, 257])
    ri, rd = ops.knn_forward(p1.cuda(), p2.cuda(), L1.cuda(), L2.cuda(), 2, K, -1)
    rd, order = rd.sort(dim=2)
    ri = ri.gather(2, order)
    i, d = C.knn_fwd(p1.cuda(), p2.cuda(), L1.cuda(), L2.cuda(), 2, K, 0)
    valid = torch.arange(90)[None, :, None] < L1[:, None, None]
    assert torch.equal(i.cpu()[valid.expand_as(i.cpu())], ri.cpu()[valid.expand_as(i.cpu())])
    assert np.array_equal(_bits(d.cpu()[valid.expand_as(d.cpu())]), _bits(rd.cpu()[valid.expand_as(d.cpu())]))


@pytest.mark.parametrize("ragged", [False, True])
def test_reference_knn_cuda_f16(ragged):
    """fp16 knn against the reference CUDA build (c10::Half arithmetic: every
    sub, mul and add rounds to half).  Half distances tie often, and the
    reference's MinK and its unstable torch.sort order equal distances freely,
    so: the sorted distances are compared bit for bit everywhere, and indices
    wherever the distance value is unique within the query's K and is not the
    K-th distance (there the reference may keep any of the tied candidates);
    every reference index must also reproduce its own distance."""
    ops = oracle.ref_knn()
    if ops is None or not oracle._ref_loaded.get("knn_cuda_ref.so"):
        pytest.skip("reference CUDA knn build not present in oracle/_ref")
    g = torch.Generator().manual_seed(16 + ragged)
    B, P1, P2, K = 3, 600, 900, 16
    p1 = torch.randn(B, P1, 3, generator=g).half()
    p2 = torch.randn(B, P2, 3, generator=g).half()
    L1 = torch.tensor([600, 401, 77]) if ragged else torch.full((B,), P1)
    L2 = torch.tensor([900, 513, 40]) if ragged else torch.full((B,), P2)
    ri, rd = ops.knn_forward(p1.cuda(), p2.cuda(), L1.cuda(), L2.cuda(), 2, K, -1)
    rd, order = rd.sort(dim=2)
    ri = ri.gather(2, order).cpu()
    rd = rd.cpu()
    i, d = C.knn_fwd(p1.cuda(), p2.cuda(), L1.cuda(), L2.cuda(), 2, K, 0)
    i, d = i.cpu(), d.cpu()
    oi, od = oracle.knn_fwd(p1.numpy(), p2.numpy(), L1.numpy(), L2.numpy(), 2, K, 0)
    assert np.array_equal(i.numpy(), oi) and np.array_equal(_bits(d), od.view(np.uint8))
    for b in range(B):
        l1, kk = int(L1[b]), min(K, int(L2[b]))
        db, rdb = d[b, :l1, :kk], rd[b, :l1, :kk]
        assert np.array_equal(_bits(db), _bits(rdb)), "sorted distances differ"
        dv = db.float().numpy()
        kth = dv[:, kk - 1:kk]
        uniq = (np.sum(dv[:, :, None] == dv[:, None, :], axis=2) == 1) & (dv != kth)
        assert np.array_equal(i[b, :l1, :kk].numpy()[uniq], ri[b, :l1, :kk].numpy()[uniq])
        # each reference index reproduces its distance with c10::Half rounding
        q = p1[b, :l1].float()[:, None, :]
        t = p2[b].float()[ri[b, :l1, :kk].long()]
        # recompute the reference neighbours' distances in half, per operation
        dx = (t[..., 0] - q[..., 0]).half().float()
        dy = (t[..., 1] - q[..., 1]).half().float()
        dz = (t[..., 2] - q[..., 2]).half().float()
        rr = ((dx * dx).half().float() + (dy * dy).half().float()).half().float()
        rr = (rr + (dz * dz).half().float()).half()
        assert np.array_equal(_bits(rr), _bits(rdb))


@pytest.mark.parametrize("cfg", ["2", "2h", "3"])
def test_reference_chamfer_cuda_full_size(cfg):
    """Benchmark configurations 2 (fp32, fp16) and 3 at full size: indices and
    distances bit-identical to the reference CUDA kernel's, every point."""
    ops = oracle.ref_chamfer()
    if ops is None:
        pytest.skip("reference CUDA build not present in oracle/_ref")
    if cfg == "3":
        x1, x2 = datagen.gmm(16, 16384, seed=30), datagen.gmm(16, 8192, seed=31)
    else:
        dt = torch.float16 if cfg == "2h" else torch.float32
        x1, x2 = datagen.sphere_noise(32, 2048, seed=20, dtype=dt), datagen.sphere_noise(32, 2048, seed=21, dtype=dt)
    rd1, rd2, ri1, ri2 = ops.chamfer_forward(x1.cuda(), x2.cuda())
    d1, d2, i1, i2 = C.chamfer_fwd(x1.cuda(), x2.cuda(), 0)
    assert torch.equal(i1.cpu(), ri1.cpu()) and torch.equal(i2.cpu(), ri2.cpu())
    assert np.array_equal(_bits(d1), _bits(rd1)) and np.array_equal(_bits(d2), _bits(rd2))


def test_reference_knn_cuda_config4_full_size():
    """Benchmark configuration 4 at full size (K=16, ragged lengths): the valid
    entries of every valid row equal the reference CUDA kernel's after its own
    python sort -- distances bit for bit, indices wherever the distance is not
    tied within the row's K (the reference orders equal distances freely)."""
    ops = oracle.ref_knn()
    if ops is None or not oracle._ref_loaded.get("knn_cuda_ref.so"):
        pytest.skip("reference CUDA knn build not present in oracle/_ref")
    p1, p2, l1, l2 = [t.cuda() for t in datagen.knn_config4(seed=4)]
    K = 16
    ri, rd = ops.knn_forward(p1, p2, l1, l2, 2, K, -1)
    rd, order = rd.sort(dim=2)
    ri = ri.gather(2, order)
    i, d = C.knn_fwd(p1, p2, l1, l2, 2, K, 0)
    for b in range(p1.shape[0]):
        L1 = int(l1[b])
        db, rdb = d[b, :L1].cpu(), rd[b, :L1].cpu()
        assert np.array_equal(_bits(db), _bits(rdb))
        dv = db.numpy()
        uniq = np.sum(dv[:, :, None] == dv[:, None, :], axis=2) == 1
        assert np.array_equal(i[b, :L1].cpu().numpy()[uniq], ri[b, :L1].cpu().numpy()[uniq])
        assert uniq.mean() > 0.999
