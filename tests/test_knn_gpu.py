"""knn_points / knn_gather parity on the B200 against the CPU oracle, through the
C ABI and the torch API.  idxs bit-exact, dists bit-exact, grad_p1 bit-exact
(summed in k order like the reference CPU), grad_p2 within tolerance."""
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
    return t.detach().cpu().contiguous().numpy().view(np.uint8)


def _case(Nb, P1, P2, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    p1 = torch.randn(Nb, P1, D, generator=g).to(dtype)
    p2 = torch.randn(Nb, P2, D, generator=g).to(dtype)
    l1 = torch.randint(0, P1 + 1, (Nb,), generator=g)
    l2 = torch.randint(0, P2 + 1, (Nb,), generator=g)
    l1[0], l2[0] = P1, P2
    return p1, p2, l1, l2


def _run(p1, p2, l1, l2, norm, K, flags=0, seed=0):
    mode = 0  # the reference knn kernels are uncontracted in both paths
    i, d = C.knn_fwd(p1.to(DEV), p2.to(DEV), l1.to(DEV), l2.to(DEV), norm, K, flags)
    torch.cuda.synchronize()
    oi, od = oracle.knn_fwd(p1.numpy(), p2.numpy(), l1.numpy(), l2.numpy(), norm, K, mode)
    assert np.array_equal(i.cpu().numpy(), oi)
    assert np.array_equal(_bits(d), od.view(np.uint8))
    g = torch.Generator().manual_seed(seed)
    gd = torch.randn(i.shape, generator=g).to(p1.dtype)
    g1, g2 = C.knn_bwd(p1.to(DEV), p2.to(DEV), l1.to(DEV), l2.to(DEV), i, norm, gd.to(DEV))
    torch.cuda.synchronize()
    o1, o2 = oracle.knn_bwd(p1.numpy(), p2.numpy(), l1.numpy(), l2.numpy(), oi, norm, gd.numpy())
    assert np.array_equal(_bits(g1), o1.view(np.uint8)), "grad_p1 must be bit-exact"
    # grad_p2: atomics; bound by the summed term magnitudes
    s2 = np.zeros(p2.shape, np.float64)
    n2 = np.zeros(p2.shape, np.float64)
    P2 = p2.shape[1]
    for n in range(p1.shape[0]):
        for k in range(K):
            j = oi[n, :, k]
            ok = j >= 0
            if norm == 2:
                t = np.abs(2 * gd[n, :, k].double().numpy()[:, None] *
                           (p1[n].double().numpy() - p2[n].double().numpy()[np.clip(j, 0, P2 - 1)]))
            else:
                t = np.repeat(np.abs(gd[n, :, k].double().numpy())[:, None], p1.shape[2], 1)
            np.add.at(s2[n], j[ok], t[ok])
            np.add.at(n2[n], j[ok], 1.0)
    e2 = np.abs(g2.cpu().double().numpy() - o2.astype(np.float64))
    assert np.all(e2 <= tolerance(p1.dtype, s2, n2))
    return i, d


@pytest.mark.parametrize("K", [1, 3, 5, 16, 32])
@pytest.mark.parametrize("norm", [1, 2])
def test_knn_f32_ragged(K, norm):
    p1, p2, l1, l2 = _case(3, 300, 450, 3, torch.float32, seed=K * 10 + norm)
    _run(p1, p2, l1, l2, norm, K)
    _run(p1, p2, l1, l2, norm, K, flags=1)


@pytest.mark.parametrize("D", [1, 2, 5, 8])
def test_knn_general_d(D):
    p1, p2, l1, l2 = _case(2, 130, 260, D, torch.float32, seed=D)
    _run(p1, p2, l1, l2, 2, 7)
    _run(p1, p2, l1, l2, 1, 7)


@pytest.mark.parametrize("D,K", [(9, 5), (16, 32), (32, 7), (64, 3), (3, 33), (3, 64),
                                 (12, 100), (2, 256), (3, 300), (4, 700), (3, 1024)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.float16])
def test_knn_large_d_and_k(D, K, dtype):
    """The general kernel: any D (the reference's V0/V1 range) and K up to 1024
    (K beyond a batch's target count pads with idx -1)."""
    p1, p2, l1, l2 = _case(2, 70, 1200 if K > 256 else 300, D, dtype, seed=D * 100 + K)
    _run(p1, p2, l1, l2, 2, K)
    _run(p1, p2, l1, l2, 1, K)


def test_knn_large_k_ties():
    g = torch.Generator().manual_seed(19)
    p1 = torch.randint(0, 2, (2, 40, 10), generator=g).float()
    p2 = torch.randint(0, 2, (2, 400, 10), generator=g).float()
    _run(p1, p2, torch.tensor([40, 17]), torch.tensor([400, 90]), 2, 130)


def test_knn_k_limit():
    import ctypes

    x = torch.zeros(1, 4, 3, device=DEV)
    L = torch.full((1,), 4, device=DEV)
    d = torch.empty(1, 4, 1025, device=DEV)
    i = torch.empty(1, 4, 1025, dtype=torch.int64, device=DEV)
    rc = C.lib().tpo_knn_fwd(0, 0, C.p(x), C.p(x), C.p(L), C.p(L), C.I64(1), C.I64(4), C.I64(4),
                             C.I64(3), C.I64(2), C.I64(1025), C.p(d), C.p(i), C.stream())
    assert rc == 2  # TPO_ERR_UNSUPPORTED


@pytest.mark.parametrize("dtype", [torch.float64, torch.float16])
@pytest.mark.parametrize("norm", [1, 2])
def test_knn_other_dtypes(dtype, norm):
    p1, p2, l1, l2 = _case(2, 200, 333, 3, dtype, seed=3)
    _run(p1, p2, l1, l2, norm, 16)


def test_knn_ties_and_k_beyond_lengths():
    g = torch.Generator().manual_seed(9)
    p1 = torch.randint(0, 3, (2, 100, 3), generator=g).float()
    p2 = torch.randint(0, 3, (2, 120, 3), generator=g).float()
    _run(p1, p2, torch.tensor([100, 50]), torch.tensor([120, 6]), 2, 16)
    _run(p1, p2, torch.tensor([100, 50]), torch.tensor([0, 3]), 1, 4)


def test_knn_known_values():
    import torch_point_ops_b200 as tpo

    p1 = torch.tensor([[[0.0, 0.0, 0.0], [1.0, 0.0, 0.0]]], device=DEV)
    p2 = torch.tensor([[[0.0, 0.0, 0.0], [0.5, 0.0, 0.0], [2.0, 0.0, 0.0]]], device=DEV)
    idxs, dists = tpo.knn_points(p1, p2, K=2)
    assert idxs.tolist() == [[[0, 1], [1, 0]]]
    assert torch.allclose(dists.cpu(), torch.tensor([[[0.0, 0.25], [0.25, 1.0]]]))


def test_knn_gather_and_module():
    import torch_point_ops_b200 as tpo

    p1, p2, l1, l2 = _case(3, 40, 50, 3, torch.float32, seed=21)
    l2[1] = 2
    p1, p2, l1, l2 = p1.to(DEV), p2.to(DEV), l1.to(DEV), l2.to(DEV)
    p2.requires_grad_()
    idxs, dists, nn = tpo.KNearestNeighbors(K=4, return_nn=True)(p1, p2, l1, l2)
    ref = oracle.knn_gather(p2.detach().cpu().numpy(), idxs.cpu().numpy(), l2.cpu().numpy())
    assert np.array_equal(nn.detach().cpu().numpy(), ref)
    gout = torch.randn_like(nn)
    nn.backward(gout, inputs=[p2])
    # gather backward = scatter-add of gout over valid (idx, k < lengths) slots
    exp = np.zeros(p2.shape, np.float64)
    I = idxs.cpu().numpy()
    G = gout.cpu().double().numpy()
    for n in range(3):
        for k in range(4):
            ok = (I[n, :, k] >= 0) & (k < int(l2[n]))
            np.add.at(exp[n], I[n, ok, k], G[n, ok, k])
    assert np.allclose(p2.grad.cpu().double().numpy(), exp, rtol=1e-5, atol=1e-5)
    # module without return_nn, functional form
    i2, d2 = tpo.KNNFunction()(p1, p2.detach(), l1, l2, K=4)
    assert torch.equal(i2, idxs)


def test_knn_config4_full_size():
    p1, p2, l1, l2 = datagen.knn_config4()
    _run(p1, p2, l1, l2, 2, 16)


def test_knn_autograd_api():
    import torch_point_ops_b200 as tpo

    p1, p2, l1, l2 = _case(2, 64, 80, 3, torch.float64, seed=2)
    a = p1.to(DEV).requires_grad_()
    b = p2.to(DEV).requires_grad_()
    f = lambda x, y: tpo.knn_points(x, y, K=3)[1]
    assert torch.autograd.gradcheck(f, (a, b), nondet_tol=1e-12)
