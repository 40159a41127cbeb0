"""The fp32 D=3 knn kernel starts each query's threshold at a seed: the K-th
smallest distance to a window of targets near the query in a Morton cell order
of the targets, an upper bound on the true K-th distance.  These cases aim at
what could break that bound or the tie rule -- ties exactly at the seed, flat or
degenerate bounding boxes, queries outside the targets' box, windows longer than
the valid targets, both scratch layouts (float4 copies for K >= 2, int32 indices
when only those fit, K=1 here) -- and require the result to equal the CPU oracle
bit for bit, forward and grad_p1 (helpers shared with test_knn_gpu)."""
import pytest
import torch

from test_knn_gpu import _run

pytestmark = pytest.mark.gpu


def _lattice(B, P, seed, side=8):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, side, (B, P, 3), generator=g).float()


def _full(B, P):
    return torch.full((B,), P, dtype=torch.int64)


@pytest.mark.parametrize("K", [2, 16, 32])
def test_seed_lattice_ties(K):
    # integer lattice: many equal distances, so the seed often equals the K-th
    # distance and ties at the K-th place must still go to the lowest index
    p1, p2 = _lattice(2, 1024, 1), _lattice(2, 2048, 2)
    _run(p1, p2, _full(2, 1024), _full(2, 2048), 2, K)


def test_seed_flat_and_identical_targets():
    g = torch.Generator().manual_seed(3)
    p1 = torch.randn(2, 1024, 3, generator=g)
    p2 = torch.randn(2, 2048, 3, generator=g)
    p2[0, :, 2] = 0.0          # flat along z: that axis has a single cell
    p2[1] = p2[1, :1].clone()  # every target the same point
    _run(p1, p2, _full(2, 1024), _full(2, 2048), 2, 8)


def test_seed_queries_outside_box():
    g = torch.Generator().manual_seed(4)
    p2 = torch.rand(2, 2048, 3, generator=g)
    p1 = torch.rand(2, 1024, 3, generator=g) * 6 - 2.5  # mostly outside [0,1)^3
    _run(p1, p2, _full(2, 1024), _full(2, 2048), 2, 16)


def test_seed_ragged_short_windows():
    g = torch.Generator().manual_seed(5)
    p1 = torch.rand(4, 1024, 3, generator=g)
    p2 = torch.rand(4, 1100, 3, generator=g)
    l1 = torch.tensor([1024, 700, 1, 0])
    l2 = torch.tensor([1100, 50, 9, 1030])  # 50 < the 128-target window, 9 < K
    _run(p1, p2, l1, l2, 2, 16)


def test_seed_k1_index_scratch():
    # K=1: the idxs buffer holds only the int32 cell order, not float4 copies
    g = torch.Generator().manual_seed(6)
    p1 = torch.randn(2, 4096, 3, generator=g)
    p2 = torch.randn(2, 2048, 3, generator=g)
    _run(p1, p2, torch.tensor([4096, 3000]), torch.tensor([2048, 1500]), 2, 1)


def test_seed_on_off_identical_config4():
    # the whole of config 4 (K=16 and K=1) with and without seeds: the seeds may
    # only remove candidates that the final list would not keep, so every index
    # and distance must agree; the unseeded run needs a fresh process because
    # the library reads TPO_KNN_SEED once
    import os
    import subprocess
    import sys

    import datagen
    import torch_point_ops_b200 as tpo

    p1, p2, l1, l2 = [t.cuda() for t in datagen.knn_config4()]
    here = os.path.dirname(os.path.abspath(__file__))
    code = (
        "import sys, torch; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
        "import datagen, torch_point_ops_b200 as tpo\n"
        "p1, p2, l1, l2 = [t.cuda() for t in datagen.knn_config4()]\n"
        "out = {}\n"
        "for K in (1, 16):\n"
        "    out[K] = [t.cpu() for t in tpo.knn_points(p1, p2, l1, l2, K=K)[:2]]\n"
        "torch.save(out, sys.argv[1])\n" % (here, os.path.dirname(here)))
    import tempfile
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "unseeded.pt")
        env = dict(os.environ, TPO_KNN_SEED="0")
        subprocess.run([sys.executable, "-c", code, path], env=env, check=True)
        ref = torch.load(path)
    for K in (1, 16):
        idx, dist = tpo.knn_points(p1, p2, l1, l2, K=K)[:2]
        assert torch.equal(idx.cpu(), ref[K][0])
        assert torch.equal(dist.cpu(), ref[K][1])
