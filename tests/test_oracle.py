"""Pins the CPU oracle (oracle/tpo_oracle.c) against the reference: golden vectors
recorded from the reference's own CPU operators (tests/golden/make_golden.py), the
known values of the reference test-suite, and -- when oracle/_ref holds a build of
the reference sources -- live comparisons.  CPU only."""
import glob
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint8)


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "chamfer_*.npz"))))
def test_oracle_chamfer_golden(path):
    z = np.load(path)
    d1, d2, i1, i2 = oracle.chamfer_fwd(z["xyz1"], z["xyz2"], mode=0)
    assert np.array_equal(i1, z["idx1"]) and np.array_equal(i2, z["idx2"])
    assert np.array_equal(_bits(d1), _bits(z["dist1"])) and np.array_equal(_bits(d2), _bits(z["dist2"]))
    # duplicated target 17 == 5: the tie must resolve to the lower index
    assert not np.any(z["idx1"] == 17)
    # backward, direction by direction (the reference CPU sums sequentially)
    zero2 = np.zeros_like(z["grad_dist2"])
    zero1 = np.zeros_like(z["grad_dist1"])
    ga, gb = oracle.chamfer_bwd(z["xyz1"], z["xyz2"], i1, i2, z["grad_dist1"], zero2)
    assert np.array_equal(ga, z["grad_xyz1_dir1"]) and np.array_equal(gb, z["grad_xyz2_dir1"])
    ga, gb = oracle.chamfer_bwd(z["xyz1"], z["xyz2"], i1, i2, zero1, z["grad_dist2"])
    assert np.array_equal(ga, z["grad_xyz1_dir2"]) and np.array_equal(gb, z["grad_xyz2_dir2"])


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "knn_*.npz"))))
def test_oracle_knn_golden(path):
    z = np.load(path)
    K, norm = int(z["K"]), int(z["norm"])
    idx, dist = oracle.knn_fwd(z["p1"], z["p2"], z["lengths1"], z["lengths2"], norm, K, mode=0)
    assert np.array_equal(idx, z["idxs"])
    assert np.array_equal(_bits(dist), _bits(z["dists"]))
    g1, g2 = oracle.knn_bwd(z["p1"], z["p2"], z["lengths1"], z["lengths2"], idx, norm,
                            z["grad_dists"], l1_zero_at_tie=False)
    assert np.array_equal(g1, z["grad_p1"]) and np.array_equal(g2, z["grad_p2"])


def test_oracle_known_values():
    # tests/test_chamfer.py:180-197 of the reference: identical clouds -> 0;
    # (0,0,0) vs (1,2,3) -> 14
    a = np.array([[[0.0, 0.0, 0.0]]], np.float32)
    b = np.array([[[1.0, 2.0, 3.0]]], np.float32)
    d1, d2, _, _ = oracle.chamfer_fwd(a, b)
    assert d1[0, 0] == 14 and d2[0, 0] == 14
    x = np.random.default_rng(0).random((2, 30, 3), dtype=np.float32)
    d1, d2, i1, i2 = oracle.chamfer_fwd(x, x)
    assert np.all(d1 == 0) and np.all(d2 == 0)
    assert np.array_equal(i1[0], np.arange(30))
    # tests/test_knn.py:187-218: K=2 known neighbours
    p1 = np.array([[[0, 0, 0], [1, 0, 0]]], np.float32)
    p2 = np.array([[[0, 0, 0], [0.5, 0, 0], [2, 0, 0]]], np.float32)
    idx, dist = oracle.knn_fwd(p1, p2, K=2)
    assert idx.tolist() == [[[0, 1], [1, 0]]]
    assert np.allclose(dist, [[[0, 0.25], [0.25, 1.0]]])


def test_oracle_knn_ties_and_padding():
    # four equidistant targets: K=2 keeps the two lowest indices, ascending
    p1 = np.zeros((1, 1, 3), np.float32)
    p2 = np.array([[[1, 0, 0], [0, 1, 0], [-1, 0, 0], [0, -1, 0]]], np.float32)
    idx, dist = oracle.knn_fwd(p1, p2, K=2)
    assert idx.tolist() == [[[0, 1]]]
    # K > lengths2 -> -1 / 0 padding; rows beyond lengths1 -> -1 / 0
    idx, dist = oracle.knn_fwd(np.ones((1, 3, 3), np.float32), p2, np.array([2]), np.array([3]), K=5)
    assert idx[0, 0].tolist() == [0, 1, 2, -1, -1] or idx[0, 0, 3:].tolist() == [-1, -1]
    assert idx[0, 2].tolist() == [-1] * 5 and np.all(dist[0, 2] == 0)


def test_oracle_fma_mode_differs_only_by_rounding():
    rng = np.random.default_rng(3)
    a = rng.random((2, 300, 3), dtype=np.float32)
    b = rng.random((2, 400, 3), dtype=np.float32)
    d_exact, _, _, _ = oracle.chamfer_fwd(a, b, 0)
    d_fma, _, _, _ = oracle.chamfer_fwd(a, b, 1)
    assert np.allclose(d_exact, d_fma, rtol=1e-6, atol=0)


def test_oracle_vs_reference_live():
    """Live pin: the reference CPU knn built from its own sources (if present)."""
    ops = oracle.ref_knn()
    if ops is None:
        pytest.skip("oracle/_ref not built (needs the reference checkout)")
    import torch

    g = torch.Generator().manual_seed(7)
    for dt in (torch.float32, torch.float16, torch.float64):
        p1 = torch.rand(2, 90, 3, generator=g).to(dt)
        p2 = torch.rand(2, 120, 3, generator=g).to(dt)
        l1 = torch.tensor([90, 40])
        l2 = torch.tensor([120, 11])
        i, d = ops.knn_forward(p1, p2, l1, l2, 2, 12, -1)
        oi, od = oracle.knn_fwd(p1.numpy(), p2.numpy(), l1.numpy(), l2.numpy(), 2, 12, 0)
        assert np.array_equal(i.numpy(), oi)
        assert np.array_equal(_bits(d.numpy()), _bits(od))


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "fps_*.npz"))))
def test_oracle_fps_golden(path):
    """FPS indices and gather_points values recorded from the reference's CPU ops."""
    z = np.load(path)
    for ci in range(3):
        x, ref = z[f"points{ci}"], z[f"idx{ci}"]
        assert np.array_equal(oracle.fps(x, ref.shape[1]), ref)
    assert np.array_equal(oracle.gather_points(z["gp_points"], z["gp_idx"]), z["gp_out"])
    assert np.array_equal(oracle.gather_points_bwd(z["gp_grad_out"], z["gp_idx"], 90), z["gp_grad_points"])


def test_oracle_fps_tie_order():
    """Equal maxima resolve like the reference CUDA kernel's halving reduction:
    smallest bit-reversed thread (k mod bs), then smallest k.  P = 6 gives bs = 4,
    threads in tie order 0 (points 0, 4), 2 (point 2), 1 (points 1, 5), 3.
    Points 1..5 are all at squared distance 2 from point 0, so step 1 picks 4
    (thread 0); every remaining point is then still at 2, and step 2 picks 2
    (thread 2 ranks before thread 1) -- neither the lowest index nor the lowest
    thread.  (This order reproduces the reference's CUDA output on lattice
    clouds; tests/test_ref_cuda_pin.py checks it on the GPU.)"""
    x = np.array([[[1, 0, 0], [0, 1, 0], [0, -1, 0], [0, 0, 1], [0, 0, -1], [1, 1, 1]]],
                 np.float32)
    for dt in (np.float32, np.float64, np.float16):
        assert oracle.fps(x.astype(dt), 3).tolist() == [[0, 4, 2]]
