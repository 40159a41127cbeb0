"""Generates tests/golden/*.npz from the UNMODIFIED reference implementation.

Run in a container that has the reference checkout: it builds (oracle/Makefile.ref)
and loads the reference's own CPU knn operator library (torch_point_ops/knn/csrc/
knn.cpp) and records its outputs on seeded inputs.  The reference's CPU path is
the only one runnable without a GPU; chamfer's CPU path is knn(K=1) in both
directions + knn_backward (chamfer itself raises on CPU, chamfer.cpp:21-24).

    python tests/golden/make_golden.py [chamfer_knn|fps|all]

fps: the reference's CPU fps_forward / gather_points_forward / _backward
(torch_point_ops/fps/csrc/fps.cpp:17-145) on clouds without degenerate points
(|p|^2 > 1e-3) and without exact ties, where its CPU path and its CUDA kernel
(which the oracle restates) select the same points.
"""
import os
import subprocess
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)


def main():
    import oracle

    if oracle.ref_knn() is None:
        subprocess.check_call(["make", "-f", os.path.join(ROOT, "oracle", "Makefile.ref"), "cpu"])
    ops = oracle.ref_knn()
    assert ops is not None, "reference knn library not available"
    g = torch.Generator().manual_seed(1234)
    dts = {"f32": torch.float32, "f64": torch.float64, "f16": torch.float16}
    for name, dt in dts.items():
        # chamfer-shaped case: unequal sizes, an exact duplicate point to force ties
        B, N, M = 2, 157, 211
        x1 = torch.rand(B, N, 3, generator=g).to(dt)
        x2 = torch.rand(B, M, 3, generator=g).to(dt)
        x2[:, 17] = x2[:, 5]          # duplicate target -> tie, lowest index must win
        x1[:, 40] = x1[:, 3]
        L1 = torch.full((B,), N)
        L2 = torch.full((B,), M)
        i1, d1 = ops.knn_forward(x1, x2, L1, L2, 2, 1, -1)
        i2, d2 = ops.knn_forward(x2, x1, L2, L1, 2, 1, -1)
        g1 = torch.randn(B, N, 1, generator=g).to(dt)
        g2 = torch.randn(B, M, 1, generator=g).to(dt)
        ga1, gb1 = ops.knn_backward(x1, x2, L1, L2, i1, 2, g1)
        gb2, ga2 = ops.knn_backward(x2, x1, L2, L1, i2, 2, g2)
        np.savez_compressed(
            os.path.join(HERE, f"chamfer_{name}.npz"), xyz1=x1.numpy(), xyz2=x2.numpy(),
            dist1=d1[..., 0].numpy(), idx1=i1[..., 0].numpy(), dist2=d2[..., 0].numpy(),
            idx2=i2[..., 0].numpy(), grad_dist1=g1[..., 0].numpy(), grad_dist2=g2[..., 0].numpy(),
            grad_xyz1_dir1=ga1.numpy(), grad_xyz2_dir1=gb1.numpy(),
            grad_xyz1_dir2=ga2.numpy(), grad_xyz2_dir2=gb2.numpy())
        # knn: ragged lengths, K larger than some lengths2, both norms
        for norm in (1, 2):
            Nb, P1, P2, K = 3, 60, 50, 16
            p1 = torch.randn(Nb, P1, 3, generator=g).to(dt)
            p2 = torch.randn(Nb, P2, 3, generator=g).to(dt)
            l1 = torch.tensor([60, 33, 7])
            l2 = torch.tensor([50, 9, 30])
            idx, dist = ops.knn_forward(p1, p2, l1, l2, norm, K, -1)
            gd = torch.randn(Nb, P1, K, generator=g).to(dt)
            gp1, gp2 = ops.knn_backward(p1, p2, l1, l2, idx, norm, gd)
            np.savez_compressed(
                os.path.join(HERE, f"knn_{name}_L{norm}.npz"), p1=p1.numpy(), p2=p2.numpy(),
                lengths1=l1.numpy(), lengths2=l2.numpy(), K=K, norm=norm, idxs=idx.numpy(),
                dists=dist.numpy(), grad_dists=gd.numpy(), grad_p1=gp1.numpy(), grad_p2=gp2.numpy())
    print("wrote", sorted(os.listdir(HERE)))


def fps_main():
    import oracle

    if oracle.ref_fps() is None:
        subprocess.check_call(["make", "-f", os.path.join(ROOT, "oracle", "Makefile.ref"), "cuda"])
    ops = oracle.ref_fps()
    assert ops is not None, "reference fps library not available"
    g = torch.Generator().manual_seed(4321)
    dts = {"f32": torch.float32, "f64": torch.float64, "f16": torch.float16}
    for name, dt in dts.items():
        out = {}
        for ci, (B, P, S) in enumerate([(2, 50, 12), (3, 333, 40), (1, 1200, 64)]):
            x = torch.randn(B, P, 3, generator=g)
            x = torch.where(x.pow(2).sum(-1, keepdim=True) < 0.01, x + 0.5, x).to(dt)
            out[f"points{ci}"] = x.numpy()
            out[f"idx{ci}"] = ops.fps_forward(x, S).numpy()
        pts = torch.randn(2, 5, 90, generator=g).to(dt)
        gidx = torch.stack([torch.randperm(90, generator=g)[:31] for _ in range(2)])
        gout = torch.randn(2, 5, 31, generator=g).to(dt)
        out.update(gp_points=pts.numpy(), gp_idx=gidx.numpy(),
                   gp_out=ops.gather_points_forward(pts, gidx).numpy(), gp_grad_out=gout.numpy(),
                   gp_grad_points=ops.gather_points_backward(gout, gidx, 90).numpy())
        np.savez_compressed(os.path.join(HERE, f"fps_{name}.npz"), **out)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    what = sys.argv[1] if len(sys.argv) > 1 else "all"
    if what in ("chamfer_knn", "all"):
        main()
    if what in ("fps", "all"):
        fps_main()
