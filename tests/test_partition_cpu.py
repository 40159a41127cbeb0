"""Work partitions for one problem over several GPUs (torch_point_ops_b200/partition.py),
on the CPU: the ragged knn units cover every valid (batch, row) exactly once and
balance lengths1*lengths2 work to within one row per rank; and on 2 and 4 gloo
ranks, the per-rank knn over its units (the oracle standing in for the CUDA
kernel) with gradients summed by all_reduce equals the whole-batch result."""
import importlib.util
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import datagen
import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _partition():
    # loaded by path: importing the package itself needs the CUDA build
    spec = importlib.util.spec_from_file_location(
        "tpo_partition", os.path.join(ROOT, "torch_point_ops_b200", "partition.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


P = _partition()


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8, 13])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_knn_units_cover_and_balance(world, seed):
    g = torch.Generator().manual_seed(seed)
    B = 8
    l1 = torch.randint(4096, 8193, (B,), generator=g).tolist()
    l2 = torch.randint(4096, 8193, (B,), generator=g).tolist()
    if seed == 2:
        l1[3], l2[5] = 0, 0  # empty query set / empty target set
    seen = [np.zeros(n, np.int64) for n in l1]
    works = []
    for r in range(world):
        w = 0
        for b, r0, r1 in P.knn_units(l1, l2, world, r):
            assert 0 <= r0 < r1 <= l1[b] and l2[b] > 0
            seen[b][r0:r1] += 1
            w += (r1 - r0) * l2[b]
        works.append(w)
    for b in range(B):
        assert np.all(seen[b] == (1 if l2[b] > 0 else 0))
    total = sum(a * c for a, c in zip(l1, l2))
    assert sum(works) == total
    assert max(works) - total / world <= max(l2)


def test_batch_and_row_ranges():
    for n in (0, 1, 7, 32, 1 << 20):
        for world in (1, 2, 3, 8):
            rs = [P.row_range(n, world, r) for r in range(world)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(rs[i][1] == rs[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in rs) - min(b - a for a, b in rs) <= 1


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, p1, p2, l1, l2, K, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g1 = np.zeros_like(p1)
    g2 = np.zeros_like(p2)
    loss = 0.0
    for b, r0, r1 in P.knn_units(l1.tolist(), l2.tolist(), world, rank):
        q1 = p1[b:b + 1, r0:r1]
        idx, d = oracle.knn_fwd(q1, p2[b:b + 1], np.array([r1 - r0]), l2[b:b + 1], 2, K, 0)
        a, c = oracle.knn_bwd(q1, p2[b:b + 1], np.array([r1 - r0]), l2[b:b + 1], idx, 2,
                              np.ones_like(d))
        g1[b, r0:r1] += a[0]
        g2[b] += c[0]
        loss += float(d.astype(np.float64).sum())
    flat = torch.from_numpy(np.concatenate([g1.ravel(), g2.ravel(), [loss]]).astype(np.float64))
    dist.all_reduce(flat)
    if rank == 0:
        q.put(flat.numpy())
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_knn_units_gloo_equals_whole_batch(world):
    p1, p2, l1, l2 = datagen.knn_config4(seed=9, B=4, P=256)
    p1, p2, l1, l2 = p1.numpy(), p2.numpy(), l1.numpy(), l2.numpy()
    K = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, p1, p2, l1, l2, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    idx, d = oracle.knn_fwd(p1, p2, l1, l2, 2, K, 0)
    g1, g2 = oracle.knn_bwd(p1, p2, l1, l2, idx, 2, np.ones_like(d))
    n1 = g1.size
    np.testing.assert_allclose(got[:n1].reshape(g1.shape), g1, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(got[n1:n1 + g2.size].reshape(g2.shape), g2, rtol=1e-6, atol=1e-6)
    assert abs(got[-1] - d.astype(np.float64).sum()) <= 1e-9 * abs(got[-1])
