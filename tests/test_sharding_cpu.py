"""The row-sharded protocol of torch_point_ops_b200.sharded on 2 CPU ranks (gloo):
partial column keys merged by all_reduce(MIN) over int64 must give the global
nearest neighbours (lowest index on ties), and the per-rank partial backward
(own rows + own column shard) summed by all_reduce(SUM) must give the full
gradient.  The oracle stands in for the CUDA kernels; the host logic (ranges,
key encoding, collectives) is the one the GPU path uses."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _row_range(n, world, rank):
    # same arithmetic as torch_point_ops_b200.sharded.row_range (importing the
    # package needs the CUDA build, so it is restated here and checked below)
    return (n * rank) // world, (n * (rank + 1)) // world


def _worker(rank, world, port, x1, x2, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, N, M = x1.shape[0], x1.shape[1], x2.shape[1]
    r0, r1 = _row_range(N, world, rank)
    c0, c1 = _row_range(M, world, rank)
    # partial column keys over this rank's rows: (dist bits << 32) | row
    keys = np.full((B, M), np.iinfo(np.int64).max, np.int64)
    for b in range(B):
        d = ((x2[b][None, :, :] - x1[b, r0:r1][:, None, :]) ** 2).astype(np.float32)
        dd = ((d[..., 0] + d[..., 1]) + d[..., 2]).astype(np.float32)  # (rows, M)
        bits = dd.view(np.uint32).astype(np.int64)
        k = (bits << 32) | np.arange(r0, r1, dtype=np.int64)[:, None]
        if r1 > r0:
            keys[b] = k.min(axis=0)
    t = torch.from_numpy(keys)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    col_idx = (t.numpy() & 0xFFFFFFFF).astype(np.int32)
    col_d = (t.numpy() >> 32).astype(np.uint32).view(np.float32)
    # partial backward: own rows (direction 1) + own column shard (direction 2)
    _, _, i1, i2 = oracle.chamfer_fwd(x1, x2, 0)
    g1 = np.zeros((B, N), np.float32)
    g2 = np.zeros((B, M), np.float32)
    g1[:, r0:r1] = 1.0 / (B * N)
    g2[:, c0:c1] = 1.0 / (B * M)
    gx1, gx2 = oracle.chamfer_bwd(x1, x2, i1, i2, g1, g2)
    flat = torch.from_numpy(np.concatenate([gx1.ravel(), gx2.ravel()]).astype(np.float64))
    dist.all_reduce(flat)
    if rank == 0:
        out["col_idx"] = col_idx
        out["col_d"] = col_d
        out["grad"] = flat.numpy()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_protocol(world):
    rng = np.random.default_rng(world)
    x1 = rng.integers(0, 6, (2, 61, 3)).astype(np.float32)   # integer grid: many ties
    x2 = rng.integers(0, 6, (2, 47, 3)).astype(np.float32)
    out = mp.Manager().dict()
    mp.spawn(_worker, args=(world, _free_port(), x1, x2, out), nprocs=world, join=True)
    od1, od2, oi1, oi2 = oracle.chamfer_fwd(x1, x2, 0)
    assert np.array_equal(out["col_idx"], oi2)
    assert np.array_equal(out["col_d"], od2)
    B, N, M = 2, 61, 47
    g1 = np.full((B, N), 1.0 / (B * N), np.float32)
    g2 = np.full((B, M), 1.0 / (B * M), np.float32)
    f1, f2 = oracle.chamfer_bwd(x1, x2, oi1, oi2, g1, g2)
    full = np.concatenate([f1.ravel(), f2.ravel()]).astype(np.float64)
    assert np.allclose(out["grad"], full, rtol=1e-6, atol=1e-7)


def test_row_range_partitions():
    for n in (0, 1, 7, 1 << 20):
        for w in (1, 2, 3, 8):
            rs = [_row_range(n, w, r) for r in range(w)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            assert max(e - s for s, e in rs) - min(e - s for s, e in rs) <= 1
