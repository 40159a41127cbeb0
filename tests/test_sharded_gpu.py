"""Row-sharded chamfer (torch_point_ops_b200.sharded) on the GPU: one rank must
reproduce the fused loss and gradients of ChamferDistance("mean"); with two or
more GPUs, ranks exchanging keys over NCCL must give the same result."""
import os
import socket

import pytest
import torch

import datagen

pytestmark = pytest.mark.gpu


def _run(rank, world, port, x1, x2, q, dtype=torch.float32):
    import torch.distributed as dist

    import torch_point_ops_b200 as tpo
    from torch_point_ops_b200.sharded import sharded_chamfer_loss

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    a, b = x1.to(dev, dtype), x2.to(dev, dtype)
    loss, g1s, g2s = sharded_chamfer_loss(a, b)
    if rank == 0:
        import numpy as np

        import capi_util as C
        from tolerances import term_scale, tolerance

        ra = a.clone().requires_grad_()
        rb = b.clone().requires_grad_()
        ref = tpo.ChamferDistance("mean")(ra, rb)
        ref.backward()
        rt = 1e-6 if dtype == torch.float32 else 1e-12
        ok = abs(float(loss) - float(ref)) <= rt * abs(float(ref))
        # gradients: both sides are sums in a free order, so each may sit the
        # per-element bound away from the exact sum -> twice the bound apart
        _, _, i1, i2 = C.chamfer_fwd(a, b)
        B, N, M = a.shape[0], a.shape[1], b.shape[1]
        g1 = torch.full((B, N), 1.0 / (B * N), dtype=dtype)
        g2 = torch.full((B, M), 1.0 / (B * M), dtype=dtype)
        s1, s2, n1, n2 = term_scale(a.cpu(), b.cpu(), i1, i2, g1, g2)
        e1 = np.abs(g1s.cpu().double().numpy() - ra.grad.cpu().double().numpy())
        e2 = np.abs(g2s.cpu().double().numpy() - rb.grad.cpu().double().numpy())
        ok = ok and bool(np.all(e1 <= 2 * tolerance(dtype, s1, n1)))
        ok = ok and bool(np.all(e2 <= 2 * tolerance(dtype, s2, n2)))
        q.put(bool(ok))
    dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("world", [1, 2])
def test_sharded_matches_single(world, dtype):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    x1 = datagen.lidar(50_000, seed=1)
    x2 = datagen.lidar(40_000, seed=2)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_run, args=(r, world, port, x1, x2, q, dtype)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert q.get(timeout=10)


@pytest.mark.parametrize("world", [1, 3, 8])
def test_knn_units_sum_to_whole_batch_on_one_gpu(world):
    """The ragged-knn split (partition.knn_units + sharded_knn_loss): the ranks'
    partial losses and gradients, computed one after another on one GPU with no
    collective and summed here, equal the whole batch through the public API
    (distances feed the loss bit-exactly; gradients are sums in a free order)."""
    import torch_point_ops_b200 as tpo
    from torch_point_ops_b200.sharded import KnnUnits, sharded_knn_loss

    p1, p2, l1, l2 = datagen.knn_config4(seed=12, B=4, P=1024)
    dev = "cuda"
    a = p1.to(dev).requires_grad_()
    b = p2.to(dev).requires_grad_()
    _, d, nn = tpo.KNearestNeighbors(K=8, return_nn=True)(a, b, l1.to(dev), l2.to(dev))
    ref = d.sum() + nn.sum()
    ga, gb = torch.autograd.grad(ref, [a, b])
    loss = 0.0
    g1 = torch.zeros_like(ga)
    g2 = torch.zeros_like(gb)
    for r in range(world):
        units = KnnUnits(l1, l2, world, r, dev)
        lo, x, y = sharded_knn_loss(p1.to(dev), p2.to(dev), units, 8, reduce=False)
        loss += float(lo)
        g1 += x
        g2 += y
    assert abs(loss - float(ref)) <= 1e-5 * abs(float(ref))
    torch.testing.assert_close(g1, ga, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(g2, gb, rtol=1e-5, atol=1e-5)
