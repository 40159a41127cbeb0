"""Row-sharded chamfer for one huge cloud pair over several GPUs (one process per
GPU, torch.distributed over NCCL).

Rank r owns rows [r0, r1) of xyz1 (row_range) and evaluates them against all of
xyz2.  Its row results are complete; its column results are partial minima.
Column keys -- (distance bits << 32) | candidate chunk, an int64 >= 0 because
distances are non-negative -- are merged with ONE all_reduce(MIN), the only
exchange of the forward.  The backward accumulates the rank's own rows and its
column shard [c0, c1) (col_range) into full-size gradient buffers, merged with
an all_reduce(SUM).  Both clouds are replicated on every rank (12 MB fp32 at
1M points each), so no point data crosses NVLink.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from .partition import knn_units, row_range

col_range = row_range


def sharded_chamfer_loss(xyz1: torch.Tensor, xyz2: torch.Tensor, group=None, flags: int = 0):
    """mean(dist1) + mean(dist2) over the full clouds, computed row-sharded.

    Returns (loss, grad_xyz1, grad_xyz2) -- the loss value and its gradients,
    identical on every rank (forward and backward fused, as a training step uses
    them).  xyz1 (B,N,3), xyz2 (B,M,3): the full clouds, replicated per rank."""
    ops = _lib.chamfer_ops
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    xyz1 = xyz1.contiguous()
    xyz2 = xyz2.contiguous()
    B, N, M = xyz1.shape[0], xyz1.shape[1], xyz2.shape[1]
    r0, r1 = row_range(N, world, rank)
    c0, c1 = col_range(M, world, rank)
    k1 = ops.chamfer_keys_empty(xyz1, B * N)
    k2 = ops.chamfer_keys_empty(xyz1, B * M)
    ops.chamfer_fwd_keys(xyz1, xyz2, r0, r1, flags, k1, k2)
    if world > 1 and r1 == r0:
        # a rank without rows folded nothing: its empty keys (all ones = -1 as a
        # signed int64) must not win the signed MIN below
        k2.fill_(torch.iinfo(torch.int64).max)
    if world > 1:
        if k2.numel() == B * M:  # 64-bit keys (fp32 / fp16): one element-wise MIN
            dist.all_reduce(k2, op=dist.ReduceOp.MIN, group=group)
        else:  # fp64: 128-bit keys {lo = index, hi = distance bits}; gather, then
            # the lexicographic (hi, lo) minimum over ranks
            allk = torch.empty((world,) + k2.shape, dtype=k2.dtype, device=k2.device)
            dist.all_gather_into_tensor(allk, k2, group=group)
            allk = allk.view(world, -1, 2)
            hi = allk[..., 1]
            best_hi = hi.min(dim=0).values
            lo = torch.where(hi == best_hi, allk[..., 0],
                             torch.full_like(allk[..., 0], torch.iinfo(torch.int64).max))
            # keys are non-negative as int64 (distance >= 0, index < 2^31)
            k2 = torch.stack([lo.min(dim=0).values, best_hi], dim=-1).reshape(-1)
    d1, d2, i1, i2 = ops.chamfer_finalize(xyz1, xyz2, r0, r1, flags, k1, k2)
    # loss: this rank's rows of dist1 + its column shard of dist2, summed over ranks
    part = d1[:, r0:r1].double().sum() / (B * N) + d2[:, c0:c1].double().sum() / (B * M)
    # backward of the mean: 1/(B*N) per row, 1/(B*M) per column
    g1 = torch.full((B, N), 1.0 / (B * N), dtype=xyz1.dtype, device=xyz1.device)
    g2 = torch.full((B, M), 1.0 / (B * M), dtype=xyz1.dtype, device=xyz1.device)
    gx1 = torch.zeros_like(xyz1)
    gx2 = torch.zeros_like(xyz2)
    ops.chamfer_bwd_partial(xyz1, xyz2, r0, r1, c0, c1, i1, i2, g1, g2, gx1, gx2)
    if world > 1:
        dist.all_reduce(part, group=group)
        flat = torch.cat([gx1.view(-1), gx2.view(-1)])
        dist.all_reduce(flat, group=group)
        gx1 = flat[: gx1.numel()].view_as(gx1)
        gx2 = flat[gx1.numel():].view_as(gx2)
    return part.to(xyz1.dtype), gx1, gx2


class KnnUnits:
    """One rank's share of a ragged knn batch, as (batch, query-row range) units
    balanced by lengths1*lengths2 work over the ranks (partition.knn_units).

    The rank's units run as ONE packed knn launch: the units' query rows are
    gathered into a (S, Lmax, D) batch and their target clouds into (S, P2, D)
    (small copies, index tensors built once here), because a launch per unit
    would leave most SMs idle (one batch of config 4 is ~200 CTAs).  Indices
    returned by the knn are indices into the unit's batch of p2, as in the
    unsplit call."""

    def __init__(self, lengths1, lengths2, world: int, rank: int, device):
        l1 = [int(v) for v in lengths1]
        l2 = [int(v) for v in lengths2]
        self.units = knn_units(l1, l2, world, rank)
        S = len(self.units)
        L = max([r1 - r0 for _, r0, r1 in self.units], default=0)
        self.L = L
        b = torch.tensor([u[0] for u in self.units], dtype=torch.int64)
        r0 = torch.tensor([u[1] for u in self.units], dtype=torch.int64)
        n = torch.tensor([u[2] - u[1] for u in self.units], dtype=torch.int64)
        k = torch.arange(L, dtype=torch.int64)[None, :]
        rows = r0[:, None] + torch.minimum(k, (n - 1).clamp_min(0)[:, None])  # pads repeat a valid row
        self.batch = b.to(device)
        self._valid = (k < n[:, None]).reshape(-1)  # packed rows that are real (host)
        self.lengths1 = n.to(device)
        self.lengths2 = torch.tensor([l2[u[0]] for u in self.units], dtype=torch.int64).to(device)
        self.work = sum((r1 - r0) * l2[bb] for bb, r0, r1 in self.units)
        self._rows = rows
        self._b = b

    def index(self, P1: int):
        """Device index tensors for a (B*P1, D) view of p1, built on the host
        once per P1: (flat row of every packed row, flat row of every real packed
        row, packed position of every real packed row)."""
        if getattr(self, "_P1", None) != P1:
            flat = (self._b[:, None] * P1 + self._rows).reshape(-1)
            pos = torch.nonzero(self._valid).reshape(-1)
            dev = self.batch.device
            self._idx = (flat.to(dev), flat[pos].to(dev), pos.to(dev))
            self._P1 = P1
        return self._idx


def sharded_knn_loss(p1, p2, units: KnnUnits, K: int, group=None, norm: int = 2,
                     reduce: bool = True):
    """sum(dists) + sum(nn) of KNearestNeighbors(K, return_nn=True) over the whole
    ragged batch, computed on this rank's units; returns (loss, grad_p1, grad_p2),
    identical on every rank after one all_reduce(SUM) of the gradients (the
    rank's units write disjoint rows of grad_p1 but may share a batch's p2).
    reduce=False returns this rank's partial sums without the collective (for a
    caller that captures the compute in a CUDA graph and reduces after it).

    The gradients are formed with the library's own backward ops (the same the
    autograd path calls): d loss/d dists = 1 and d loss/d nn = 1."""
    ops = _lib.knn_ops
    B, P1, D = p1.shape
    P2 = p2.shape[1]
    ga = torch.zeros_like(p1)
    gb = torch.zeros_like(p2)
    if len(units.units):
        flat, dst, src = units.index(P1)
        S, L = len(units.units), units.L
        pa = p1.reshape(B * P1, D).index_select(0, flat).view(S, L, D)
        pb = p2.index_select(0, units.batch)
        idx, d = ops.knn_forward(pa, pb, units.lengths1, units.lengths2, norm, K, -1)
        nn = ops.knn_gather_forward(pb, idx, units.lengths2)
        loss = d.sum() + nn.sum()
        g1, g2 = ops.knn_backward(pa, pb, units.lengths1, units.lengths2, idx, norm, torch.ones_like(d))
        g2 = g2 + ops.knn_gather_backward(torch.ones_like(nn), idx, units.lengths2, P2)
        # packed rows back to their places: real rows are disjoint; p2 grads of
        # units sharing a batch add up
        ga.view(B * P1, D).index_copy_(0, dst, g1.reshape(S * L, D).index_select(0, src))
        gb.index_add_(0, units.batch, g2)
    else:
        loss = torch.zeros((), dtype=p1.dtype, device=p1.device)
    if reduce and dist.is_initialized() and dist.get_world_size(group) > 1:
        flat = torch.cat([ga.reshape(-1), gb.reshape(-1), loss.reshape(1)])
        dist.all_reduce(flat, group=group)
        ga = flat[: ga.numel()].view_as(ga)
        gb = flat[ga.numel(): ga.numel() + gb.numel()].view_as(gb)
        loss = flat[-1]
    return loss, ga, gb
