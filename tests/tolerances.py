"""Gradient tolerances.  Indices and distances are compared bit for bit; gradients
are sums whose order is free in the reference too (it scatters with atomics,
chamfer.cu:235-245, knn.cu:440-470), so they are compared against the oracle's
sequential sum within

    rel * S  +  2 * n * u * S

where S is the sum of the magnitudes of the n terms entering the element, rel the
contract's relative tolerance (1e-6 fp32, 1e-12 fp64, 1e-3 fp16) and u the unit
roundoff of the dtype (2^-24, 2^-53, 2^-11).  The second part is the standard
bound on reordering a recursive sum of n terms (each order is within (n-1)*u*S of
the exact sum, so two orders are within twice that); it matters only where a
point is the nearest neighbour of very many others (clustered clouds: config 3's
Gaussian mixture has points referenced by ~4000 others)."""
import numpy as np
import torch

REL = {torch.float32: 1e-6, torch.float64: 1e-12, torch.float16: 1e-3}
UNIT = {torch.float32: 2.0 ** -24, torch.float64: 2.0 ** -53, torch.float16: 2.0 ** -11}


def tolerance(dtype, term_sum, n_terms):
    tol = REL[dtype] * term_sum + 2.0 * n_terms * UNIT[dtype] * term_sum
    if dtype == torch.float16:
        tol = tol + np.finfo(np.float16).tiny
    return tol


def term_scale(x1, x2, i1, i2, g1, g2):
    """Chamfer backward: per gradient element, the sum of |terms| entering it and
    their count (float64 numpy), from CPU tensors x1 (B,N,3), x2 (B,M,3), the
    indices i1 (B,N), i2 (B,M) and the upstream gradients g1 (B,N), g2 (B,M)."""
    a, b = x1.double().numpy(), x2.double().numpy()
    i1, i2 = i1.cpu().numpy().astype(np.int64), i2.cpu().numpy().astype(np.int64)
    g1, g2 = g1.cpu().double().numpy(), g2.cpu().double().numpy()
    s1, s2 = np.zeros_like(a), np.zeros_like(b)
    n1, n2 = np.ones_like(a), np.ones_like(b)
    for bi in range(a.shape[0]):
        t = np.abs(2 * g1[bi][:, None] * (a[bi] - b[bi][i1[bi]]))
        s1[bi] += t
        np.add.at(s2[bi], i1[bi], t)
        np.add.at(n2[bi], i1[bi], 1.0)
        t = np.abs(2 * g2[bi][:, None] * (b[bi] - a[bi][i2[bi]]))
        s2[bi] += t
        np.add.at(s1[bi], i2[bi], t)
        np.add.at(n1[bi], i2[bi], 1.0)
    return s1, s2, n1, n2
