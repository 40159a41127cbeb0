"""Gradient tolerances.  Indices and distances are compared bit for bit; gradients
are sums whose order is free in the reference too (it scatters with atomics), so
they are compared against the oracle's sequential sum within
    rel * S  (+ for fp16: n * 2^-10 * S, the bound on the reordering error of n
    half-precision additions, each rounding at most 2^-11 of the running sum)
where S is the sum of the magnitudes of the n terms entering the element.
rel = 1e-6 (fp32), 1e-12 (fp64), 1e-3 (fp16)."""
import numpy as np
import torch

REL = {torch.float32: 1e-6, torch.float64: 1e-12, torch.float16: 1e-3}


def tolerance(dtype, term_sum, n_terms):
    tol = REL[dtype] * term_sum
    if dtype == torch.float16:
        tol = tol + n_terms * 2.0 ** -10 * term_sum + np.finfo(np.float16).tiny
    return tol
