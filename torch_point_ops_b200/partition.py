"""Work partitions for running one fixed problem on several GPUs (one process per
GPU).  Pure host arithmetic on plain integers: no CUDA, no collectives, so the
same functions serve the GPU ranks and the CPU tests.

* row_range    -- contiguous, balanced share of n rows (one huge cloud pair,
                  sharded by query rows; both clouds replicated on every rank).
* batch_range  -- contiguous share of B independent batch elements.
* knn_units    -- the ragged knn case: (batch, query-row range) units whose
                  work, sum over the unit's rows of lengths2[b], is balanced over
                  the ranks.  The reference launches a fixed grid over every
                  (batch, row) slot regardless of lengths (knn/csrc/cuda/knn.cu:
                  340-341); with one batch per GPU and lengths in [P/2, P] a
                  batch split would leave up to 4x imbalance between ranks.
"""
from __future__ import annotations


def row_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced [begin, end) share of n items for `rank`."""
    return (n * rank) // world, (n * (rank + 1)) // world


batch_range = row_range


def knn_units(lengths1, lengths2, world: int, rank: int) -> list[tuple[int, int, int]]:
    """Rank `rank`'s units (b, r0, r1) over query rows r0..r1-1 of batch b.

    The valid rows of all batches, in (b, row) order, are cut into `world`
    contiguous pieces of (nearly) equal work, a row of batch b costing
    lengths2[b] pairs.  Cut points fall on row boundaries, so each rank's work
    is within one row's cost (max lengths2) of the ideal share.  Batches with no
    valid rows or no valid targets produce no units."""
    l1 = [int(v) for v in lengths1]
    l2 = [int(v) for v in lengths2]
    total = sum(a * c for a, c in zip(l1, l2))
    lo = total * rank // world
    hi = total * (rank + 1) // world
    units = []
    cum = 0  # work of all rows before batch b
    for b, (n, w) in enumerate(zip(l1, l2)):
        if n <= 0 or w <= 0:
            continue
        span = n * w
        if cum + span > lo and cum < hi:
            # rows whose start offset cum + r*w lies in [lo, hi)
            r0 = max(0, -(-(lo - cum) // w))
            r1 = min(n, -(-(hi - cum) // w))
            if r1 > r0:
                units.append((b, r0, r1))
        cum += span
    return units
