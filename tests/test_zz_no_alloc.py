"""tpo_chamfer_fwd_noalloc: the chamfer forward for callers that may not allocate
device memory (inside allocators or memory pools, allocation-free serving loops,
FFI hosts that are only handed buffers).  It must give exactly the results of
tpo_chamfer_fwd -- indices and distances bit for bit, the same bar as every
other chamfer parity test here -- on consecutive calls that reuse the library's
fixed scratch array, and must refuse problems larger than that array.

Collected last on purpose (file name), so a run that stops at the first failure
has already run every other test; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

import capi_util as C
import datagen

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _noalloc(x1, x2, flags=0):
    B, N, _ = x1.shape
    M = x2.shape[1]
    d1 = torch.empty(B, N, dtype=x1.dtype, device=DEV)
    d2 = torch.empty(B, M, dtype=x1.dtype, device=DEV)
    i1 = torch.empty(B, N, dtype=torch.int32, device=DEV)
    i2 = torch.empty(B, M, dtype=torch.int32, device=DEV)
    rc = C.lib().tpo_chamfer_fwd_noalloc(C.DT[x1.dtype], flags, C.p(x1), C.p(x2), C.I64(B),
                                          C.I64(N), C.I64(M), C.p(d1), C.p(d2), C.p(i1), C.p(i2),
                                          C.stream())
    C.check(rc)
    return d1, d2, i1, i2


def _same(a, b):
    for x, y in zip(a, b):
        assert x.shape == y.shape
        assert np.array_equal(x.cpu().numpy().view(np.uint8), y.cpu().numpy().view(np.uint8))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.float64])
def test_noalloc_matches_workspace_entry_point_twice(dtype):
    # two consecutive calls of different sizes: the second must not see the first's keys
    cases = [(4, 3000, 2500, 11), (2, 700, 1900, 12)]
    for flags in (0, 1):
        for B, N, M, seed in cases:
            x1 = datagen.sphere_noise(B, N, seed, dtype=dtype).to(DEV)
            x2 = datagen.sphere_noise(B, M, seed + 100, dtype=dtype).to(DEV)
            got = _noalloc(x1, x2, flags)
            torch.cuda.synchronize()
            ref = C.chamfer_fwd(x1, x2, flags)
            torch.cuda.synchronize()
            _same(got, ref)


def test_noalloc_rejects_oversize_problem():
    # 8 B of keys per point for f32: 3M points exceed the 16 MiB array
    x = torch.empty(1, 1, 3, device=DEV)
    rc = C.lib().tpo_chamfer_fwd_noalloc(0, 0, C.p(x), C.p(x), C.I64(1), C.I64(1_500_000),
                                          C.I64(1_500_000), C.p(x), C.p(x), C.p(x), C.p(x),
                                          C.stream())
    assert rc == 3  # TPO_ERR_WORKSPACE
    assert b"16 MiB" in C.lib().tpo_status_string(rc)


@pytest.mark.parametrize("dtype,N,M", [(torch.float32, 1_048_575, 1_048_577),
                                       (torch.float64, 524_287, 524_289)])
def test_noalloc_exact_point_limit_with_unaligned_halves(dtype, N, M):
    """B*(N+M) exactly at the stated limit, split so that neither key region is a
    multiple of 256 bytes: accepted, and equal to the workspace entry point; one
    point more is refused."""
    x1 = datagen.lidar(N, seed=3, dtype=dtype).to(DEV)
    x2 = datagen.lidar(M, seed=4, dtype=dtype).to(DEV)
    got = _noalloc(x1, x2)
    torch.cuda.synchronize()
    _same(got, C.chamfer_fwd(x1, x2))
    x = torch.empty(1, 1, 3, dtype=dtype, device=DEV)
    rc = C.lib().tpo_chamfer_fwd_noalloc(C.DT[dtype], 0, C.p(x), C.p(x), C.I64(1), C.I64(N),
                                          C.I64(M + 1), C.p(x), C.p(x), C.p(x), C.p(x), C.stream())
    assert rc == 3


def test_noalloc_rejects_sizes_whose_product_would_wrap():
    # B*(N+M) wraps a 64-bit size for these values; must be refused, not launched
    x = torch.empty(1, 1, 3, device=DEV)
    for B, N, M in [(1 << 40, 1 << 30, 1 << 30), (1 << 62, 4, 4), (3, 1 << 61, 0)]:
        rc = C.lib().tpo_chamfer_fwd_noalloc(0, 0, C.p(x), C.p(x), C.I64(B), C.I64(N), C.I64(M),
                                              C.p(x), C.p(x), C.p(x), C.p(x), C.stream())
        assert rc in (1, 3)  # TPO_ERR_INVALID_ARGUMENT or TPO_ERR_WORKSPACE
