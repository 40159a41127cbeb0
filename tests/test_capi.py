"""C-ABI library: loads, exports every symbol include/tpo_b200.h declares, and
rejects bad arguments with status codes (no kernel is launched).  CPU only."""
import ctypes
import subprocess

import pytest

from capi_util import I64, LIB, VP, declared_symbols, lib


def test_exports_every_declared_symbol():
    syms = declared_symbols()
    assert len(syms) >= 14
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if l.strip()}
    missing = [s for s in syms if s not in exported]
    assert not missing, missing
    for s in syms:
        assert hasattr(lib(), s)


def test_abi_version_and_status_strings():
    assert lib().tpo_abi_version() == 1
    assert lib().tpo_status_string(0) == b"ok"
    assert lib().tpo_status_string(99) == b"unknown status"


def test_workspace_size():
    ws = lib().tpo_chamfer_fwd_workspace_size
    assert ws(0, 2, 100, 300) == 1792 + 4864  # 8 B keys, each part 256-B aligned
    assert ws(0, 32, 2048, 2048) == 8 * 32 * 4096
    assert ws(2, 1, 10, 10) >= 16 * 20
    assert ws(7, 1, 1, 1) == 0
    assert lib().tpo_chamfer_key_bytes(0) == 8 and lib().tpo_chamfer_key_bytes(2) == 16


@pytest.mark.parametrize("dtype", [3, -1])
def test_bad_dtype_rejected(dtype):
    rc = lib().tpo_chamfer_fwd(dtype, 0, VP(0), VP(0), I64(1), I64(1), I64(1), VP(0), VP(0),
                               VP(0), VP(0), VP(0), ctypes.c_size_t(0), VP(0))
    assert rc == 1
    assert b"dtype" in lib().tpo_status_string(rc)


def test_knn_argument_checks():
    L = lib()
    args = lambda norm, K, D: (0, 0, VP(1), VP(1), VP(0), VP(0), I64(1), I64(4), I64(4), I64(D),
                               I64(norm), I64(K), VP(1), VP(1), VP(0))
    assert L.tpo_knn_fwd(*args(3, 1, 3)) == 1          # bad norm
    assert L.tpo_knn_fwd(*args(2, 0, 3)) == 1          # K < 1
    assert L.tpo_knn_fwd(*args(2, 1025, 3)) == 2       # K > 1024: unsupported
    assert L.tpo_knn_fwd(*args(2, 4, 0)) == 1          # D < 1


def test_fps_argument_checks():
    L = lib()
    f = lambda B, P, S: L.tpo_fps_fwd(0, VP(1), I64(B), I64(P), I64(S), VP(1), VP(0),
                                      ctypes.c_size_t(0), VP(0))
    assert f(1, 10, 0) == 1      # nsamples must be positive
    assert f(1, 10, 11) == 1     # nsamples > P
    assert f(-1, 10, 5) == 1     # bad shape
    assert L.tpo_fps_fwd(7, VP(1), I64(1), I64(10), I64(5), VP(1), VP(0), ctypes.c_size_t(0),
                         VP(0)) == 1   # bad dtype
    assert f(0, 10, 5) == 0      # empty batch: nothing to do
    g = lambda N, C, P, M: L.tpo_gather_points_fwd(0, VP(1), VP(1), I64(N), I64(C), I64(P),
                                                   I64(M), VP(1), VP(0))
    assert g(1, -2, 4, 4) == 1
    assert g(0, 3, 4, 4) == 0


def test_workspace_checked():
    rc = lib().tpo_chamfer_fwd(0, 0, VP(16), VP(16), I64(1), I64(8), I64(8), VP(16), VP(16),
                               VP(16), VP(16), VP(0), ctypes.c_size_t(0), VP(0))
    assert rc == 3


def test_empty_problem_is_a_noop():
    # B == 0: nothing to do, no device work, success
    rc = lib().tpo_chamfer_fwd(0, 0, VP(0), VP(0), I64(0), I64(5), I64(5), VP(0), VP(0),
                               VP(0), VP(0), VP(0), ctypes.c_size_t(0), VP(0))
    assert rc == 0


def test_device_error_flags_null_rejected():
    assert lib().tpo_device_error_flags(VP(0), 0) == 1
