"""tpo_probe_pipe_peak (the roofline denominator bench.py uses): every kind
returns a rate in a plausible range for the device and a live SM clock, and an
unknown kind is refused."""
import ctypes

import pytest

import capi_util as C

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", [0, 1, 2, 3])
def test_pipe_probe_rates(kind):
    import torch

    r, mhz = ctypes.c_double(), ctypes.c_double()
    assert C.lib().tpo_probe_pipe_peak(kind, ctypes.byref(r), ctypes.byref(mhz)) == 0
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    lanes = 64 if kind == 3 else 128  # element results per SM per clock, upper bound
    assert 200.0 < mhz.value < 3000.0
    assert 0.3 * sms * lanes * mhz.value * 1e6 * (0.5 if kind == 3 else 1.0) < r.value
    assert r.value < 1.1 * sms * lanes * 2 * mhz.value * 1e6


def test_pipe_probe_rejects_unknown_kind():
    r, mhz = ctypes.c_double(), ctypes.c_double()
    assert C.lib().tpo_probe_pipe_peak(7, ctypes.byref(r), ctypes.byref(mhz)) == 1
