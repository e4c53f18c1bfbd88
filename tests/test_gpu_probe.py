"""The mxf4 tensor-pipe peak probe runs and returns a plausible rate."""

import pytest

pytestmark = pytest.mark.gpu


def test_mxf4_peak_probe_plausible():
    from mbs_b200.probe import mxf4_peak_probe
    r = mxf4_peak_probe(groups=2000)
    # 256x256x64 pair MMA: ~128 cycles at the nominal FP4 rate; anything far
    # outside means the probe did not run what it claims
    assert 64 <= r["cycles_per_mma"] <= 1024, r
    assert 500 <= r["sm_mhz"] <= 2500, r
    assert 1000 <= r["tflops"] <= 20000, r


def test_mxf4_peak_probe_rejects_bad_groups():
    import ctypes
    from mbs_b200 import _lib
    d = [ctypes.c_double(0.0) for _ in range(3)]
    assert _lib.lib().mbs_mxf4_peak_probe(3, *(ctypes.byref(x) for x in d), None) == 1
