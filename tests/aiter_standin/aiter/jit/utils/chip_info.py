"""aiter.jit.utils.chip_info stand-in.

The reference test runs its sweep only when this returns "gfx950"
(test_gemm_a4w4.py:129-132), the one architecture its HIP kernel targets.
Here the operator is the B200 build, so the stand-in reports "gfx950" for an
sm_100 device, i.e. "the device the operator under test was built for", and
the name of the device otherwise."""

from __future__ import annotations

import torch


def get_gfx_runtime() -> str:
    if torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0):
        return "gfx950"
    return torch.cuda.get_device_name() if torch.cuda.is_available() else "cpu"


get_gfx = get_gfx_runtime
