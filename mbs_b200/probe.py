"""Tensor-pipe peak probe (diagnostic): the measured roofline denominator for
compute-bound MXFP4 GEMMs on the current device (include/mbs_gemm_a4w4.h,
mbs_mxf4_peak_probe)."""

from __future__ import annotations

import ctypes

import torch

from . import _lib

__all__ = ["mxf4_peak_probe"]


def mxf4_peak_probe(groups: int = 20000, device: torch.device | None = None) -> dict:
    """Run the probe on `device` (default: current) and return
    {"tflops", "cycles_per_mma", "sm_mhz"}.  Synchronises the device's current stream."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    out = [ctypes.c_double(0.0) for _ in range(3)]
    with torch.cuda.device(device):
        _lib.call("mbs_mxf4_peak_probe", int(groups), *(ctypes.byref(o) for o in out),
                  torch.cuda.current_stream(device).cuda_stream)
    return {"tflops": out[0].value, "cycles_per_mma": out[1].value, "sm_mhz": out[2].value}
