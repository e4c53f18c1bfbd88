"""A stand-in for the parts of AMD's `aiter` package that the reference's
drivers call around the operator (test_gemm_a4w4.py:14-18,134-163 and
bench_one.py:13-25), built on this repository's CUDA kernels so those call
sequences run on a B200 against `mbs_gemm_a4w4`.

aiter itself is AMD-only, unpinned and absent here.  This package is test
infrastructure: it restates the published behaviour the drivers rely on
(per-1x32 MXFP4 quantisation with plain or shuffled e8m0 scales, the 16x16
weight preshuffle, fp4/e8m0 decoding, a timing decorator and an allclose
check) and nothing else.  Put `tests/aiter_standin` on `sys.path` to use it.

    quant = aiter.get_triton_quant(aiter.QuantType.per_1x32)
    x_fp4, x_scales = quant(x_bf16, shuffle=True)
"""

from __future__ import annotations

import enum
import logging
import os
import sys

import torch

_REPO = os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
if _REPO not in sys.path:
    sys.path.insert(0, _REPO)

from . import dtypes  # noqa: E402

logger = logging.getLogger("aiter")

__all__ = ["QuantType", "get_triton_quant", "gemm_a4w4", "dtypes", "logger"]


class QuantType(enum.Enum):
    """The quantisation kinds the drivers name; only per_1x32 (MXFP4) exists here."""
    per_1x32 = "per_1x32"


def _fp4_view(t: torch.Tensor) -> torch.Tensor:
    return t.view(dtypes.fp4x2) if dtypes.fp4x2 is not None else t


def _e8m0_view(t: torch.Tensor) -> torch.Tensor:
    return t.view(dtypes.fp8_e8m0) if dtypes.fp8_e8m0 is not None else t


def get_triton_quant(qtype: QuantType):
    """Returns quant(x, shuffle=False) -> (fp4x2 [R, K/2], e8m0 scales):
    plain scales are [R, K/32], shuffled ones the flatS buffer
    [roundup(R, 32), scaleN_pad].  Runs mbs_b200.quantize_mxfp4 (CUDA)."""
    if qtype is not QuantType.per_1x32:
        raise NotImplementedError(f"only QuantType.per_1x32 is provided, got {qtype}")
    import mbs_b200

    def quant(x: torch.Tensor, shuffle: bool = False, **_unused):
        q, s = mbs_b200.quantize_mxfp4(x.to(torch.bfloat16), shuffle=shuffle)
        return _fp4_view(q), _e8m0_view(s)
    return quant


def gemm_a4w4(A, B, A_scale, B_scale, out=None, bias=None, alpha=1.0, beta=0.0, bpreshuffle=True, **_unused):
    """The unified gemm_a4w4 API the reference test times beside its own
    kernel (test_gemm_a4w4.py:158-165): preshuffled B and shuffled scales,
    bf16 [M, N] out; here it is this repository's operator."""
    if not bpreshuffle:
        raise NotImplementedError("this stand-in takes the preshuffled weight layout only")
    if beta != 0.0:
        raise NotImplementedError("beta != 0 is not provided")
    import mbs_b200
    M = A.shape[0]
    res = mbs_b200.gemm_a4w4(A, B, A_scale, B_scale, alpha=alpha,
                             bias=None if bias is None else bias.to(torch.bfloat16))
    if out is not None:
        out[:M].copy_(res)
        return out
    return res
