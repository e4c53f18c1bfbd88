"""aiter.utility.fp4_utils stand-in: decoding used by the reference's torch
oracle (test_gemm_a4w4.py:28-69).  Written from the OCP MX definitions:
e2m1 code c -> (-1)^(c>>3) * {0, .5, 1, 1.5, 2, 3, 4, 6}[c & 7], two codes per
byte with element 2j in the low nibble; e8m0 byte e -> 2^(e - 127), 0xFF -> NaN."""

from __future__ import annotations

import torch

_E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]


def mxfp4_to_f32(x: torch.Tensor) -> torch.Tensor:
    """fp4x2 [R, K/2] -> float32 [R, K]."""
    b = x.view(torch.uint8).to(torch.int64)
    table = torch.tensor(_E2M1, dtype=torch.float32, device=b.device)
    lo, hi = table[b & 0xF], table[b >> 4]
    return torch.stack((lo, hi), dim=-1).reshape(*b.shape[:-1], b.shape[-1] * 2)


def e8m0_to_f32(s: torch.Tensor) -> torch.Tensor:
    """e8m0 bytes -> float32 2^(e - 127) (exact; byte 0xFF is NaN, byte 0 is 2^-127)."""
    e = s.view(torch.uint8).to(torch.int32)
    # 2^(e-127): biased exponent e in the float's exponent field; e = 0 is the subnormal 2^-127
    bits = torch.where(e > 0, e << 23, torch.full_like(e, 0x00400000))
    f = bits.view(torch.float32)
    return torch.where(e == 255, torch.full_like(f, float("nan")), f)
