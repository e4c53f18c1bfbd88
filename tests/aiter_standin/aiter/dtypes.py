"""Data-type names of aiter.dtypes that the reference's drivers use."""

from __future__ import annotations

import torch

bf16 = torch.bfloat16
fp16 = torch.float16
fp32 = torch.float32
fp4x2 = getattr(torch, "float4_e2m1fn_x2", None)
fp8_e8m0 = getattr(torch, "float8_e8m0fnu", None)
d_dtypes = {"bf16": bf16, "fp16": fp16, "fp32": fp32}


def str2Dtype(name: str) -> torch.dtype:
    return d_dtypes[name]


def str2tuple(text: str) -> tuple:
    return tuple(int(v) for v in text.split(","))
