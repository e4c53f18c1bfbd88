"""aiter.ops.shuffle stand-in: the 16x16 weight preshuffle (flatB,
kernel/gemm_a4w4.hip:84-95) on the GPU via mbs_b200.shuffle_weight."""

from __future__ import annotations

import torch


def shuffle_weight(x: torch.Tensor, layout=(16, 16), use_int4: bool = False) -> torch.Tensor:
    if tuple(layout) != (16, 16) or use_int4:
        raise NotImplementedError("only the (16, 16) fp4x2 preshuffle is provided")
    import mbs_b200
    out = mbs_b200.shuffle_weight(x)
    return out.view(x.dtype) if x.dtype != torch.uint8 else out
