"""N-sharded MXFP4 GEMM over a process group.

Each rank holds a contiguous slice of the weight's rows (output columns): in
the preshuffled layout every 16-row tile is one contiguous block and in the
shuffled scale layout every 32-row group is one contiguous block, so a shard
aligned to 256 rows is a plain byte range of both buffers -- sharding needs
no re-layout.  A forward pass quantises the bf16 activations on each rank
(A is replicated: quantising it locally costs less than broadcasting it),
runs the GEMM on the local slice and combines the bf16 C shards with one
all-gather (NCCL over NVLink for CUDA tensors).

The all-gather returns the shards stacked as [world, M, N/world]; `layout=
"blocked"` hands that back as is (a view per rank is C[:, r*N/w:(r+1)*N/w]),
`layout="rows"` pays one permute copy for a row-major [M, N].
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

SHARD_ALIGN = 256


def shard_rows(N: int, world: int, rank: int, align: int = SHARD_ALIGN) -> tuple[int, int]:
    """Row range [n0, n1) of the weight held by `rank`; N/world must be a multiple of `align`."""
    if N % world != 0 or (N // world) % align != 0:
        raise ValueError(f"N={N} must split into {world} shards that are multiples of {align} rows")
    per = N // world
    return rank * per, (rank + 1) * per


def scale_n_pad(K: int) -> int:
    return ((K + 31) // 32 + 7) // 8 * 8


def shard_weight(B_shuffled: torch.Tensor, B_scale_shuffled: torch.Tensor, N: int, K: int,
                 world: int, rank: int):
    """Slice the full preshuffled weight [N, K/2] and its shuffled scales
    (roundup(N,32) x scaleN_pad bytes) down to this rank's rows.  Returns
    contiguous (B_shard [N/world, K/2], B_scale_shard [(N/world) * scaleN_pad])."""
    n0, n1 = shard_rows(N, world, rank)
    kp = K // 2
    snp = scale_n_pad(K)
    b = B_shuffled.reshape(-1)[n0 * kp: n1 * kp].reshape(n1 - n0, kp)
    s = B_scale_shuffled.reshape(-1)[n0 * snp: n1 * snp]
    return b.contiguous(), s.contiguous()


class ShardedA4W4:
    """One rank's part of an N-sharded A4W4 linear layer.

    `local_gemm(A_fp4, B, A_scale_shuffled, B_scale, A_factor, B_factor) -> C`
    and `quantize(x) -> (A_fp4, A_scale_shuffled)` default to the CUDA
    operators of this package; they are parameters so that the collective and
    layout logic can be exercised on CPU process groups in tests.
    """

    def __init__(self, B_shard: torch.Tensor, B_scale_shard: torch.Tensor, N: int, K: int,
                 group: Optional[dist.ProcessGroup] = None, B_factor_shard: Optional[torch.Tensor] = None,
                 local_gemm: Optional[Callable] = None, quantize: Optional[Callable] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.N, self.K = N, K
        self.n0, self.n1 = shard_rows(N, self.world, self.rank)
        if B_shard.shape[0] != self.n1 - self.n0 or B_shard.shape[1] != K // 2:
            raise ValueError(f"B_shard must be [{self.n1 - self.n0}, {K // 2}], got {tuple(B_shard.shape)}")
        self.B, self.B_scale, self.B_factor = B_shard, B_scale_shard, B_factor_shard
        if local_gemm is None or quantize is None:
            from .mbs_gemm_a4w4 import gemm_a4w4
            from .quant import quantize_mxfp4
            local_gemm = local_gemm or gemm_a4w4
            quantize = quantize or (lambda x: quantize_mxfp4(x, shuffle=True))
        self._gemm = local_gemm
        self._quant = quantize

    def local(self, x: torch.Tensor, A_factor: Optional[torch.Tensor] = None) -> torch.Tensor:
        """bf16 x [M, K] -> this rank's bf16 C columns [M, N/world]."""
        q, s = self._quant(x)
        return self._gemm(q, self.B, s, self.B_scale, A_factor, self.B_factor)

    def forward(self, x: torch.Tensor, A_factor: Optional[torch.Tensor] = None,
                layout: str = "blocked") -> torch.Tensor:
        c = self.local(x, A_factor).contiguous()
        M, nl = c.shape
        flat = torch.empty((self.world * M, nl), dtype=c.dtype, device=c.device)
        dist.all_gather_into_tensor(flat, c, group=self.group)
        gathered = flat.view(self.world, M, nl)
        if layout == "blocked":
            return gathered
        if layout == "rows":
            return gathered.permute(1, 0, 2).reshape(M, self.world * nl)
        raise ValueError(f"layout must be 'blocked' or 'rows', got {layout!r}")

    __call__ = forward
