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

`exchange="copy"` (CUDA GPUs) moves the rows with copy engines instead:
every rank maps its peers' output buffers through CUDA IPC and pushes each
chunk of its block into them with cudaMemcpyAsync on a side stream while
the next chunk's GEMM runs on all SMs; one-word NCCL all-reduces serve as
device-side barriers.  With layout="blocked" the result is the layer's
exchange buffer and stays valid until the next forward call.

`exchange="fused"` (CUDA GPUs; the default from 2 ranks up) takes the
exchange into the GEMM itself: every rank maps its peers' copies of the full
output [M, N] through CUDA IPC and launches one GEMM whose epilogue writes
each finished tile into all of them (mbs_gemm_a4w4_launch_multi), so the
NVLink traffic runs beside the tensor-core work of the following tiles and
no copy or collective kernel follows the GEMM; two one-word NCCL
all-reduces serve as the device-side barriers around it.  The result is
row-major [M, N] on every rank (layout="blocked" views it as
[world, M, N/world]) and stays valid until the next forward call.

`chunks > 1` (with exchange="nccl") pipelines the exchange with the compute: A is processed in
row chunks, each chunk's GEMM writes straight into this rank's block of the
output, and its rows are exchanged with every peer by NCCL point-to-point
sends/receives (straight into the peers' blocks) while the next chunk's
GEMM runs.  The GEMM then runs on all SMs but `comm_sms`, which the NCCL
kernels need to run alongside it (the GEMM's CTAs fill an SM each).
"""

from __future__ import annotations

import contextlib
from typing import Callable, Optional

import torch
import torch.distributed as dist

SHARD_ALIGN = 256


def _lib_call(name, *args):
    from . import _lib
    return _lib.call(name, *args)


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

    `local_gemm(A_fp4, B, A_scale_shuffled, B_scale, A_factor, B_factor, out=None) -> C`
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
        self._default_gemm = local_gemm is None
        if local_gemm is None or quantize is None:
            from .mbs_gemm_a4w4 import gemm_a4w4
            from .quant import quantize_mxfp4
            local_gemm = local_gemm or gemm_a4w4
            quantize = quantize or (lambda x: quantize_mxfp4(x, shuffle=True))
        self._gemm = local_gemm
        self._quant = quantize
        self._peerbuf = None   # PeerBuffer of the copy exchange, sized on first use
        self._side = None
        self._flag = None

    def local(self, x: torch.Tensor, A_factor: Optional[torch.Tensor] = None) -> torch.Tensor:
        """bf16 x [M, K] -> this rank's bf16 C columns [M, N/world]."""
        q, s = self._quant(x)
        return self._gemm(q, self.B, s, self.B_scale, A_factor, self.B_factor)

    def forward(self, x: torch.Tensor, A_factor: Optional[torch.Tensor] = None,
                layout: str = "blocked", chunks: int = 1, comm_sms: int = 16,
                exchange: str = "nccl") -> torch.Tensor:
        if layout not in ("blocked", "rows"):
            raise ValueError(f"layout must be 'blocked' or 'rows', got {layout!r}")
        if exchange not in ("nccl", "copy", "fused", "auto"):
            raise ValueError(f"exchange must be 'nccl', 'copy', 'fused' or 'auto', got {exchange!r}")
        if exchange == "auto":
            # measured on B200 (config[4]): copy engines win at 2 ranks
            # (2.14 vs 3.73 ms), NCCL's all-gather from 4 ranks up (3.29 vs 3.65 ms)
            exchange = self.default_exchange(x)
            if exchange == "copy" and chunks < 2:
                chunks = self.default_chunks(exchange)
        if exchange == "fused" and self.world > 1:
            return self._forward_fused(x, A_factor, layout)
        if exchange == "copy" and self.world > 1:
            return self._forward_copy(x, A_factor, layout, max(1, chunks))
        if chunks > 1:
            return self._forward_pipelined(x, A_factor, layout, chunks, comm_sms)
        c = self.local(x, A_factor).contiguous()
        M, nl = c.shape
        if self.world == 1:
            # nothing to exchange: the local block is the whole output
            return c.view(1, M, nl) if layout == "blocked" else c
        flat = torch.empty((self.world * M, nl), dtype=c.dtype, device=c.device)
        dist.all_gather_into_tensor(flat, c, group=self.group)
        gathered = flat.view(self.world, M, nl)
        if layout == "blocked":
            return gathered
        if layout == "rows":
            return gathered.permute(1, 0, 2).reshape(M, self.world * nl)
        raise ValueError(f"layout must be 'blocked' or 'rows', got {layout!r}")

    def default_exchange(self, x: torch.Tensor) -> str:
        """The exchange `forward(exchange="auto")` takes: the GEMM-fused one on
        CUDA tensors with peers to exchange with, NCCL otherwise."""
        return "fused" if self.world > 1 and x.is_cuda and self._default_gemm else "nccl"

    @staticmethod
    def default_chunks(exchange: str) -> int:
        return 4 if exchange == "copy" else 1

    def describe_exchange(self, exchange: str, chunks: int) -> str:
        if exchange == "fused":
            return (f"fused into the GEMM: the epilogue stores every output tile into all {self.world} ranks' "
                    f"copies of C (CUDA IPC peer memory over NVLink); NCCL one-word barriers before and after")
        if exchange == "copy":
            return (f"{chunks} row chunks pushed into the peers' buffers by copy engines (CUDA IPC), "
                    f"overlapped with the next chunk's GEMM")
        if chunks > 1:
            return f"{chunks} row chunks, NCCL send/recv overlapped with the next chunk's GEMM"
        return f"NCCL all-gather over {self.world} ranks after the GEMM"

    def close(self):
        """Release the peer buffers (collective: call on every rank once no
        rank uses the layer's results any more)."""
        if self._peerbuf is not None:
            torch.cuda.synchronize(self.B.device)
            self._peerbuf.close()
            self._peerbuf = None

    def _global_rank(self, r: int) -> int:
        return r if self.group is None else dist.get_global_rank(self.group, r)

    def _forward_pipelined(self, x, A_factor, layout, chunks, comm_sms):
        M = int(x.shape[0])
        nl = self.n1 - self.n0
        step = max(32, (-(-M // chunks) + 31) // 32 * 32)  # chunk rows, a multiple of 32
        out = torch.empty((self.world, M, nl), dtype=torch.bfloat16, device=x.device)
        limit = contextlib.nullcontext()
        if x.is_cuda and comm_sms > 0 and self.world > 1 and self._default_gemm:
            from .mbs_gemm_a4w4 import grid_limit
            sms = torch.cuda.get_device_properties(x.device).multi_processor_count
            limit = grid_limit(max(2, sms - comm_sms))
        works = []
        with limit:
            for r0 in range(0, M, step):
                r1 = min(M, r0 + step)
                q, s = self._quant(x[r0:r1])
                fa = None if A_factor is None else A_factor[r0:r1]
                mine = out[self.rank, r0:r1]
                self._gemm(q, self.B, s, self.B_scale, fa, self.B_factor, out=mine)
                ops = []
                for r in range(self.world):
                    if r != self.rank:
                        ops.append(dist.P2POp(dist.isend, mine, self._global_rank(r), group=self.group))
                        ops.append(dist.P2POp(dist.irecv, out[r, r0:r1], self._global_rank(r), group=self.group))
                if ops:
                    works.extend(dist.batch_isend_irecv(ops))
        for w in works:
            w.wait()
        if layout == "blocked":
            return out
        return out.permute(1, 0, 2).reshape(M, self.world * nl)

    def _barrier(self):
        """Barrier between the ranks' streams: on an NCCL group a one-word
        all-reduce, which completes on a rank only after every rank's stream
        has reached it (no host synchronisation); on other groups (gloo: ranks
        that share a GPU, as in the single-GPU tests) the host waits for this
        device's work and then for the other ranks."""
        if dist.get_backend(self.group) == "nccl":
            if self._flag is None:
                self._flag = torch.zeros(1, dtype=torch.int32, device=self.B.device)
            dist.all_reduce(self._flag, group=self.group)
        else:
            torch.cuda.synchronize(self.B.device)
            dist.barrier(group=self.group)

    def _peer_buffer(self, nbytes: int, device: torch.device):
        """The layer's IPC-shared buffer on every rank, (re)allocated collectively."""
        from .peer import PeerBuffer
        if self._peerbuf is None or self._peerbuf.nbytes < nbytes:
            if self._peerbuf is not None:
                torch.cuda.synchronize(device)
                self._barrier()
                torch.cuda.synchronize(device)
                self._peerbuf.close()
            self._peerbuf = PeerBuffer(nbytes, device, self.group)
        return self._peerbuf

    def _forward_fused(self, x, A_factor, layout):
        """One GEMM writes this rank's column block of C into every rank's copy
        of C (its own first, then the peers in rank order after its own, so the
        ranks spread their traffic over different links)."""
        import ctypes

        from . import _lib
        from .mbs_gemm_a4w4 import scale_n_pad, workspace_for
        if not x.is_cuda or not self._default_gemm:
            raise ValueError("exchange='fused' needs CUDA tensors and this package's GEMM")
        M = int(x.shape[0])
        nl = self.n1 - self.n0
        buf = self._peer_buffer(M * self.N * 2, x.device)
        out = buf.tensor((M, self.N))
        q, s = self._quant(x)
        qu, su = q.view(torch.uint8).contiguous(), s.view(torch.uint8).contiguous()
        fa = None if A_factor is None else A_factor.view(torch.uint8).contiguous()
        fb = None if self.B_factor is None else self.B_factor.view(torch.uint8).contiguous()
        order = [(self.rank + i) % self.world for i in range(self.world)]
        dst = (ctypes.c_void_p * self.world)(*[buf.ptrs[r] + self.n0 * 2 for r in order])
        K = self.K
        Mpad = (M + 31) // 32 * 32
        ws = workspace_for(M, nl, K, x.device)
        # nobody may write into a rank's copy of C before that rank is done with
        # the previous result (anything it queued before this call)
        self._barrier()
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.call("mbs_gemm_a4w4_launch_multi", qu.data_ptr(), self.B.data_ptr(), su.data_ptr(),
                  self.B_scale.data_ptr(), None if fa is None else fa.data_ptr(),
                  None if fb is None else fb.data_ptr(), dst, self.world, self.N, M, nl, K, Mpad,
                  scale_n_pad(K), 1.0, None, None if ws is None else ws.data_ptr(),
                  0 if ws is None else ws.numel(), stream)
        self._barrier()  # every rank's GEMM (and with it every store into every copy) has completed
        if layout == "rows":
            return out
        return out.view(M, self.world, nl).permute(1, 0, 2)

    def _forward_copy(self, x, A_factor, layout, chunks):
        """Copy-engine exchange: every chunk's rows go straight into each peer's
        copy of the gathered output (CUDA IPC mapping, cudaMemcpyAsync on a side
        stream), beside the next chunk's GEMM, which keeps every SM."""
        M = int(x.shape[0])
        nl = self.n1 - self.n0
        nbytes = self.world * M * nl * 2
        self._peer_buffer(nbytes, x.device)
        if self._side is None:
            # one side stream: copies to different peers issued on separate
            # streams measured slower at 4 GPUs (4.15 vs 3.65 ms)
            self._side = torch.cuda.Stream(x.device)
        out = self._peerbuf.tensor((self.world, M, nl))
        compute = torch.cuda.current_stream(x.device)
        # nobody may write into a rank's buffer before that rank is done with the
        # previous result (anything it queued before this call)
        self._barrier()
        step = max(32, (-(-M // chunks) + 31) // 32 * 32)
        for r0 in range(0, M, step):
            r1 = min(M, r0 + step)
            q, s = self._quant(x[r0:r1])
            fa = None if A_factor is None else A_factor[r0:r1]
            mine = out[self.rank, r0:r1]
            self._gemm(q, self.B, s, self.B_scale, fa, self.B_factor, out=mine)
            self._side.wait_stream(compute)
            off = (self.rank * M + r0) * nl * 2
            for r in range(self.world):
                if r != self.rank:
                    _lib_call("mbs_copy_async", self._peerbuf.ptrs[r] + off, mine.data_ptr(), (r1 - r0) * nl * 2,
                              self._side.cuda_stream)
        with torch.cuda.stream(self._side):
            self._barrier()  # every rank's copies into every buffer are complete
        compute.wait_stream(self._side)
        if layout == "blocked":
            return out  # the layer's exchange buffer: valid until the next forward call
        return out.permute(1, 0, 2).reshape(M, self.world * nl)

    __call__ = forward
