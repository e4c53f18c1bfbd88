"""torchrun worker for tests/test_sharded.py: one rank per GPU, NCCL.

Builds a seeded weight, shards it, runs the sharded forward (quantise A on
each rank, local GEMM, exchange of the C shards: NCCL all-gather, NCCL
send/recv, copy engines, or stores into the peers' copies from the GEMM's
epilogue) and checks the gathered C against the CPU oracle on a sample of
columns from every shard.  Prints SHARDED_OK per rank.
"""

import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import mbs_b200  # noqa: E402
from mbs_b200.sharded import ShardedA4W4, shard_weight  # noqa: E402
from oracle import mxfp4_oracle as O  # noqa: E402


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        M, N, K = 96, 512 * world, 1024
        g = torch.Generator().manual_seed(1234)  # identical on every rank
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        wq, ws = O.quantize_mxfp4(bits(w))
        xq, xs = O.quantize_mxfp4(bits(x))
        Bsh = torch.from_numpy(O.shuffle_weight(wq))
        Ssh = torch.from_numpy(O.shuffle_scales(ws, K))
        b, s = shard_weight(Bsh, Ssh, N, K, world, rank)
        layer = ShardedA4W4(b.cuda(), s.cuda(), N, K)
        cols = np.concatenate([np.arange(r * N // world, r * N // world + 64) for r in range(world)])
        ref = O.gemm_ref(xq, wq[cols], xs, ws[cols])
        bound = O.gemm_abs_bound(xq, wq[cols], xs, ws[cols])
        # one all-gather, the pipelined point-to-point exchange, the copy-engine
        # exchange through peer memory (twice, reusing its buffer) and the exchange
        # fused into the GEMM's epilogue (twice, reusing its buffer)
        for exchange, chunks in (("nccl", 1), ("nccl", 3), ("copy", 1), ("copy", 3), ("copy", 3),
                                 ("fused", 1), ("fused", 1)):
            out = layer(x.cuda(), layout="rows", chunks=chunks, exchange=exchange)
            torch.cuda.synchronize()
            got = out[:, torch.from_numpy(cols).cuda()].float().cpu().numpy()
            ok, ratio, nbad = O.check_gemm(got, ref, bound)
            assert ok, f"rank {rank} {exchange} chunks {chunks}: {nbad} bad elements (max ratio {ratio})"
            blocked = layer(x.cuda(), layout="blocked", chunks=chunks, exchange=exchange)
            torch.cuda.synchronize()
            assert torch.equal(blocked.permute(1, 0, 2).reshape(M, N), out), f"{exchange} blocked vs rows"
        dist.barrier()
        if layer._peerbuf is not None:
            torch.cuda.synchronize()
            dist.barrier()
            layer._peerbuf.close()
        print(f"SHARDED_OK rank={rank} world={world}", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
