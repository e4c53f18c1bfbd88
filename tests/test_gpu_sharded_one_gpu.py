"""The N-sharded layer's exchanges through peer memory, run by two ranks that
share one GPU (a gloo group; the layer's barriers then synchronise on the
host).  The GEMM-fused exchange (each rank's GEMM stores its tiles into both
ranks' copies of C through CUDA IPC mappings) and the copy-engine exchange
need no NCCL in their data path, so this runs wherever one GPU is visible,
which the multi-GPU worker (tests/sharded_worker.py) needs two for.  No
kernel waits on another rank: the ranks only meet at host barriers.  Every
rank checks the whole gathered C against the CPU oracle on sampled columns
of both shards, and that both ranks hold the same bytes."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    sys.path.insert(0, REPO)
    import torch.distributed as dist

    from mbs_b200.sharded import ShardedA4W4, shard_weight
    from oracle import mxfp4_oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M, N, K = 300, 512 * world, 1024
        g = torch.Generator().manual_seed(4321)  # identical on every rank
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        wq, ws = O.quantize_mxfp4(bits(w))
        xq, xs = O.quantize_mxfp4(bits(x))
        b, s = shard_weight(torch.from_numpy(O.shuffle_weight(wq)), torch.from_numpy(O.shuffle_scales(ws, K)),
                            N, K, world, rank)
        layer = ShardedA4W4(b.cuda(), s.cuda(), N, K)
        cols = np.concatenate([np.arange(r * N // world, r * N // world + 96) for r in range(world)])
        ref = O.gemm_ref(xq, wq[cols], xs, ws[cols])
        bound = O.gemm_abs_bound(xq, wq[cols], xs, ws[cols])
        res = []
        for exchange, chunks in (("fused", 1), ("fused", 1), ("copy", 3)):
            out = layer(x.cuda(), layout="rows", chunks=chunks, exchange=exchange)
            torch.cuda.synchronize()
            got = out[:, torch.from_numpy(cols).cuda()].float().cpu().numpy()
            ok, ratio, nbad = O.check_gemm(got, ref, bound)
            digest = int(out.view(torch.int16).to(torch.int64).sum().item())
            res.append((exchange, bool(ok), float(ratio), int(nbad), digest))
            dist.barrier()
        layer.close()
        dist.barrier()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_peer_memory_exchanges_with_two_ranks_on_one_gpu(cuda_ok):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, res in results.items():
        for exchange, ok, ratio, nbad, _ in res:
            assert ok, f"rank {rank} {exchange}: {nbad} elements outside the oracle tolerance (max ratio {ratio})"
    for i in range(len(results[0])):
        assert results[0][i][4] == results[1][i][4], f"ranks hold different C after {results[0][i][0]}"
