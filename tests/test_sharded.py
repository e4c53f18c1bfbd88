"""N-sharded path: host logic on CPU (gloo, world size 2) and, on GPUs, the
NCCL all-gather of real shards (run by tests/sharded_worker.py under torchrun)."""

import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import mxfp4_oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shard_rows_and_alignment():
    from mbs_b200.sharded import shard_rows
    assert shard_rows(57344, 8, 3) == (21504, 28672)
    assert shard_rows(1024, 2, 1) == (512, 1024)
    with pytest.raises(ValueError):
        shard_rows(1024, 3, 0)
    with pytest.raises(ValueError):
        shard_rows(768, 2, 0)  # 384-row shards are not multiples of 256


def test_shard_is_a_byte_range_of_both_layouts():
    """Slicing the preshuffled weight and shuffled scales equals shuffling the
    sliced plain weight: sharding needs no re-layout."""
    from mbs_b200.sharded import shard_weight
    rng = np.random.default_rng(0)
    N, K, world = 1024, 512, 4
    w = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    s = rng.integers(100, 140, size=(N, K // 32), dtype=np.uint8)
    Bsh = torch.from_numpy(O.shuffle_weight(w))
    Ssh = torch.from_numpy(O.shuffle_scales(s, K))
    for r in range(world):
        b, sc = shard_weight(Bsh, Ssh, N, K, world, r)
        n0, n1 = r * N // world, (r + 1) * N // world
        assert np.array_equal(b.numpy(), O.shuffle_weight(w[n0:n1]))
        assert np.array_equal(sc.numpy().reshape(-1), O.shuffle_scales(s[n0:n1], K).reshape(-1))


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _gloo_worker(rank, world, port, M, N, K, q):
    import torch.distributed as dist

    from mbs_b200.sharded import ShardedA4W4, shard_weight
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(7)  # same weights on every rank
        xq = rng.integers(0, 256, size=(M, K // 2), dtype=np.uint8)
        xs = rng.integers(120, 134, size=(M, K // 32), dtype=np.uint8)
        w = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
        ws = rng.integers(120, 134, size=(N, K // 32), dtype=np.uint8)
        Bsh, Ssh = shard_weight(torch.from_numpy(O.shuffle_weight(w)),
                                torch.from_numpy(O.shuffle_scales(ws, K)), N, K, world, rank)

        # CPU stand-ins for the CUDA operators: the oracle on unshuffled bytes
        def quant(x):
            r0 = int(x.data_ptr() - base.data_ptr()) // (x.element_size() * K)  # row offset of the view
            rows = x.shape[0]
            return (torch.from_numpy(xq[r0:r0 + rows].copy()),
                    torch.from_numpy(O.shuffle_scales(xs[r0:r0 + rows], K)))

        def gemm(A, B, As, Bs, Af, Bf, out=None):
            nl = B.shape[0]
            rows = A.shape[0]
            bp = O.unshuffle_weight(B.numpy())
            bs = O.unshuffle_scales(Bs.numpy(), nl, K)
            a_s = O.unshuffle_scales(As.numpy(), rows, K)
            c = torch.from_numpy(O.gemm_ref(A.numpy(), bp, a_s, bs)).to(torch.bfloat16)
            if out is not None:
                out.copy_(c)
                return out
            return c

        base = torch.zeros(M, K)
        layer = ShardedA4W4(Bsh, Ssh, N, K, local_gemm=gemm, quantize=quant)
        ref = O.gemm_ref(xq, w, xs, ws)
        res = []
        for chunks in (1, 3):
            out_rows = layer(base, layout="rows", chunks=chunks)
            out_blocked = layer(base, layout="blocked", chunks=chunks)
            res.append((np.array_equal(out_rows.float().numpy(), ref), tuple(out_blocked.shape),
                        np.array_equal(out_blocked[rank].float().numpy(),
                                       ref[:, rank * N // world:(rank + 1) * N // world]),
                        all(np.array_equal(out_blocked[r].float().numpy(),
                                           ref[:, r * N // world:(r + 1) * N // world]) for r in range(world))))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_sharded_allgather_on_gloo_world2():
    M, N, K, world = 80, 512, 128, 2   # 3 chunks of 32, 32 and 16 rows
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, M, N, K, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, res in results:
        for chunks, (rows_ok, bshape, block_ok, all_ok) in zip((1, 3), res):
            assert rows_ok, f"rank {rank} chunks {chunks}: row-major gather differs from the oracle"
            assert bshape == (world, M, N // world) and block_ok and all_ok, f"rank {rank} chunks {chunks}"


@pytest.mark.gpu
def test_sharded_nccl_on_available_gpus():
    """Runs tests/sharded_worker.py with one rank per visible GPU (at least 1):
    every rank checks its gathered C against the oracle on sampled columns."""
    n = torch.cuda.device_count()
    assert n >= 1
    port = _free_port()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(REPO, "tests", "sharded_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert res.stdout.count("SHARDED_OK") == n, res.stdout[-2000:]
