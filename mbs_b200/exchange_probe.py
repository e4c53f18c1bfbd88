"""Rate at which one GEMM's epilogue stores reach another GPU (the GEMM-fused
exchange of the N-sharded layer, mbs_gemm_a4w4_launch_multi).

    python -m torch.distributed.run --nproc-per-node 2 -m mbs_b200.exchange_probe

Two ranks, each running the config[4] shard GEMM of an 8-GPU layer
(16384 x 7168 x 8192) with its output written to its own buffer plus
copies - 1 copies in the other rank's buffer (CUDA IPC), for copies = 1, 2,
4, 8, both ranks at once (traffic in both directions, as in the layer).
Prints one JSON line: per copy count the time per call (CUDA events, max
over ranks) and the outbound GB/s of peer stores, (copies - 1) x M x N x 2
bytes per call.  With 7 peer copies the GEMM is store-bound, so that figure
is the NVLink rate this store path reaches.
"""

from __future__ import annotations

import ctypes
import json
import os
from datetime import timedelta


def main():
    import torch
    import torch.distributed as dist

    from . import _lib, quantize_mxfp4, shuffle_scales, shuffle_weight
    from .mbs_gemm_a4w4 import scale_n_pad, workspace_for
    from .peer import PeerBuffer

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != 2:
        raise SystemExit("run with exactly 2 ranks")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    M, nl, K = 16384, 7168, 8192
    g = torch.Generator(device=dev).manual_seed(rank)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(nl, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    qa, sa = quantize_mxfp4(x, shuffle=True)
    qw, sw = quantize_mxfp4(w, shuffle=False)
    B, Bs = shuffle_weight(qw), shuffle_scales(sw, K)
    del x, w, qw, sw
    ldc = 16 * nl  # room for 8 column blocks per rank
    buf = PeerBuffer(M * ldc * 2, dev)
    peer = 1 - rank
    L = _lib.lib()
    ws = workspace_for(M, nl, K, dev)
    res = {}
    for n in (1, 2, 4, 8):
        ptrs = [buf.ptrs[rank] + rank * 8 * nl * 2] + [buf.ptrs[peer] + (rank * 8 + j) * nl * 2 for j in range(1, n)]
        dst = (ctypes.c_void_p * n)(*ptrs)

        def call():
            _lib.check("mbs_gemm_a4w4_launch_multi", L.mbs_gemm_a4w4_launch_multi(
                qa.data_ptr(), B.data_ptr(), sa.data_ptr(), Bs.data_ptr(), None, None, dst, n, ldc, M, nl, K, M,
                scale_n_pad(K), ctypes.c_float(1.0), None, None if ws is None else ws.data_ptr(),
                0 if ws is None else ws.numel(), torch.cuda.current_stream().cuda_stream))
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            call()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / 10], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        res[n] = {"ms": round(ms, 4), "peer_store_gbs": round((n - 1) * M * nl * 2 / (ms * 1e-3) / 1e9, 1)}
    torch.cuda.synchronize()
    dist.barrier()
    buf.close()
    dist.barrier()
    if rank == 0:
        print(json.dumps({"probe": "GEMM epilogue stores into a peer", "shape": [M, nl, K], "copies": res}),
              flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
