"""Per-call time of gemm_a4w4 on a list of shapes.

    python -m mbs_b200.bench_shapes [--shapes MxNxK,...] [--calls 20] [--reps 5]

Two numbers per shape, one JSON line each:
  * `b2b_us`: `--calls` calls captured in one CUDA graph and replayed back to
    back with the operands hot in L2, CUDA events around the replay, divided
    by the number of calls (median of `--reps` replays) -- how the
    reference's tuning log times its kernels (asm_vs_wg_kernel.md:179-182);
  * `one_call_us`: one call after a 256 MB write that evicts L2, events
    around the call (median of `--reps`).

The default shapes are the ones the reference publishes MI355X numbers for
(asm_vs_wg_kernel.md:191-196).  Operands: seeded N(0,1) bf16 quantised to
MXFP4 on the device (weights N(0,0.02) for M <= 64), factors off.
"""

from __future__ import annotations

import argparse
import json
import statistics

REFERENCE_SHAPES = "8192x17408x5120,8192x5120x17408,8192x10240x5120,8192x12288x5120,1024x17408x5120,1024x1024x5120"


def make_operands(M: int, N: int, K: int, seed: int, device):
    import torch

    from . import quantize_mxfp4, shuffle_scales, shuffle_weight

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=device, generator=g) * (0.02 if M <= 64 else 1.0)).to(torch.bfloat16)
    qa, sa = quantize_mxfp4(x, shuffle=True)
    qw, sw = quantize_mxfp4(w, shuffle=False)
    return qa, shuffle_weight(qw), sa, shuffle_scales(sw, K)


def time_shape(M: int, N: int, K: int, calls: int, reps: int) -> dict:
    import torch

    from . import gemm_a4w4

    dev = torch.device("cuda")
    A, B, As, Bs = make_operands(M, N, K, 0, dev)
    out = torch.empty(((M + 31) // 32 * 32, N), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def call():
        gemm_a4w4(A, B, As, Bs, out=out)

    for _ in range(3):
        call()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(calls):
            call()
    graph.replay()
    torch.cuda.synchronize()
    b2b = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        b2b.append(e0.elapsed_time(e1) * 1e3 / calls)
    del graph
    one = []
    for r in range(reps):
        flush.fill_(r & 0xFF)
        torch.cuda._sleep(200000)  # the host queues the call while the GPU is busy
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        call()
        e1.record()
        torch.cuda.synchronize()
        one.append(e0.elapsed_time(e1) * 1e3)
    t_b2b, t_one = statistics.median(b2b), statistics.median(one)
    flop = 2.0 * M * N * K
    return {"shape": f"{M}x{N}x{K}", "b2b_us": round(t_b2b, 2), "b2b_tflops": round(flop / t_b2b / 1e6, 1),
            "one_call_us": round(t_one, 2), "calls": calls, "reps": reps}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--shapes", default=REFERENCE_SHAPES, help="comma-separated MxNxK list")
    ap.add_argument("--calls", type=int, default=20)
    ap.add_argument("--reps", type=int, default=5)
    a = ap.parse_args()
    for s in a.shapes.split(","):
        M, N, K = (int(v) for v in s.split("x"))
        print(json.dumps(time_shape(M, N, K, a.calls, a.reps)), flush=True)


if __name__ == "__main__":
    main()
