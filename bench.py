"""Benchmark of the MXFP4 A4W4 GEMM (BASELINE.json metric: TFLOPS at 8192^3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mbs|reference]
                    [--workload prefill|decode] [--m M]

One step = one gemm_a4w4 call on the workload (default: BASELINE config[2],
M = N = K = 8192, MXFP4 A and B quantised from seeded N(0,1) bf16, bf16 out).
`value` is device-timed (CUDA events on the launching stream) with inputs
resident in HBM; prefill flushes L2 before every step, decode (whose weights
alone exceed L2) replays its K steps back to back from one CUDA graph with
events around all of them (the reference's bench_one.py:34-47 also times
back-to-back iterations), and also reports one isolated
call after a flush (`isolated_call`); `e2e` times the public
operator with host (pinned) operands copied in and the result copied out
inside the timed region.  Under torchrun every rank runs its own workload
(weak scaling: replicas, no collective in the timed region) and the JSON
line reports the max time over ranks.

The default line carries three more measurements beside the headline:
`decode` (config[1], M = 1/4/16/32: HBM GB/s per call back to back from a
CUDA graph, eager back to back as bench_one.py:34-47 times, and one call
after an L2 flush) and `configs` (config[0] per call, config[3] TFLOPS), both
on one GPU only, and `sharded` on every rank count (config[4]: quantise +
N-sharded GEMM + exchange of the C shards so every rank holds all of C;
strong scaling, max over ranks, with parity against the oracle on each
rank's shard and checksums of the exchanged blocks).

`--impl reference` times the reference's CPU path (the dequantise-then-matmul
oracle of test_gemm_a4w4.py:28-44, restated in oracle/) on the host cores on
a bounded row sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

FP4_PER_BF16 = 4.0  # dense FP4 : BF16 tensor throughput on B200 (9 : 2.25 PFLOP/s nominal)
L2_FLUSH_BYTES = 256 << 20
L2_BYTES = 126 * 1000 * 1000  # B200 L2

THROTTLE_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["mbs", "reference"], default="mbs")
    ap.add_argument("--workload", choices=["prefill", "decode", "decode-fused", "sharded"], default="prefill",
                    help="decode-fused: config[1] from bf16 activations, quantised inside the GEMM "
                         "(quant_gemm_a4w4)")
    ap.add_argument("--m", type=int, default=None, help="M for --workload decode (default 16)")
    ap.add_argument("--packed", action="store_true",
                    help="decode workloads: the weights in the one-time packed layout (gemm_a4w4_packed, "
                         "or quant_gemm_a4w4_packed from bf16 activations, up to 16 rows)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--chunks", type=int, default=None,
                    help="--workload sharded: row chunks whose exchange overlaps the next chunk's GEMM "
                         "(default 4 on more than one GPU, 1 on one)")
    ap.add_argument("--exchange", choices=["nccl", "copy", "fused", "auto"], default="auto",
                    help="config[4]: exchange the C shards with NCCL, with copy engines through peer "
                         "memory, inside the GEMM's epilogue (fused), or auto (fused from 2 GPUs up)")
    ap.add_argument("--comm-sms", type=int, default=16,
                    help="--workload sharded with chunks > 1: SMs left free for the NCCL kernels")
    ap.add_argument("--skip-extras", action="store_true",
                    help="skip the e2e and CPU-baseline legs (profiling runs)")
    ap.add_argument("--no-extra-configs", action="store_true",
                    help="skip the decode, other-config and sharded objects of the default line")
    ap.add_argument("--sharded-steps", type=int, default=10)
    ap.add_argument("--soak-s", type=float, default=1.5,
                    help="seconds of untimed steps right before the timed region, so the "
                         "clock sampler sees the GPU under this load")
    args = ap.parse_args()
    if args.packed and args.workload not in ("decode", "decode-fused"):
        ap.error("--packed applies to --workload decode and decode-fused")
    if args.packed and args.workload == "decode-fused" and (args.m or 16) > 16:
        ap.error("--packed with decode-fused: one launch per call up to M = 16")
    return args


def workload_shape(args):
    packed = " with packed weights" if getattr(args, "packed", False) else ""
    if args.workload == "decode":
        M = args.m or 16
        return M, 57344, 8192, f"cfg1 decode M={M} N=57344 K=8192 (Llama-3-70B gate+up){packed}"
    if args.workload == "decode-fused":
        M = args.m or 16
        op = "quant_gemm_a4w4_packed" if packed else "quant_gemm_a4w4"
        return M, 57344, 8192, (f"cfg1 decode M={M} N=57344 K=8192 from bf16 activations, quantised inside "
                                f"the GEMM ({op}){packed}")
    return 8192, 8192, 8192, "cfg2 prefill M=N=K=8192"


def load_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d, "MEASURED_PEAKS.json"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 4:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
                bits = int(parts[3], 16) if parts[3].startswith("0x") else int(parts[3])
            except ValueError:
                continue
            for b, name in THROTTLE_BITS.items():
                if bits & b and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def load_traffic(workload, M):
    """DRAM bytes per launch of the main kernel from the committed ncu summary
    (profiles/traffic.json: dram__bytes_read.sum + dram__bytes_write.sum)."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            d = json.load(f)
        key = {"prefill": "prefill_8192", "decode": f"decode_m{M}", "decode-fused": f"decode_fused_m{M}",
               "decode-packed": f"decode_packed_m{M}",
               "decode-fused-packed": f"decode_fused_packed_m{M}"}.get(workload)
        return d.get(key) if key else None
    except (OSError, ValueError):
        return None


def dist_setup(args):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def make_inputs(M, N, K, seed, device):
    import torch

    import mbs_b200
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(M, K, device=device, generator=g).to(torch.bfloat16)
    std = 0.02 if M <= 64 else 1.0
    w = (torch.randn(N, K, device=device, generator=g) * std).to(torch.bfloat16)
    qa, sa = mbs_b200.quantize_mxfp4(x, shuffle=True)
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    del x, w
    B = mbs_b200.shuffle_weight(qw)
    Bs = mbs_b200.shuffle_scales(sw, K)
    del qw, sw
    return qa, B, sa, Bs


def run_mbs(args):
    import torch
    import torch.distributed as dist

    import mbs_b200
    from mbs_b200 import _lib

    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", local)
    M, N, K, wl_name = workload_shape(args)
    A, B, As, Bs = make_inputs(M, N, K, seed=1234 + rank, device=dev)
    x_bf16 = None
    if args.workload == "decode-fused":
        x_bf16 = torch.randn(M, K, device=dev, generator=torch.Generator(device=dev).manual_seed(5)).to(
            torch.bfloat16)
    packed_w = mbs_b200.pack_weight(B, Bs) if args.packed else None
    out = torch.empty(((M + 31) // 32 * 32, N), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    flush_rd = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)

    def flush_l2(i):
        # write a buffer larger than L2 (126 MB), then read another one so the
        # dirty lines are written back here rather than inside the timed step
        flush.fill_(i)
        flush_rd.sum()
    stream = torch.cuda.current_stream(dev)

    def step():
        if x_bf16 is not None and packed_w is not None:
            mbs_b200.quant_gemm_a4w4_packed(x_bf16, packed_w, out=out)
        elif x_bf16 is not None:
            mbs_b200.quant_gemm_a4w4(x_bf16, B, Bs, out=out)
        elif packed_w is not None:
            mbs_b200.gemm_a4w4_packed(A, packed_w, As, out=out)
        else:
            mbs_b200.gemm_a4w4(A, B, As, Bs, out=out)

    # Decode: the weights alone are larger than L2, so steps run back to back
    # with events around all of them (the reference's bench_one.py:34-47 times
    # this way); every other workload flushes L2 before each timed step.
    w_bytes = N * K // 2 + N * K // 32
    b2b = args.workload != "prefill" and w_bytes > L2_BYTES

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    # events the library records around the main GEMM kernel of each step
    k_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    k_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for ev in k_starts + k_ends:
        ev.record(stream)  # materialise the CUDA events
    torch.cuda.synchronize()
    L = _lib.lib()
    graph = None
    if b2b:
        # the K back-to-back steps replay from one CUDA graph, so host-side
        # launch cost cannot starve the GPU between them
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                step()
        graph.replay()
        torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        # untimed soak: keeps the GPU under this load while the sampler starts
        t_soak = time.perf_counter() + (0.0 if args.skip_extras else args.soak_s)
        while time.perf_counter() < t_soak:
            for _ in range(20):
                flush_l2(0)
                step()
            if graph is not None:
                graph.replay()
            torch.cuda.synchronize()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t_wall = time.perf_counter()
        if b2b:
            starts[0].record(stream)
            graph.replay()
            ends[0].record(stream)
        else:
            for i in range(args.steps):
                flush_l2(i)  # evict the operands from L2 before every timed step
                L.mbs_set_profile_events(k_starts[i].cuda_event, k_ends[i].cuda_event)
                starts[i].record(stream)
                step()
                ends[i].record(stream)
        L.mbs_set_profile_events(None, None)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t_wall = time.perf_counter() - t_wall
        if not args.skip_extras:
            time.sleep(0.25)  # let the sampler record the end of the timed region
    launches = launches_per_call(M, N, K)
    if b2b:
        total_ms = starts[0].elapsed_time(ends[0])
        kernel_ms = total_ms / args.steps  # one GEMM kernel per step, back to back
        assert launches == 1, "back-to-back timing assumes one kernel per call"
    else:
        total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
        kernel_ms = sum(s.elapsed_time(e) for s, e in zip(k_starts, k_ends)) / args.steps
    isolated = None
    if b2b and not args.skip_extras:
        # beside the headline: one call at a time after an L2 flush (median of 5)
        iso = []
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for i in range(5):
            flush_l2(i)
            L.mbs_set_profile_events(k_starts[0].cuda_event, k_ends[0].cuda_event)
            c0.record(stream)
            step()
            c1.record(stream)
            L.mbs_set_profile_events(None, None)
            torch.cuda.synchronize()
            iso.append((c0.elapsed_time(c1), k_starts[0].elapsed_time(k_ends[0])))
        iso.sort()
        isolated = {"call_ms": round(iso[2][0], 5), "kernel_ms": round(iso[2][1], 5),
                    "what": "one call after an L2 flush, events around the call and around its kernel"}
    if world > 1:
        t = torch.tensor([total_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms = total_ms / args.steps
    flops = 2.0 * M * N * K
    value = world * flops * args.steps / (total_ms * 1e-3) / 1e12
    kernel_tflops = flops / (kernel_ms * 1e-3) / 1e12  # main GEMM kernel alone

    if args.skip_extras:
        if rank == 0:
            print(json.dumps({"metric": "profiling run", "ms_per_step": ms, "kernel_ms": kernel_ms,
                              "kernel_tflops": kernel_tflops}), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    # e2e: public operator on host operands (pinned), copies inside the timed
    # region.  Consecutive steps alternate between two streams, each with its
    # own device and host buffers, so one step's result copy (device to host)
    # overlaps the next step's operand copies (host to device) on the other
    # copy engine, as a serving loop would run them.
    # the same operator as the timed step: activations (quantised, or bf16 for
    # the dynamic-quant call) and weights (preshuffled, or packed) from the host
    acts = [x_bf16] if x_bf16 is not None else [A, As]
    wts = [packed_w.data] if packed_w is not None else [B, Bs]
    hosts = [t.cpu().pin_memory() for t in acts + wts]
    n_act = len(acts)
    lanes = []
    for _ in range(2):
        lanes.append({
            "stream": torch.cuda.Stream(dev),
            "dev": [torch.empty_like(t, device=dev) for t in hosts],
            "out": torch.empty(((M + 31) // 32 * 32, N), dtype=torch.bfloat16, device=dev),
            "hout": torch.empty((M, N), dtype=torch.bfloat16).pin_memory(),
        })

    def e2e_step(i):
        ln = lanes[i % 2]
        with torch.cuda.stream(ln["stream"]):
            for d, h in zip(ln["dev"], hosts):
                d.copy_(h, non_blocking=True)
            da, dw = ln["dev"][:n_act], ln["dev"][n_act:]
            pw = mbs_b200.PackedWeight(dw[0], N, K) if packed_w is not None else None
            if x_bf16 is not None:
                o = (mbs_b200.quant_gemm_a4w4_packed(da[0], pw, out=ln["out"]) if pw is not None
                     else mbs_b200.quant_gemm_a4w4(da[0], dw[0], dw[1], out=ln["out"]))
            else:
                o = (mbs_b200.gemm_a4w4_packed(da[0], pw, da[1], out=ln["out"]) if pw is not None
                     else mbs_b200.gemm_a4w4(da[0], dw[0], da[1], dw[1], out=ln["out"]))
            ln["hout"].copy_(o, non_blocking=True)

    e2e_step(0)
    e2e_step(1)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for ln in lanes:
        ln["stream"].wait_event(ev0)
    for i in range(args.e2e_steps):
        e2e_step(i)
    for ln in lanes:
        stream.wait_stream(ln["stream"])
    ev1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = ev0.elapsed_time(ev1) / args.e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    hout = lanes[0]["hout"]
    h2d = sum(t.numel() * t.element_size() for t in hosts)
    d2h = hout.numel() * hout.element_size()

    peaks, src = load_peaks()
    traffic = load_traffic(args.workload + ("-packed" if args.packed else ""), M)
    if args.workload == "prefill":
        # MEASURED_PEAKS.json holds no FP4 figure: the denominator is the mxf4
        # tensor-pipe rate measured here by the probe (the prefill kernel's own
        # instruction, operands resident, no memory traffic); 4 x the measured
        # bf16 cuBLAS rate is reported beside it
        from mbs_b200.probe import mxf4_peak_probe
        pr = mxf4_peak_probe(groups=20000, device=dev)
        peak = float(pr["tflops"])
        peak4 = FP4_PER_BF16 * float(peaks["bf16_tflops"])
        roof = {"bound": "tensor", "achieved": round(kernel_tflops, 2), "peak": round(peak, 1),
                "unit": "TFLOP/s", "frac": round(kernel_tflops / peak, 4), "traffic": traffic,
                "peak_source": "measured this run: mbs_mxf4_peak_probe (back-to-back 256x256x64 "
                               "tcgen05 kind::mxf4 pair MMAs, operands resident in shared memory)",
                "peak_probe": {"tflops": round(peak, 1), "sm_mhz": round(pr["sm_mhz"], 1),
                               "cycles_per_mma": round(pr["cycles_per_mma"], 2)},
                "peak_4x_bf16": {"tflops": round(peak4, 1), "frac": round(kernel_tflops / peak4, 4),
                                 "source": f"4 x bf16_tflops of {src} (dense FP4:BF16 = 4:1)"},
                "kernel_ms": round(kernel_ms, 5)}
    else:
        # weights + their scales + activations (fp4 + scales, or bf16 when quantised in the GEMM) + bf16 out
        a_bytes = M * K * 2 if args.workload == "decode-fused" else M * K // 2 + M * K // 32
        nbytes = N * K // 2 + N * K // 32 + a_bytes + M * N * 2
        gbs = nbytes / (kernel_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(gbs, 1), "peak": float(peaks["hbm_gbs"]),
                "unit": "GB/s", "frac": round(gbs / float(peaks["hbm_gbs"]), 4), "traffic": traffic,
                "peak_source": src, "algorithmic_bytes": nbytes, "kernel_ms": round(kernel_ms, 5)}
    line = {
        "metric": "A4W4 MXFP4 GEMM TFLOPS" if args.workload == "prefill"
                  else "A4W4 MXFP4 GEMM decode TFLOPS",
        "value": round(value, 2), "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "e2m1 (fp32 accumulate, bf16 out)",
        "data": "synthetic (seeded N(0,1) bf16 quantised to MXFP4 on device)",
        "config": {"workload": wl_name, "M": M, "N": N, "K": K,
                   "l2": (f"weights ({w_bytes} B) larger than L2: steps back to back (one CUDA graph of the K "
                          "steps), events around all of them"
                          if b2b else "flushed before every step (256 MB write + 256 MB read)"),
                   "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
        "roofline": roof,
        "clocks": clk.summary(),
        "e2e": {"value": round(world * flops / (e2e_ms * 1e-3) / 1e12, 3), "unit": "TFLOPS",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": round(e2e_ms, 4)},
        "gpu_launches": args.steps * launches,
        "wall_s": round(t_wall, 3),
    }
    if isolated is not None:
        line["isolated_call"] = isolated
    if rank == 0 and world == 1:
        line["cpu_baseline"] = cpu_baseline(M, N, K)
    if args.workload == "prefill" and not args.no_extra_configs:
        del A, B, As, Bs, out, flush, flush_rd, lanes, hosts, acts, wts
        torch.cuda.empty_cache()
        if world == 1:
            line["decode"] = decode_object(dev, peaks)
            line["configs"] = configs_object(dev)
        line["sharded"] = sharded_object(args, world, rank, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    del _lib


def launches_per_call(M, N, K):
    """Kernels one gemm_a4w4 call launches (the library's own plan: the GEMM,
    plus the scale-image kernel on the CTA-pair path)."""
    from mbs_b200 import _lib
    return int(_lib.lib().mbs_gemm_a4w4_kernels_per_call(M, N, K))


def _cpu_sample(M, N, K, rows, seed=0):
    """Oracle inputs for a row sample of the workload (random fp4 codes/scales)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    qa = rng.integers(0, 256, size=(rows, K // 2), dtype=np.uint8)
    qb = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    sa = rng.integers(120, 130, size=(rows, K // 32), dtype=np.uint8)
    sb = rng.integers(120, 130, size=(N, K // 32), dtype=np.uint8)
    return qa, qb, sa, sb


def _cpu_call_s(M, N, K, rows, cols, reps=2):
    """Host seconds one full-size call of the oracle port (the reference's CPU
    path) takes, timed on a sample of `rows` rows of A against `cols` rows of
    B (best of `reps`) and scaled by (M / rows) * (N / cols): the dequantise
    and matmul costs are linear in both.  Returns (seconds, sample text)."""
    from oracle import mxfp4_oracle as O
    rows, cols = min(M, rows), min(N, cols)
    qa, qb, sa, sb = _cpu_sample(M, cols, K, rows)
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        O.gemm_ref(qa, qb, sa, sb)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    scale = (M / rows) * (N / cols)
    return best * scale, f"{rows} of {M} rows x {cols} of {N} columns, scaled x{scale:.0f}, best of {reps}"


def cpu_baseline(M, N, K, budget_s=20.0):
    """The oracle's dequantise-then-matmul on the host cores, on a row sample of A."""
    from oracle import mxfp4_oracle as O
    rows = min(M, 512)
    qa, qb, sa, sb = _cpu_sample(M, N, K, rows)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        O.gemm_ref(qa, qb, sa, sb)
        times.append(time.perf_counter() - t0)
    best = min(times)
    return {"value": round(2.0 * rows * N * K / best / 1e12, 5), "unit": "TFLOPS",
            "cores": os.cpu_count(), "kind": "port",
            "sample": f"{rows} of {M} rows of A against all of B (dequant + fp32 matmul + bf16 "
                      f"cast), best of {len(times)}"}


def _events(n):
    import torch
    return [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]


def _per_call_us(call, flush_fn, steps=20, reps=3, eager_iters=50):
    """Three per-call times of one operator call (microseconds):
    graph  -- `steps` calls captured in one CUDA graph, replayed back to back
              (median of `reps` replays): the launch cost overlaps the
              previous call, as in a serving step;
    eager  -- bench_one.py:34-47's method: 10 warm-up calls, then events
              around `eager_iters` back-to-back eager calls;
    isolated -- one call after an L2 flush, events around it (median of 5)."""
    import torch
    stream = torch.cuda.current_stream()
    for _ in range(10):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(eager_iters):
        call()
    e1.record(stream)
    torch.cuda.synchronize()
    eager = e0.elapsed_time(e1) * 1e3 / eager_iters
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(steps):
            call()
    graph.replay()
    torch.cuda.synchronize()
    g = []
    for _ in range(reps):
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        g.append(e0.elapsed_time(e1) * 1e3 / steps)
    del graph
    iso = []
    for i in range(5):
        flush_fn(i)
        torch.cuda._sleep(100000)  # the host queues the call while the GPU is still busy
        e0.record(stream)
        call()
        e1.record(stream)
        torch.cuda.synchronize()
        iso.append(e0.elapsed_time(e1) * 1e3)
    return statistics.median(g), eager, statistics.median(iso)


def _flusher(dev):
    import torch
    buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    rd = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)

    def flush(i):
        buf.fill_(i)
        rd.sum()
    return flush


def _two_calls(mbs_b200, x, B, Bs, out):
    q, s = mbs_b200.quantize_mxfp4(x, shuffle=True)
    return mbs_b200.gemm_a4w4(q, B, s, Bs, out=out)


def decode_object(dev, peaks):
    """BASELINE config[1] (decode, N = 57344, K = 8192, M in {1, 4, 16, 32};
    activations N(0,1), weights N(0,0.02), both quantised on the device).
    HBM-bound: algorithmic bytes = weights + their scales + activations +
    their scales + bf16 out, against the measured copy rate and 8 TB/s."""
    import torch

    import mbs_b200
    N, K = 57344, 8192
    g = torch.Generator(device=dev).manual_seed(4242)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    del w
    B, Bs = mbs_b200.shuffle_weight(qw), mbs_b200.shuffle_scales(sw, K)
    del qw, sw
    flush = _flusher(dev)
    hbm = float(peaks["hbm_gbs"])
    res = {"workload": "cfg1 decode N=57344 K=8192 (Llama-3-70B gate+up), MBS factors off",
           "method": "graph: 20 calls in one CUDA graph replayed back to back (median of 3); eager: "
                     "bench_one.py:34-47 (10 warm-up, 50 eager calls back to back); isolated: one call "
                     "after an L2 flush (median of 5); GB/s = algorithmic bytes / per-call time",
           "peak_measured_gbs": hbm}
    packed = mbs_b200.pack_weight(B, Bs)  # the optional one-time re-layout of static weights
    for M in (1, 4, 16, 32):
        x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        A, As = mbs_b200.quantize_mxfp4(x, shuffle=True)
        out = torch.empty(((M + 31) // 32 * 32, N), dtype=torch.bfloat16, device=dev)
        nbytes = N * K // 2 + N * K // 32 + M * K // 2 + M * K // 32 + M * N * 2
        gus, eus, ius = _per_call_us(lambda: mbs_b200.gemm_a4w4(A, B, As, Bs, out=out), flush)
        # activations in bf16: quantise + GEMM as two calls, and fused in one launch
        q2_us = _per_call_us(lambda: _two_calls(mbs_b200, x, B, Bs, out), flush)
        qf_us = _per_call_us(lambda: mbs_b200.quant_gemm_a4w4(x, B, Bs, out=out), flush)
        pk_us = _per_call_us(lambda: mbs_b200.gemm_a4w4_packed(A, packed, As, out=out), flush)
        pkq_us = _per_call_us(lambda: mbs_b200.quant_gemm_a4w4_packed(x, packed, out=out), flush)
        gbs = nbytes / (gus * 1e-6) / 1e9
        cpu_s, cpu_sample = _cpu_call_s(M, N, K, rows=M, cols=2048)
        res[f"M={M}"] = {"graph_us": round(gus, 2), "eager_us": round(eus, 2), "isolated_us": round(ius, 2),
                         "gbs": round(gbs, 1), "frac_measured": round(gbs / hbm, 4),
                         "frac_8tbs": round(gbs / 8000.0, 4),
                         "eager_gbs": round(nbytes / (eus * 1e-6) / 1e9, 1),
                         "isolated_gbs": round(nbytes / (ius * 1e-6) / 1e9, 1),
                         "algorithmic_bytes": nbytes,
                         "quant_gemm": {"two_calls_us": [round(v, 2) for v in q2_us],
                                        "fused_us": [round(v, 2) for v in qf_us],
                                        "what": "bf16 activations: quantize_mxfp4 + gemm_a4w4 vs quant_gemm_a4w4 "
                                                "(one launch); [graph, eager, isolated] per call"},
                         "packed_weights": {"us": [round(v, 2) for v in pk_us],
                                            "gbs_graph": round(nbytes / (pk_us[0] * 1e-6) / 1e9, 1),
                                            "from_bf16_us": [round(v, 2) for v in pkq_us],
                                            "what": "gemm_a4w4_packed on the one-time packed weight layout, "
                                                    "and quant_gemm_a4w4_packed from bf16 activations (one "
                                                    "launch up to 16 rows); [graph, eager, isolated] per call"},
                         "cpu_baseline_us": round(cpu_s * 1e6, 1), "cpu_sample": cpu_sample}
    del B, Bs, packed
    torch.cuda.empty_cache()
    return res


def configs_object(dev):
    """The other single-GPU configs of BASELINE.json: config[0] (256x512x1024
    with MBS factors, latency-bound) per call, and config[3] (4096x7168x18432,
    macro-block B scales, activations with 1 % x20 outliers, MBS factors) in
    TFLOPS with L2 flushed before every call."""
    import torch

    import mbs_b200
    from mbs_b200 import _lib
    flush = _flusher(dev)
    g = torch.Generator(device=dev).manual_seed(99)
    res = {}
    M, N, K = 256, 512, 1024
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    w = torch.randn(N, K, device=dev, generator=g).to(torch.bfloat16)
    A, As = mbs_b200.quantize_mxfp4(x, shuffle=True)
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    B, Bs = mbs_b200.shuffle_weight(qw), mbs_b200.shuffle_scales(sw, K)
    fa = torch.randint(0, 256, (M,), dtype=torch.uint8, device=dev, generator=g)
    fb = torch.randint(0, 256, (N,), dtype=torch.uint8, device=dev, generator=g)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    gus, eus, ius = _per_call_us(lambda: mbs_b200.gemm_a4w4(A, B, As, Bs, fa, fb, out=out), flush)
    cpu_s, cpu_sample = _cpu_call_s(M, N, K, rows=M, cols=N, reps=3)
    res["cfg0"] = {"workload": "256x512x1024 + MBS factors", "graph_us": round(gus, 2),
                   "eager_us": round(eus, 2), "isolated_us": round(ius, 2),
                   "tflops_graph": round(2.0 * M * N * K / (gus * 1e-6) / 1e12, 2),
                   "cpu_baseline_us": round(cpu_s * 1e6, 1), "cpu_sample": cpu_sample}
    M, N, K = 4096, 7168, 18432
    x = torch.randn(M, K, device=dev, generator=g)
    x = torch.where(torch.rand(M, K, device=dev, generator=g) < 0.01, x * 20, x).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    A, As = mbs_b200.quantize_mxfp4(x, shuffle=True)
    qw, mb = mbs_b200.quantize_mxfp4_macro(w)
    del x, w
    B = mbs_b200.shuffle_weight(qw)
    fa = torch.randint(0, 256, (M,), dtype=torch.uint8, device=dev, generator=g)
    fb = torch.randint(0, 256, (N,), dtype=torch.uint8, device=dev, generator=g)
    out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)

    def call():
        mbs_b200.gemm_a4w4_macro(A, B, As, mb, fa, fb, out=out)
    for _ in range(3):
        call()
    L = _lib.lib()
    steps = 10
    ev, kev = _events(steps), _events(steps)
    for a, b in kev:
        a.record()
        b.record()
    torch.cuda.synchronize()
    for i in range(steps):
        flush(i)
        L.mbs_set_profile_events(kev[i][0].cuda_event, kev[i][1].cuda_event)
        ev[i][0].record()
        call()
        ev[i][1].record()
    L.mbs_set_profile_events(None, None)
    torch.cuda.synchronize()
    ms = statistics.median(a.elapsed_time(b) for a, b in ev)
    kms = statistics.median(a.elapsed_time(b) for a, b in kev)
    flops = 2.0 * M * N * K
    cpu_s, cpu_sample = _cpu_call_s(M, N, K, rows=128, cols=1024)
    res["cfg3"] = {"workload": "4096x7168x18432 macro-block B scales + MBS factors, L2 flushed per call",
                   "call_ms": round(ms, 4), "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
                   "kernel_ms": round(kms, 4), "kernel_tflops": round(flops / (kms * 1e-3) / 1e12, 1),
                   "cpu_baseline_ms": round(cpu_s * 1e3, 1), "cpu_sample": cpu_sample + " (per-row block scales)"}
    torch.cuda.empty_cache()
    return res


def sharded_object(args, world, rank, dev):
    """BASELINE config[4] on all `world` ranks: A bf16 [16384, 8192] N(0,1),
    the same on every rank and quantised on each; the MXFP4 weight
    [57344, 8192] (N(0,0.02)) split by output columns, N/world rows per rank;
    each rank's GEMM writes its C shard and the shards are exchanged so every
    rank holds all of C.  Timed with CUDA events per step, max over ranks.
    Parity: each rank's shard against the CPU oracle on sampled rows/columns,
    and the exchange by checksums (every block a rank received equals the
    block its owner computed)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    import mbs_b200
    from mbs_b200.sharded import ShardedA4W4
    from oracle import mxfp4_oracle as O

    own_group = False
    if not dist.is_initialized():
        import socket
        with socket.socket() as s_:
            s_.bind(("127.0.0.1", 0))
            port = s_.getsockname()[1]
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                                device_id=dev)
        own_group = True
    M, N, K = 16384, 57344, 8192
    nl = N // world
    x = torch.randn(M, K, device=dev, generator=torch.Generator(device=dev).manual_seed(77)).to(torch.bfloat16)
    gw = torch.Generator(device=dev).manual_seed(1000 + rank)
    w = (torch.randn(nl, K, device=dev, generator=gw) * 0.02).to(torch.bfloat16)
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    B, Bs = mbs_b200.shuffle_weight(qw), mbs_b200.shuffle_scales(sw, K)
    del w
    layer = ShardedA4W4(B, Bs, N, K)
    exchange = args.exchange
    if exchange == "auto":
        exchange = layer.default_exchange(x)
    chunks = args.chunks if args.chunks is not None else layer.default_chunks(exchange)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        ev = _events(args.sharded_steps)
        for a, b in ev:
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        return statistics.median(a.elapsed_time(b) for a, b in ev)

    local_ms = timed(lambda: layer.local(x))
    # one rank: the layer is the quantiser and the GEMM alone (nothing to exchange)
    layer_ms = local_ms if world == 1 else timed(
        lambda: layer(x, chunks=chunks, comm_sms=args.comm_sms, exchange=exchange))
    t = torch.tensor([local_ms, layer_ms], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    local_ms, layer_ms = float(t[0]), float(t[1])
    # parity
    out = layer(x, chunks=chunks, comm_sms=args.comm_sms, exchange=exchange)  # [world, M, nl]
    torch.cuda.synchronize()
    mine = out[rank]
    rows = np.sort(np.random.default_rng(rank).choice(M, 64, replace=False))
    cols = np.sort(np.random.default_rng(100 + rank).choice(nl, 256, replace=False))
    qa, sa = mbs_b200.quantize_mxfp4(x[torch.from_numpy(rows).to(dev)], shuffle=False)
    tc = torch.from_numpy(cols).to(dev)
    ref = O.gemm_ref(qa.cpu().numpy(), qw[tc].cpu().numpy(), sa.cpu().numpy(), sw[tc].cpu().numpy())
    bound = O.gemm_abs_bound(qa.cpu().numpy(), qw[tc].cpu().numpy(), sa.cpu().numpy(), sw[tc].cpu().numpy())
    got = mine[torch.from_numpy(rows).to(dev)][:, tc].float().cpu().numpy()
    ok, ratio, nbad = O.check_gemm(got, ref, bound)
    # exchange: int64 sums of the bf16 bit patterns, exact and order-independent
    sums = torch.stack([out[r].view(torch.int16).sum(dtype=torch.int64) for r in range(world)])
    owner_sums = torch.empty(world, dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(owner_sums, sums[rank].reshape(1))
    xchg_ok = bool(torch.equal(sums, owner_sums))
    flags = torch.tensor([1 if ok else 0, 1 if xchg_ok else 0], device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    rat = torch.tensor([ratio], device=dev)
    dist.all_reduce(rat, op=dist.ReduceOp.MAX)
    flops = 2.0 * M * N * K
    res = {"workload": "cfg4 M=16384 N=57344 K=8192: quantise A on every rank + N-sharded GEMM + exchange of "
                       "the bf16 C shards (every rank ends with all of C)",
           "scaling": "strong", "n_ranks": world, "layer_ms": round(layer_ms, 4),
           "tflops": round(flops / (layer_ms * 1e-3) / 1e12, 1),
           "quant_gemm_ms": round(local_ms, 4),
           "quant_gemm_tflops_per_rank": round(flops / world / (local_ms * 1e-3) / 1e12, 1),
           "exposed_exchange_ms": round(layer_ms - local_ms, 4),
           "exchange": "none (one rank holds all of C)" if world == 1 else layer.describe_exchange(exchange, chunks),
           "bytes_received_per_rank": (world - 1) * M * nl * 2,
           # what bounds the layer: the exchange volume at the pool's peer-copy rate
           # (770 GB/s per direction) against quantise + GEMM alone
           "nvlink_bound_ms": round((world - 1) * M * nl * 2 / 770e9 * 1e3, 4),
           "layer_over_bound": round(layer_ms / max(local_ms, (world - 1) * M * nl * 2 / 770e9 * 1e3), 3),
           "parity": {"oracle_sample_ok": bool(flags[0].item()), "max_ratio": round(float(rat.item()), 4),
                      "sample": "64 rows x 256 columns of every rank's shard against the CPU oracle",
                      "exchange_checksums_ok": bool(flags[1].item())},
           "steps": args.sharded_steps, "timing": "median of per-step CUDA events, max over ranks"}
    if rank == 0 and world == 1:
        cpu_s, cpu_sample = _cpu_call_s(M, N, K, rows=64, cols=4096)
        res["cpu_baseline_ms"] = round(cpu_s * 1e3, 1)
        res["cpu_sample"] = cpu_sample + " (GEMM only, activations already quantised)"
    del out, mine
    dist.barrier()
    layer.close()
    dist.barrier()
    if own_group:
        dist.destroy_process_group()
    return res


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    M, N, K, wl_name = workload_shape(args)
    from oracle import mxfp4_oracle as O
    rows = min(M, 256)
    qa, qb, sa, sb = _cpu_sample(M, N, K, rows)
    for _ in range(args.warmup):
        O.gemm_ref(qa[:8], qb, sa[:8], sb)
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.gemm_ref(qa, qb, sa, sb)
        ts.append(time.perf_counter() - t0)
    ms = statistics.mean(ts) * 1e3
    value = 2.0 * rows * N * K / (ms * 1e-3) / 1e12
    sample = (f"{rows} of {M} rows of A per step (oracle port of test_gemm_a4w4.py:28-44: "
              f"dequant + fp32 matmul + bf16 cast)")
    print(json.dumps({
        "impl": "reference", "metric": "A4W4 MXFP4 GEMM TFLOPS", "value": round(value, 5),
        "unit": "TFLOPS", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (dequantised e2m1)", "data": "synthetic",
        "config": {"workload": wl_name, "M": M, "N": N, "K": K},
        "cpu_baseline": {"value": round(value, 5), "unit": "TFLOPS", "cores": os.cpu_count(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 5), "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }), flush=True)


def run_sharded(args):
    """`--workload sharded`: BASELINE config[4] alone (the `sharded` object of
    the default line, printed as its own line)."""
    import torch
    import torch.distributed as dist
    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", local)
    res = sharded_object(args, world, rank, dev)
    if rank == 0:
        print(json.dumps({
            "metric": "A4W4 MXFP4 quant + N-sharded GEMM + exchange TFLOPS (config[4])",
            "value": res["tflops"], "unit": "TFLOPS", "n_gpus": world, "steps": args.sharded_steps,
            "warmup": 3, "ms_per_step": res["layer_ms"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "e2m1 (fp32 accumulate, bf16 out)", "data": "synthetic",
            "config": {"workload": res["workload"], "parallelism": f"N-shards x{world}"},
            "sharded": res}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "sharded":
        run_sharded(args)
    else:
        run_mbs(args)


if __name__ == "__main__":
    main()
