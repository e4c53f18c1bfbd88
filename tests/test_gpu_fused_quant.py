"""Dynamic-quant + GEMM in one call (mbs_quant_gemm_a4w4_launch, Python
quant_gemm_a4w4) against the two-call sequence it replaces
(bench_one.py:20-31: quantise with shuffled scales, then gemm_a4w4): the
outputs must be bit-identical, on every schedule -- up to 8 rows quantised
in shared memory from the bf16 rows each pipeline stage brings (stream-K,
data-parallel, cluster split-K; 1, 4, 5 and 8 rows, a K tail shorter than a
stage), more rows quantising A in global memory behind a grid barrier
(stream-K, data-parallel single CTAs) or per CTA (cluster split-K), and the
stand-alone quantiser in front of the CTA-pair GEMM -- and one workspace
serves a sequence of shapes (the grid barrier words are left zero)."""

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O
from tests.gpu_helpers import assert_gemm_close, bf16_bits, seeded_bf16

pytestmark = pytest.mark.gpu

PLANS = {
    "auto": dict(),
    "stream_k": dict(schedule=1, grid=17),
    "dp_single": dict(schedule=2, pair=0),
    "ksplit": dict(ksplit=4),
    "pair": dict(schedule=2, pair=1),
}


def _two_call(x, B, Bs, fa, fb):
    import mbs_b200
    q, s = mbs_b200.quantize_mxfp4(x, shuffle=True)
    return mbs_b200.gemm_a4w4(q, B, s, Bs, fa, fb)


def _weights(N, K, seed):
    import mbs_b200
    w = seeded_bf16(N, K, seed, std=0.02).cuda()
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    return qw, sw, mbs_b200.shuffle_weight(qw), mbs_b200.shuffle_scales(sw, K)


@pytest.mark.parametrize("sched,M,N,K", [
    ("auto", 1, 57344, 8192), ("auto", 16, 57344, 8192), ("auto", 32, 57344, 8192),  # config[1]: stream-K
    ("auto", 16, 8192, 8192),      # skinny cluster split-K
    ("auto", 256, 512, 1024),      # config[0]: data-parallel single CTAs
    ("auto", 1024, 1024, 5120),    # cluster split-K, 128-row tiles
    ("auto", 1000, 2048, 1024),    # CTA pairs: stand-alone quantiser first
    ("stream_k", 40, 2048, 2048), ("stream_k", 300, 272, 1088),
    ("dp_single", 200, 768, 512), ("dp_single", 33, 96, 576),
    ("ksplit", 129, 784, 4160), ("ksplit", 24, 1280, 3072),
    ("pair", 300, 1040, 1024),
    # in-stage quantiser (M <= 8): one and two blocks per lane, K tails, every schedule
    ("auto", 4, 57344, 8192), ("auto", 8, 57344, 8192), ("auto", 5, 8192, 8192),
    ("stream_k", 5, 1024, 1088), ("dp_single", 1, 256, 64), ("dp_single", 7, 272, 320),
    ("ksplit", 8, 2048, 4096), ("stream_k", 3, 4096, 576),
    # the grid-shared quantiser just past that: 9 to 64 rows
    ("auto", 9, 57344, 1024), ("auto", 64, 4096, 2048), ("stream_k", 63, 1024, 1088),
    ("dp_single", 31, 272, 320), ("ksplit", 48, 2048, 4096),
])
def test_fused_matches_two_calls(plan, sched, M, N, K):
    import mbs_b200
    qw, sw, B, Bs = _weights(N, K, seed=N + K)
    x = seeded_bf16(M, K, seed=M, outlier_frac=0.01).cuda()
    g = torch.Generator(device="cuda").manual_seed(M + 1)
    fa = torch.randint(0, 256, (M,), dtype=torch.uint8, device="cuda", generator=g)
    fb = torch.randint(0, 256, (N,), dtype=torch.uint8, device="cuda", generator=g)
    plan(**PLANS[sched])
    ref2 = _two_call(x, B, Bs, fa, fb)
    for call in range(2):  # the second call reuses the workspace the first left behind
        got = mbs_b200.quant_gemm_a4w4(x, B, Bs, fa, fb)
        torch.cuda.synchronize()
        assert torch.equal(got, ref2), f"call {call}: differs from quantise + gemm_a4w4"
    assert mbs_b200.device_error() == 0
    if M * N <= 1 << 22:  # and against the CPU oracle where it is cheap
        qa, sa = O.quantize_mxfp4(bf16_bits(x.cpu()))
        ref = O.gemm_ref(qa, qw.cpu().numpy(), sa, sw.cpu().numpy(), fa.cpu().numpy(), fb.cpu().numpy())
        bound = O.gemm_abs_bound(qa, qw.cpu().numpy(), sa, sw.cpu().numpy())
        assert_gemm_close(got, ref, bound, f"fused quant {sched} {M}x{N}x{K}")


def test_one_workspace_across_shapes_and_strided_x():
    """A sequence of shapes and schedules on one cached workspace (grid
    barrier words and stream-K flags must be left zero by every call), with
    activations given as a row-strided view."""
    import mbs_b200
    for i, (M, N, K) in enumerate([(16, 4096, 2048), (1, 57344, 1024), (300, 1024, 2048), (8, 8192, 8192),
                                   (16, 4096, 2048)]):
        qw, sw, B, Bs = _weights(N, K, seed=7 + i)
        big = seeded_bf16(M, K + 64, seed=i).cuda()
        x = big[:, 32:32 + K]  # row stride K + 64, 64-byte aligned start
        assert x.stride(0) == K + 64 and x.stride(1) == 1
        got = mbs_b200.quant_gemm_a4w4(x, B, Bs)
        ref2 = _two_call(x.contiguous(), B, Bs, None, None)
        torch.cuda.synchronize()
        assert torch.equal(got, ref2), f"step {i} {M}x{N}x{K}"
    assert mbs_b200.device_error() == 0


@pytest.mark.parametrize("M", [40, 7])
@pytest.mark.parametrize("sched", ["auto", "stream_k", "ksplit", "dp_single"])
def test_fused_special_values_bit_identical(plan, sched, M):
    """Blocks holding Inf or NaN (scale 0xFF, codes 0), all-zero blocks, -0,
    and values near the bf16 maximum: the in-kernel quantiser writes the same
    bytes as the stand-alone one, so the outputs agree bit for bit (NaN
    patterns included)."""
    import mbs_b200
    N, K = 2048, 2048
    qw, sw, B, Bs = _weights(N, K, seed=9)
    x = seeded_bf16(M, K, seed=3).cuda()
    x[0, 5] = float("inf")
    x[1, 40] = float("-inf")
    x[2, 77] = float("nan")
    x[3, :64] = 0.0
    x[4, 64:96] = -0.0
    x[5, 96:128] = 3.0e38
    x[6, 128:160] = -1.0e-38
    plan(**PLANS[sched])
    ref2 = _two_call(x, B, Bs, None, None)
    got = mbs_b200.quant_gemm_a4w4(x, B, Bs)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref2.view(torch.int16))
    assert mbs_b200.device_error() == 0
