"""Output epilogue extensions (mbs_gemm_a4w4_launch_ex): alpha scaling and a
bf16 bias, on every schedule, against the oracle's
((c * (a_f * b_f)) * alpha + bias) -> bf16."""

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O
from tests.gpu_helpers import Case, assert_gemm_close, bf16_bits

pytestmark = pytest.mark.gpu

SCHEDULES = {
    "pair": dict(schedule="2", pair="1", pair_bn="256"),  # CTA pairs
    "pair384": dict(schedule="2", pair="1", pair_bn="384"),
    "pair_mix": dict(schedule="2", pair="1", pair_wide="1"),
    "dp_single": dict(schedule="2", pair="0"),
    "stream_k": dict(schedule="1", grid="17"),
    "swap": dict(swap="1"),
    "ksplit": dict(ksplit="4"),  # cluster split-K
}


@pytest.mark.parametrize("sched,M,N,K", [("pair", 512, 512, 1024), ("pair384", 300, 1040, 1024),
                                         ("pair_mix", 300, 1040, 1024),
                                         ("dp_single", 200, 768, 512),
                                         ("stream_k", 40, 2048, 2048), ("swap", 24, 1024, 512),
                                         ("ksplit", 200, 768, 2048)])
@pytest.mark.parametrize("alpha,with_bias", [(0.5, False), (-3.25, True), (1.0, True), (7.0, True)])
def test_alpha_bias(plan, sched, M, N, K, alpha, with_bias):
    import mbs_b200
    plan(**SCHEDULES[sched])
    c = Case(M, N, K, seed=M + N, factors=True)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(N)) * 4).to(torch.bfloat16)
    out = mbs_b200.gemm_a4w4(c.A, c.B, c.A_scale, c.B_scale, c.A_factor, c.B_factor,
                             alpha=alpha, bias=bias.cuda() if with_bias else None)
    torch.cuda.synchronize()
    ref = O.gemm_ref_ex(c.qa, c.qb, c.sa, c.sb, c.fa, c.fb, alpha,
                        bf16_bits(bias) if with_bias else None)
    bound = O.gemm_abs_bound(c.qa, c.qb, c.sa, c.sb) * np.float32(abs(alpha))
    assert_gemm_close(out, ref, bound, f"{sched} alpha={alpha} bias={with_bias}")


def test_defaults_are_bit_identical_to_the_plain_operator():
    import ctypes
    import mbs_b200
    from mbs_b200 import _lib
    from mbs_b200.mbs_gemm_a4w4 import scale_n_pad
    c = Case(100, 512, 512, seed=3, factors=True)
    plain = mbs_b200.gemm_a4w4(c.A, c.B, c.A_scale, c.B_scale, c.A_factor, c.B_factor)
    out = torch.empty((128, 512), dtype=torch.bfloat16, device="cuda")
    st = _lib.lib().mbs_gemm_a4w4_launch_ex(
        c.A.data_ptr(), c.B.data_ptr(), c.A_scale.data_ptr(), c.B_scale.data_ptr(),
        c.A_factor.data_ptr(), c.B_factor.data_ptr(), out.data_ptr(), 100, 512, 512, 128,
        scale_n_pad(512), ctypes.c_float(1.0), None, None, 0,
        torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert st == 0
    assert torch.equal(out[:100], plain)


def test_bias_checks():
    import mbs_b200
    c = Case(32, 256, 256, seed=4)
    with pytest.raises(RuntimeError, match="bias must be bf16"):
        mbs_b200.gemm_a4w4(c.A, c.B, c.A_scale, c.B_scale, bias=torch.zeros(255, dtype=torch.bfloat16,
                                                                               device="cuda"))
