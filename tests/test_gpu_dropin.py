"""The reference's drivers' call sequences against this library on a B200.

bench_one.py:11-31 and test_gemm_a4w4.py:12-18,129-171 quantise with aiter,
preshuffle the weight, then `import mbs_gemm_a4w4` from a directory put on
sys.path and call `gemm_a4w4` with 4 or 6 arguments.  These tests take the
same steps (aiter is the CUDA-backed stand-in in tests/aiter_standin) and
check the operator's result with the reference's own check (checkAllclose
against its torch oracle, restated over the stand-in's decoders) and with
the CPU oracle's tolerance.
"""

import os
import sys

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O
from tests.test_dropin import PKG, STANDIN, _run_torch_mbs

pytestmark = pytest.mark.gpu


@pytest.fixture
def driver_env():
    added = [p for p in (PKG, STANDIN) if p not in sys.path]
    for p in added:
        sys.path.insert(0, p)
    torch.set_default_device("cuda")
    try:
        import aiter
        import mbs_gemm_a4w4
        yield aiter, mbs_gemm_a4w4
    finally:
        torch.set_default_device("cpu")
        for p in added:
            sys.path.remove(p)


def _oracle_check(out, x, w, xs, ws, fa=None, fb=None):
    u8 = lambda t: t.view(torch.uint8).cpu().numpy()  # noqa: E731
    ref = O.gemm_ref(u8(x), u8(w), u8(xs), u8(ws), None if fa is None else u8(fa), None if fb is None else u8(fb))
    bound = O.gemm_abs_bound(u8(x), u8(w), u8(xs), u8(ws))
    ok, ratio, nbad = O.check_gemm(out.float().cpu().numpy(), ref, bound)
    assert ok, f"{nbad} elements outside the oracle tolerance (max ratio {ratio})"


@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (16, 4096, 2048)])
def test_bench_one_sequence(driver_env, M, N, K):
    aiter, mbs_gemm_a4w4 = driver_env
    from aiter.ops.shuffle import shuffle_weight
    from aiter.utility import fp4_utils
    torch.manual_seed(M + N)
    quant_func = aiter.get_triton_quant(aiter.QuantType.per_1x32)
    x = torch.randn((M, K), dtype=torch.bfloat16)
    w = torch.randn((N, K), dtype=torch.bfloat16)
    _, x_scales = quant_func(x, shuffle=False)
    _, w_scales = quant_func(w, shuffle=False)
    x, x_scales_shuffle = quant_func(x, shuffle=True)
    w, w_scales_shuffle = quant_func(w, shuffle=True)
    wshuffle = shuffle_weight(w, layout=(16, 16))
    out = mbs_gemm_a4w4.gemm_a4w4(x, wshuffle, x_scales_shuffle, w_scales_shuffle)  # bench_one.py:31
    torch.cuda.synchronize()
    assert out.shape == (M, N) and out.dtype == torch.bfloat16
    ref = _run_torch_mbs(fp4_utils, x, w, x_scales.view(torch.uint8), w_scales.view(torch.uint8))
    from aiter.test_common import checkAllclose
    assert checkAllclose(ref, out, msg="mbs b200", catastrophic_check=True) == 0.0
    _oracle_check(out, x, w, x_scales, w_scales)


@pytest.mark.parametrize("M,N,K", [(1024, 1024, 5120), (300, 272, 1088)])
def test_test_gemm_a4w4_sequence(driver_env, M, N, K):
    aiter, mbs_gemm_a4w4 = driver_env
    from aiter.ops.shuffle import shuffle_weight
    from aiter.test_common import checkAllclose, run_perftest
    from aiter.utility import fp4_utils
    torch.manual_seed(M)
    quant_func = aiter.get_triton_quant(aiter.QuantType.per_1x32)
    x = torch.randn((M, K), dtype=torch.bfloat16)
    w = torch.randn((N, K), dtype=torch.bfloat16)
    _, x_scales = quant_func(x, shuffle=False)
    _, w_scales = quant_func(w, shuffle=False)
    x, x_scales_shuffle = quant_func(x, shuffle=True)
    w, w_scales_shuffle = quant_func(w, shuffle=True)
    wshuffle = shuffle_weight(w, layout=(16, 16))
    x_scales, w_scales = x_scales.view(torch.uint8), w_scales.view(torch.uint8)
    a_factor = torch.randint(0, 256, (M, 1), dtype=torch.uint8)
    b_factor = torch.randint(0, 256, (N, 1), dtype=torch.uint8)
    a_mbs = _run_torch_mbs(fp4_utils, x, w, x_scales, w_scales, a_factor, b_factor)
    f, us = run_perftest(mbs_gemm_a4w4.gemm_a4w4, x, wshuffle, x_scales_shuffle, w_scales_shuffle,
                         a_factor, b_factor, num_iters=5)
    assert us > 0
    assert checkAllclose(a_mbs, f, msg="mbs b200", catastrophic_check=True) == 0.0
    _oracle_check(f, x, w, x_scales, w_scales, a_factor, b_factor)
    # the unified API the reference test times beside its kernel (no factors)
    c, _ = run_perftest(aiter.gemm_a4w4, x, wshuffle, x_scales_shuffle, w_scales_shuffle, bpreshuffle=True,
                        num_iters=2)
    a = _run_torch_mbs(fp4_utils, x, w, x_scales, w_scales)
    assert checkAllclose(a, c, msg="unified api", catastrophic_check=True) == 0.0
