"""CPU tests of the drop-in boundary as the reference's drivers use it.

bench_one.py:11,27 and test_gemm_a4w4.py:12,80 put the extension's directory
on sys.path and `import mbs_gemm_a4w4`; with this package's directory there
instead, the same import must give this library's operator.  The aiter
stand-in (tests/aiter_standin) must decode fp4/e8m0 exactly as the oracle
does, so the reference's own torch oracle restated over it reproduces the
golden outputs the reference's run_torch/run_torch_mbs produced.
"""

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "mbs_b200")
STANDIN = os.path.join(REPO, "tests", "aiter_standin")
GOLDEN = os.path.join(REPO, "tests", "golden")


def test_top_level_import_like_the_reference_drivers():
    code = (
        "import inspect, sys\n"
        f"sys.path.insert(0, {PKG!r})\n"
        "import mbs_gemm_a4w4\n"
        "import mbs_b200.mbs_gemm_a4w4 as pkg\n"
        "assert mbs_gemm_a4w4 is pkg, 'two module objects'\n"
        "p = list(inspect.signature(mbs_gemm_a4w4.gemm_a4w4).parameters)\n"
        "assert p[:6] == ['A', 'B', 'A_scale', 'B_scale', 'A_factor', 'B_factor'], p\n"
        "print('ok')\n")
    res = subprocess.run([sys.executable, "-c", code], cwd="/tmp" if os.path.isdir("/tmp") else REPO,
                         capture_output=True, text=True, timeout=300)
    assert res.returncode == 0 and res.stdout.strip().endswith("ok"), res.stderr + res.stdout


@pytest.fixture
def aiter_mod():
    sys.path.insert(0, STANDIN)
    try:
        import aiter
        from aiter.utility import fp4_utils
        yield aiter, fp4_utils
    finally:
        sys.path.remove(STANDIN)


def test_standin_decoders_match_the_oracle(aiter_mod):
    _, fp4_utils = aiter_mod
    b = np.arange(256, dtype=np.uint8).reshape(4, 64)
    got = fp4_utils.mxfp4_to_f32(torch.from_numpy(b)).numpy()
    assert np.array_equal(got.view(np.uint32), O.mxfp4_to_f32(b).view(np.uint32))
    e = np.arange(256, dtype=np.uint8)
    got = fp4_utils.e8m0_to_f32(torch.from_numpy(e)).numpy()
    ref = O.e8m0_to_f32(e)
    assert np.isnan(got[255]) and np.array_equal(got[:255].view(np.uint32), ref[:255].view(np.uint32))


def _run_torch_mbs(fp4_utils, x, w, xs, ws, a_factor=None, b_factor=None):
    # the reference's oracle, test_gemm_a4w4.py:28-44 / 54-69, over the stand-in's decoders
    m, n = x.shape[0], w.shape[0]
    x_f32 = fp4_utils.mxfp4_to_f32(x) * fp4_utils.e8m0_to_f32(xs[:m].repeat_interleave(32, dim=1))
    w_f32 = fp4_utils.mxfp4_to_f32(w) * fp4_utils.e8m0_to_f32(ws[:n].repeat_interleave(32, dim=1))
    c = torch.mm(x_f32, w_f32.T)
    if a_factor is not None:
        one = lambda b: 1.0 / (b.to(torch.int32) << 15 | 0x3F800000).view(torch.float32)  # noqa: E731
        c = c * (one(a_factor).view(m, 1) * one(b_factor).view(n, 1).T)
    return c.to(torch.bfloat16)[:m, :n]


@pytest.mark.parametrize("tag", ["5x16x64", "33x48x128", "64x32x256", "17x64x512"])
def test_standin_oracle_reproduces_reference_goldens(aiter_mod, tag):
    _, fp4_utils = aiter_mod
    g = np.load(os.path.join(GOLDEN, "gemm_oracle_golden.npz"))
    a, w, sa, sw, fa, fw = (torch.from_numpy(g[f"{k}_{tag}"]) for k in ("a", "w", "sa", "sw", "fa", "fw"))
    out = _run_torch_mbs(fp4_utils, a, w, sa, sw)
    out_mbs = _run_torch_mbs(fp4_utils, a, w, sa, sw, fa, fw)
    assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), g[f"out_{tag}"])
    assert np.array_equal(out_mbs.view(torch.int16).numpy().view(np.uint16), g[f"outmbs_{tag}"])


def test_standin_check_and_timer(aiter_mod):
    aiter, _ = aiter_mod
    from aiter.test_common import checkAllclose, perftest
    a = torch.ones(100)
    assert checkAllclose(a, a) == 0.0
    b = a.clone()
    b[:10] = 5.0
    assert checkAllclose(a, b) == pytest.approx(0.1)
    with pytest.raises(AssertionError):
        checkAllclose(a, b, catastrophic_check=True)

    @perftest(num_iters=3)
    def f(x):
        return x + 1
    res, us = f(torch.zeros(3))
    assert torch.equal(res, torch.ones(3)) and us >= 0.0
    assert aiter.QuantType.per_1x32.name == "per_1x32"
