import ctypes
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda_ok():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return True


@pytest.fixture
def plan():
    """plan(**fields) forces parts of the GEMM schedule (mbs_set_plan_override:
    schedule, grid, pair, swap, pair_bn, pair_wide, ksplit, split_bn) for the
    calls that follow on this thread; each call replaces the previous override
    and the planner's own choice is restored after the test."""
    from mbs_b200 import _lib

    def set_(**fields):
        _lib.call("mbs_set_plan_override", ctypes.byref(_lib.PlanOverride(**fields)))
    yield set_
    _lib.call("mbs_set_plan_override", None)


def pytest_terminal_summary(terminalreporter):
    """Per GEMM check: the largest tolerance ratio and the reduction-order
    slack the result needed beyond 2 bf16 ulp (in units of sum_k |a_k b_k|)."""
    helpers = sys.modules.get("tests.gpu_helpers")
    if helpers is None or not helpers.OBSERVED:
        return
    import math
    from oracle import mxfp4_oracle as O
    tr = terminalreporter
    tr.section("GEMM parity: observed tolerance use")
    worst = max(e for _, e in helpers.OBSERVED.values())
    worst_ratio = max(r for r, _ in helpers.OBSERVED.values())
    tr.write_line(f"slack allowed 2^{math.log2(O.GEMM_SLACK):.0f}; largest needed "
                  f"{'0' if worst == 0 else f'2^{math.log2(worst):.1f}'}, largest tolerance ratio "
                  f"{worst_ratio:.3g}, over {len(helpers.OBSERVED)} checks")
    for what, (ratio, ex) in sorted(helpers.OBSERVED.items(), key=lambda kv: -kv[1][1])[:12]:
        tr.write_line(f"  {what}: max ratio {ratio:.3g}, slack needed "
                      f"{'0' if ex == 0 else f'2^{math.log2(ex):.1f}'}")
