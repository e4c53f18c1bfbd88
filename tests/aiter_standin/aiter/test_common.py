"""aiter.test_common stand-in: the timing decorator and the allclose check
the reference's drivers use (test_gemm_a4w4.py:27-101,155-171)."""

from __future__ import annotations

import functools
import time

import torch


def _timed(fn, args, kwargs, num_iters, num_warmup):
    out = None
    for _ in range(num_warmup):
        out = fn(*args, **kwargs)
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(num_iters):
            out = fn(*args, **kwargs)
        end.record()
        torch.cuda.synchronize()
        us = start.elapsed_time(end) * 1e3 / num_iters
    else:
        t0 = time.perf_counter()
        for _ in range(num_iters):
            out = fn(*args, **kwargs)
        us = (time.perf_counter() - t0) * 1e6 / num_iters
    return out, us


def perftest(num_iters: int = 101, num_warmup: int = 2, **_unused):
    """Decorator: the wrapped call returns (result, average microseconds)."""
    def deco(fn):
        @functools.wraps(fn)
        def wrapper(*args, **kwargs):
            return _timed(fn, args, kwargs, num_iters, num_warmup)
        return wrapper
    return deco


def run_perftest(fn, *args, num_iters: int = 101, num_warmup: int = 2, **kwargs):
    """(result, average microseconds) of fn(*args, **kwargs)."""
    return _timed(fn, args, kwargs, num_iters, num_warmup)


def benchmark(**_unused):
    """Decorator kept for the drivers' structure: calls pass through."""
    def deco(fn):
        return fn
    return deco


def checkAllclose(a, b, rtol: float = 1e-2, atol: float = 1e-2, msg: str = "", catastrophic_check: bool = False,
                  printNum: int = 8, tol_err_ratio: float = 0.05):
    """Fraction of elements outside |a - b| <= atol + rtol * |b| (0 = all close).
    With catastrophic_check, more than tol_err_ratio of them raises."""
    a = a.float()
    b = b.float()
    bad = ~torch.isclose(a, b, rtol=rtol, atol=atol, equal_nan=True)
    ratio = float(bad.float().mean().item()) if bad.numel() else 0.0
    if ratio > 0:
        print(f"{msg} {int(bad.sum())} of {bad.numel()} elements outside tolerance ({ratio:.2%})")
        if catastrophic_check and ratio > tol_err_ratio:
            raise AssertionError(f"{msg} catastrophic mismatch: {ratio:.2%} of elements")
    return ratio
