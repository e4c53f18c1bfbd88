"""Drop-in ``mbs_gemm_a4w4`` operator module (host side of the C ABI).

Mirrors the reference's pybind11 module ``mbs_gemm_a4w4``
(interface/gemm_a4w4_pybind.cpp:19-74): same function name, argument order,
byte-reinterpretation of fp4/e8m0 tensors, shape checks and ``RuntimeError``
messages, and the same output contract (bf16 ``out[Mpad, N]`` allocated on
A's device, returned as ``out[:M]``).  Two additions: the MBS factors are
optional (the reference's 6-argument form and the 4-argument form used by
bench_one.py:31 both work), and ``out=`` accepts a caller buffer.

    import mbs_b200.mbs_gemm_a4w4 as mbs_gemm_a4w4
    out = mbs_gemm_a4w4.gemm_a4w4(A, B, A_scale, B_scale, A_factor, B_factor)

The reference's drivers import their extension as a top-level module after
putting its directory on the path (`sys.path.insert(0, <dir>); import
mbs_gemm_a4w4`, bench_one.py:11,27 and test_gemm_a4w4.py:12,80).  The same
works with this package's directory on the path: imported that way, this file
loads the package and makes `mbs_gemm_a4w4` an alias of
`mbs_b200.mbs_gemm_a4w4`, so both names share one module (one workspace
cache, one library handle).

Launches go to the current torch CUDA stream of A's device, asynchronously.
"""

from __future__ import annotations

import contextlib
import ctypes
import importlib
import os
import sys
import threading

import torch

if not __package__:
    # top-level import from the package directory: become the package's module
    _root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    if _root not in sys.path:
        sys.path.insert(0, _root)
    sys.modules[__name__] = importlib.import_module("mbs_b200.mbs_gemm_a4w4")
else:
    from . import _lib

__all__ = ["gemm_a4w4", "gemm_a4w4_macro", "workspace_for", "device_error", "grid_limit", "plan_override"]

# Workspace layout of include/mbs_gemm_a4w4.h: the first WS_FLAG_BYTES bytes
# are the stream-K flag words (zero between launches), the rest is scratch.
WS_FLAG_BYTES = 4096

_ws_lock = threading.Lock()
_ws_cache: dict = {}


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


def scale_n_pad(K: int) -> int:
    """roundup(ceil(K/32), 8) -- interface/gemm_a4w4_pybind.cpp:46-48."""
    return _round_up((K + 31) // 32, 8)


def _bytes(t: torch.Tensor) -> torch.Tensor:
    # .view(kByte).contiguous() as in interface/gemm_a4w4_pybind.cpp:25-30 (each torch
    # call costs a few microseconds of host time per launch, so skip the no-op ones)
    if t.dtype != torch.uint8:
        t = t.view(torch.uint8)
    return t if t.is_contiguous() else t.contiguous()


class _on_device:
    """`with torch.cuda.device(dev)` only when dev is not already current
    (switching costs host time on every launch)."""
    __slots__ = ("idx", "prev")

    def __init__(self, device: torch.device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


@contextlib.contextmanager
def grid_limit(max_ctas: int):
    """Run the GEMMs launched inside the block (from this thread) on at most
    `max_ctas` CTAs, leaving the other SMs to concurrent kernels such as an
    overlapped NCCL all-gather.  0 = no limit."""
    _lib.call("mbs_set_grid_limit", int(max_ctas))
    try:
        yield
    finally:
        _lib.call("mbs_set_grid_limit", 0)


@contextlib.contextmanager
def plan_override(**fields):
    """Force parts of the GEMM schedule for the calls made (from this thread)
    inside the block: schedule (1 stream-K, 2 data-parallel), grid, pair,
    swap, pair_bn, pair_wide, ksplit, split_bn -- the fields of
    mbs_plan_override in include/mbs_gemm_a4w4.h.  A tuning and test hook; the
    planner's own choice is restored on exit."""
    ov = _lib.PlanOverride(**fields)
    _lib.call("mbs_set_plan_override", ctypes.byref(ov))
    try:
        yield
    finally:
        _lib.call("mbs_set_plan_override", None)


def cached_workspace(need: int, device: torch.device) -> torch.Tensor | None:
    """The (device, current stream) workspace, grown to at least `need` bytes.

    Zero-filled when allocated; every completed launch leaves its flag words
    zero again, so one buffer serves every shape and schedule on that stream.
    """
    if need == 0:
        return None
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, _stream_ptr(device))
    buf = _ws_cache.get(key)
    if buf is not None and buf.numel() >= need:
        return buf
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < need:
            buf = torch.zeros(max(need, 1 << 22), dtype=torch.uint8, device=device)
            _ws_cache[key] = buf
    return buf


_ws_size_cache: dict = {}


def workspace_for(M: int, N: int, K: int, device: torch.device) -> torch.Tensor | None:
    """Workspace for a drop-in launch of this shape on the current stream."""
    return _remembered_workspace(M, N, K, device, fresh=True)


def _remembered_workspace(M: int, N: int, K: int, device: torch.device, fresh: bool = False):
    """As workspace_for with the size remembered per (shape, device), which
    saves a library call per launch.  The plan behind a size can change with
    this thread's plan override or grid limit, so a launch that reports
    MBS_ERR_WORKSPACE asks again with fresh=True (see _launch)."""
    key = (M, N, K, device.index)
    need = None if fresh else _ws_size_cache.get(key)
    if need is None:
        need = int(_lib.lib().mbs_gemm_a4w4_workspace_size(M, N, K))
        _ws_size_cache[key] = need
    return cached_workspace(need, device)


def _stream_ptr(device: torch.device) -> int:
    """Raw handle of the current stream of `device` (the cheap accessor when
    this torch build has it)."""
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return raw(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _launch(func: str, args_before_ws: tuple, M: int, N: int, K: int, device: torch.device,
            ws_fn=None) -> None:
    """Launch `func` with the cached workspace of the shape; on MBS_ERR_WORKSPACE
    (a cached size from before a plan override or grid limit) size it afresh once."""
    ws_fn = ws_fn or _remembered_workspace
    fn = getattr(_lib.lib(), func)
    stream = _stream_ptr(device)
    for fresh in (False, True):
        ws = ws_fn(M, N, K, device, fresh=fresh)
        st = fn(*args_before_ws, None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), stream)
        if st != MBS_ERR_WORKSPACE or fresh:
            _lib.check(func, st)
            return


MBS_ERR_WORKSPACE = 5


def device_error(reset: bool = False) -> int:
    """Sticky device error code of the current device (0 = none; synchronises).

    With reset=True the code is cleared, and so are the flag words of this
    module's cached workspaces: a launch that stopped on a device error may
    have left some set.
    """
    code = ctypes.c_int(0)
    _lib.call("mbs_device_error", ctypes.byref(code), 1 if reset else 0)
    if reset and code.value != 0:
        with _ws_lock:
            for buf in _ws_cache.values():
                buf[:WS_FLAG_BYTES].zero_()
        torch.cuda.synchronize()  # cleared before any stream's next launch
    return code.value


def _check_inputs(A, B, A_scale, B_scale, A_factor, B_factor):
    if not (A.is_cuda and B.is_cuda):
        raise RuntimeError("gemm_a4w4: A, B must be on device")
    if A.dim() != 2 or B.dim() != 2:
        raise RuntimeError("gemm_a4w4: A, B must be 2D")
    Au, Bu = _bytes(A), _bytes(B)
    Asc, Bsc = _bytes(A_scale), _bytes(B_scale)
    M, Kp = int(Au.size(0)), int(Au.size(1))
    K, N = 2 * Kp, int(Bu.size(0))
    if int(Bu.size(1)) != Kp:
        raise RuntimeError(f"gemm_a4w4: A, B must share K/2, got {Au.size(1)} vs {Bu.size(1)}")
    if K % 32 != 0:
        raise RuntimeError(f"gemm_a4w4: K must be a multiple of 32, got {K}")
    if N % 16 != 0:
        raise RuntimeError(f"gemm_a4w4: N must be a multiple of 16, got {N}")
    Afc = Bfc = None
    if A_factor is not None:
        Afc = _bytes(A_factor)
        if not (Afc.is_cuda and Afc.numel() == M):
            raise RuntimeError(f"gemm_a4w4: A_factor must hold M = {M} bytes on device, got {Afc.numel()}")
    if B_factor is not None:
        Bfc = _bytes(B_factor)
        if not (Bfc.is_cuda and Bfc.numel() == N):
            raise RuntimeError(f"gemm_a4w4: B_factor must hold N = {N} bytes on device, got {Bfc.numel()}")
    for name, t in (("A_scale", Asc), ("B_scale", Bsc)):
        if not t.is_cuda or t.get_device() != A.get_device():
            raise RuntimeError(f"gemm_a4w4: {name} must be on A's device")
    return Au, Bu, Asc, Bsc, Afc, Bfc, M, N, K


def _out_buffer(out, Mpad, M, N, device):
    if out is None:
        return torch.empty((Mpad, N), dtype=torch.bfloat16, device=device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if out.dtype != torch.bfloat16 or not out.is_cuda or out.get_device() != idx \
            or not out.is_contiguous() or out.dim() != 2 or out.size(0) < M or out.size(1) != N:
        raise RuntimeError(f"gemm_a4w4: out must be a contiguous bf16 [>= {M}, {N}] tensor on {device}")
    return out


def _ptr(t):
    return None if t is None else t.data_ptr()


def gemm_a4w4(A: torch.Tensor, B: torch.Tensor, A_scale: torch.Tensor, B_scale: torch.Tensor,
              A_factor: torch.Tensor | None = None, B_factor: torch.Tensor | None = None,
              out: torch.Tensor | None = None, alpha: float = 1.0,
              bias: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] bf16 = dequant(A) @ dequant(B)^T * f(A_factor) * f(B_factor)^T.

    A: [M, K/2] fp4x2 plain; B: [N, K/2] fp4x2 preshuffled (16x16);
    A_scale / B_scale: e8m0 in the shuffled layout (>= Mpad*scaleN_pad and
    roundup(N,32)*scaleN_pad bytes); factors: uint8 [M] / [N] or None,
    f(b) = 1 / (1 + b/256).  (interface/gemm_a4w4_pybind.cpp:7-18)
    Extensions (keyword only in spirit; defaults leave the result unchanged):
    `alpha` scales the fp32 result and `bias` (bf16 [N]) is added to every
    row before the bf16 rounding.
    """
    if alpha != 1.0 or bias is not None:
        return _gemm_ex(A, B, A_scale, B_scale, A_factor, B_factor, out, float(alpha), bias)
    Au, Bu, Asc, Bsc, Afc, Bfc, M, N, K = _check_inputs(A, B, A_scale, B_scale, A_factor, B_factor)
    Mpad = _round_up(M, 32)
    snp = scale_n_pad(K)
    if Asc.numel() < Mpad * snp:
        raise RuntimeError(f"gemm_a4w4: A_scale must hold Mpad*scaleN_pad = {Mpad * snp} bytes, "
                           f"got {Asc.numel()}")
    if Bsc.numel() < _round_up(N, 32) * snp:
        raise RuntimeError(f"gemm_a4w4: B_scale must hold roundup(N,32)*scaleN_pad = "
                           f"{_round_up(N, 32) * snp} bytes, got {Bsc.numel()}")
    dev = A.device
    o = _out_buffer(out, Mpad, M, N, dev)
    with _on_device(dev):
        _launch("mbs_gemm_a4w4_launch_ws", (_ptr(Au), _ptr(Bu), _ptr(Asc), _ptr(Bsc), _ptr(Afc), _ptr(Bfc),
                                            o.data_ptr(), M, N, K, Mpad, snp), M, N, K, dev)
    return o if o.size(0) == M else o.narrow(0, 0, M)


def _gemm_ex(A, B, A_scale, B_scale, A_factor, B_factor, out, alpha, bias):
    Au, Bu, Asc, Bsc, Afc, Bfc, M, N, K = _check_inputs(A, B, A_scale, B_scale, A_factor, B_factor)
    Mpad = _round_up(M, 32)
    snp = scale_n_pad(K)
    if Asc.numel() < Mpad * snp or Bsc.numel() < _round_up(N, 32) * snp:
        raise RuntimeError("gemm_a4w4: scale buffers too small for the shape")
    bias_t = None
    if bias is not None:
        if not bias.is_cuda or bias.device != A.device:
            raise RuntimeError("gemm_a4w4: bias must be on A's device")
        if bias.dtype != torch.bfloat16 or bias.numel() != N:
            raise RuntimeError(f"gemm_a4w4: bias must be bf16 with N = {N} elements")
        bias_t = bias.contiguous()
    dev = A.device
    o = _out_buffer(out, Mpad, M, N, dev)
    with _on_device(dev):
        _launch("mbs_gemm_a4w4_launch_ex", (_ptr(Au), _ptr(Bu), _ptr(Asc), _ptr(Bsc), _ptr(Afc), _ptr(Bfc),
                                            o.data_ptr(), M, N, K, Mpad, snp, alpha, _ptr(bias_t)), M, N, K, dev)
    return o if o.size(0) == M else o.narrow(0, 0, M)


def gemm_a4w4_macro(A: torch.Tensor, B: torch.Tensor, A_scale: torch.Tensor,
                    B_scale_macro: torch.Tensor, A_factor: torch.Tensor | None = None,
                    B_factor: torch.Tensor | None = None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """Macro-block-scaling variant: B's scales are one e8m0 per 32 rows x 32 K,
    given plainly as [ceil(N/32), roundup(K/32, 16)] (see quantize_mxfp4_macro)."""
    Au, Bu, Asc, Bsc, Afc, Bfc, M, N, K = _check_inputs(A, B, A_scale, B_scale_macro, A_factor,
                                                        B_factor)
    Mpad = _round_up(M, 32)
    snp = scale_n_pad(K)
    mb_ld = _round_up(K // 32, 16)
    if Asc.numel() < Mpad * snp:
        raise RuntimeError(f"gemm_a4w4: A_scale must hold {Mpad * snp} bytes, got {Asc.numel()}")
    if Bsc.numel() < ((N + 31) // 32) * mb_ld:
        raise RuntimeError(f"gemm_a4w4: B_scale_macro must hold {((N + 31) // 32) * mb_ld} bytes, "
                           f"got {Bsc.numel()}")
    o = _out_buffer(out, Mpad, M, N, A.device)
    with torch.cuda.device(A.device):
        ws = workspace_for(M, N, K, A.device)
        stream = torch.cuda.current_stream(A.device).cuda_stream
        _lib.call("mbs_gemm_a4w4_macro_launch_ws", _ptr(Au), _ptr(Bu), _ptr(Asc), _ptr(Bsc),
                  _ptr(Afc), _ptr(Bfc), o.data_ptr(), M, N, K, Mpad, snp, mb_ld, _ptr(ws),
                  0 if ws is None else ws.numel(), stream)
    return o.narrow(0, 0, M)
