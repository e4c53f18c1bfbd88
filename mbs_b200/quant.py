"""bf16 -> MXFP4 quantisers and layout shuffles (CUDA kernels via the C ABI).

These replace the aiter helpers the reference's drivers call before the GEMM
(test_gemm_a4w4.py:134-141, bench_one.py:20-25): ``get_triton_quant
(QuantType.per_1x32)`` and ``shuffle_weight(layout=(16, 16))``.  aiter itself
is third-party and absent; the arithmetic is OCP MX per-1x32 (see
include/mbs_gemm_a4w4.h).
"""

from __future__ import annotations

import torch

from . import _lib
from .mbs_gemm_a4w4 import _round_up, scale_n_pad

__all__ = ["quantize_mxfp4", "quantize_mxfp4_mbs", "quantize_mxfp4_macro", "shuffle_weight", "shuffle_scales",
           "macro_scale_ld", "quant_gemm_a4w4"]


def macro_scale_ld(K: int) -> int:
    return _round_up(K // 32, 16)


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _check_x(x: torch.Tensor):
    if not x.is_cuda or x.dtype != torch.bfloat16 or x.dim() != 2:
        raise RuntimeError("quantize_mxfp4: x must be a 2-D bf16 CUDA tensor")
    if x.stride(1) != 1:
        x = x.contiguous()
    R, K = int(x.size(0)), int(x.size(1))
    if K % 32 != 0:
        raise RuntimeError(f"quantize_mxfp4: K must be a multiple of 32, got {K}")
    return x, R, K


def quantize_mxfp4(x: torch.Tensor, shuffle: bool = False):
    """bf16 [R, K] -> (fp4x2 uint8 [R, K/2], e8m0 uint8 scales).

    shuffle=False: scales [R, K/32].  shuffle=True: scales
    [roundup(R,32), scaleN_pad] in the reference's shuffled layout.
    """
    x, R, K = _check_x(x)
    q = torch.empty((R, K // 2), dtype=torch.uint8, device=x.device)
    if shuffle:
        s = torch.empty((_round_up(R, 32), scale_n_pad(K)), dtype=torch.uint8, device=x.device)
    else:
        s = torch.empty((R, K // 32), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("mbs_quantize_mxfp4", x.data_ptr(), R, K, int(x.stride(0)), q.data_ptr(),
                  s.data_ptr(), 1 if shuffle else 0, _stream(x.device))
    return q, s


def quantize_mxfp4_mbs(x: torch.Tensor, shuffle: bool = False):
    """bf16 [R, K] -> (fp4x2 [R, K/2], e8m0 scales, MBS factor bytes [R]).

    Each row is quantised as x * (1 + b/256) with b its MBS factor (the top 8
    mantissa bits of 6 / max|row|); pass the factors to gemm_a4w4 as A_factor
    (activations) or B_factor (weight rows) to undo the scaling.  Scales as in
    quantize_mxfp4."""
    x, R, K = _check_x(x)
    q = torch.empty((R, K // 2), dtype=torch.uint8, device=x.device)
    if shuffle:
        s = torch.empty((_round_up(R, 32), scale_n_pad(K)), dtype=torch.uint8, device=x.device)
    else:
        s = torch.empty((R, K // 32), dtype=torch.uint8, device=x.device)
    f = torch.empty((R,), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("mbs_quantize_mxfp4_mbs", x.data_ptr(), R, K, int(x.stride(0)), q.data_ptr(),
                  s.data_ptr(), f.data_ptr(), 1 if shuffle else 0, _stream(x.device))
    return q, s, f


def quantize_mxfp4_macro(x: torch.Tensor):
    """bf16 [N, K] -> (fp4x2 [N, K/2], macro scales [ceil(N/32), roundup(K/32, 16)])."""
    x, R, K = _check_x(x)
    q = torch.empty((R, K // 2), dtype=torch.uint8, device=x.device)
    s = torch.empty(((R + 31) // 32, macro_scale_ld(K)), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("mbs_quantize_mxfp4_macro", x.data_ptr(), R, K, int(x.stride(0)), q.data_ptr(),
                  s.data_ptr(), _stream(x.device))
    return q, s


def shuffle_weight(w: torch.Tensor) -> torch.Tensor:
    """Plain fp4x2 [N, K/2] -> preshuffled [N, K/2] (the 16x16 weight layout)."""
    wu = w.view(torch.uint8).contiguous()
    N, Kp = int(wu.size(0)), int(wu.size(1))
    out = torch.empty_like(wu)
    with torch.cuda.device(wu.device):
        _lib.call("mbs_shuffle_weight", wu.data_ptr(), out.data_ptr(), N, 2 * Kp, _stream(wu.device))
    return out


def shuffle_scales(s: torch.Tensor, K: int | None = None) -> torch.Tensor:
    """Plain scales [R, K/32] -> shuffled [roundup(R,32), scaleN_pad]."""
    su = s.view(torch.uint8).contiguous()
    R = int(su.size(0))
    K = int(su.size(1)) * 32 if K is None else K
    out = torch.empty((_round_up(R, 32), scale_n_pad(K)), dtype=torch.uint8, device=su.device)
    with torch.cuda.device(su.device):
        _lib.call("mbs_shuffle_scales", su.data_ptr(), out.data_ptr(), R, K, _stream(su.device))
    return out


_qws_size_cache: dict = {}


def quant_gemm_a4w4(x: torch.Tensor, B: torch.Tensor, B_scale: torch.Tensor,
                    A_factor=None, B_factor=None, out=None) -> torch.Tensor:
    """Dynamic-quant + GEMM in one call (mbs_quant_gemm_a4w4_launch): bf16
    activations x [M, K] against a preshuffled MXFP4 weight B [N, K/2] with
    shuffled scales.  Bit-identical to quantize_mxfp4(x, shuffle=True)
    followed by gemm_a4w4; for skinny and small M the quantiser runs inside
    the GEMM kernel (one launch: up to 8 rows each pipeline stage converts
    its bf16 rows in shared memory, more rows are quantised by idle warps
    behind a grid barrier)."""
    from .mbs_gemm_a4w4 import _bytes, _launch, _on_device, _out_buffer, _ptr, cached_workspace
    x, M, K = _check_x(x)
    Bu, Bsc = _bytes(B), _bytes(B_scale)
    N = int(Bu.size(0))
    if int(Bu.size(1)) * 2 != K:
        raise RuntimeError(f"quant_gemm_a4w4: B must be [N, K/2] = [{N}, {K // 2}], got {tuple(Bu.shape)}")
    if N % 16 != 0:
        raise RuntimeError(f"quant_gemm_a4w4: N must be a multiple of 16, got {N}")
    snp = scale_n_pad(K)
    if Bsc.numel() < _round_up(N, 32) * snp:
        raise RuntimeError(f"quant_gemm_a4w4: B_scale must hold {_round_up(N, 32) * snp} bytes")
    fa = None if A_factor is None else _bytes(A_factor)
    fb = None if B_factor is None else _bytes(B_factor)
    if fa is not None and fa.numel() != M:
        raise RuntimeError(f"quant_gemm_a4w4: A_factor must hold M = {M} bytes")
    if fb is not None and fb.numel() != N:
        raise RuntimeError(f"quant_gemm_a4w4: B_factor must hold N = {N} bytes")
    o = _out_buffer(out, _round_up(M, 32), M, N, x.device)
    with _on_device(x.device):
        _launch("mbs_quant_gemm_a4w4_launch", (x.data_ptr(), int(x.stride(0)), Bu.data_ptr(), Bsc.data_ptr(),
                                               _ptr(fa), _ptr(fb), o.data_ptr(), M, N, K, snp),
                M, N, K, x.device, ws_fn=_quant_gemm_workspace)
    return o if o.size(0) == M else o.narrow(0, 0, M)


def _quant_gemm_workspace(M, N, K, device, fresh=False):
    from .mbs_gemm_a4w4 import cached_workspace
    key = (M, N, K, device.index)
    need = None if fresh else _qws_size_cache.get(key)
    if need is None:
        need = int(_lib.lib().mbs_quant_gemm_a4w4_workspace_size(M, N, K))
        _qws_size_cache[key] = need
    # the fused call always needs a workspace (at least its barrier words)
    return cached_workspace(max(need, 1), device)
