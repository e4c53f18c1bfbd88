"""Packed weights for skinny (decode) GEMMs.

`pack_weight` turns a preshuffled weight and its shuffled scales (the
reference's formats) into the packed format of include/mbs_gemm_a4w4.h: per
256-row tile and 256-element K stage one contiguous 34 KB block, which the
GEMM streams with a single bulk copy.  Packing is a one-time step for static
weights, like the preshuffle itself.
"""

from __future__ import annotations

import torch

from . import _lib
from .mbs_gemm_a4w4 import _bytes, _out_buffer, _ptr, _round_up, cached_workspace, scale_n_pad

__all__ = ["PackedWeight", "pack_weight", "gemm_a4w4_packed", "quant_gemm_a4w4_packed"]


class PackedWeight:
    """A packed MXFP4 weight of logical shape [N, K]."""

    def __init__(self, data: torch.Tensor, N: int, K: int):
        self.data, self.N, self.K = data, N, K

    @property
    def device(self):
        return self.data.device


def pack_weight(B: torch.Tensor, B_scale: torch.Tensor) -> PackedWeight:
    """B: preshuffled fp4x2 [N, K/2]; B_scale: shuffled e8m0 (>= roundup(N,32)*scaleN_pad bytes)."""
    Bu, Bs = _bytes(B), _bytes(B_scale)
    N, K = int(Bu.size(0)), 2 * int(Bu.size(1))
    snp = scale_n_pad(K)
    if Bs.numel() < _round_up(N, 32) * snp:
        raise RuntimeError(f"pack_weight: B_scale must hold {_round_up(N, 32) * snp} bytes, got {Bs.numel()}")
    L = _lib.lib()
    out = torch.empty(int(L.mbs_packed_weight_bytes(N, K)), dtype=torch.uint8, device=Bu.device)
    with torch.cuda.device(Bu.device):
        _lib.call("mbs_pack_weight", Bu.data_ptr(), Bs.data_ptr(), N, K, snp, out.data_ptr(),
                  torch.cuda.current_stream(Bu.device).cuda_stream)
    return PackedWeight(out, N, K)


def _workspace(M, N, K, device):
    return cached_workspace(int(_lib.lib().mbs_gemm_a4w4_packed_workspace_size(M, N, K)), device)


def gemm_a4w4_packed(A: torch.Tensor, W: PackedWeight, A_scale: torch.Tensor,
                     A_factor: torch.Tensor | None = None, B_factor: torch.Tensor | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """out[M, N] bf16 = dequant(A) @ dequant(W)^T * f(A_factor) * f(B_factor)^T with a packed W."""
    if not A.is_cuda or A.device != W.device:
        raise RuntimeError("gemm_a4w4_packed: A and the packed weight must be on the same CUDA device")
    Au, Asc = _bytes(A), _bytes(A_scale)
    M, K, N = int(Au.size(0)), 2 * int(Au.size(1)), W.N
    if K != W.K:
        raise RuntimeError(f"gemm_a4w4_packed: A has K={K}, the packed weight K={W.K}")
    Mpad = _round_up(M, 32)
    snp = scale_n_pad(K)
    if Asc.numel() < Mpad * snp:
        raise RuntimeError(f"gemm_a4w4_packed: A_scale must hold {Mpad * snp} bytes, got {Asc.numel()}")
    Afc = None if A_factor is None else _bytes(A_factor)
    Bfc = None if B_factor is None else _bytes(B_factor)
    if Afc is not None and Afc.numel() != M:
        raise RuntimeError(f"gemm_a4w4_packed: A_factor must hold M = {M} bytes")
    if Bfc is not None and Bfc.numel() != N:
        raise RuntimeError(f"gemm_a4w4_packed: B_factor must hold N = {N} bytes")
    o = _out_buffer(out, Mpad, M, N, A.device)
    with torch.cuda.device(A.device):
        ws = _workspace(M, N, K, A.device)
        _lib.call("mbs_gemm_a4w4_packed_launch_ws", _ptr(Au), W.data.data_ptr(), _ptr(Asc), _ptr(Afc),
                  _ptr(Bfc), o.data_ptr(), M, N, K, Mpad, snp, _ptr(ws), 0 if ws is None else ws.numel(),
                  torch.cuda.current_stream(A.device).cuda_stream)
    return o.narrow(0, 0, M)


_qws_size_cache: dict = {}


def _quant_workspace(M, N, K, device, fresh=False):
    key = (M, N, K, device.index)
    need = None if fresh else _qws_size_cache.get(key)
    if need is None:
        need = int(_lib.lib().mbs_quant_gemm_a4w4_packed_workspace_size(M, N, K))
        _qws_size_cache[key] = need
    return cached_workspace(max(need, 1), device)


def quant_gemm_a4w4_packed(x: torch.Tensor, W: PackedWeight, A_factor: torch.Tensor | None = None,
                           B_factor: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Dynamic-quant + GEMM with a packed weight (mbs_quant_gemm_a4w4_packed_launch):
    bf16 activations x [M, K]; bit-identical to quantize_mxfp4(x, shuffle=True)
    followed by gemm_a4w4_packed.  Up to 16 rows, one launch that converts
    each stage's bf16 rows in shared memory."""
    from .mbs_gemm_a4w4 import _launch, _on_device
    from .quant import _check_x
    if not x.is_cuda or x.device != W.device:
        raise RuntimeError("quant_gemm_a4w4_packed: x and the packed weight must be on the same CUDA device")
    x, M, K = _check_x(x)
    N = W.N
    if K != W.K:
        raise RuntimeError(f"quant_gemm_a4w4_packed: x has K={K}, the packed weight K={W.K}")
    fa = None if A_factor is None else _bytes(A_factor)
    fb = None if B_factor is None else _bytes(B_factor)
    if fa is not None and fa.numel() != M:
        raise RuntimeError(f"quant_gemm_a4w4_packed: A_factor must hold M = {M} bytes")
    if fb is not None and fb.numel() != N:
        raise RuntimeError(f"quant_gemm_a4w4_packed: B_factor must hold N = {N} bytes")
    o = _out_buffer(out, _round_up(M, 32), M, N, x.device)
    with _on_device(x.device):
        _launch("mbs_quant_gemm_a4w4_packed_launch", (x.data_ptr(), int(x.stride(0)), W.data.data_ptr(),
                                                      _ptr(fa), _ptr(fb), o.data_ptr(), M, N, K),
                M, N, K, x.device, ws_fn=_quant_workspace)
    return o if o.size(0) == M else o.narrow(0, 0, M)
