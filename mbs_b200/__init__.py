"""mbs_b200 -- B200 (sm_100a) MXFP4 A4W4 GEMM behind the mbs operator API.

Compute lives in libmbs_gemm_kernel.so (hand-written CUDA, C ABI declared in
include/mbs_gemm_a4w4.h); this package is the host side: the drop-in
``mbs_gemm_a4w4.gemm_a4w4`` operator, the quantiser/shuffle ops and the
N-sharded multi-GPU wrapper.
"""

from .mbs_gemm_a4w4 import device_error, gemm_a4w4, gemm_a4w4_macro  # noqa: F401
from .packed import PackedWeight, gemm_a4w4_packed, pack_weight, quant_gemm_a4w4_packed  # noqa: F401
from .quant import (quant_gemm_a4w4, quantize_mxfp4, quantize_mxfp4_macro,  # noqa: F401
                    quantize_mxfp4_mbs, shuffle_scales, shuffle_weight)

__all__ = ["gemm_a4w4", "gemm_a4w4_macro", "quantize_mxfp4", "quantize_mxfp4_macro",
           "shuffle_weight", "shuffle_scales", "quant_gemm_a4w4", "pack_weight",
           "gemm_a4w4_packed", "quant_gemm_a4w4_packed", "PackedWeight", "device_error",
           "quantize_mxfp4_mbs"]
