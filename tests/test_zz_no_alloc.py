"""The allocation-free GEMM entry point, through the C ABI.

mbs_gemm_a4w4_launch_noalloc exists for callers that may not allocate device
memory (a plugin whose host framework owns every device allocation, or a loop
that cannot afford cudaMalloc's implicit synchronisation).  Its scratch is a
static buffer inside the library; the caller passes only inputs and outputs.
Here its output must match the CPU oracle within the GEMM parity tolerance,
and the workspace entry point's output bit for bit, on two calls in a row
(the second call reuses the scratch the first one left behind).  This file is collected last
and also passes when run alone in a fresh process.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O
from tests.gpu_helpers import Case

pytestmark = pytest.mark.gpu


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _args(c, out):
    return (c.A.data_ptr(), c.B.data_ptr(), c.A_scale.data_ptr(), c.B_scale.data_ptr(),
            c.A_factor.data_ptr(), c.B_factor.data_ptr(), out.data_ptr(),
            c.M, c.N, c.K, (c.M + 31) // 32 * 32, O.scale_n_pad(c.K))


# (8, 4096, 1024) and (48, 2048, 1024) take the stream-K schedule (too few K
# stages for cluster split-K), so their scratch lives in the static buffer;
# (512, 512, 1024) the CTA-pair schedule, whose scale images live there too;
# (256, 512, 1024) data-parallel single CTAs, which need no scratch.
@pytest.mark.parametrize("M,N,K,needs_scratch", [(8, 4096, 1024, True), (48, 2048, 1024, True),
                                                 (512, 512, 1024, True), (256, 512, 1024, False)])
def test_noalloc_matches_oracle_and_workspace_entry_point(M, N, K, needs_scratch):
    from mbs_b200 import _lib
    L = _lib.lib()
    need = int(L.mbs_gemm_a4w4_workspace_size(M, N, K))
    assert (need > 0) == needs_scratch, f"planner changed: {M}x{N}x{K} needs {need} bytes of scratch"
    assert need <= 8 << 20
    c = Case(M, N, K, seed=M + K, factors=True)
    Mpad = (M + 31) // 32 * 32
    ws_out = torch.empty((Mpad, N), dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    st = L.mbs_gemm_a4w4_launch_ws(*_args(c, ws_out), ws.data_ptr(), ws.numel(), _stream())
    assert st == 0, L.mbs_last_error_message()
    torch.cuda.synchronize()
    ref, bound = c.reference()  # the CPU oracle (the reference's fp32 dequantise-then-matmul)
    for call in range(2):
        out = torch.full((Mpad, N), -3.0, dtype=torch.bfloat16, device="cuda")
        st = L.mbs_gemm_a4w4_launch_noalloc(*_args(c, out), _stream())
        assert st == 0, L.mbs_last_error_message()
        torch.cuda.synchronize()
        ok, ratio, nbad = O.check_gemm(out[:M].float().cpu().numpy(), ref, bound)
        assert ok, f"call {call}: {nbad} elements outside the oracle tolerance (max ratio {ratio})"
        # same plan, same kernel: bit-identical to the workspace entry point
        assert torch.equal(out[:M], ws_out[:M]), f"call {call}: differs from mbs_gemm_a4w4_launch_ws"
        assert torch.all(out[M:] == -3.0), "rows >= M were written"


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from mbs_b200 import _lib
    L = _lib.lib()
    # 64x57344x1024: skinny stream-K on every SM with 64-row partials,
    # 148 x 64 KB, more than the 8 MiB static buffer.  The entry point refuses
    # before reading any operand, so zero-filled buffers of the right sizes do.
    M, N, K = 64, 57344, 1024
    assert L.mbs_gemm_a4w4_workspace_size(M, N, K) > 8 << 20
    snp = O.scale_n_pad(K)
    A = torch.zeros((M, K // 2), dtype=torch.uint8, device="cuda")
    B = torch.zeros((N, K // 2), dtype=torch.uint8, device="cuda")
    As = torch.zeros((M * snp,), dtype=torch.uint8, device="cuda")
    Bs = torch.zeros((N * snp,), dtype=torch.uint8, device="cuda")
    out = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    st = L.mbs_gemm_a4w4_launch_noalloc(A.data_ptr(), B.data_ptr(), As.data_ptr(), Bs.data_ptr(), None,
                                        None, out.data_ptr(), M, N, K, M, snp, _stream())
    assert st == 5  # MBS_ERR_WORKSPACE
    assert b"static buffer" in L.mbs_last_error_message()
