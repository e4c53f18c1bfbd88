"""mbs_gemm_a4w4_launch_multi on one GPU: the output written to several
buffers at once with a row stride larger than N (the N-sharded layer's
fused exchange, where the copies are the ranks' full outputs and this GEMM
fills one column block of each).  Here the copies are local buffers; every
copy must equal the single-output launch bit for bit, match the oracle, and
leave everything outside its column block untouched, on every schedule."""

import ctypes

import pytest
import torch

from oracle import mxfp4_oracle as O
from tests.gpu_helpers import Case, assert_gemm_close

pytestmark = pytest.mark.gpu

PLANS = {
    "pair256": dict(schedule=2, pair=1, pair_bn=256),
    "pair384": dict(schedule=2, pair=1, pair_bn=384),
    "pair_mix": dict(schedule=2, pair=1, pair_wide=1),
    "dp_single": dict(schedule=2, pair=0),
    "stream_k": dict(schedule=1, grid=17),
    "swap": dict(swap=1),
    "ksplit": dict(ksplit=4),
    "auto": dict(),
}


@pytest.mark.parametrize("sched,M,N,K", [("pair256", 300, 1040, 1024), ("pair384", 512, 768, 512),
                                         ("pair_mix", 300, 1040, 1024), ("dp_single", 200, 768, 512),
                                         ("stream_k", 40, 2048, 2048), ("swap", 24, 1024, 512),
                                         ("ksplit", 200, 768, 2048), ("auto", 16, 4096, 4096)])
@pytest.mark.parametrize("copies,col0,extra", [(3, 64, 96), (1, 0, 16), (8, 256, 0)])
def test_multi_output_copies(plan, sched, M, N, K, copies, col0, extra):
    import mbs_b200
    from mbs_b200 import _lib
    from mbs_b200.mbs_gemm_a4w4 import scale_n_pad, workspace_for
    L = _lib.lib()
    c = Case(M, N, K, seed=M + N + copies, factors=True)
    plan(**PLANS[sched])
    single = mbs_b200.gemm_a4w4(c.A, c.B, c.A_scale, c.B_scale, c.A_factor, c.B_factor)
    ldc = col0 + N + extra
    rows = (M + 31) // 32 * 32 + 8
    bufs = [torch.full((rows, ldc), -5.0 - d, dtype=torch.bfloat16, device="cuda") for d in range(copies)]
    dst = (ctypes.c_void_p * copies)(*[b.data_ptr() + col0 * 2 for b in bufs])
    ws = workspace_for(M, N, K, torch.device("cuda"))
    st = L.mbs_gemm_a4w4_launch_multi(
        c.A.data_ptr(), c.B.data_ptr(), c.A_scale.data_ptr(), c.B_scale.data_ptr(), c.A_factor.data_ptr(),
        c.B_factor.data_ptr(), dst, copies, ldc, M, N, K, (M + 31) // 32 * 32, scale_n_pad(K),
        ctypes.c_float(1.0), None, None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
        torch.cuda.current_stream().cuda_stream)
    assert st == 0, L.mbs_last_error_message()
    torch.cuda.synchronize()
    ref, bound = c.reference()
    for d, b in enumerate(bufs):
        blk = b[:M, col0:col0 + N]
        assert torch.equal(blk, single), f"copy {d} differs from the single-output launch"
        fill = -5.0 - d
        assert torch.all(b[:, :col0] == fill) and torch.all(b[:, col0 + N:] == fill) and torch.all(b[M:] == fill), \
            f"copy {d}: written outside its block"
    assert_gemm_close(bufs[0][:M, col0:col0 + N], ref, bound, f"multi-output {sched}")


def test_multi_output_rejects_bad_arguments():
    from mbs_b200 import _lib
    L = _lib.lib()
    c = Case(32, 256, 512, seed=1)
    buf = torch.empty((32, 512), dtype=torch.bfloat16, device="cuda")

    def call(n, ldc, ptrs=None):
        ptrs = ptrs or [buf.data_ptr()] * max(n, 1)
        dst = (ctypes.c_void_p * len(ptrs))(*ptrs)
        return L.mbs_gemm_a4w4_launch_multi(
            c.A.data_ptr(), c.B.data_ptr(), c.A_scale.data_ptr(), c.B_scale.data_ptr(), None, None, dst, n, ldc,
            32, 256, 512, 32, O.scale_n_pad(512), ctypes.c_float(1.0), None, None, 0,
            torch.cuda.current_stream().cuda_stream)
    assert call(9, 512, [buf.data_ptr()] * 9) == 1       # more than 8 copies
    assert call(0, 512) == 1                               # no copies
    assert call(1, 200) == 1                               # ldc < N
    assert call(1, 260) == 1                               # ldc not a multiple of 8
    assert call(2, 512, [buf.data_ptr(), buf.data_ptr() + 2]) == 3  # misaligned copy


@pytest.mark.parametrize("sched", ["pair384", "pair_mix", "dp_single", "stream_k"])
def test_multi_output_with_alpha_and_bias(plan, sched):
    """The alpha/bias epilogue on the multi-copy path (the staged pair
    epilogue included): every copy equals the single-output
    mbs_gemm_a4w4_launch_ex result bit for bit."""
    import mbs_b200
    from mbs_b200 import _lib
    from mbs_b200.mbs_gemm_a4w4 import scale_n_pad, workspace_for
    L = _lib.lib()
    M, N, K = 300, 1040, 1024
    c = Case(M, N, K, seed=77, factors=True)
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(5)) * 3).to(torch.bfloat16).cuda()
    plan(**PLANS[sched])
    single = mbs_b200.gemm_a4w4(c.A, c.B, c.A_scale, c.B_scale, c.A_factor, c.B_factor, alpha=-1.75, bias=bias)
    copies, col0, ldc = 3, 32, N + 96
    bufs = [torch.full((M + 8, ldc), 9.0, dtype=torch.bfloat16, device="cuda") for _ in range(copies)]
    dst = (ctypes.c_void_p * copies)(*[b.data_ptr() + col0 * 2 for b in bufs])
    ws = workspace_for(M, N, K, torch.device("cuda"))
    st = L.mbs_gemm_a4w4_launch_multi(
        c.A.data_ptr(), c.B.data_ptr(), c.A_scale.data_ptr(), c.B_scale.data_ptr(), c.A_factor.data_ptr(),
        c.B_factor.data_ptr(), dst, copies, ldc, M, N, K, (M + 31) // 32 * 32, scale_n_pad(K),
        ctypes.c_float(-1.75), bias.data_ptr(), None if ws is None else ws.data_ptr(),
        0 if ws is None else ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert st == 0, L.mbs_last_error_message()
    torch.cuda.synchronize()
    for d, b in enumerate(bufs):
        assert torch.equal(b[:M, col0:col0 + N], single), f"copy {d} differs from launch_ex"
        assert torch.all(b[:, :col0] == 9.0) and torch.all(b[:, col0 + N:] == 9.0) and torch.all(b[M:] == 9.0)
