"""GPU GEMM parity: the tcgen05 kernel against the CPU oracle.

Tolerance (written here and in oracle/mxfp4_oracle.py::gemm_tolerance):
    |gpu - ref| <= 2 bf16 ulp(|ref|) + 2^-20 * sum_k |a_k b_k|
where ref is the reference oracle (fp32 dequant-matmul, factor multiply, RNE
bf16; test_gemm_a4w4.py:28-69).
"""

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O
from tests.gpu_helpers import Case, assert_gemm_close, full_check

pytestmark = pytest.mark.gpu


def _gemm(case, factors=True, out=None):
    import mbs_b200
    return mbs_b200.gemm_a4w4(case.A, case.B, case.A_scale, case.B_scale,
                              case.A_factor if factors else None,
                              case.B_factor if factors else None, out=out)


@pytest.mark.parametrize("factors", [False, True])
def test_config0_256x512x1024(factors):
    c = Case(256, 512, 1024, seed=0, factors=factors)
    out = _gemm(c)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, "cfg0")


@pytest.mark.parametrize("M,N,K", [
    (1, 16, 64), (4, 48, 128), (16, 256, 256), (32, 128, 512), (33, 64, 320),
    (64, 512, 1024), (65, 32, 192), (127, 1040, 256), (200, 96, 576), (300, 272, 1088),
])
def test_ragged_shapes_with_factors(M, N, K):
    c = Case(M, N, K, seed=M + N + K, factors=True)
    out = _gemm(c)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, f"{M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K", [(777, 1040, 2048), (8000, 48, 512), (1000, 48, 1024), (8000, 1040, 256)])
def test_tuning_log_ragged_shapes(M, N, K):
    """The ragged M and N the reference's tuning log lists as passing
    (asm_vs_wg_kernel.md:184-187: M = 1000, 777, 33, 300, 8000; N = 48, 1040),
    on the planner's own schedule, full output against the oracle."""
    c = Case(M, N, K, seed=M + 7 * N + K, factors=True)
    out = _gemm(c)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, f"tuning-log {M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K", [(2, 2048, 4096), (24, 1024, 2048), (48, 4096, 1024),
                                   (512, 1024, 2048)])
@pytest.mark.parametrize("grid", [3, 17, 148])
def test_stream_k_splits(plan, M, N, K, grid):
    plan(schedule=1, grid=grid)
    c = Case(M, N, K, seed=grid, factors=True)
    out = _gemm(c)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, f"sk G={grid}")
    # the workspace is left zeroed: a second launch gives the same result
    out2 = _gemm(c)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_one_workspace_serves_every_schedule(plan):
    """Shapes and schedules in sequence on one stream share the cached
    workspace: scale images and wide stream-K partial slots written by one
    launch must never read as another schedule's completion flags."""
    seq = [
        (dict(pair=1), (512, 512, 1024)),                         # CTA pairs: scale images
        (dict(), (300, 1024, 2048)),                                        # cluster split-K: no workspace
        (dict(schedule=1), (300, 1024, 2048)),                    # stream-K, 128-row slots
        (dict(schedule=1, grid=17), (2, 2048, 4096)),   # 3 CTAs per tile
        (dict(schedule=1, grid=29), (48, 1024, 4096)),  # 64-row slots
        (dict(schedule=1, grid=17), (2, 2048, 4096)),
    ]
    for i, (env, (M, N, K)) in enumerate(seq):
        plan(**env)
        c = Case(M, N, K, seed=100 + i, factors=True)
        out = _gemm(c)
        torch.cuda.synchronize()
        ref, bound = c.reference()
        assert_gemm_close(out, ref, bound, f"step {i} {M}x{N}x{K} {env}")


@pytest.mark.parametrize("bn", [256, 384, "mix"])
@pytest.mark.parametrize("M,N,K,macro,grid", [(512, 1024, 2048, False, 0), (300, 1024, 1088, False, 0),
                                              (256, 1040, 512, False, 0), (512, 1024, 2048, True, 0),
                                              (700, 768, 1600, True, 0), (1000, 2000, 768, False, 6)])
def test_cta_pair_path(plan, M, N, K, macro, grid, bn):
    """The CTA-pair kernel with all tiles 256 columns wide, all 384 (an N=256
    plus an N=128 MMA), and mixed (one 384-wide column tile, then 256-wide
    ones in the 384-column configuration): ragged M (rows past M are computed
    from padding and never stored), ragged N inside a tile's second MMA and
    inside a narrow tile, a partial last K stage, both B scale layouts, and
    several tiles per cluster."""
    import mbs_b200
    env = dict(schedule=2, pair=1)
    if bn == "mix":
        env["pair_wide"] = 1
    else:
        env["pair_bn"] = bn
    if grid:
        env["grid"] = grid
    plan(**env)
    c = Case(M, N, K, seed=M + K + (1 if bn == "mix" else bn), factors=True, macro=macro)
    if macro:
        out = mbs_b200.gemm_a4w4_macro(c.A, c.B, c.A_scale, c.B_scale, c.A_factor, c.B_factor)
    else:
        out = _gemm(c)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, f"pair{bn} {M}x{N}x{K} macro={macro} grid={grid}")


@pytest.mark.parametrize("S,M,N,K,kind,bn", [
    (2, 300, 272, 1088, "plain", 256),    # ragged M and N, partial last K stage, 5 stages over 2
    (4, 129, 784, 4160, "plain", 256),    # one row past a tile, 17 stages over 4
    (8, 256, 512, 2048, "plain", 256),    # one stage per rank
    (8, 200, 1024, 2304, "macro", 256),   # macro-block B scales, 9 stages over 8
    (4, 160, 1280, 3072, "packed", 256),  # packed weights
    (4, 1024, 1024, 5120, "plain", 0),    # the reference's small deep-K shape (default plan)
    (2, 300, 272, 1088, "plain", 128),    # 128-column tiles: a last tile of 16 columns
    (4, 129, 784, 4160, "plain", 128),
    (2, 200, 1024, 2304, "macro", 128),
    (4, 1024, 1024, 5120, "plain", 128),
    (4, 16, 784, 4160, "plain", 256),     # skinny tiles (32 rows), 17 stages over 4
    (2, 48, 1024, 2304, "macro", 256),    # 64-row tiles, macro-block scales
    (8, 1, 512, 2048, "plain", 256),      # M = 1, 4 rows per rank
    (4, 24, 1280, 3072, "packed", 256),   # skinny packed weights
    (4, 16, 8192, 8192, "plain", 0),      # skinny, default plan
])
def test_cluster_split_k(plan, S, M, N, K, kind, bn):
    """Cluster split-K: the S CTAs of a cluster take S K ranges of one tile
    (128 x 256, 128 x 128, or a skinny tile of 32 or 64 rows by 256) and add
    their fp32 partials through distributed shared memory, each finishing
    1/S of the tile's rows."""
    import mbs_b200
    if bn:
        plan(ksplit=S, split_bn=bn)
    c = Case(M, N, K, seed=M + N + S + bn, factors=True, macro=kind == "macro",
             b_std=0.02 if kind == "packed" else 1.0)
    if kind == "macro":
        out = mbs_b200.gemm_a4w4_macro(c.A, c.B, c.A_scale, c.B_scale, c.A_factor, c.B_factor)
    elif kind == "packed":
        pw = mbs_b200.pack_weight(c.B, c.B_scale)
        out = mbs_b200.gemm_a4w4_packed(c.A, pw, c.A_scale, c.A_factor, c.B_factor)
    else:
        out = _gemm(c)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, f"ksplit{S} bn{bn} {M}x{N}x{K} {kind}")


@pytest.mark.parametrize("M,N,K", [(384, 1024, 512), (1000, 2048, 256)])
def test_data_parallel_schedule(plan, M, N, K):
    plan(schedule=2, grid=7)
    c = Case(M, N, K, seed=3, factors=True)
    out = _gemm(c)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, "dp")


def test_output_canary_rows_untouched():
    M, N, K = 45, 64, 256
    c = Case(M, N, K, seed=9, factors=True)
    buf = torch.full((96, N), -7.0, dtype=torch.bfloat16, device="cuda")
    out = _gemm(c, out=buf)
    torch.cuda.synchronize()
    assert out.data_ptr() == buf.data_ptr()
    assert torch.all(buf[M:] == -7.0)
    ref, bound = c.reference()
    assert_gemm_close(buf[:M], ref, bound, "canary")


@pytest.mark.parametrize("env", [dict(schedule=2, pair=1, pair_bn=256),
                                 dict(schedule=2, pair=1, pair_bn=384),
                                 dict(schedule=2, pair=0),
                                 dict(schedule=1, grid=5)])
def test_output_only_16_byte_aligned(plan, env):
    """The epilogues store 32 bytes per instruction when `out` is 32-byte
    aligned; an output 16 bytes past such a boundary takes the 16-byte
    stores, with the same values and nothing written outside it."""
    plan(**env)
    M, N, K = 300, 1040, 512
    c = Case(M, N, K, seed=21, factors=True)
    Mpad = (M + 31) // 32 * 32
    flat = torch.full((Mpad * N + 16,), -7.0, dtype=torch.bfloat16, device="cuda")
    buf = flat[8:8 + Mpad * N].view(Mpad, N)
    assert buf.data_ptr() % 32 == 16
    out = _gemm(c, out=buf)
    torch.cuda.synchronize()
    assert out.data_ptr() == buf.data_ptr()
    assert torch.all(flat[:8] == -7.0) and torch.all(flat[8 + Mpad * N:] == -7.0)
    assert torch.all(buf[M:] == -7.0)
    ref, bound = c.reference()
    assert_gemm_close(buf[:M], ref, bound, f"16-byte aligned out {env}")


def test_four_argument_call_and_dtype_views():
    """bench_one.py:31 calls with 4 args; fp4/e8m0 dtypes are byte-reinterpreted."""
    import mbs_b200
    c = Case(64, 256, 512, seed=11)
    out = mbs_b200.gemm_a4w4(c.A.view(torch.float4_e2m1fn_x2), c.B.view(torch.float4_e2m1fn_x2),
                             c.A_scale.view(torch.float8_e8m0fnu), c.B_scale.view(torch.float8_e8m0fnu))
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, "4-arg")


def test_reference_entry_point_internal_workspace():
    """The reference-signature C entry (library-owned scratch) matches the _ws entry."""
    import ctypes

    from mbs_b200 import _lib
    c = Case(8, 1024, 2048, seed=13, factors=True)
    out = torch.empty((32, 1024), dtype=torch.bfloat16, device="cuda")
    st = _lib.lib().gemm_a4w4_mxfp4_launch(
        c.A.data_ptr(), c.B.data_ptr(), c.A_scale.data_ptr(), c.B_scale.data_ptr(),
        c.A_factor.data_ptr(), c.B_factor.data_ptr(), out.data_ptr(), 8, 1024, 2048, 32,
        O.scale_n_pad(2048), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, _lib.lib().mbs_last_error_message()
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out[:8], ref, bound, "c-abi")


def test_rejects_bad_shapes():
    import mbs_b200
    c = Case(8, 32, 64, seed=1)
    with pytest.raises(RuntimeError, match="multiple of 16"):
        mbs_b200.gemm_a4w4(c.A, c.B[:24], c.A_scale, c.B_scale)
    a = torch.zeros(8, 48, dtype=torch.uint8, device="cuda")  # K = 96: not a whole 64-K tile
    b = torch.zeros(16, 48, dtype=torch.uint8, device="cuda")
    s = torch.zeros(64, 8, dtype=torch.uint8, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 64"):
        mbs_b200.gemm_a4w4(a, b, s, s)
    with pytest.raises(RuntimeError, match="A_scale must hold"):
        mbs_b200.gemm_a4w4(c.A, c.B, c.A_scale[:1], c.B_scale)


def test_device_error_word_clear():
    import ctypes

    from mbs_b200 import _lib
    code = ctypes.c_int(-1)
    assert _lib.lib().mbs_device_error(ctypes.byref(code), 0) == 0
    assert code.value == 0


@pytest.mark.parametrize("M", [1, 4, 16, 32])
def test_decode_full_size(M):
    """Decode shape N=57344, K=8192 at full size with
    MBS factors: every output element against the oracle (its weight rows
    dequantised in blocks of 8192)."""
    import mbs_b200
    N, K = 57344, 8192
    g = torch.Generator(device="cuda").manual_seed(100 + M)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    qa, sa_sh = mbs_b200.quantize_mxfp4(x, shuffle=True)
    _, sa = mbs_b200.quantize_mxfp4(x, shuffle=False)
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    B = mbs_b200.shuffle_weight(qw)
    B_scale = mbs_b200.shuffle_scales(sw, K)
    fa = torch.randint(0, 256, (M,), dtype=torch.uint8, device="cuda", generator=g)
    fb = torch.randint(0, 256, (N,), dtype=torch.uint8, device="cuda", generator=g)
    out = mbs_b200.gemm_a4w4(qa, B, sa_sh, B_scale, fa, fb)
    torch.cuda.synchronize()
    full_check(out, qa.cpu().numpy(), sa.cpu().numpy(), qw.cpu().numpy(), sw.cpu().numpy(),
               fa.cpu().numpy(), fb.cpu().numpy(), what=f"config[1] decode M={M}")


def test_prefill_8192_cubed_full_and_scale_property():
    """M=N=K=8192 on the planner's own CTA-pair layout:
    every output element against the oracle, and the size-independent
    property that adding 1 to every B scale byte doubles every output exactly."""
    import mbs_b200
    n = 8192
    g = torch.Generator(device="cuda").manual_seed(8192)
    x = torch.randn(n, n, device="cuda", generator=g).to(torch.bfloat16)
    w = torch.randn(n, n, device="cuda", generator=g).to(torch.bfloat16)
    qa, sa_sh = mbs_b200.quantize_mxfp4(x, shuffle=True)
    _, sa = mbs_b200.quantize_mxfp4(x, shuffle=False)
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    del x, w
    B = mbs_b200.shuffle_weight(qw)
    B_scale = mbs_b200.shuffle_scales(sw, n)
    out = mbs_b200.gemm_a4w4(qa, B, sa_sh, B_scale)
    out2 = mbs_b200.gemm_a4w4(qa, B, sa_sh, B_scale + 1)
    torch.cuda.synchronize()
    assert torch.equal(out2.float(), out.float() * 2)
    full_check(out, qa.cpu().numpy(), sa.cpu().numpy(), qw.cpu().numpy(), sw.cpu().numpy(),
               what="config[2] 8192^3")


def test_config3_macro_full_size():
    """BASELINE config[3] at full size (4096 x 7168 x 18432; macro-block B
    scales, N(0, 0.02) weights, activations with 1 % x20 outliers, MBS
    factors) on the planner's own mixed 384/256-column CTA-pair layout: every
    output element against the oracle, and adding 1 to every A scale byte
    doubles every output exactly."""
    import mbs_b200
    M, N, K = 4096, 7168, 18432
    g = torch.Generator(device="cuda").manual_seed(33)
    x = torch.randn(M, K, device="cuda", generator=g)
    x = torch.where(torch.rand(M, K, device="cuda", generator=g) < 0.01, x * 20, x).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    qa, sa_sh = mbs_b200.quantize_mxfp4(x, shuffle=True)
    _, sa = mbs_b200.quantize_mxfp4(x, shuffle=False)
    qw, mb = mbs_b200.quantize_mxfp4_macro(w)
    del x, w
    B = mbs_b200.shuffle_weight(qw)
    fa = torch.randint(0, 256, (M,), dtype=torch.uint8, device="cuda", generator=g)
    fb = torch.randint(0, 256, (N,), dtype=torch.uint8, device="cuda", generator=g)
    out = mbs_b200.gemm_a4w4_macro(qa, B, sa_sh, mb, fa, fb)
    # shuffled A scales: bytes past the real ones are padding (127), +1 keeps the ratio exact
    # only where scales exist, so double the plain scale bytes and re-shuffle
    sa2 = mbs_b200.shuffle_scales(sa + 1, K)
    out2 = mbs_b200.gemm_a4w4_macro(qa, B, sa2, mb, fa, fb)
    torch.cuda.synchronize()
    assert torch.equal(out2.float(), out.float() * 2)
    sb = O.expand_macro_scales(mb.cpu().numpy(), N, K)
    full_check(out, qa.cpu().numpy(), sa.cpu().numpy(), qw.cpu().numpy(), sb,
               fa.cpu().numpy(), fb.cpu().numpy(), what="config[3] macro 4096x7168x18432")


def test_bounded_wait_runs_out_and_the_next_launch_is_clean(plan):
    """The failure path of a bounded device wait: with the stream-K
    contributors' completion flags withheld (mbs_set_withhold_release, a flag
    that nothing sets), each split tile's owner waits until its 2 s limit,
    records MBS_ERR_DEVICE_TIMEOUT and ends its kernel.  The context stays
    usable: after the error is read and cleared, the next launch on the same
    workspace matches the oracle (the flag words were never set)."""
    import ctypes

    import mbs_b200
    from mbs_b200 import _lib
    L = _lib.lib()
    plan(schedule=1, grid=17)  # 16 tiles x 8 K stages over 17 CTAs: every tile is split
    c = Case(16, 4096, 2048, seed=5, factors=True)
    assert mbs_b200.device_error(reset=True) == 0
    assert L.mbs_set_withhold_release(1) == 0
    try:
        _gemm(c)
        code = ctypes.c_int(0)
        assert L.mbs_device_error(ctypes.byref(code), 0) == 0  # synchronises
        assert code.value == 7, f"expected MBS_ERR_DEVICE_TIMEOUT (7), got {code.value}"
    finally:
        assert L.mbs_set_withhold_release(0) == 0
    assert mbs_b200.device_error(reset=True) == 7  # read and clear (also zeroes cached flag words)
    assert mbs_b200.device_error() == 0
    out = _gemm(c)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, "after a device timeout")
    assert mbs_b200.device_error() == 0


@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (33, 96, 576), (8, 256, 512)])
def test_macro_block_variant(M, N, K):
    import mbs_b200
    c = Case(M, N, K, seed=21, factors=True, b_std=0.02, outlier_frac=0.01, macro=True)
    out = mbs_b200.gemm_a4w4_macro(c.A, c.B, c.A_scale, c.B_scale, c.A_factor, c.B_factor)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, "macro")
