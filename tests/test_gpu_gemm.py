"""GPU GEMM parity: the tcgen05 kernel against the CPU oracle.

Tolerance (written here and in oracle/mxfp4_oracle.py::gemm_tolerance):
    |gpu - ref| <= 2 bf16 ulp(|ref|) + 2^-16 * sum_k |a_k b_k|
where ref is the reference oracle (fp32 dequant-matmul, factor multiply, RNE
bf16; test_gemm_a4w4.py:28-69).
"""

import os

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O
from tests.gpu_helpers import Case, assert_gemm_close

pytestmark = pytest.mark.gpu


def _gemm(case, factors=True, out=None):
    import mbs_b200
    return mbs_b200.gemm_a4w4(case.A, case.B, case.A_scale, case.B_scale,
                              case.A_factor if factors else None,
                              case.B_factor if factors else None, out=out)


@pytest.fixture
def force_env():
    saved = {}

    def set_(**kw):
        for k, v in kw.items():
            saved.setdefault(k, os.environ.get(k))
            os.environ[k] = str(v)
    yield set_
    for k, v in saved.items():
        if v is None:
            os.environ.pop(k, None)
        else:
            os.environ[k] = v


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


@pytest.mark.parametrize("M,N,K", [(2, 2048, 4096), (24, 1024, 2048), (48, 4096, 1024),
                                   (512, 1024, 2048)])
@pytest.mark.parametrize("grid", [3, 17, 148])
def test_stream_k_splits(force_env, M, N, K, grid):
    force_env(MBS_FORCE_SCHEDULE=1, MBS_FORCE_GRID=grid)
    c = Case(M, N, K, seed=grid, factors=True)
    out = _gemm(c)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, f"sk G={grid}")
    # the workspace is left zeroed: a second launch gives the same result
    out2 = _gemm(c)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


def test_one_workspace_serves_every_schedule(force_env):
    """Shapes and schedules in sequence on one stream share the cached
    workspace: scale images and wide stream-K partial slots written by one
    launch must never read as another schedule's completion flags."""
    seq = [
        (dict(MBS_FORCE_PAIR=1), (512, 512, 1024)),                         # CTA pairs: scale images
        (dict(), (300, 1024, 2048)),                                        # cluster split-K: no workspace
        (dict(MBS_FORCE_SCHEDULE=1), (300, 1024, 2048)),                    # stream-K, 128-row slots
        (dict(MBS_FORCE_SCHEDULE=1, MBS_FORCE_GRID=17), (2, 2048, 4096)),   # 3 CTAs per tile
        (dict(MBS_FORCE_SCHEDULE=1, MBS_FORCE_GRID=29), (48, 1024, 4096)),  # 64-row slots
        (dict(MBS_FORCE_SCHEDULE=1, MBS_FORCE_GRID=17), (2, 2048, 4096)),
    ]
    for i, (env, (M, N, K)) in enumerate(seq):
        for k in ("MBS_FORCE_SCHEDULE", "MBS_FORCE_GRID", "MBS_FORCE_PAIR"):
            force_env(**{k: ""})
            os.environ.pop(k)
        force_env(**env)
        c = Case(M, N, K, seed=100 + i, factors=True)
        out = _gemm(c)
        torch.cuda.synchronize()
        ref, bound = c.reference()
        assert_gemm_close(out, ref, bound, f"step {i} {M}x{N}x{K} {env}")


@pytest.mark.parametrize("bn", [256, 384, "mix"])
@pytest.mark.parametrize("M,N,K,macro,grid", [(512, 1024, 2048, False, 0), (300, 1024, 1088, False, 0),
                                              (256, 1040, 512, False, 0), (512, 1024, 2048, True, 0),
                                              (700, 768, 1600, True, 0), (1000, 2000, 768, False, 6)])
def test_cta_pair_path(force_env, M, N, K, macro, grid, bn):
    """The CTA-pair kernel with all tiles 256 columns wide, all 384 (an N=256
    plus an N=128 MMA), and mixed (one 384-wide column tile, then 256-wide
    ones in the 384-column configuration): ragged M (rows past M are computed
    from padding and never stored), ragged N inside a tile's second MMA and
    inside a narrow tile, a partial last K stage, both B scale layouts, and
    several tiles per cluster."""
    import mbs_b200
    env = dict(MBS_FORCE_SCHEDULE=2, MBS_FORCE_PAIR=1)
    if bn == "mix":
        env["MBS_PAIR_WIDE"] = 1
    else:
        env["MBS_PAIR_BN"] = bn
    if grid:
        env["MBS_FORCE_GRID"] = grid
    force_env(**env)
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
def test_cluster_split_k(force_env, S, M, N, K, kind, bn):
    """Cluster split-K: the S CTAs of a cluster take S K ranges of one tile
    (128 x 256, 128 x 128, or a skinny tile of 32 or 64 rows by 256) and add
    their fp32 partials through distributed shared memory, each finishing
    1/S of the tile's rows."""
    import mbs_b200
    if bn:
        force_env(MBS_KSPLIT=S, MBS_SPLIT_BN=bn)
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
def test_data_parallel_schedule(force_env, M, N, K):
    force_env(MBS_FORCE_SCHEDULE=2, MBS_FORCE_GRID=7)
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


@pytest.mark.parametrize("env", [dict(MBS_FORCE_SCHEDULE=2, MBS_FORCE_PAIR=1, MBS_PAIR_BN=256),
                                 dict(MBS_FORCE_SCHEDULE=2, MBS_FORCE_PAIR=1, MBS_PAIR_BN=384),
                                 dict(MBS_FORCE_SCHEDULE=2, MBS_FORCE_PAIR=0),
                                 dict(MBS_FORCE_SCHEDULE=1, MBS_FORCE_GRID=5)])
def test_output_only_16_byte_aligned(force_env, env):
    """The epilogues store 32 bytes per instruction when `out` is 32-byte
    aligned; an output 16 bytes past such a boundary takes the 16-byte
    stores, with the same values and nothing written outside it."""
    force_env(**env)
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
def test_decode_full_size_sampled(M):
    """Decode shape N=57344, K=8192 at full size; parity on
    a sample of output columns (the oracle dequantises only those weight rows)."""
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
    cols = np.sort(np.random.default_rng(M).choice(N, 2048, replace=False))
    tc = torch.from_numpy(cols).cuda()
    ref = O.gemm_ref(qa.cpu().numpy(), qw[tc].cpu().numpy(), sa.cpu().numpy(), sw[tc].cpu().numpy(),
                     fa.cpu().numpy(), fb[tc].cpu().numpy())
    bound = O.gemm_abs_bound(qa.cpu().numpy(), qw[tc].cpu().numpy(), sa.cpu().numpy(),
                             sw[tc].cpu().numpy())
    assert_gemm_close(out[:, tc], ref, bound, f"decode M={M}")


def test_prefill_8192_cubed_sampled_and_scale_property():
    """M=N=K=8192: parity on a 256x256 sample, and the
    size-independent property that adding 1 to every B scale byte doubles
    every output exactly."""
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
    rows = np.sort(np.random.default_rng(1).choice(n, 256, replace=False))
    cols = np.sort(np.random.default_rng(2).choice(n, 256, replace=False))
    tr, tcol = torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()
    ref = O.gemm_ref(qa[tr].cpu().numpy(), qw[tcol].cpu().numpy(), sa[tr].cpu().numpy(),
                     sw[tcol].cpu().numpy())
    bound = O.gemm_abs_bound(qa[tr].cpu().numpy(), qw[tcol].cpu().numpy(), sa[tr].cpu().numpy(),
                             sw[tcol].cpu().numpy())
    assert_gemm_close(out[tr][:, tcol], ref, bound, "8192^3")


def test_config3_macro_full_size_sampled():
    """BASELINE config[3] at full size (4096 x 7168 x 18432; macro-block B
    scales, N(0, 0.02) weights, activations with 1 % x20 outliers, MBS
    factors): the planner's own mixed 384/256-column CTA-pair layout, parity
    on a 128 x 128 sample of rows and columns."""
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
    torch.cuda.synchronize()
    rows = np.sort(np.random.default_rng(3).choice(M, 128, replace=False))
    cols = np.sort(np.random.default_rng(4).choice(N, 128, replace=False))
    tr, tcol = torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()
    sb = O.expand_macro_scales(mb.cpu().numpy(), N, K)[cols]
    qa_s, qw_s, sa_s = qa[tr].cpu().numpy(), qw[tcol].cpu().numpy(), sa[tr].cpu().numpy()
    ref = O.gemm_ref(qa_s, qw_s, sa_s, sb, fa[tr].cpu().numpy().reshape(-1, 1),
                     fb[tcol].cpu().numpy().reshape(-1, 1))
    bound = O.gemm_abs_bound(qa_s, qw_s, sa_s, sb)
    assert_gemm_close(out[tr][:, tcol], ref, bound, "config[3] full size")


@pytest.mark.parametrize("M,N,K", [(256, 512, 1024), (33, 96, 576), (8, 256, 512)])
def test_macro_block_variant(M, N, K):
    import mbs_b200
    c = Case(M, N, K, seed=21, factors=True, b_std=0.02, outlier_frac=0.01, macro=True)
    out = mbs_b200.gemm_a4w4_macro(c.A, c.B, c.A_scale, c.B_scale, c.A_factor, c.B_factor)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, "macro")
