"""CPU tests of the C ABI: the library builds, loads, exports every declared
symbol, and rejects bad arguments before touching a device."""

import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = []
    inc = os.path.join(REPO, "include")
    for fn in sorted(os.listdir(inc)):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(inc, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(",
                             text, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from mbs_b200 import _lib, build
    build.build()
    return _lib.lib()


def test_every_declared_symbol_is_exported(lib):
    from mbs_b200 import _lib
    declared = _declared_functions()
    assert "gemm_a4w4_mxfp4_launch" in declared and len(declared) >= 11
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_status_strings(lib):
    assert lib.mbs_status_string(0) == b"MBS_OK"
    assert lib.mbs_status_string(2) == b"MBS_ERR_UNSUPPORTED_SHAPE"
    assert lib.mbs_status_string(99) == b"MBS_ERR_UNKNOWN"


def _gemm(lib, A=1024, B=1024, AS=1024, BS=1024, out=1024, M=32, N=64, K=128, Mpad=32, snp=8):
    return lib.mbs_gemm_a4w4_launch_ws(A, B, AS, BS, None, None, out, M, N, K, Mpad, snp, None, 0,
                                      None)


def test_gemm_argument_validation_without_device(lib):
    # all of these fail in host-side validation, before any CUDA call
    assert _gemm(lib, A=None) == 1
    assert _gemm(lib, M=0) == 1
    assert _gemm(lib, N=40) == 2                      # N % 16
    assert _gemm(lib, K=96) == 2                      # K % 64
    assert _gemm(lib, Mpad=16) == 1                   # Mpad < roundup(M, 32)
    assert _gemm(lib, snp=4) == 1                     # scaleN_pad < K/32
    assert _gemm(lib, A=1024 + 8) == 3                # misaligned operand
    assert b"multiple of 16" in lib.mbs_last_error_message() or True
    assert _gemm(lib, N=40) == 2
    assert b"N must be a multiple of 16" in lib.mbs_last_error_message()
    st = lib.gemm_a4w4_mxfp4_launch(1024, 1024, 1024, 1024, None, None, 1024, 8, 16, 64, 32, 7,
                                    None)
    assert st == 1 and b"scaleN_pad" in lib.mbs_last_error_message()


def test_quant_and_shuffle_validation_without_device(lib):
    assert lib.mbs_quantize_mxfp4(None, 4, 64, 64, 1024, 1024, 0, None) == 1
    assert lib.mbs_quantize_mxfp4(1024, 4, 48, 48, 1024, 1024, 0, None) == 2
    assert lib.mbs_quantize_mxfp4(1024 + 2, 4, 64, 64, 1024, 1024, 0, None) == 3
    assert lib.mbs_shuffle_weight(1024, 2048, 24, 64, None) == 2
    assert lib.mbs_shuffle_weight(1024, 2048, 32, 96, None) == 2
    assert lib.mbs_shuffle_scales(1024, 2048, 4, 40, None) == 2
    assert lib.mbs_quantize_mxfp4_macro(1024, 4, 40, 64, 1024, 1024, None) == 2


def test_multi_output_and_fused_quant_validation_without_device(lib):
    """The several-copies entry point and the dynamic-quant entry points reject
    bad arguments in host-side validation, before any CUDA call."""
    def multi(dsts, n=None, ldc=16):
        arr = None if dsts is None else (ctypes.c_void_p * max(1, len(dsts)))(*dsts)
        n = len(dsts) if n is None and dsts is not None else (n or 0)
        return lib.mbs_gemm_a4w4_launch_multi(1024, 1024, 1024, 1024, None, None, arr, n, ldc,
                                              8, 16, 64, 32, 8, 1.0, None, None, 0, None)
    assert multi(None) == 1                                   # no output copies
    assert multi([4096], n=0) == 1
    assert multi([4096] * 9) == 1 and b"at most 8" in lib.mbs_last_error_message()
    assert multi([4096], ldc=8) == 1 and b"ldc" in lib.mbs_last_error_message()   # ldc < N
    assert multi([4096], ldc=20) == 1                         # ldc % 8
    assert multi([4096, None]) == 1 and b"copy 1 is NULL" in lib.mbs_last_error_message()
    assert multi([4096, 4096 + 8]) == 3                       # misaligned copy

    def qg(x=4096, ld_x=64, K=64, ws=8192):
        return lib.mbs_quant_gemm_a4w4_launch(x, ld_x, 1024, 1024, None, None, 2048, 8, 16, K, 8, ws,
                                              1 << 20, None)
    assert qg(x=None) == 1
    assert qg(ws=None) == 1
    assert qg(ld_x=32) == 1 and b"ld_x" in lib.mbs_last_error_message()  # ld_x < K
    assert qg(ld_x=68) == 1                                   # ld_x % 8
    assert qg(x=4096 + 2) == 1                                # x not 16-byte aligned
    assert qg(ws=8192 + 16) == 3                              # workspace not 256-byte aligned

    def qp(x=4096, ld_x=64, K=64, ws=8192):
        return lib.mbs_quant_gemm_a4w4_packed_launch(x, ld_x, 1024, None, None, 2048, 8, 16, K, ws, 1 << 20, None)
    assert qp(x=None) == 1
    assert qp(ws=None) == 1
    assert qp(ld_x=32) == 1 and b"ld_x" in lib.mbs_last_error_message()
    assert qp(x=4096 + 2) == 1
    assert qp(ws=8192 + 16) == 3


def test_workspace_size_is_host_only(lib):
    lib.mbs_gemm_a4w4_workspace_size.restype = ctypes.c_size_t
    # decode shapes use stream-K partials; a large prefill runs on CTA pairs
    # whose workspace holds the scale images (1 KB per 128-row block of A or B
    # per 256-element K stage; B's blocks cover whole pair tiles)
    assert lib.mbs_gemm_a4w4_workspace_size(16, 57344, 8192) > 0
    # flag words first, then the pair path's A and B scale images: 8192^3
    # takes 18 column tiles 384 wide and 5 tiles 256 wide (the busiest of 74
    # clusters does 8 wide + 2 narrow tiles, against 14 tiles of 256 or 10 of
    # 384), so B's images cover 8192 / 128 = 64 blocks, plus one
    assert lib.mbs_gemm_a4w4_workspace_size(8192, 8192, 8192) == 4096 + 64 * 32 * 1024 + 65 * 32 * 1024
    # 256-column tiles where both widths take one round: 2048 x 2048 x 1024
    # is 64 tiles of 256 columns (8 x 2 B blocks per stage) against 48 of 384
    assert lib.mbs_gemm_a4w4_workspace_size(2048, 2048, 1024) == 4096 + 16 * 4 * 1024 + 16 * 4 * 1024
    # stream-K: flag words, then one [BN=256][32 rows] fp32 partial slot per CTA (G = 148 SMs
    # is not known without a device, so only the layout's lower bound is checked)
    for shape in [(16, 57344, 8192), (1, 16, 64), (300, 272, 1088)]:
        ws = lib.mbs_gemm_a4w4_workspace_size(*shape)
        assert ws == 0 or ws >= 4096
    assert lib.mbs_gemm_a4w4_workspace_size(0, 16, 64) == 0


def test_kernels_per_call_is_host_only(lib):
    # the CTA-pair path adds its scale-image pass; decode and small shapes launch one kernel
    assert lib.mbs_gemm_a4w4_kernels_per_call(8192, 8192, 8192) == 2
    assert lib.mbs_gemm_a4w4_kernels_per_call(16, 57344, 8192) == 1
    assert lib.mbs_gemm_a4w4_kernels_per_call(256, 512, 1024) == 1
    assert lib.mbs_gemm_a4w4_kernels_per_call(1024, 1024, 5120) == 1  # cluster split-K
    assert lib.mbs_gemm_a4w4_kernels_per_call(2048, 2048, 8192) == 2
    assert lib.mbs_gemm_a4w4_kernels_per_call(0, 16, 64) == -1


def test_workspace_flag_region_matches_header():
    from mbs_b200 import mbs_gemm_a4w4
    hdr = open(os.path.join(REPO, "include", "mbs_gemm_a4w4.h")).read()
    m = re.search(r"#define MBS_GEMM_WS_FLAG_BYTES (\d+)", hdr)
    assert m and int(m.group(1)) == mbs_gemm_a4w4.WS_FLAG_BYTES


def test_python_layer_fails_loudly_without_library(monkeypatch, tmp_path):
    from mbs_b200 import _lib
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    with pytest.raises(RuntimeError, match="no non-CUDA fallback"):
        _lib.lib()


def test_plan_override_is_validated_and_steers_the_planner(lib):
    """mbs_set_plan_override: values outside the documented sets are refused
    (a cluster split-K factor that does not divide the tile rows would address
    CTAs outside the cluster); accepted ones steer the host-side planner, seen
    through the workspace-size and kernels-per-call queries (no device needed:
    without one the planner assumes 148 SMs)."""
    from mbs_b200 import _lib

    def setov(**kw):
        return lib.mbs_set_plan_override(ctypes.byref(_lib.PlanOverride(**kw)))
    try:
        for bad in (dict(ksplit=3), dict(ksplit=5), dict(ksplit=16), dict(split_bn=64), dict(pair_bn=320),
                    dict(schedule=3), dict(grid=-1), dict(swap=2), dict(pair=2)):
            assert setov(**bad) == 1, bad
        auto_ws = lib.mbs_gemm_a4w4_workspace_size(16, 57344, 8192)
        assert auto_ws > 4096  # config[1]: stream-K with 32-row partials
        # forced cluster split-K on a skinny tile: no workspace; split_bn 128 is
        # ignored there (skinny configurations exist only 256 wide)
        assert setov(ksplit=4, split_bn=128) == 0
        assert lib.mbs_gemm_a4w4_workspace_size(16, 1024, 4096) == 0
        assert lib.mbs_gemm_a4w4_kernels_per_call(16, 1024, 4096) == 1
        # forced stream-K on 17 CTAs: flags + 17 partial slots of 32 x 256 fp32
        assert setov(schedule=1, grid=17) == 0
        assert lib.mbs_gemm_a4w4_workspace_size(16, 1024, 4096) == 4096 + 17 * 32 * 256 * 4
        # forced CTA pairs: two launches (scale images + GEMM)
        assert setov(schedule=2, pair=1) == 0
        assert lib.mbs_gemm_a4w4_kernels_per_call(512, 512, 1024) == 2
        assert setov(schedule=2, pair=0) == 0
        assert lib.mbs_gemm_a4w4_kernels_per_call(512, 512, 1024) == 1
    finally:
        assert lib.mbs_set_plan_override(None) == 0
    assert lib.mbs_gemm_a4w4_workspace_size(16, 57344, 8192) == auto_ws
