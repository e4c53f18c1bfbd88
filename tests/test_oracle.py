"""CPU tests of the oracle: pinned against the reference's own known answers.

Pins:
  * tests/golden/factor_table.npy -- the reference's convert_byte_to_float
    (test_gemm_a4w4.py:47-51) executed on all 256 bytes.
  * tests/golden/gemm_oracle_golden.npz -- the reference's run_torch /
    run_torch_mbs (test_gemm_a4w4.py:28-69) executed on seeded inputs.
  * the reference's MFMA probe known answers (kernel/mfma_probe.hip:40-45,
    95-106): A = B = +1.0 (code 0x2), K = 128, scale 127 -> C = 128;
    A scales {127,128,129,130} over the four 32-K groups -> C = 480.
"""

import os

import numpy as np
import pytest

from oracle import mxfp4_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_factor_table_matches_reference_function():
    ref = np.load(os.path.join(GOLDEN, "factor_table.npy"))
    mine = O.factor_table()
    assert ref.dtype == np.float32 and ref.shape == (256,)
    assert np.array_equal(ref.view(np.uint32), mine.view(np.uint32))
    # the reference kernel's claim: 1/x exactly for all 256 bytes
    x = ((np.arange(256, dtype=np.uint32) << 15) | 0x3F800000).view(np.float32)
    assert np.array_equal(mine, (1.0 / x.astype(np.float64)).astype(np.float32))


@pytest.mark.parametrize("tag", ["5x16x64", "33x48x128", "64x32x256", "17x64x512"])
def test_gemm_oracle_matches_reference_run_torch(tag):
    g = np.load(os.path.join(GOLDEN, "gemm_oracle_golden.npz"))
    a, w, sa, sw, fa, fw = (g[f"{k}_{tag}"] for k in ("a", "w", "sa", "sw", "fa", "fw"))
    out = O.f32_to_bf16_bits(O.gemm_f32(a, w, sa, sw))
    out_mbs = O.f32_to_bf16_bits(O.gemm_f32(a, w, sa, sw, fa, fw))
    assert np.array_equal(out, g[f"out_{tag}"])
    assert np.array_equal(out_mbs, g[f"outmbs_{tag}"])


def test_mfma_probe_known_answers():
    K = 128
    ones = np.full((16, K // 2), 0x22, dtype=np.uint8)  # every nibble = 0x2 = +1.0
    unity = np.full((16, K // 32), 127, dtype=np.uint8)
    c = O.gemm_f32(ones, ones, unity, unity)
    assert np.all(c == 128.0)
    packed = np.tile(np.array([127, 128, 129, 130], dtype=np.uint8), (16, 1))
    c2 = O.gemm_f32(ones, ones, packed, unity)
    assert np.all(c2 == 480.0)


def test_e2m1_and_e8m0_tables():
    assert list(O.E2M1_VALUES[:8]) == [0, 0.5, 1, 1.5, 2, 3, 4, 6]
    assert np.array_equal(O.E2M1_VALUES[8:], -O.E2M1_VALUES[:8])
    e = np.arange(256, dtype=np.uint8)
    v = O.e8m0_to_f32(e)
    assert np.isnan(v[255])
    assert v[127] == 1.0 and v[128] == 2.0 and v[0] == np.float32(2.0 ** -127)
    assert np.all(v[1:255] == np.ldexp(np.float32(1), e[1:255].astype(np.int32) - 127))


def test_fp4_pack_roundtrip():
    rng = np.random.default_rng(0)
    codes = rng.integers(0, 16, size=(7, 64), dtype=np.uint8)
    p = O.pack_fp4(codes)
    assert p.shape == (7, 32)
    assert np.array_equal(p[:, 0], codes[:, 0] | (codes[:, 1] << 4))  # low nibble first
    assert np.array_equal(O.unpack_fp4(p), codes)


def _bf16(vals):
    return O.f32_to_bf16_bits(np.asarray(vals, dtype=np.float32))


def test_quantiser_rne_ties_and_saturation():
    # amax = 4 -> E(4)=129 -> scale byte 127 (2^0): values map straight onto the grid
    vals = [4.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 0.3, 2.6, -3.5, -0.0] + [0.0] * 20
    q, s = O.quantize_mxfp4(_bf16([vals]))
    assert s[0, 0] == 127
    codes = O.unpack_fp4(q)[0, :12]
    # 4->6, .25->0 (tie down), .75->2 (tie up), 1.25->2, 1.75->4, 2.5->4, 3.5->6, 5->6,
    # .3->1, 2.6->5, -3.5->sign|6, -0.0->sign|0
    assert list(codes) == [6, 0, 2, 2, 4, 4, 6, 6, 1, 5, 0x8 | 6, 0x8]
    # amax in [4, 8): 7.9 / 2^0 saturates to 6
    q2, s2 = O.quantize_mxfp4(_bf16([[7.9] + [0.0] * 31]))
    assert s2[0, 0] == 127 and O.unpack_fp4(q2)[0, 0] == 7


def test_quantiser_scale_rule():
    for amax, byte in [(1.0, 125), (6.0, 127), (1e-30, 25), (1e-39, 0), (2.0 ** -126, 0), (2.0 ** -124, 1), (2.0 ** 100, 225), (3.0e38, 252)]:
        _, s = O.quantize_mxfp4(_bf16([[amax] + [0.0] * 31]))
        assert s[0, 0] == byte, (amax, s[0, 0])
    _, s = O.quantize_mxfp4(_bf16([[0.0] * 32]))
    assert s[0, 0] == 0
    q, s = O.quantize_mxfp4(_bf16([[np.inf] + [1.0] * 31, [np.nan] + [1.0] * 31]))
    assert list(s[:, 0]) == [255, 255] and not q.any()


def test_quantiser_dequant_error_bound():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((64, 256)).astype(np.float32)
    xb = O.f32_to_bf16_bits(x)
    q, s = O.quantize_mxfp4(xb)
    xr = O.dequant(q, s)
    xf = O.bf16_bits_to_f32(xb)
    scale = O.e8m0_to_f32(s).repeat(32, axis=1)
    # RNE onto a grid whose spacing is <= 2*scale (spacing 2 at [4,6]); saturation <= 2*scale
    assert np.all(np.abs(xr - xf) <= 2.0 * scale + 1e-30)


def test_flatb_and_flats_are_bijections_and_roundtrip():
    N, K = 48, 320 - 64  # K % 64 == 0
    offs = O.flat_b_offsets(N, K).ravel()
    assert np.array_equal(np.sort(offs), np.arange(N * K // 2))
    rng = np.random.default_rng(2)
    w = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    assert np.array_equal(O.unshuffle_weight(O.shuffle_weight(w)), w)
    R, K2 = 45, 320
    s = rng.integers(0, 256, size=(R, K2 // 32), dtype=np.uint8)
    flat = O.shuffle_scales(s)
    assert flat.shape == (64, O.scale_n_pad(K2))
    assert np.array_equal(O.unshuffle_scales(flat, R, K2), s)
    so = O.flat_s_offsets(64, O.scale_n_pad(K2), O.scale_n_pad(K2)).ravel()
    assert np.array_equal(np.sort(so), np.arange(64 * O.scale_n_pad(K2)))
    # padding is 127
    mask = np.ones(flat.size, bool)
    mask[O.flat_s_offsets(R, K2 // 32, O.scale_n_pad(K2)).ravel()] = False
    assert np.all(flat.ravel()[mask] == 127)


def test_flatb_formula_spot_values():
    # kernel/gemm_a4w4.hip:85-95: (n/16)*(KT*512) + (kp/32)*512 + ((kp%32)/16)*256 + (n%16)*16 + kp%16
    N, K = 32, 256
    off = O.flat_b_offsets(N, K)
    KT = K // 64
    for n, kp in [(0, 0), (1, 0), (0, 16), (0, 32), (17, 45), (31, 127)]:
        exp = (n // 16) * KT * 512 + (kp // 32) * 512 + ((kp % 32) // 16) * 256 + (n % 16) * 16 + kp % 16
        assert off[n, kp] == exp


def test_macro_quantiser_consistency():
    rng = np.random.default_rng(3)
    N, K = 70, 96
    x = rng.standard_normal((N, K)).astype(np.float32)
    xb = O.f32_to_bf16_bits(x)
    q, mb = O.quantize_mxfp4_macro(xb)
    assert mb.shape == (3, O.macro_scale_ld(K))
    assert np.all(mb[:, K // 32:] == 127)
    srow = O.expand_macro_scales(mb, N, K)
    # every row of a 32-row block shares the block's scale; codes equal a per-row
    # quantisation with that scale
    codes = O.quantize_blocks(O.bf16_bits_to_f32(xb).reshape(N, K // 32, 32), srow[..., None])
    assert np.array_equal(O.pack_fp4(codes.reshape(N, K)), q)
    # the block scale is derived from the block amax (rows past N ignored)
    amax = np.abs(O.bf16_bits_to_f32(xb)[64:70, 0:32]).max()
    assert mb[2, 0] == O.scale_byte_from_amax(np.array([amax], np.float32))[0]


def test_check_gemm_detects_single_block_error():
    rng = np.random.default_rng(4)
    M, N, K = 8, 16, 2048
    xb = O.f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    wb = O.f32_to_bf16_bits(rng.standard_normal((N, K)).astype(np.float32))
    qa, sa = O.quantize_mxfp4(xb)
    qw, sw = O.quantize_mxfp4(wb)
    ref = O.gemm_ref(qa, qw, sa, sw)
    bound = O.gemm_abs_bound(qa, qw, sa, sw)
    ok, _, _ = O.check_gemm(ref, ref, bound)
    assert ok
    sw_bad = sw.copy()
    sw_bad[3, 17] += 1  # one 32-K block of one weight row scaled by 2
    bad = O.gemm_ref(qa, qw, sa, sw_bad)
    ok, _, nbad = O.check_gemm(bad, ref, bound)
    assert not ok and nbad >= M // 2


def test_mbs_factor_known_values():
    """6.0 / max: max 1 -> 6 = 1.5 * 4 -> b = 128; max 6 or 3 -> mantissa 0;
    max 5 -> 1.2 -> b = floor(0.2 * 256) = 51 (bits truncated); zero, Inf and
    NaN rows -> 0."""
    rows = np.zeros((7, 32), np.float32)
    rows[0, 3] = -1.0
    rows[1, 0] = 6.0
    rows[2, 9] = 3.0
    rows[3, 1] = 5.0
    rows[5, 2] = np.inf
    rows[6, 2] = np.nan
    b = O.mbs_row_factor(rows)
    assert b.tolist() == [128, 0, 0, 51, 0, 0, 0]
    assert O.mbs_multiplier(np.array([51], np.uint8))[0] == np.float32(1.0 + 51 / 256)
    # the factor table is the inverse of the multiplier, exactly as the reference defines it
    assert np.all(O.byte_to_factor(np.arange(256)) ==
                  (np.float32(1.0) / O.mbs_multiplier(np.arange(256))).astype(np.float32))


def test_mbs_scaled_row_max_lands_just_below_six():
    """After the multiplier the row max is 6 * 2^k * (1 - e) with 0 <= e < 2^-8
    (truncated mantissa), so the largest code of the row is 6 or 4, never the
    saturated spill of a max in (6, 8)."""
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((64, 256)) * np.exp2(rng.integers(-20, 20, (64, 1)))).astype(np.float32)
    xb = O.f32_to_bf16_bits(x)
    xf = O.bf16_bits_to_f32(xb)
    b = O.mbs_row_factor(xf)
    scaled = np.max(np.abs(xf), axis=1) * O.mbs_multiplier(b)
    mant = scaled / np.exp2(np.floor(np.log2(scaled)))      # in [1, 2)
    assert np.all((mant <= 1.5) & (mant > 1.5 * (1 - 2.0 ** -7)))


def test_mbs_quantiser_roundtrip_and_gemm_identity():
    """dequant(q) * f(b) reconstructs x within the MXFP4 error, and the GEMM
    oracle with the factors approximates the bf16 product at least as well as
    plain per-1x32 quantisation on average."""
    rng = np.random.default_rng(12)
    M, N, K = 32, 48, 512
    xa = O.f32_to_bf16_bits(rng.standard_normal((M, K)).astype(np.float32))
    xw = O.f32_to_bf16_bits((rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    qa, sa, fa = O.quantize_mxfp4_mbs(xa)
    qw, sw, fw = O.quantize_mxfp4_mbs(xw)
    rec = O.dequant(qa, sa) * O.byte_to_factor(fa)[:, None]
    xf = O.bf16_bits_to_f32(xa)
    blk_max = np.repeat(np.max(np.abs(xf.reshape(M, K // 32, 32)), axis=-1), 32, axis=1)
    assert np.all(np.abs(rec - xf) <= 0.25 * blk_max + 1e-30)
    exact = xf @ O.bf16_bits_to_f32(xw).T
    mbs = O.gemm_f32(qa, qw, sa, sw, fa, fw)
    pa, psa = O.quantize_mxfp4(xa)
    pw, psw = O.quantize_mxfp4(xw)
    plain = O.gemm_f32(pa, pw, psa, psw)
    assert np.mean(np.abs(mbs - exact)) <= np.mean(np.abs(plain - exact)) * 1.05


def test_mbs_factor_zero_when_scaling_would_overflow():
    big = np.full((2, 32), 3.0e38, np.float32)
    big[1] = 1.0e38
    b = O.mbs_row_factor(big)
    assert b[0] == 0 and b[1] != 0
    assert np.isfinite(1.0e38 * O.mbs_multiplier(b[1:]))
    q, s, f = O.quantize_mxfp4_mbs(O.f32_to_bf16_bits(big))
    assert np.all(s != 0xFF)
