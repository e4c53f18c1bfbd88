"""GPU quantiser and layout kernels: bit-exact against the CPU oracle."""

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O
from tests.gpu_helpers import bf16_bits, seeded_bf16

pytestmark = pytest.mark.gpu


def _special_rows(K: int) -> torch.Tensor:
    """Rows exercising ties, saturation, zero / subnormal / Inf / NaN blocks."""
    grid = torch.tensor([4.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.9, -3.5, -0.0, 0.3],
                        dtype=torch.float32)
    rows = []
    r = torch.zeros(K)
    r[: grid.numel()] = grid
    rows.append(r)
    rows.append(torch.zeros(K))                          # zero blocks -> scale 0
    rows.append(torch.full((K,), 1e-39))                 # subnormal blocks
    r = torch.randn(K)
    r[5] = float("inf")
    rows.append(r)
    r = torch.randn(K)
    r[K - 1] = float("nan")
    rows.append(r)
    rows.append(torch.full((K,), 3.0e38))                # near the top of the range
    rows.append(torch.randn(K) * 1e-30)
    return torch.stack(rows).to(torch.bfloat16)


@pytest.mark.parametrize("R,K", [(1, 32), (7, 64), (33, 96), (64, 1024), (300, 2080)])
@pytest.mark.parametrize("shuffle", [False, True])
def test_quantize_bit_exact(R, K, shuffle):
    x = seeded_bf16(R, K, seed=R * 31 + K)
    if R >= 7:
        x[:7] = _special_rows(K)
    q_ref, s_ref = O.quantize_mxfp4(bf16_bits(x))
    q, s = __import__("mbs_b200").quantize_mxfp4(x.cuda(), shuffle=shuffle)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), q_ref)
    if shuffle:
        assert np.array_equal(s.cpu().numpy(), O.shuffle_scales(s_ref, K))
    else:
        assert np.array_equal(s.cpu().numpy(), s_ref)


def _from_bits(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("macro", [False, True])
def test_quantize_every_bf16_pattern(macro):
    """All 65536 bf16 bit patterns (in order, 32 per block: zero, subnormal,
    normal, Inf and NaN blocks of both signs) against the oracle."""
    import mbs_b200
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(64, 1024)
    x = _from_bits(bits)
    if macro:
        q, s = mbs_b200.quantize_mxfp4_macro(x.cuda())
        q_ref, s_ref = O.quantize_mxfp4_macro(bits)
    else:
        q, s = mbs_b200.quantize_mxfp4(x.cuda(), shuffle=False)
        q_ref, s_ref = O.quantize_mxfp4(bits)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)


def test_quantize_ties_and_saturation_at_every_scale():
    """Blocks whose amax is 4 * 2^k hold every rounding midpoint of the e2m1
    grid (ties to even), values just off the midpoints, values that saturate
    and values that round to zero, at scales k = -126..126, both signs."""
    import mbs_b200
    mids = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, 0.125, 0.2, 0.3, 6.5, 5.5, 4.5, 2.75]
    rows = []
    for k in range(-126, 127):
        blk = np.zeros(32, dtype=np.float32)
        blk[0] = 4.0
        blk[1:1 + len(mids)] = mids
        blk[16:16 + len(mids)] = [-m for m in mids]
        blk[31] = -7.9
        rows.append(np.ldexp(blk, k))
    xf = torch.from_numpy(np.stack(rows)).to(torch.bfloat16)   # [253, 32] rows of one block each
    x = xf.repeat(1, 2)                                         # K = 64
    bits = x.view(torch.int16).numpy().view(np.uint16)
    q, s = mbs_b200.quantize_mxfp4(x.cuda(), shuffle=False)
    q_ref, s_ref = O.quantize_mxfp4(bits)
    torch.cuda.synchronize()
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)


def test_quantize_strided_rows():
    import mbs_b200
    big = seeded_bf16(40, 512, seed=5)
    view = big[:, :256]  # row stride 512 elements
    q, s = mbs_b200.quantize_mxfp4(view.cuda(), shuffle=False)
    q_ref, s_ref = O.quantize_mxfp4(bf16_bits(view))
    assert np.array_equal(q.cpu().numpy(), q_ref) and np.array_equal(s.cpu().numpy(), s_ref)


@pytest.mark.parametrize("N,K", [(32, 64), (70, 96), (256, 1024), (1000, 4096)])
def test_quantize_macro_bit_exact(N, K):
    import mbs_b200
    x = seeded_bf16(N, K, seed=N + K, outlier_frac=0.01)
    q_ref, mb_ref = O.quantize_mxfp4_macro(bf16_bits(x))
    q, mb = mbs_b200.quantize_mxfp4_macro(x.cuda())
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(mb.cpu().numpy(), mb_ref)


@pytest.mark.parametrize("N,K", [(16, 64), (48, 320), (1040, 1024)])
def test_shuffle_weight_bit_exact(N, K):
    import mbs_b200
    rng = np.random.default_rng(N * K)
    w = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    out = mbs_b200.shuffle_weight(torch.from_numpy(w).cuda())
    assert np.array_equal(out.cpu().numpy(), O.shuffle_weight(w))


@pytest.mark.parametrize("R,K", [(1, 32), (45, 320), (256, 8192)])
def test_shuffle_scales_bit_exact(R, K):
    import mbs_b200
    rng = np.random.default_rng(R + K)
    s = rng.integers(0, 256, size=(R, K // 32), dtype=np.uint8)
    out = mbs_b200.shuffle_scales(torch.from_numpy(s).cuda(), K)
    assert np.array_equal(out.cpu().numpy(), O.shuffle_scales(s, K))


def test_quantize_rejects_bad_k():
    import mbs_b200
    with pytest.raises(RuntimeError, match="multiple of 32"):
        mbs_b200.quantize_mxfp4(torch.zeros(4, 48, dtype=torch.bfloat16, device="cuda"))


@pytest.mark.parametrize("R,K", [(1, 32), (33, 96), (300, 2080), (64, 8192), (5, 16384)])
@pytest.mark.parametrize("shuffle", [False, True])
def test_quantize_mbs_bit_exact(R, K, shuffle):
    """Fused MBS factor producer + quantiser against the oracle: codes, scales
    and factor bytes, including zero / subnormal / Inf / NaN / huge rows."""
    import mbs_b200
    x = seeded_bf16(R, K, seed=R * 7 + K)
    x = x * torch.exp2(torch.randint(-30, 30, (R, 1))).to(torch.bfloat16)
    if R >= 7:
        x[:7] = _special_rows(K)
    q, s, f = mbs_b200.quantize_mxfp4_mbs(x.cuda(), shuffle=shuffle)
    torch.cuda.synchronize()
    q_ref, s_ref, f_ref = O.quantize_mxfp4_mbs(bf16_bits(x))
    assert np.array_equal(f.cpu().numpy(), f_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    if shuffle:
        assert np.array_equal(s.cpu().numpy(), O.shuffle_scales(s_ref, K))
    else:
        assert np.array_equal(s.cpu().numpy(), s_ref)


def test_quantize_mbs_every_bf16_pattern():
    import mbs_b200
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16).reshape(64, 1024)
    q, s, f = mbs_b200.quantize_mxfp4_mbs(_from_bits(bits).cuda())
    torch.cuda.synchronize()
    q_ref, s_ref, f_ref = O.quantize_mxfp4_mbs(bits)
    assert np.array_equal(f.cpu().numpy(), f_ref)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)


def test_mbs_end_to_end_gemm():
    """MBS-quantised activations and weights through the GEMM with their factor
    bytes: matches the oracle GEMM on the same bytes, and the factors undo
    the row scaling (close to the bf16 product)."""
    import mbs_b200
    from tests.gpu_helpers import assert_gemm_close
    M, N, K = 96, 512, 1024
    g = torch.Generator().manual_seed(21)
    xa = torch.randn(M, K, generator=g).to(torch.bfloat16)
    xw = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    qa, sa_sh, fa = mbs_b200.quantize_mxfp4_mbs(xa.cuda(), shuffle=True)
    qw, sw, fw = mbs_b200.quantize_mxfp4_mbs(xw.cuda(), shuffle=False)
    B = mbs_b200.shuffle_weight(qw)
    Bs = mbs_b200.shuffle_scales(sw, K)
    out = mbs_b200.gemm_a4w4(qa, B, sa_sh, Bs, fa, fw)
    torch.cuda.synchronize()
    qa_r, sa_r, fa_r = O.quantize_mxfp4_mbs(bf16_bits(xa))
    qw_r, sw_r, fw_r = O.quantize_mxfp4_mbs(bf16_bits(xw))
    ref = O.gemm_ref(qa_r, qw_r, sa_r, sw_r, fa_r, fw_r)
    bound = O.gemm_abs_bound(qa_r, qw_r, sa_r, sw_r)
    assert_gemm_close(out, ref, bound, "mbs gemm")
    exact = xa.float() @ xw.float().T
    rel = (out.float().cpu() - exact).abs().mean() / exact.abs().mean()
    assert rel < 0.2
