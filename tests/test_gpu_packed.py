"""Packed weight format and the GEMM that streams it (decode-oriented path)."""

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O
from tests.gpu_helpers import Case, assert_gemm_close

pytestmark = pytest.mark.gpu

PACK_STAGE = 256 * 128 + 4 * 512


def packed_reference(w_plain: np.ndarray, s_plain: np.ndarray, N: int, K: int) -> np.ndarray:
    """numpy restatement of the packed layout (include/mbs_gemm_a4w4.h)."""
    flat = O.shuffle_weight(w_plain).reshape(-1)
    tiles, kst = (N + 255) // 256, (K + 255) // 256
    out = np.zeros((tiles, kst, PACK_STAGE), dtype=np.uint8)
    chunks = K // 32
    for t in range(tiles):
        for ks in range(kst):
            blk = out[t, ks]
            for c in range(8):
                for nt in range(16):
                    ntile, chunk = t * 16 + nt, ks * 8 + c
                    if ntile * 16 < N and chunk < chunks:
                        src = ntile * K * 8 + chunk * 256
                        blk[(c * 16 + nt) * 256:(c * 16 + nt + 1) * 256] = flat[src:src + 256]
            for q in range(2):
                for rb in range(2):
                    for r in range(128):
                        row = 256 * t + 128 * rb + r
                        if row >= N:
                            continue
                        base = 32768 + (2 * q + rb) * 512 + (r % 32) * 16 + (r // 32) * 4
                        for k in range(4):
                            kb = 8 * ks + 4 * q + k
                            if kb < s_plain.shape[1]:
                                blk[base + k] = s_plain[row, kb]
    return out.reshape(-1)


@pytest.mark.parametrize("N,K", [(256, 256), (272, 576), (512, 1024)])
def test_pack_layout_bit_exact(N, K):
    import mbs_b200
    rng = np.random.default_rng(N + K)
    w = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    s = rng.integers(110, 140, size=(N, K // 32), dtype=np.uint8)
    B = torch.from_numpy(O.shuffle_weight(w)).cuda()
    Bs = torch.from_numpy(O.shuffle_scales(s, K)).cuda()
    pw = mbs_b200.pack_weight(B, Bs)
    got = pw.data.cpu().numpy()
    ref = packed_reference(w, s, N, K)
    # scale bytes of K groups beyond K/32 come from the flatS padding (127) on the GPU
    assert got.shape == ref.shape
    tiles, kst = (N + 255) // 256, (K + 255) // 256
    g = got.reshape(tiles, kst, PACK_STAGE)
    r = ref.reshape(tiles, kst, PACK_STAGE)
    assert np.array_equal(g[:, :, :32768], r[:, :, :32768])
    if K % 256 == 0:
        assert np.array_equal(g, r)


@pytest.mark.parametrize("M,N,K", [(1, 512, 1024), (16, 4096, 2048), (32, 272, 576), (48, 1024, 512),
                                   (100, 768, 512), (300, 2048, 1024)])
def test_packed_gemm_matches_oracle(M, N, K):
    import mbs_b200
    c = Case(M, N, K, seed=M * 7 + N, factors=True, b_std=0.02)
    pw = mbs_b200.pack_weight(c.B, c.B_scale)
    out = mbs_b200.gemm_a4w4_packed(c.A, pw, c.A_scale, c.A_factor, c.B_factor)
    torch.cuda.synchronize()
    ref, bound = c.reference()
    assert_gemm_close(out, ref, bound, f"packed {M}x{N}x{K}")
    # same inputs through the drop-in operator
    out2 = mbs_b200.gemm_a4w4(c.A, c.B, c.A_scale, c.B_scale, c.A_factor, c.B_factor)
    torch.cuda.synchronize()
    assert_gemm_close(out2, ref, bound, "drop-in")


def test_packed_decode_full_size_sampled():
    import mbs_b200
    M, N, K = 16, 57344, 8192
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    qa, sa_sh = mbs_b200.quantize_mxfp4(x, shuffle=True)
    _, sa = mbs_b200.quantize_mxfp4(x, shuffle=False)
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    pw = mbs_b200.pack_weight(mbs_b200.shuffle_weight(qw), mbs_b200.shuffle_scales(sw, K))
    out = mbs_b200.gemm_a4w4_packed(qa, pw, sa_sh)
    torch.cuda.synchronize()
    cols = np.sort(np.random.default_rng(3).choice(N, 2048, replace=False))
    tc = torch.from_numpy(cols).cuda()
    ref = O.gemm_ref(qa.cpu().numpy(), qw[tc].cpu().numpy(), sa.cpu().numpy(), sw[tc].cpu().numpy())
    bound = O.gemm_abs_bound(qa.cpu().numpy(), qw[tc].cpu().numpy(), sa.cpu().numpy(), sw[tc].cpu().numpy())
    assert_gemm_close(out[:, tc], ref, bound, "packed decode")


_PACKED_FUSED_PLANS = {
    "auto": dict(),
    "stream_k": dict(schedule=1, grid=17),
    "dp_single": dict(schedule=2, pair=0),
    "ksplit": dict(ksplit=4),
}


@pytest.mark.parametrize("sched,M,N,K", [
    ("auto", 1, 57344, 8192), ("auto", 8, 57344, 8192), ("auto", 16, 57344, 8192),  # config[1]
    ("auto", 12, 8192, 8192),                        # skinny cluster split-K
    ("stream_k", 9, 2048, 1088), ("stream_k", 16, 1024, 576),
    ("dp_single", 13, 272, 320), ("dp_single", 5, 256, 64),
    ("ksplit", 16, 2048, 4096), ("ksplit", 3, 2048, 4096),
    ("auto", 17, 4096, 2048), ("auto", 40, 2048, 1024),  # past 16 rows: the stand-alone quantiser first
])
def test_fused_quant_with_packed_weights(plan, sched, M, N, K):
    """quant_gemm_a4w4_packed (bf16 activations, packed weights) is bit-identical
    to quantize_mxfp4 + gemm_a4w4_packed: up to 8 rows converted in shared memory
    by one warp, up to 16 by two, more by the stand-alone quantiser first; and
    within the oracle's tolerance where that is cheap to compute."""
    import mbs_b200
    from tests.gpu_helpers import seeded_bf16, bf16_bits
    w = seeded_bf16(N, K, N + K, std=0.02).cuda()
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    W = mbs_b200.pack_weight(mbs_b200.shuffle_weight(qw), mbs_b200.shuffle_scales(sw, K))
    x = seeded_bf16(M, K, M, outlier_frac=0.01).cuda()
    g = torch.Generator(device="cuda").manual_seed(M + 3)
    fa = torch.randint(0, 256, (M,), dtype=torch.uint8, device="cuda", generator=g)
    fb = torch.randint(0, 256, (N,), dtype=torch.uint8, device="cuda", generator=g)
    plan(**_PACKED_FUSED_PLANS[sched])
    q, s = mbs_b200.quantize_mxfp4(x, shuffle=True)
    ref2 = mbs_b200.gemm_a4w4_packed(q, W, s, fa, fb)
    for call in range(2):  # the second call reuses the cached workspace
        got = mbs_b200.quant_gemm_a4w4_packed(x, W, fa, fb)
        torch.cuda.synchronize()
        assert torch.equal(got, ref2), f"call {call}: differs from quantise + gemm_a4w4_packed"
    assert mbs_b200.device_error() == 0
    if M * N <= 1 << 22:
        qa, sa = O.quantize_mxfp4(bf16_bits(x.cpu()))
        wq, ws = qw.cpu().numpy(), sw.cpu().numpy()
        ref = O.gemm_ref(qa, wq, sa, ws, fa.cpu().numpy(), fb.cpu().numpy())
        assert_gemm_close(got, ref, O.gemm_abs_bound(qa, wq, sa, ws), f"fused packed {sched} {M}x{N}x{K}")


@pytest.mark.parametrize("M", [14, 6])
def test_fused_quant_with_packed_weights_special_values(M):
    """Inf / NaN / zero / -0 / near-maximum blocks through the in-stage
    quantiser with packed weights: the same bytes as the stand-alone quantiser,
    so the outputs agree bit for bit (NaN patterns included)."""
    import mbs_b200
    from tests.gpu_helpers import seeded_bf16
    N, K = 2048, 2048
    w = seeded_bf16(N, K, 9, std=0.02).cuda()
    qw, sw = mbs_b200.quantize_mxfp4(w, shuffle=False)
    W = mbs_b200.pack_weight(mbs_b200.shuffle_weight(qw), mbs_b200.shuffle_scales(sw, K))
    x = seeded_bf16(M, K, 3).cuda()
    x[0, 5] = float("inf")
    x[1, 40] = float("-inf")
    x[2, 77] = float("nan")
    x[3, :64] = 0.0
    x[4, 64:96] = -0.0
    x[5, 96:128] = 3.0e38
    x[M - 1, 128:160] = -1.0e-38
    q, s = mbs_b200.quantize_mxfp4(x, shuffle=True)
    ref2 = mbs_b200.gemm_a4w4_packed(q, W, s)
    got = mbs_b200.quant_gemm_a4w4_packed(x, W)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref2.view(torch.int16))
    assert mbs_b200.device_error() == 0
