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
