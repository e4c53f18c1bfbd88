"""Shared helpers of the GPU parity tests: seeded inputs and oracle comparison."""

from __future__ import annotations

import numpy as np
import torch

from oracle import mxfp4_oracle as O


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def seeded_bf16(rows: int, cols: int, seed: int, std: float = 1.0, outlier_frac: float = 0.0,
                outlier_mult: float = 20.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g) * std
    if outlier_frac > 0:
        mask = torch.rand(rows, cols, generator=g) < outlier_frac
        x = torch.where(mask, x * outlier_mult, x)
    return x.to(torch.bfloat16)


class Case:
    """Quantised GEMM inputs built with the oracle (so GEMM tests do not depend
    on the GPU quantiser), uploaded in the reference's device layouts."""

    def __init__(self, M, N, K, seed=0, factors=False, a_std=1.0, b_std=1.0, outlier_frac=0.0,
                 macro=False, device="cuda"):
        self.M, self.N, self.K = M, N, K
        xa = seeded_bf16(M, K, seed, a_std, outlier_frac)
        xb = seeded_bf16(N, K, seed + 1, b_std)
        self.qa, self.sa = O.quantize_mxfp4(bf16_bits(xa))
        if macro:
            self.qb, self.mb = O.quantize_mxfp4_macro(bf16_bits(xb))
            self.sb = O.expand_macro_scales(self.mb, N, K)
        else:
            self.qb, self.sb = O.quantize_mxfp4(bf16_bits(xb))
            self.mb = None
        rng = np.random.default_rng(seed + 7)
        self.fa = rng.integers(0, 256, size=(M, 1), dtype=np.uint8) if factors else None
        self.fb = rng.integers(0, 256, size=(N, 1), dtype=np.uint8) if factors else None
        dev = torch.device(device)
        up = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        self.A = up(self.qa)
        self.B = up(O.shuffle_weight(self.qb))
        self.A_scale = up(O.shuffle_scales(self.sa, K))
        self.B_scale = up(self.mb) if macro else up(O.shuffle_scales(self.sb, K))
        self.A_factor = up(self.fa) if factors else None
        self.B_factor = up(self.fb) if factors else None

    def reference(self, rows=None, cols=None):
        qa, sa = self.qa, self.sa
        qb, sb = self.qb, self.sb
        fa, fb = self.fa, self.fb
        if rows is not None:
            qa, sa = qa[rows], sa[rows]
            fa = None if fa is None else fa[rows]
        if cols is not None:
            qb, sb = qb[cols], sb[cols]
            fb = None if fb is None else fb[cols]
        ref = O.gemm_ref(qa, qb, sa, sb, fa, fb)
        bound = O.gemm_abs_bound(qa, qb, sa, sb)
        return ref, bound


# what -> (largest tolerance ratio, largest slack needed beyond 2 bf16 ulp):
# printed at the end of the session (tests/conftest.py) so the reduction-order
# slack the GPU results actually needed can be compared with O.GEMM_SLACK.
OBSERVED: dict = {}


def _record(what, ratio, excess):
    r0, e0 = OBSERVED.get(what, (0.0, 0.0))
    OBSERVED[what] = (max(r0, ratio), max(e0, excess))


def assert_gemm_close(out, ref: np.ndarray, bound: np.ndarray, what: str = ""):
    got = out if isinstance(out, np.ndarray) else out.float().cpu().numpy()
    ok, ratio, nbad = O.check_gemm(got, ref, bound)
    _record(what, ratio, O.excess_over_ulps(got, ref, bound))
    if not ok:
        d = np.abs(got - ref)
        idx = np.unravel_index(np.nanargmax(np.where(np.isnan(d), np.inf, d)), d.shape)
        raise AssertionError(
            f"{what}: {nbad}/{got.size} elements outside tolerance (max ratio {ratio:.3g}); "
            f"worst at {idx}: got {got[idx]} ref {ref[idx]}")
    return ratio


def full_check(out: torch.Tensor, qa, sa, qb, sb, fa=None, fb=None, what: str = "",
               row_chunk: int = 1024, col_chunk: int = 8192):
    """Every output element against the oracle, in blocks: each block of B
    rows is dequantised once, each block of A rows once per B block, and the
    oracle's own steps (O.matmul_factors, then RNE to bf16) give the block's
    reference.  Returns the largest tolerance ratio."""
    got_all = out.float().cpu().numpy()
    M, N = got_all.shape
    worst = 0.0
    for c0 in range(0, N, col_chunk):
        c1 = min(N, c0 + col_chunk)
        xb = O.dequant(qb[c0:c1], sb[c0:c1])
        xb_abs = np.abs(xb)
        fbc = None if fb is None else np.asarray(fb).reshape(N)[c0:c1]
        for r0 in range(0, M, row_chunk):
            r1 = min(M, r0 + row_chunk)
            xa = O.dequant(qa[r0:r1], sa[r0:r1])
            fac = None if fa is None else np.asarray(fa).reshape(M)[r0:r1]
            ref = O.bf16_round(O.matmul_factors(xa, xb, fac, fbc))
            with np.errstate(invalid="ignore", over="ignore"):
                bound = (np.abs(xa) @ xb_abs.T).astype(np.float32)
            got = got_all[r0:r1, c0:c1]
            ok, ratio, nbad = O.check_gemm(got, ref, bound)
            _record(what, ratio, O.excess_over_ulps(got, ref, bound))
            if not ok:
                assert_gemm_close(got, ref, bound, f"{what} block [{r0}:{r1}, {c0}:{c1}]")
            worst = max(worst, ratio)
    return worst
