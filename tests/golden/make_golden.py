"""Generate the golden fixtures under tests/golden/ from the reference's own code.

Run in a container that has the reference checkout (it is read, never
modified, and is not needed at test time):

    python tests/golden/make_golden.py /path/to/reference

What it executes: the bodies of ``convert_byte_to_float``, ``run_torch`` and
``run_torch_mbs`` taken verbatim (by ``ast``) from the reference's
test_gemm_a4w4.py:28-69, with the aiter ``@perftest`` decorators stripped.  The
two aiter helpers those bodies call (``fp4_utils.mxfp4_to_f32`` and
``fp4_utils.e8m0_to_f32``; aiter is third-party and absent here) are supplied
by the small torch stand-in below, written from the OCP MX definitions.  The
inputs are seeded random fp4 bytes, scale bytes and factor bytes; the outputs
are the reference oracle's bf16 results.  The CPU oracle in oracle/ is pinned
against these files by tests/test_oracle.py.
"""

from __future__ import annotations

import ast
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (M, N, K) cases: ragged M, the smallest legal N/K, several 32-K groups.
CASES = [(5, 16, 64), (33, 48, 128), (64, 32, 256), (17, 64, 512)]


def _fp4_utils_standin() -> types.ModuleType:
    """torch stand-in for aiter.utility.fp4_utils (OCP MX definitions)."""
    mod = types.ModuleType("fp4_utils")
    lut = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float32)

    def mxfp4_to_f32(x):
        x = x.view(torch.uint8)
        lo = (x & 0xF).long()
        hi = (x >> 4).long()
        out = torch.stack([lut[lo], lut[hi]], dim=-1)
        return out.reshape(*x.shape[:-1], x.shape[-1] * 2)

    def e8m0_to_f32(s):
        s = s.view(torch.uint8).to(torch.int32)
        out = torch.pow(torch.tensor(2.0, dtype=torch.float64), (s - 127).double()).float()
        return torch.where(s == 255, torch.tensor(float("nan")), out)

    mod.mxfp4_to_f32 = mxfp4_to_f32
    mod.e8m0_to_f32 = e8m0_to_f32
    return mod


def load_reference_functions(ref_root: str) -> dict:
    src_path = os.path.join(ref_root, "test_gemm_a4w4.py")
    with open(src_path, "r", encoding="utf-8") as f:
        tree = ast.parse(f.read(), filename=src_path)
    wanted = {"convert_byte_to_float", "run_torch", "run_torch_mbs"}
    body = []
    for node in tree.body:
        if isinstance(node, ast.FunctionDef) and node.name in wanted:
            node.decorator_list = []  # drop aiter's @perftest
            body.append(node)
    assert {n.name for n in body} == wanted, "reference functions not found"
    ns = {"torch": torch, "SCALE_GROUP_SIZE": 32, "fp4_utils": _fp4_utils_standin()}
    exec(compile(ast.Module(body=body, type_ignores=[]), src_path, "exec"), ns)
    return ns


def main(ref_root: str) -> None:
    ns = load_reference_functions(ref_root)
    # 1) factor table: all 256 bytes through the reference's own function
    b = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    ftab = ns["convert_byte_to_float"](b).numpy().astype(np.float32)
    np.save(os.path.join(HERE, "factor_table.npy"), ftab)

    # 2) GEMM oracle outputs on seeded inputs
    rng = np.random.default_rng(20261201)
    arrays = {}
    for (M, N, K) in CASES:
        a = rng.integers(0, 256, size=(M, K // 2), dtype=np.uint8)
        w = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
        sa = rng.integers(118, 136, size=(M, K // 32), dtype=np.uint8)
        sw = rng.integers(118, 136, size=(N, K // 32), dtype=np.uint8)
        fa = rng.integers(0, 256, size=(M, 1), dtype=np.uint8)
        fw = rng.integers(0, 256, size=(N, 1), dtype=np.uint8)
        ta, tw = torch.from_numpy(a), torch.from_numpy(w)
        tsa, tsw = torch.from_numpy(sa), torch.from_numpy(sw)
        out = ns["run_torch"](ta, tw, tsa, tsw, torch.bfloat16)
        out_mbs = ns["run_torch_mbs"](ta, tw, tsa, tsw, torch.from_numpy(fa),
                                      torch.from_numpy(fw), torch.bfloat16)
        tag = f"{M}x{N}x{K}"
        arrays[f"a_{tag}"] = a
        arrays[f"w_{tag}"] = w
        arrays[f"sa_{tag}"] = sa
        arrays[f"sw_{tag}"] = sw
        arrays[f"fa_{tag}"] = fa
        arrays[f"fw_{tag}"] = fw
        arrays[f"out_{tag}"] = out.view(torch.int16).numpy().view(np.uint16)
        arrays[f"outmbs_{tag}"] = out_mbs.view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "gemm_oracle_golden.npz"), **arrays)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
