"""Regenerate tests/golden/golden.json (run from the repo root).

    python tests/golden/make_golden.py

Sources of truth:
  * glibc's own srand()/rand() called through ctypes -- the reference draws
    every input from exactly this stream (src/persistent.cu:132-135 of
    AyaanFaisal21/APK), so these prefixes are the reference generator's
    output on this platform, not a restatement;
  * exact rational arithmetic for small products: inputs drawn from glibc's
    rand() above and converted as the reference converts them
    ((float)(r/(double)RAND_MAX*2-1)), every product a_ik*b_kj summed exactly
    (fractions.Fraction) and rounded once to double.  Nothing here calls the
    oracle, so these values pin the oracle's float64 i-k-j loop
    (src/persistent.cu:221-227) from outside: the loop must land within a
    few ulps of the exact sums;
  * the known-answer value ref[0] = 12.687869863082142 at M=N=K=1024, seed
    21, from the reference's own loop.
"""
from __future__ import annotations

import ctypes
import json
import os
import sys
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402


def glibc_prefix(seed: int, n: int):
    libc = ctypes.CDLL("libc.so.6")
    libc.srand.argtypes = [ctypes.c_uint]
    libc.rand.restype = ctypes.c_int
    libc.srand(seed)
    return [int(libc.rand()) for _ in range(n)]


def glibc_operands(M: int, N: int, K: int, seed: int):
    """A (MxK) then B (KxN) from glibc's own srand/rand, converted as in
    src/persistent.cu:132-135."""
    libc = ctypes.CDLL("libc.so.6")
    libc.srand.argtypes = [ctypes.c_uint]
    libc.rand.restype = ctypes.c_int
    libc.srand(seed)
    vals = [np.float32(libc.rand() / 2147483647.0 * 2.0 - 1.0) for _ in range(M * K + K * N)]
    v = np.array(vals, np.float32)
    return v[:M * K].reshape(M, K), v[M * K:].reshape(K, N)


def main():
    out = {"glibc_rand": {}, "gemm": {}, "kat": {}}
    for seed in (0, 1, 21, 12345):
        out["glibc_rand"][str(seed)] = glibc_prefix(seed, 64)
    for (M, N, K) in [(128, 128, 128), (256, 128, 64), (128, 256, 256)]:
        A, B = glibc_operands(M, N, K, 21)
        Af = [[Fraction(float(x)) for x in row] for row in A[:8]]
        Bt = [[Fraction(float(B[k, j])) for k in range(K)] for j in range(8)]
        exact = lambda i, j: sum(a * b for a, b in zip(Af[i], Bt[j]))  # noqa: E731
        # sum of all of C = sum_k (sum_i A_ik) (sum_j B_kj), exactly
        colA = [sum(Fraction(float(x)) for x in A[:, k]) for k in range(K)]
        rowB = [sum(Fraction(float(x)) for x in B[k, :]) for k in range(K)]
        out["gemm"][f"{M}x{N}x{K}"] = {
            "seed": 21,
            "A_head": [float(x) for x in A.ravel()[:8]],
            "B_head": [float(x) for x in B.ravel()[:8]],
            "C_row0_head": [float(exact(0, j)) for j in range(8)],
            "C_diag_head": [float(exact(i, i)) for i in range(8)],
            "C_sum": float(sum(a * b for a, b in zip(colA, rowB))),
            "source": "exact rational sums over glibc rand() inputs, rounded once to double",
        }
    out["kat"]["1024x1024x1024_seed21_ref0"] = oracle.KAT_1024_REF0
    bf = oracle.gen_normal_bf16(16, 21)
    out["normal_bf16_seed21_head"] = [int(x) for x in bf]
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", os.path.join(HERE, "golden.json"))


if __name__ == "__main__":
    main()
