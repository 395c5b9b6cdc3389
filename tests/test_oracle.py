"""The CPU oracle, pinned against the reference's known answers (no GPU)."""
import json
import math
import os

import numpy as np
import pytest

import oracle

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))


def test_kat_1024_seed21():
    # ref[0] of the reference's own float64 loop, src/persistent.cu:221-227
    A, B = oracle.gen_uniform(1024, 1024, 1024, 21)
    C = oracle.gemm_f64(A, B)
    assert C[0, 0] == oracle.KAT_1024_REF0 == GOLDEN["kat"]["1024x1024x1024_seed21_ref0"]


def test_omp_loop_bit_identical_to_single_thread():
    A, B = oracle.gen_uniform(256, 384, 512, 3)
    assert np.array_equal(oracle.gemm_f64(A, B), oracle.gemm_f64_omp(A, B))


def test_rows_variant_matches_full():
    A, B = oracle.gen_uniform(256, 128, 64, 5)
    C = oracle.gemm_f64(A, B)
    assert np.array_equal(oracle.gemm_f64_rows(A, B, 40, 17), C[40:57])


@pytest.mark.parametrize("shape", list(GOLDEN["gemm"].keys()))
def test_golden_small_products(shape):
    M, N, K = map(int, shape.split("x"))
    g = GOLDEN["gemm"][shape]
    A, B = oracle.gen_uniform(M, N, K, g["seed"])
    assert A.ravel()[:8].tolist() == pytest.approx(g["A_head"], abs=0)
    assert B.ravel()[:8].tolist() == pytest.approx(g["B_head"], abs=0)
    C = oracle.gemm_f64(A, B)
    # golden values are exact sums rounded once (no oracle involved); the
    # loop's K sequential double roundings stay within K ulps of the sum of
    # |terms| (|a|, |b| <= 1, so that sum is at most K)
    tol = K * 2.0 ** -52 * K
    assert np.allclose(C[0, :8], g["C_row0_head"], rtol=0, atol=tol)
    assert np.allclose([C[i, i] for i in range(8)], g["C_diag_head"], rtol=0, atol=tol)
    assert abs(float(C.sum()) - g["C_sum"]) <= M * N * tol


def test_generator_is_glibc_rand():
    # the oracle's generator is the C library's rand(): compare its first
    # values with the recorded glibc stream
    seq = GOLDEN["glibc_rand"]["21"]
    A, _ = oracle.gen_uniform(1, 1, 64, 21)  # A holds 64 draws
    want = np.array([(np.float32(r / 2147483647.0 * 2.0 - 1.0)) for r in seq], np.float32)
    assert np.array_equal(A.ravel(), want)


def test_check_metric_and_nan_accounting():
    ref = np.array([0.5, -3.0, 100.0, 2.0], np.float64)
    got = np.array([0.5 + 1e-6, -3.0 + 1.5e-5, 100.0 * (1 + 2e-5), np.nan], np.float32)
    mr, bad, nans = oracle.check(got, ref, 1e-5)
    assert nans == 1
    # rel = err / max(1, |ref|): ~1e-6, ~5e-6 (pass), ~2e-5 (fail)
    assert bad == 1
    assert mr == pytest.approx(2e-5, rel=0.05)


def test_fp32_tolerance_formula():
    assert oracle.fp32_tol(4096) == pytest.approx(6.4e-4)
    assert oracle.fp32_tol(1024) == pytest.approx(3.2e-4)


def test_nearest_rank_percentile():
    v = list(range(1, 101))
    assert oracle.percentile(v, 0.5) == 51  # v[min(50, 99)]
    assert oracle.percentile(v, 0.99) == 100
    assert oracle.percentile([7.0], 0.99) == 7.0
    assert math.isnan(oracle.percentile([], 0.5))


def test_exactly_once_verdict():
    ok = oracle.exactly_once([1, 1, 1], [4, 4, 0], [3, 9, 0], [10, 20, 0], 4, 2)
    assert ok["pass"]
    dup = oracle.exactly_once([1, 2, 0], [4, 4, 0], [3, 9, 0], [10, 20, 0], 4, 2)
    assert not dup["pass"] and dup["dup"] == 1 and dup["missed"] == 1
    bad = oracle.exactly_once([1], [4, 3], [3, 0], [10, 20], 4, 2)
    assert not bad["pass"] and bad["bad_urgent"] == 1 and bad["unclaimed"] == 1


def test_bf16_round_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.0, 3.0e38, 1e-40], np.float32)
    h = oracle.round_bf16(x)
    # 1 + 2^-8 is a tie between 1.0 and 1 + 2^-7 -> even (1.0)
    assert oracle.bf16_to_f32(h).tolist()[:4] == [1.0, 1.0, 1.0078125, -2.0]


def test_normal_bf16_golden_and_moments():
    h = oracle.gen_normal_bf16(16, 21)
    assert h.tolist() == GOLDEN["normal_bf16_seed21_head"]
    f = oracle.bf16_to_f32(oracle.gen_normal_bf16(1 << 20, 7))
    assert abs(f.mean()) < 0.01 and abs(f.std() - 1.0) < 0.01
