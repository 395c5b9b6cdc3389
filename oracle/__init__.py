"""CPU oracle for the preemptible persistent-GEMM runtime (test infrastructure).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s cpu_baseline /
reference arm may import this package.  It is the checker, never the thing
measured or shipped: ``apk_b200`` does not import it and has no CPU fallback.

It wraps ``oracle/liboracle.so`` (built from ``gemm_ref.c`` by
``oracle/Makefile``), whose functions restate the reference's float64 host GEMM
(``src/persistent.cu:221-227``), its ``srand(21)``/``rand()`` input generator
(``src/persistent.cu:132-135``) and its error metric
(``src/persistent.cu:230-234``).  The pure-Python helpers below restate the
reference's nearest-rank percentile (``src/yield.cu:322-325``) and its
exactly-once scheduler verdict (``src/yield.cu:630-663``).
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

# Known-answer value pinned from the reference's own loop: M=N=K=1024,
# srand(21), ref[0] of the float64 product (see gemm_ref.c header).
KAT_1024_REF0 = 12.687869863082142


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "gemm_ref.c"))
        ):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        sz = ctypes.c_size_t
        i32 = ctypes.c_int
        L.oracle_gen_uniform_glibc.argtypes = [ctypes.c_uint, P, sz, P, sz]
        L.oracle_gen_uniform_glibc.restype = None
        L.oracle_gemm_f64.argtypes = [P, P, P, i32, i32, i32]
        L.oracle_gemm_f64.restype = None
        L.oracle_gemm_f64_rows.argtypes = [P, P, P, i32, i32, i32, i32]
        L.oracle_gemm_f64_rows.restype = None
        L.oracle_gemm_f64_omp.argtypes = [P, P, P, i32, i32, i32, i32]
        L.oracle_gemm_f64_omp.restype = None
        L.oracle_max_threads.argtypes = []
        L.oracle_max_threads.restype = i32
        L.oracle_check_f32.argtypes = [P, P, sz, ctypes.c_double, P, P]
        L.oracle_check_f32.restype = ctypes.c_double
        L.oracle_round_bf16.argtypes = [P, P, sz]
        L.oracle_round_bf16.restype = None
        L.oracle_bf16_to_f32.argtypes = [P, P, sz]
        L.oracle_bf16_to_f32.restype = None
        L.oracle_gemm_f64_bf16_rows.argtypes = [P, P, P, i32, i32, i32, i32, i32]
        L.oracle_gemm_f64_bf16_rows.restype = None
        L.oracle_gen_normal_bf16.argtypes = [ctypes.c_uint64, P, sz]
        L.oracle_gen_normal_bf16.restype = None
        L.oracle_gen_uniform_glibc_bf16.argtypes = [ctypes.c_uint, P, sz, P, sz]
        L.oracle_gen_uniform_glibc_bf16.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def gen_uniform(M: int, N: int, K: int, seed: int = 21):
    """A (MxK) then B (KxN), uniform[-1,1) via glibc srand/rand."""
    A = np.empty((M, K), np.float32)
    B = np.empty((K, N), np.float32)
    lib().oracle_gen_uniform_glibc(seed, _p(A), A.size, _p(B), B.size)
    return A, B


def gen_uniform_bf16(M: int, N: int, K: int, seed: int = 21):
    A = np.empty((M, K), np.uint16)
    B = np.empty((K, N), np.uint16)
    lib().oracle_gen_uniform_glibc_bf16(seed, _p(A), A.size, _p(B), B.size)
    return A, B


def gen_normal_bf16(n: int, seed: int) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().oracle_gen_normal_bf16(seed, _p(out), n)
    return out


def gemm_f64(A: np.ndarray, B: np.ndarray) -> np.ndarray:
    """Single-threaded reference loop (src/persistent.cu:221-227)."""
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    C = np.empty((M, N), np.float64)
    lib().oracle_gemm_f64(_p(A), _p(B), _p(C), M, N, K)
    return C


def gemm_f64_rows(A: np.ndarray, B: np.ndarray, row0: int, nrows: int) -> np.ndarray:
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((nrows, N), np.float64)
    lib().oracle_gemm_f64_rows(_p(A), _p(B), _p(C), N, K, row0, nrows)
    return C


def gemm_f64_omp(A: np.ndarray, B: np.ndarray, nthreads: int = 0) -> np.ndarray:
    M, K = A.shape
    N = B.shape[1]
    C = np.empty((M, N), np.float64)
    lib().oracle_gemm_f64_omp(_p(A), _p(B), _p(C), M, N, K, nthreads)
    return C


def gemm_f64_bf16_rows(A16, B16, row0: int, nrows: int, nthreads: int = 0) -> np.ndarray:
    K = A16.shape[1]
    N = B16.shape[1]
    C = np.empty((nrows, N), np.float64)
    lib().oracle_gemm_f64_bf16_rows(_p(A16), _p(B16), _p(C), N, K, row0, nrows, nthreads)
    return C


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().oracle_round_bf16(_p(x), _p(out), x.size)
    return out


def fp32_tol(K: int) -> float:
    """North-star fp32 tolerance: relative error <= 1e-5 * sqrt(K)."""
    return 1e-5 * math.sqrt(K)


BF16_TOL = 1e-2


def check(got: np.ndarray, ref: np.ndarray, tol: float):
    """Reference metric err/max(1,|ref|) (src/persistent.cu:230-234).

    Returns (max_rel, n_bad, n_nan)."""
    got = np.ascontiguousarray(got, np.float32)
    ref = np.ascontiguousarray(ref, np.float64)
    assert got.size == ref.size
    nb = ctypes.c_longlong(0)
    nn = ctypes.c_longlong(0)
    mr = lib().oracle_check_f32(_p(got), _p(ref), got.size, tol, ctypes.byref(nb), ctypes.byref(nn))
    return float(mr), int(nb.value), int(nn.value)


def percentile(values, q: float) -> float:
    """Nearest-rank percentile v[min(q*n, n-1)] of src/yield.cu:322-325."""
    v = sorted(values)
    if not v:
        return float("nan")
    return v[min(int(q * len(v)), len(v) - 1)]


def exactly_once(exec_counts, uexec_counts, claims, set_ns, urgent_items: int, n_events: int):
    """Scheduler verdict of src/yield.cu:630-663.

    Every task id below the bound ran exactly once; every fired event
    (set_ns != 0) executed exactly ``urgent_items`` urgent work items and has
    a claimer; the number of fired events equals ``n_events``."""
    ex = np.asarray(exec_counts)
    dup = int(np.count_nonzero(ex > 1))
    missed = int(np.count_nonzero(ex < 1))
    fired = bad_u = unclaimed = 0
    for e in range(len(set_ns)):
        if set_ns[e] == 0:
            continue
        fired += 1
        if uexec_counts[e] != urgent_items:
            bad_u += 1
        if claims[e] == 0:
            unclaimed += 1
    ok = dup == 0 and missed == 0 and bad_u == 0 and unclaimed == 0 and fired == n_events
    return {"dup": dup, "missed": missed, "fired": fired, "bad_urgent": bad_u,
            "unclaimed": unclaimed, "pass": ok}
