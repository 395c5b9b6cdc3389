"""The C ABI library: loads, exports every declared symbol, host-side logic
that needs no GPU (generators, config defaults, clean failure paths)."""
import ctypes
import json
import os
import re

import numpy as np
import pytest

import oracle
from conftest import has_gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = json.load(open(os.path.join(ROOT, "tests", "golden", "golden.json")))


def header_symbols():
    txt = open(os.path.join(ROOT, "include", "apk.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(apk_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_header_symbol(libapk):
    syms = header_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(libapk, s)]
    assert not missing, missing


def test_python_binding_covers_header():
    from apk_b200 import _lib
    assert set(header_symbols()) == set(_lib.SIGNATURES)


def test_abi_version(libapk):
    assert libapk.apk_abi_version() == 4


def test_config_defaults(libapk):
    from apk_b200 import _lib
    c = _lib.Config()
    libapk.apk_config_default(ctypes.byref(c))
    assert (c.dtype, c.k_tile, c.poll, c.discipline, c.set_mode) == (
        _lib.APK_F32, 0, _lib.APK_POLL_STAGE, _lib.APK_DISC_DRAIN, _lib.APK_SET_HOST_MEMCPY)
    assert c.max_events == 4096 and c.urgent_split_k == 8 and c.wait_limit_ns == 2_000_000_000
    assert c.scheduler == _lib.APK_SCHED_QUEUE and c.f32_kernel == 0  # queue, fp32 kernel auto


@pytest.mark.parametrize("seed,shape", [(21, (1024, 1024, 1024)), (0, (128, 256, 64)), (7, (256, 128, 512))])
def test_product_uniform_generator_matches_glibc(libapk, seed, shape):
    import apk_b200
    M, N, K = shape
    A, B = apk_b200.fill_uniform(M, N, K, seed)
    A2, B2 = oracle.gen_uniform(M, N, K, seed)
    assert np.array_equal(A, A2) and np.array_equal(B, B2)


def test_product_uniform_generator_golden_prefix(libapk):
    import apk_b200
    A, _ = apk_b200.fill_uniform(1, 1, 64, 12345)
    want = np.array([np.float32(r / 2147483647.0 * 2.0 - 1.0) for r in GOLDEN["glibc_rand"]["12345"]])
    assert np.array_equal(A.ravel(), want)


@pytest.mark.parametrize("n", [1, 7, 4096, (1 << 21) + 3])
def test_product_normal_generator_matches_oracle(libapk, n):
    import apk_b200
    assert np.array_equal(apk_b200.fill_normal_bf16(n, 21), oracle.gen_normal_bf16(n, 21))


def test_product_bf16_rounding_matches_oracle(libapk):
    import apk_b200
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 1e3
    assert np.array_equal(apk_b200.round_bf16(x), oracle.round_bf16(x))


@pytest.mark.skipif(has_gpu(), reason="checks the no-device failure path")
def test_create_fails_cleanly_without_gpu(libapk):
    import apk_b200
    with pytest.raises(apk_b200.ApkError) as ei:
        apk_b200.Context()
    assert ei.value.status in (2, 7)  # APK_ECUDA / APK_EUNSUPPORTED, no crash


def test_invalid_arguments_are_rejected(libapk):
    from apk_b200 import _lib
    assert libapk.apk_create(None, None) == _lib.APK_EINVAL
    assert libapk.apk_launch(None, 1) == _lib.APK_EINVAL
    assert libapk.apk_destroy(None) == _lib.APK_OK
