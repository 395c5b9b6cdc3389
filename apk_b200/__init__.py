"""apk_b200 -- preemptible persistent-GEMM runtime for NVIDIA B200 (sm_100a).

The product is the native library ``libapk.so`` (C ABI in ``include/apk.h``):
hand-written sm_100a kernels (fp32 CUDA-core SGEMM, bf16 tcgen05 GEMM) drained
by a persistent scheduler that yields to injected urgent GEMMs at tile
boundaries or mid-pipeline with an accumulator checkpoint.  This package is
the Python mirror of that ABI; it has no compute path of its own.
"""
from ._lib import LIB_PATH, load  # noqa: F401
from .runtime import (ApkError, Context, fill_normal_bf16, fill_uniform,  # noqa: F401
                      pinned_empty, round_bf16)

__all__ = ["Context", "ApkError", "fill_uniform", "fill_normal_bf16", "round_bf16", "pinned_empty",
           "load", "LIB_PATH"]
