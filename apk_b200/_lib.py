"""ctypes binding of include/apk.h (libapk.so, built in-tree).

The library is the product; this module only declares its C signatures.
There is no fallback: if libapk.so is missing, importing raises.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libapk.so")

c_int, c_uint, c_ll, c_ull, c_double, c_size_t, c_void_p, c_char_p = (
    ctypes.c_int, ctypes.c_uint, ctypes.c_longlong, ctypes.c_ulonglong, ctypes.c_double,
    ctypes.c_size_t, ctypes.c_void_p, ctypes.c_char_p)

# enums (apk.h)
APK_OK, APK_EINVAL, APK_ECUDA, APK_ETIMEDOUT, APK_ESTATE, APK_EDEVICE, APK_ENOMEM, APK_EUNSUPPORTED = range(8)
STATUS_NAMES = {0: "APK_OK", 1: "APK_EINVAL", 2: "APK_ECUDA", 3: "APK_ETIMEDOUT", 4: "APK_ESTATE",
                5: "APK_EDEVICE", 6: "APK_ENOMEM", 7: "APK_EUNSUPPORTED"}
APK_F32, APK_BF16 = 0, 1
APK_POLL_OFF, APK_POLL_BOUNDARY, APK_POLL_STAGE = 0, 1, 2
APK_DISC_DRAIN, APK_DISC_POISON = 0, 2
APK_SET_DEVICE, APK_SET_HOST_MAPPED, APK_SET_HOST_MEMCPY = 0, 1, 2
APK_MEM_HOST, APK_MEM_DEVICE = 0, 1
APK_SCHED_QUEUE, APK_SCHED_CLC = 0, 1
APK_TASKS_UNBOUNDED = 0xFFFFFFFFFFFFFFFF


class Config(ctypes.Structure):
    _fields_ = [("device", c_int), ("dtype", c_int), ("ctas_per_sm", c_int), ("grid", c_int),
                ("k_tile", c_int), ("poll", c_int), ("discipline", c_int), ("set_mode", c_int),
                ("max_events", c_int), ("oracle", c_int), ("urgent_split_k", c_int),
                ("wait_limit_ns", c_ll), ("scheduler", c_int), ("f32_kernel", c_int),
                ("bf16_kernel", c_int)]


class DeviceInfo(ctypes.Structure):
    _fields_ = [("sms", c_int), ("grid", c_int), ("ctas_per_sm", c_int), ("max_ctas_per_sm", c_int),
                ("cc_major", c_int), ("cc_minor", c_int), ("smem_per_cta", c_int),
                ("threads_per_cta", c_int), ("tile_m", c_int), ("tile_n", c_int), ("k_tile", c_int),
                ("stages", c_int), ("name", ctypes.c_char * 128), ("slot_k", c_int)]


class EventLog(ctypes.Structure):
    _fields_ = [("n_injected", c_int), ("n_fired", c_int), ("grid", c_int),
                ("set_ns", c_void_p), ("host_set_ns", c_void_p), ("host_ack_ns", c_void_p),
                ("host_done_ns", c_void_p), ("claim_ns", c_void_p), ("done_ns", c_void_p),
                ("claimer", c_void_p), ("claim_site", c_void_p), ("inflight", c_void_p),
                ("obs_ns", c_void_p)]


class RunStats(ctypes.Structure):
    _fields_ = [("start_ns", c_ll), ("end_ns", c_ll), ("tiles_done", c_ull), ("yields", c_ull),
                ("bg_flops", c_double), ("bg_tflops", c_double), ("exited", c_int),
                ("device_status", c_int), ("launch_ms", c_double),
                ("ckpt_spill_bytes", c_ull), ("ckpt_restore_bytes", c_ull),
                ("ckpt_spill_ns", c_ll), ("ckpt_restore_ns", c_ll), ("parks", c_ull)]


class LatencyConfig(ctypes.Structure):
    _fields_ = [("events", c_int), ("period_ns", c_ll), ("seed", c_uint), ("warmup_events", c_int),
                ("settle_ns", c_ll), ("bg_tasks", c_ull), ("probe_reps", c_int), ("poisson", c_int)]


class LatencyResult(ctypes.Structure):
    _fields_ = [("n", c_int), ("anomalies", c_int), ("unclaimed", c_int),
                ("claim_p50_us", c_double), ("claim_p99_us", c_double),
                ("last_obs_p50_us", c_double), ("last_obs_p99_us", c_double),
                ("done_p50_us", c_double), ("done_p99_us", c_double),
                ("rt_claim_p50_us", c_double), ("rt_claim_p99_us", c_double),
                ("rt_done_p50_us", c_double), ("rt_done_p99_us", c_double),
                ("bg_tflops", c_double), ("vis_offset_ns", c_double)]


class VisibilityConfig(ctypes.Structure):
    _fields_ = [("events", c_int), ("gap_min_ns", c_ll), ("gap_max_ns", c_ll), ("seed", c_uint),
                ("warmup_events", c_int), ("work_iters", c_int), ("loaded", c_int), ("traffic_bytes", c_ll)]


class VisibilityResult(ctypes.Structure):
    _fields_ = [("n", c_int), ("unset", c_int), ("anomalies", c_int), ("cadence_ns", c_double),
                ("dmin_p50_us", c_double), ("d50_p50_us", c_double), ("d95_p50_us", c_double),
                ("dmax_p50_us", c_double), ("dmax_p99_us", c_double), ("hbm_gbs", c_double),
                ("device_status", c_int)]


P = c_void_p
# name -> (restype, argtypes); every symbol include/apk.h declares
SIGNATURES = {
    "apk_abi_version": (c_int, []),
    "apk_config_default": (None, [ctypes.POINTER(Config)]),
    "apk_create": (c_int, [ctypes.POINTER(Config), ctypes.POINTER(P)]),
    "apk_destroy": (c_int, [P]),
    "apk_last_error": (c_char_p, [P]),
    "apk_get_info": (c_int, [P, ctypes.POINTER(DeviceInfo)]),
    "apk_set_background": (c_int, [P, P, P, P, c_int, c_int, c_int, c_int]),
    "apk_set_urgent": (c_int, [P, P, P, c_int, c_int, c_int, c_int]),
    "apk_launch": (c_int, [P, c_ull]),
    "apk_schedule_device_events": (c_int, [P, P, c_int]),
    "apk_schedule_count_events": (c_int, [P, P, c_int]),
    "apk_inject_urgent": (c_int, [P, ctypes.POINTER(c_int), ctypes.POINTER(c_ll)]),
    "apk_wait_ack": (c_int, [P, c_int, c_int, c_ll, ctypes.POINTER(c_ll)]),
    "apk_stop": (c_int, [P]),
    "apk_wait": (c_int, [P, c_ll]),
    "apk_read_output": (c_int, [P, P]),
    "apk_read_urgent_output": (c_int, [P, c_int, P]),
    "apk_read_events": (c_int, [P, ctypes.POINTER(EventLog)]),
    "apk_read_oracle": (c_int, [P, P, P]),
    "apk_read_run_stats": (c_int, [P, ctypes.POINTER(RunStats)]),
    "apk_gemm": (c_int, [P, P, P, P, c_int, c_int, c_int, c_int]),
    "apk_probe_copy": (c_int, [P, P, P, P, c_int, P]),
    "apk_run_latency": (c_int, [P, ctypes.POINTER(LatencyConfig), ctypes.POINTER(LatencyResult)]),
    "apk_probe_visibility": (c_int, [P, c_int, P]),
    "apk_run_visibility": (c_int, [P, ctypes.POINTER(VisibilityConfig), ctypes.POINTER(VisibilityResult), P, P]),
    "apk_selftest_wait_timeout": (c_int, [P, c_ll, ctypes.POINTER(c_int)]),
    "apk_run_overhead": (c_int, [P, c_ull, c_int, ctypes.POINTER(c_double), ctypes.POINTER(c_double)]),
    "apk_run_baseline": (c_int, [P, c_ull, c_int, c_uint, P]),
    "apk_run_reserved": (c_int, [P, c_ull, c_int, c_int, c_uint, P, ctypes.POINTER(c_double)]),
    "apk_set_task_pool": (c_int, [P, P, c_int, c_int, P, c_int, c_int, c_int, c_int, c_int]),
    "apk_set_tasks": (c_int, [P, P, c_int, c_ll, ctypes.POINTER(c_ull)]),
    "apk_read_checksums": (c_int, [P, P, c_ll]),
    "apk_read_pool_window": (c_int, [P, c_int, c_int, c_int, c_int, P]),
    "apk_gen_tasks": (c_ll, [c_ull, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                             c_int, P]),
    "apk_shard_tasks": (c_int, [P, c_int, c_int, c_int, P]),
    "apk_sgemm_f32_noalloc": (c_int, [P, P, P, c_int, c_int, c_int, c_int, P]),
    "apk_sgemm_f32_noalloc_status": (c_int, [P, ctypes.POINTER(c_int)]),
    "apk_sgemm_f32_noalloc_selftest": (c_int, [c_ll, P]),
    "apk_fill_uniform": (None, [c_uint, P, c_size_t, P, c_size_t]),
    "apk_fill_normal_bf16": (None, [c_ull, P, c_size_t]),
    "apk_round_bf16": (None, [P, P, c_size_t]),
    "apk_host_alloc": (P, [c_size_t]),
    "apk_host_free": (None, [P]),
}

_lib = None


def load():
    """Load libapk.so.  Raises if it has not been built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m apk_b200.build` "
                "(the runtime has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib
