"""Host-side checks of bench.py that need no GPU: the reference arm
(`--impl reference`) runs the reference's float64 host GEMM single-threaded
and prints the JSON line the driver parses."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_its_line():
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "TFLOP/s" and line["value"] > 0
    assert line["cpu_baseline"]["cores"] == 1 and line["cpu_baseline"]["kind"] == "port"
    assert line["all_cores"]["cores"] >= 1 and line["all_cores"]["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["gpu_launches"] == 0


def test_numa_local_cpus_reads_sysfs_or_declines():
    """The e2e buffers are allocated on the GPU's NUMA node: the helper maps
    a PCI address (nvidia-smi form) to the CPUs this process may use there,
    and answers None for an address sysfs does not know."""
    import os
    import sys
    sys.path.insert(0, ROOT)
    import bench
    allowed = os.sched_getaffinity(0)
    host_bridge = bench.numa_local_cpus("00000000:00:00.0")
    if os.path.exists("/sys/bus/pci/devices/0000:00:00.0/local_cpulist"):
        assert host_bridge is not None and host_bridge <= allowed
    assert bench.numa_local_cpus("not-a-bus-id") is None
    assert bench.numa_local_cpus("0000FFFF:FF:1F.7") is None
