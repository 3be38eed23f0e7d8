"""Host-side pieces of bench.py that need no GPU: the CPU legs' thread count
and the workload description both arms print."""
import importlib
import os
import subprocess
import sys

from conftest import ROOT


def _bench():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    return importlib.import_module("bench")


def test_host_threads_ignores_omp_num_threads():
    """torchrun sets OMP_NUM_THREADS=1 for its workers; the reference arm and
    the CPU baselines still use every core the process may run on."""
    code = "import bench; print(bench.host_threads())"
    env = dict(os.environ, OMP_NUM_THREADS="1")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=300, check=True)
    assert int(out.stdout.strip().splitlines()[-1]) == len(os.sched_getaffinity(0))


def test_both_arms_describe_the_same_workload():
    b = _bench()
    for world in (1, 2, 8):
        c = b.bench_config(world)
        assert c == b.bench_config(world)
        assert c["rows"] == 8192 and f"over {world} rank(s)" in c["partition"]
