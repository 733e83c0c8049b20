"""bench.py on the CPU: the reference arm times the reference's csr_omp on a
matrix built by the oracle's own generator, so it maps neither this
library's CUDA code nor torch, and prints the line the driver compares
(same metric, unit and config as the GPU arm but for `kernel`)."""
from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import ROOT

PROBE = """
import sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "3", "--warmup", "3"]
import bench
rc = bench.main()
maps = open("/proc/self/maps").read()
print("MAPS", "libspmvb" in maps, "libtorch" in maps)
sys.exit(rc)
"""


def test_reference_arm_loads_neither_the_library_nor_torch():
    out = subprocess.run([sys.executable, "-c", PROBE], cwd=ROOT, capture_output=True, text=True, timeout=600,
                         env=dict(os.environ, OMP_NUM_THREADS="4"))
    assert out.returncode == 0, out.stderr
    lines = out.stdout.strip().splitlines()
    line = json.loads(next(ln for ln in lines if ln.startswith("{")))
    assert lines[-1] == "MAPS False False", lines[-1]
    sys.path.insert(0, ROOT)
    import bench
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "GFLOP/s"
    assert line["value"] > 0 and line["ms_per_step"] > 0 and line["higher_is_better"] is True
    ours = bench.bench_config(1, "ELL")
    assert {k: v for k, v in line["config"].items() if k != "kernel"} == \
        {k: v for k, v in ours.items() if k != "kernel"}
    assert line["e2e"] == {"value": line["value"], "unit": "GFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["cpu_baseline"]["omp_proc_bind"] == "close"
