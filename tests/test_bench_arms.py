"""The bench's reference arm runs the oracle alone, on the product arm's
workload.

* The oracle's block manager and the product's hand out the same block
  tables and slot mappings for the seeded workload (FIFO reuse of the same
  permuted free list), so both arms measure the same config.
* ``bench.py --impl reference`` honours the driver's --steps/--warmup and
  never loads the product library (checked in the process's own memory
  map), for the decode-style workloads and the prefix workload.
"""
import json
import os
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_oracle_and_product_build_the_same_workload():
    import bench
    import oracle as orc
    for name in ("decode", "config1", "quant8"):
        w = bench.WORKLOADS[name]
        a = bench.make_workload(w, 9)
        b = bench.make_workload(w, 9, manager=orc.PagedCacheManager)
        assert a["num_blocks"] == b["num_blocks"]
        assert np.array_equal(a["lens0"], b["lens0"])
        assert np.array_equal(a["bt"], b["bt"])
        assert np.array_equal(a["slots"], b["slots"])


def _run_reference(*argv):
    code = ("import runpy, sys; sys.argv = ['bench.py'] + sys.argv[1:]; "
            "runpy.run_path('bench.py', run_name='__main__'); "
            "print('PRODUCT_LOADED', 'librmlx_kv' in open('/proc/self/maps').read())")
    r = subprocess.run([sys.executable, "-c", code, "--impl", "reference", *argv], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.strip().splitlines()
    rec = json.loads(next(ln for ln in lines if ln.startswith("{")))
    loaded = next(ln for ln in lines if ln.startswith("PRODUCT_LOADED")).split()[1]
    return rec, loaded == "True"


def test_reference_arm_is_oracle_only_and_honours_steps():
    rec, loaded = _run_reference("--workload", "config1", "--steps", "4", "--warmup", "3")
    assert not loaded
    assert rec["impl"] == "reference" and rec["steps"] == 4 and rec["warmup"] == 3
    assert rec["value"] > 0 and rec["single_thread"]["cores"] == 1
    import bench
    w = bench.WORKLOADS["config1"]
    assert rec["config"] == bench.config_of(w, w.heads, bench.make_workload(w, 7)["num_blocks"], 1, True)


def test_prefix_reference_arm_is_oracle_only():
    rec, loaded = _run_reference("--workload", "prefix", "--steps", "1", "--warmup", "3")
    assert not loaded
    assert rec["steps"] == 1 and rec["warmup"] == 3 and rec["value"] > 0
