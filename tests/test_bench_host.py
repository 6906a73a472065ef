"""CPU checks of bench.py's contract: the CPU reference arm never loads the product library, and
both arms describe the same workload with the same `config` dict."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


@pytest.mark.parametrize("name", ["cfg0", "cfg1"])
def test_both_arms_print_the_same_config(name):
    import bench
    import bigtea_b200 as bt
    from oracle import workloads

    w = workloads.workload(name)
    c = bt.config(name)
    for world in (1, 8):
        assert bench.workload_config(name, w, w.shape_name(), 8192, world) == \
            bench.workload_config(name, c, bench.shape_name(c), 8192, world)
    assert bench.decode_bytes_per_token(w, 8192) == bench.decode_bytes_per_token(c, 8192)


def test_reference_arm_does_not_load_the_product_library():
    code = (
        "import sys, json; sys.argv = ['bench.py', '--impl', 'reference', '--config', 'cfg0', '--ctx', '64', "
        "'--steps', '1', '--warmup', '1']\n"
        "import bench\n"
        "bench.main()\n"
        "assert not any(m == 'bigtea_b200' or m.startswith('bigtea_b200.') for m in sys.modules), "
        "sorted(m for m in sys.modules if m.startswith('bigtea'))\n"
        "maps = open('/proc/self/maps').read()\n"
        "assert 'libbigtea_decode' not in maps\n"
    )
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["host_copy_gbs"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0
