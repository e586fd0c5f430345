"""profiles/traffic.json, the DRAM bytes bench.py reports as roofline.traffic:
every config's entry names a committed summary and kernel sources, and every
kernel it lists is a kernel those sources define (a renamed or removed kernel
leaves the entry pointing at nothing)."""
import json
import os
import re

from conftest import ROOT

import bench


def _entries():
    with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
        t = json.load(f)
    return {k: v for k, v in t.items() if not k.startswith("_")}


def test_every_bench_config_has_a_traffic_entry():
    assert set(_entries()) == set(bench.ORDER)


def test_traffic_entries_name_committed_files_and_defined_kernels():
    for key, ent in _entries().items():
        assert ent["dram_bytes_per_launch"] > 0, key
        assert os.path.exists(os.path.join(ROOT, ent["capture"])), (key, ent["capture"])
        text = ""
        for src in ent["sources"]:
            path = os.path.join(ROOT, src)
            assert os.path.exists(path), (key, src)
            with open(path) as f:
                text += f.read()
        defined = set(re.findall(r"__global__\s+void\s+(?:__launch_bounds__\([^)]*\)\s+)?(\w+)\s*\(", text))
        for kernel in ent["kernels"]:
            name = re.sub(r"<.*$", "", kernel).split("::")[-1]
            assert name in defined, (key, kernel)
