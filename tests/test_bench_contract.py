"""bench.py's contract on CPU: the reference arm's workloads equal the package's, and that arm runs the
reference algorithm (the oracle) without importing or loading anything of the GPU package."""
import json
import os
import subprocess
import sys

import pytest

from tests.helpers import pkg

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


@pytest.mark.parametrize("name", sorted(bench.WORKLOADS))
def test_workload_tables_agree(name):
    wd = bench.WORKLOADS[name]
    w = pkg.configs.WORKLOADS[name]
    m = w.model
    assert wd["name"] == w.name
    for k in bench._SHAPE_KEYS:
        assert wd[k] == (m.kv if k == "kv_heads" else getattr(m, k)), k
    for k in ("weight_seed", "seqs", "prompt_len", "new_tokens"):
        assert wd[k] == getattr(w, k), k


def test_reference_prompts_are_the_bench_prompts():
    wd = bench.WORKLOADS["microchat"]
    w = pkg.configs.MICROCHAT
    assert (bench.ref_prompts(wd, 0, 3) == pkg.sharding.shard_prompts(w, 0)[:3]).all()
    assert (bench.ref_prompts(wd, 1, 2) == pkg.sharding.shard_prompts(w, 1)[:2]).all()


def test_reference_arm_never_touches_the_gpu_package():
    code = ("import runpy, sys, json; sys.argv = ['bench.py', '--impl', 'reference', '--workload', 'foundry', "
            "'--steps', '1', '--warmup', '3'];\n"
            "try:\n    runpy.run_path('bench.py', run_name='__main__')\nfinally:\n"
            "    bad = [m for m in sys.modules if 'shahd-llm-stack_b200' in m]\n"
            "    maps = open('/proc/self/maps').read()\n"
            "    print('LEAK' if bad or 'libshahd_b200' in maps else 'CLEAN')\n")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.strip().splitlines()
    assert lines[-1] == "CLEAN", out.stdout
    line = json.loads(lines[-2])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["config"]["seqs_per_gpu"] == bench.WORKLOADS["foundry"]["seqs"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
