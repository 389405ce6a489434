"""bench.py's output contract on the CPU: the reference arm (the reference's
own CPU decoder, built under oracle/_ref by the build step) prints exactly one
JSON line on stdout, whatever native libraries write to their standard output,
with the keys and types the benchmark driver reads."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.mark.skipif(not (ROOT / "oracle" / "_ref" / "libxksv_native.so").exists(),
                    reason="oracle/_ref not built (the build step compiles it)")
def test_reference_arm_prints_one_json_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "3", "--warmup", "3"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.splitlines()
    assert len(lines) == 1, r.stdout[:2000]
    d = json.loads(lines[0])
    for key, kind in [("metric", str), ("value", (int, float)), ("unit", str), ("n_gpus", int), ("steps", int),
                      ("warmup", int), ("ms_per_step", (int, float)), ("higher_is_better", bool),
                      ("scaling", str), ("dtype", str), ("data", str), ("config", dict), ("impl", str),
                      ("cpu_baseline", dict), ("e2e", dict)]:
        assert isinstance(d[key], kind), key
    assert d["impl"] == "reference" and d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert "vs_baseline" in d
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["bytes_match"] is True
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0
    assert "workload" in d["config"]


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun the reference arm runs on rank 0 alone; any other rank
    exits 0 without work or output."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", WORLD_SIZE="2", RANK="1", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "3",
                        "--warmup", "3"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout == ""
