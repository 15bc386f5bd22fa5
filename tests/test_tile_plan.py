"""Host check of the ancestor kernel's tile planner (tests/native/plan_check.cu).

The planner decides which K/V rows a tile stages and which key columns each
warp's walk uses; a node missing from a window would make the kernel read an
unrelated shared-memory row. The C++ harness plans every tile of ~1200 tree
shapes with the same header the kernel compiles and checks coverage exactly.
"""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


@pytest.mark.skipif(shutil.which(NVCC) is None and not Path(NVCC).exists(), reason="nvcc not available")
def test_tile_planner_covers_every_walk(tmp_path):
    exe = tmp_path / "plan_check"
    subprocess.run([NVCC, "-O2", "-std=c++17", f"-I{ROOT / 'include'}", str(ROOT / "tests/native/plan_check.cu"),
                    "-o", str(exe)], check=True, capture_output=True, timeout=600)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:]
    assert "fails 0" in r.stdout
    # the benchmark trees stage fewer rows with subtree tiles (C2: 4-ary depth 5, C3: binary depth 9)
    caps = {}
    for line in r.stdout.splitlines():
        if line.startswith("b="):
            f = dict(kv.split("=", 1) for kv in line.replace("(", " ").replace(")", " ").split() if "=" in kv)
            caps[(int(f["b"]), int(f["d"]), int(f["sub"]))] = int(f["rows_cap"])
    assert caps[(4, 5, 1)] < caps[(4, 5, 0)]
    assert caps[(2, 9, 1)] < caps[(2, 9, 0)] // 2 + 1
