"""The GEMM kernel's work-unit plan and the K split of its last wave
(macrograd_b200/csrc/mg_plan.h), checked on the CPU: the same header the
kernel and the launcher compile is built into tests/plan_check.cpp with g++
and run over thousands of (tiles, units, K-blocks) cases -- every (tile,
K-block) covered once, partial slots written once and read by their tile's
final range, the split never slower than whole-tile waves -- plus the plans
of the row-sharded 8192^3 shapes, and the column bands of the copy-engine
all-gather (contiguous, covering, never growing towards the end)."""
import os
import shutil
import subprocess
import tempfile

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "macrograd_b200", "csrc")


def test_unit_plan_covers_every_k_block_once():
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "plan_check")
        subprocess.run([cxx, "-std=c++17", "-O2", "-I", CSRC, os.path.join(HERE, "plan_check.cpp"), "-o", exe],
                       check=True)
        out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.startswith("ok"), out.stdout + out.stderr
