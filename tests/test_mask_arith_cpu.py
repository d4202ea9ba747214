"""The kernels' mask arithmetic (csrc/attn_common.cuh) against the element-wise mask definition,
compiled for the host with g++ (no GPU): key-tile ranges, full-tile tests, the per-query-tile
full range used to skip the mask test per key tile, and per-row admissible column intervals;
and the persistent kernel's work-item order (item_coords)."""

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_mask_arithmetic_matches_elementwise_definition(tmp_path):
    exe = tmp_path / "mask_ranges_check"
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", str(ROOT / "mlx-primitives_b200" / "csrc"),
                    "-o", str(exe), str(ROOT / "tests" / "native" / "mask_ranges_check.cpp")],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe), "3000"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 mismatches" in r.stdout


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_work_item_order_is_a_bijection_in_equal_groups(tmp_path):
    exe = tmp_path / "item_order_check"
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", str(ROOT / "mlx-primitives_b200" / "csrc"),
                    "-o", str(exe), str(ROOT / "tests" / "native" / "item_order_check.cpp")],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe), "2000"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 violations" in r.stdout
