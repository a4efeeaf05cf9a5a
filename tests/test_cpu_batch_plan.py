"""The batched kernel's merge-slice plan, checked on the host: tests/probes/batch_plan_probe.cu
includes the kernel header, calls batch_merge_width for every model shape the batched kernel
takes (head_dim 32 / 64 / 128, groups of 2 to 8 query heads, up to 8 KV heads, 1 to 16 columns,
several SM counts) and checks the slice width against the merge loop's thread mapping, load
alignment and shared-memory area. Built with nvcc for the host side only; no GPU."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_merge_width_fits_the_merge_loop(tmp_path):
    from voxgen_b200 import _build
    try:
        nvcc = _build.nvcc()
    except FileNotFoundError:
        pytest.skip("nvcc not found")
    exe = tmp_path / "batch_plan_probe"
    subprocess.run([nvcc, "-std=c++17", "--expt-relaxed-constexpr", *_build.ARCH, "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "probes" / "batch_plan_probe.cu"), "-o", str(exe)],
                   check=True, capture_output=True, timeout=300)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.startswith("ok "), r.stdout + r.stderr
