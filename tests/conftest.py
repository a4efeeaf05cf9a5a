"""Shared pytest configuration.

``-m gpu`` tests need a B200 and the native library; everything else runs on the CPU.
"""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# Parity tolerance of the decode step (hidden states, attention outputs, projections):
# |cuda - oracle| <= ATOL + RTOL * |oracle|, elementwise, in fp32.
ATOL = 2e-3
RTOL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the native library")


def assert_close(got, want, atol=ATOL, rtol=RTOL, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    if bad.any():
        i = int(np.argmax(err - (atol + rtol * np.abs(want))))
        raise AssertionError(
            f"{what}: {int(bad.sum())}/{bad.size} elements outside atol={atol} rtol={rtol}; "
            f"max abs err {err.max():.3e}; worst index {i}: got {got.flat[i]!r} want {want.flat[i]!r}")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    d = os.environ.get("VOXGEN_MODEL_CACHE")
    return Path(d) if d else tmp_path_factory.mktemp("models")


def spec_path(model_dir, name, **over):
    from voxgen_b200 import synth
    return synth.model_path(synth.preset(name, **over), model_dir)
