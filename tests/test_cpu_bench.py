"""Host logic of bench.py that decides what a bench line measures: how the timed steps are
spread over a config's positions, the algorithmic bytes the roofline divides, and where the
roofline's peak comes from."""
import importlib.util
import json
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("k", [1, 4, 15, 16, 17, 20, 300, 3000, 3072, 5000])
def test_spread_blocks_cover_the_range(bench, k):
    """cfg2 decodes positions 1024..4095: the k timed steps run in blocks whose starts are spread
    over that range, every step inside it, the first block at its start and (with two or more
    blocks) the last one ending at its end, whatever k the caller passes."""
    lo, hi = 1024, 4095
    blocks = bench.spread_blocks(k, lo, hi)
    assert sum(n for _, n in blocks) == k
    starts = [b for b, _ in blocks]
    assert starts == sorted(starts) and starts[0] == lo
    for b, n in blocks:
        assert n >= 1 and lo <= b and b + n - 1 <= hi or k > hi - lo + 1
    if k <= hi - lo + 1:
        assert len(blocks) <= 16
        if len(blocks) > 1:
            b, n = blocks[-1]
            assert b + n - 1 == hi
        # no two blocks overlap
        for (b0, n0), (b1, _) in zip(blocks, blocks[1:]):
            assert b0 + n0 <= b1


def test_spread_blocks_short_range(bench):
    """cfg1 spans 256 positions; more steps than positions need more than 16 blocks."""
    blocks = bench.spread_blocks(600, 128, 383)
    assert sum(n for _, n in blocks) == 600
    assert all(128 <= b and b + n - 1 <= 383 for b, n in blocks)


def test_algorithmic_bytes(bench):
    """Weights + norm weights once per token, plus the K/V rows read (position + 1 of them per
    layer) and the row written: 2 (K, V) x 2 bytes x kv_dim per layer and position."""
    info = {"block_count": 28, "kv_dim": 256, "layer_weight_bytes": 1_403_781_120, "norm_weight_bytes": 466_944}
    per_pos = 28 * 256 * 2 * 2
    b = bench.algorithmic_bytes(info, [0, 1023, 4095])
    base = 1_403_781_120 + 466_944
    assert b == [base + per_pos * 1 + per_pos, base + per_pos * 1024 + per_pos, base + per_pos * 4096 + per_pos]


def test_measured_peak_source(bench, tmp_path, monkeypatch):
    """The roofline divides by MEASURED_PEAKS.json's copy bandwidth when the file exists, and by
    the stated fallback otherwise, and says which."""
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.measured_peaks() == (6650.0, "fallback")
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6551.7}))
    assert bench.measured_peaks() == (6551.7, "measured")
