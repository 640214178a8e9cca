"""Host-side logic of bench.py (no GPU): the strong-scaling batch split, the
host identity and the roofline peak arithmetic."""

from __future__ import annotations

import importlib.util
import os

from conftest import REPO


def _bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(REPO, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_strong_scaling_split_covers_the_batch_once():
    bench = _bench()
    for world in (1, 2, 3, 4, 8):
        parts = [bench.rank_slice(r, world) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == bench.B
        assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
        sizes = [hi - lo for lo, hi in parts]
        assert max(sizes) - min(sizes) <= 1
    assert [bench.rank_slice(r, 8) for r in range(2)] == [(0, 4), (4, 8)]


def test_host_identity_and_peaks():
    bench = _bench()
    h = bench.host_identity()
    assert h["nproc"] == os.cpu_count()
    fp32, sfu = bench.peaks_at(1965.0, 148)
    assert abs(fp32 - 148 * 128 * 2 * 1.965e9) < 1.0
    assert abs(sfu - 148 * 16 * 1.965e9) < 1.0
    line = bench.config_line("c", "w", 2.0, 1000, 500, 1965.0, 148)
    assert abs(line["bbox_pair_evals_per_s"] - 500 / 2e-3) < 1e-6
    assert abs(line["fp32_frac"] - 500 * 170 / 2e-3 / fp32) < 1e-12
