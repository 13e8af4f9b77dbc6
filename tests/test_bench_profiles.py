"""The committed ncu summaries that ``bench.py`` reads its ``roofline.traffic``
figures from: every timed window the bench can run is covered, and each
side leg's per-launch traffic line parses. (CPU only: nothing is launched.)"""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


@pytest.mark.parametrize("steps", [1, 20, 128, 1024])
def test_dense_traffic_covers_every_timed_window(steps: int) -> None:
    traffic, source = bench._profile_traffic(steps)
    assert traffic is not None, source
    # between the writes alone (~204 MB) and the algorithmic bytes of a launch
    assert 2.0e8 < traffic < bench.ROWS_PER_GPU * bench.ALGO_BYTES_PER_ROW_STEP
    assert f"steps 0..{min(steps, bench.EPISODE) - 1}" in source


def test_driver_window_traffic_is_the_mean_of_its_steps() -> None:
    """The 20-step window's figure is the mean of the summary's lines 0..19."""
    per = {}
    with open(os.path.join(ROOT, "profiles", "dense_step_config2.md")) as f:
        for line in f:
            if line.strip().startswith("step_dram_bytes:"):
                k, rd, wr = line.split(":", 1)[1].split()[:3]
                per[int(k)] = float(rd) + float(wr)
    assert sorted(per) == list(range(bench.EPISODE))
    traffic, _ = bench._profile_traffic(20)
    assert traffic == pytest.approx(sum(per[k] for k in range(20)) / 20)


@pytest.mark.parametrize("name", ["pda_step_config4.md", "dense_step_config3.md",
                                  "soft_step_lookahead.md"])
def test_side_leg_traffic_lines_parse(name: str) -> None:
    value = bench._profile_bytes(name)
    assert value is not None and value > 1e6
