"""bench.py's clock sampler, on the CPU with a stand-in for nvidia-smi.

The bench line must carry the SM clock seen while the timed steps ran. With
eight ranks the headline's timed region lasts about 0.1 s, shorter than one
sampling interval of a sampler that only starts with it; the sampler now starts
before the region, counts samples from its start, and, when the region held
fewer than two, keeps running the same step untimed until two arrive.
"""

from __future__ import annotations

import os
import stat
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402

FAKE = """#!{py}
import sys, time
while True:
    print("0, 1965, 1965, 480.00, 0x0000000000000000, Not Active, Not Active, Not Active, Active",
          flush=True)
    time.sleep({period})
"""


def fake_smi(tmp_path, monkeypatch, period):
    exe = tmp_path / "nvidia-smi"
    exe.write_text(FAKE.format(py=sys.executable, period=period))
    exe.chmod(exe.stat().st_mode | stat.S_IEXEC)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")


def test_samples_in_the_region_are_counted_from_the_mark(tmp_path, monkeypatch):
    fake_smi(tmp_path, monkeypatch, 0.01)
    c = bench.ClockSampler(0)
    c.start()
    assert c.lines, "start() returns once the first sample is in"
    time.sleep(0.1)
    c.mark()
    time.sleep(0.15)  # the "timed region"
    c.extend(lambda: None)
    info = c.stop()
    assert info["window"] == "timed region"
    assert info["samples"] >= 2
    assert info["sm_mhz"] == 1965.0 and info["sm_max_mhz"] == 1965.0
    assert info["reasons"] == ["sw_power_cap"]
    assert info["samples"] < len(c.lines)  # samples before the mark are left out


def test_a_short_region_is_extended_with_untimed_steps(tmp_path, monkeypatch):
    fake_smi(tmp_path, monkeypatch, 0.2)
    c = bench.ClockSampler(0)
    c.start()
    c.mark()
    steps = []
    c.extend(lambda: (steps.append(1), time.sleep(0.01)))
    info = c.stop()
    assert steps, "the same step ran until samples arrived"
    assert info["samples"] >= 2
    assert info["window"].startswith("timed steps, continued untimed")


def test_no_nvidia_smi_gives_no_clock_record(monkeypatch, tmp_path):
    monkeypatch.setenv("PATH", str(tmp_path))
    c = bench.ClockSampler(0)
    c.start()
    c.mark()
    c.extend(lambda: None)
    assert c.stop() is None
