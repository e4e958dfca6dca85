"""CPU: the parts of bench.py that need no GPU — the traffic figures it reads
from the committed ncu summaries, the clock / throttle-reason parsing, and
the reference arm's JSON line (the numpy oracle on a one-step sample)."""

from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import REPO

sys.path.insert(0, REPO)
import bench  # noqa: E402


def test_profile_traffic_keys_parse():
    """bench.py's roofline.traffic comes from these lines of profiles/: the B=1
    cluster kernel's (captured as a plain cluster launch), the flat kernel's
    and the batched step's."""
    b1c = bench.profile_traffic("decode_b1_cfg1.md")
    flat = bench.profile_traffic("decode_b1_flat_cfg1.md")
    step = bench.profile_traffic("paged_step_b256_pos80.md", "traffic_bytes_per_step")
    assert isinstance(b1c, int) and 600_000_000 < b1c < 620_000_000  # one pass over the 607 MB of weights
    assert isinstance(flat, int) and flat > 600_000_000
    assert isinstance(step, int) and step > 1_000_000_000
    assert bench.profile_traffic("no_such_summary.md") is None


class _FakeProc:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0


def test_clock_sampler_parses_reasons():
    cs = bench.ClockSampler(0)
    cs.proc = _FakeProc()
    cs.lines = [
        "0, 1965, 1965, 700.1, 0x0, Not Active, Not Active, Not Active, Not Active",
        "0, 1890, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1800, 1965, 999.0, 0x4, Not Active, Not Active, Not Active, Active",
        "garbage",
    ]
    got = cs.stop()
    assert got["sm_mhz"] == 1890.0 and got["sm_max_mhz"] == 1965.0
    assert got["reasons"] == ["sw_power_cap"] and got["samples"] == 3


def test_reference_arm_line():
    """`bench.py --impl reference` prints one JSON line with the contract's
    keys, the oracle timed on a bounded sample (one decode step of 32
    sequences here)."""
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "1"],
                         capture_output=True, text=True, timeout=600, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["value"] > 0
    assert line["metric"] == bench.METRIC and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["workload"].startswith("serve (config 5)")
    # the line's step is the sample step it timed: K steps of ms_per_step fit in the run
    assert line["steps"] == 2 and line["warmup"] == 1
    assert abs(line["ms_per_step"] - line["cpu_baseline"]["ms_per_step"]) < 1e-9
    assert abs(line["value"] - 1000.0 * bench.REF_SAMPLE_SEQS / line["ms_per_step"]) < 1e-6 * line["value"]


def test_timed_positions_span_config5():
    """The K timed steps of the headline cover config 5's decode positions
    64..319 (evenly for K < 256, every position in turn from 256 on)."""
    for k in (1, 2, 3, 20, 255):
        p = bench.timed_positions(k)
        assert len(p) == k and all(64 <= x <= 319 for x in p)
        if k > 1:
            assert p[0] == 64 and p[-1] == 319 and p == sorted(p)
    assert bench.timed_positions(256) == list(range(64, 320))
    assert bench.timed_positions(300)[256:] == list(range(64, 108))
