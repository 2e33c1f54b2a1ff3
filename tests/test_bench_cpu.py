"""bench.py helpers that need no GPU: the algorithmic byte count and roofline record of
the column loops, and the clock-sample filter."""

import os
import sys
import tempfile
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


def test_column_loop_bytes_and_roofline():
    per_matrix = 11008 * 4096 * 4.5 + 11008 * 4096 // 32
    expected = 2 * (per_matrix + 4 * 32 * 4096) + (per_matrix + 4 * 32 * 11008)
    assert bench.column_loop_bytes() == expected
    r = bench.column_loop_roofline(2.8, 7000.0, "measured")
    assert abs(r["achieved"] - expected / 2.8e-3 / 1e9) < 1e-6
    assert abs(r["frac"] - r["achieved"] / 7000.0) < 1e-12 and r["unit"] == "GB/s"


def test_clock_samples_inside_the_timed_region():
    import datetime

    c = bench.ClockSampler(0)
    fd, c.path = tempfile.mkstemp()
    os.close(fd)
    now = time.time()

    def stamp(t):
        return datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]

    with open(c.path, "w") as f:
        for i in range(10):
            mhz = 1800 if 3 <= i <= 6 else 900
            cap = "Active" if i == 4 else "Not Active"
            f.write(f"{stamp(now + 0.05 * i)}, 0, {mhz}, 1965, 700, 0x4, Not Active, Not Active, Not Active, {cap}\n")

    class Proc:
        def terminate(self):
            pass

        def wait(self, timeout=None):
            pass

    c.proc, c.t0, c.t1 = Proc(), now + 0.15, now + 0.30
    out = c.stop()
    assert out["sm_mhz"] == 1800.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"] and out["samples"] == 6
