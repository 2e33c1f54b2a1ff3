"""bench.py helpers that need no GPU: the CPU-sample record, the executed-tile count of
the Hessian roofline, and the clock-sample filter."""

import os
import sys
import tempfile
import time

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


def test_cpu_sample_record_reports_what_ran():
    class Sample:
        elems = 1000

    rec = bench.cpu_sample_record(Sample(), [2.0, 1.0, 3.0])
    assert rec["value"] == 1000 / 2.0 and rec["kind"] == "port" and rec["cores"] >= 1
    assert rec["seconds_per_sample"] == 2.0 and "median of 3 runs" in rec["sample"]


def test_hessian_executed_elems_counts_upper_tiles():
    assert bench.hessian_executed_elems(2048) == 256 * 256 * 36
    assert bench.hessian_executed_elems(768) == 256 * 256 * 6


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
