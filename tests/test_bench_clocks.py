"""The bench's nvidia-smi clock sampler: the samples it keeps are those whose
timestamps fall inside the marked timed region (or, for a region shorter than
the sampling period, those around it), filtered to the bench's GPU, with the
throttle reasons seen among them. Runs on a synthetic nvidia-smi CSV."""
import datetime
import time

import bench


class _Done:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        pass


def _sampler(tmp_path, rows):
    path = tmp_path / "clocks.csv"
    path.write_text("".join(r + "\n" for r in rows))
    s = bench.ClockSampler(str(path))
    s.proc = _Done()
    s.f = open(tmp_path / "unused", "w")
    return s


def _row(t, uuid, mhz, power_cap):
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    cap = "Active" if power_cap else "Not Active"
    return f"{ts}, 0, {uuid}, {mhz} MHz, 1965 MHz, 900.00 W, 0x4, Not Active, Not Active, Not Active, {cap}"


def test_keeps_samples_inside_the_region(tmp_path):
    t0 = time.time()
    rows = [_row(t0 + 0.05 * i, "GPU-a", 1500 + 10 * i, i == 5) for i in range(20)]
    rows += [_row(t0 + 0.05 * i, "GPU-b", 1000, True) for i in range(20)]  # another GPU
    s = _sampler(tmp_path, rows)
    s.mark(t0 + 0.199, t0 + 0.401)  # samples 4..8
    clk = s.stop("GPU-a")
    assert clk["samples"] == 5
    assert clk["sm_mhz"] == 1560.0
    assert clk["sm_max_mhz"] == 1965.0
    assert clk["reasons"] == ["sw_power_cap"]


def test_short_region_takes_the_samples_around_it(tmp_path):
    t0 = time.time()
    rows = [_row(t0 + 0.2 * i, "GPU-a", 1700, False) for i in range(5)]
    s = _sampler(tmp_path, rows)
    s.mark(t0 + 0.25, t0 + 0.30)  # between two samples
    clk = s.stop("GPU-a")
    assert clk["samples"] >= 1 and clk["reasons"] == []


def test_no_samples_gives_none(tmp_path):
    s = _sampler(tmp_path, ["garbage line"])
    s.mark(0.0, 1.0)
    assert s.stop("GPU-a") is None
