"""bench.py's clock record: one nvidia-smi sampler for the job, each timed
region summarised from the samples stamped inside it (CPU only: the rows are
given, no nvidia-smi runs)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


def _sampler():
    c = bench.ClockSampler([0, 1])
    c.proc = object()  # rows are supplied directly below
    return c


POWER_CAP = [False, False, False, True]
NONE = [False] * 4


def test_stamp_parses_nvidia_smi_timestamps():
    a = bench.ClockSampler._stamp("2026/12/02 10:11:12.345")
    b = bench.ClockSampler._stamp("2026/12/02 10:11:13.095")
    assert abs((b - a) - 0.75) < 1e-6


def test_region_uses_samples_inside_it_and_drops_idle_ones():
    rows = [(10.0, 1965.0, 1965.0, NONE), (10.2, 1965.0, 1965.0, POWER_CAP), (10.2, 1900.0, 1965.0, NONE),
            (10.4, 345.0, 1965.0, NONE), (11.0, 1200.0, 1965.0, [True, False, False, False])]
    s = _sampler().summary(rows, 10.1, 10.45)
    assert s["window"] == "inside the timed region"
    assert s["samples"] == 2  # the 345 MHz idle sample is not "under load"
    assert s["sm_mhz"] == 1932.5 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"] and s["gpus"] == 2


def test_short_region_takes_neighbouring_samples():
    rows = [(10.0, 1965.0, 1965.0, NONE), (12.0, 1965.0, 1965.0, [False, True, False, False])]
    s = _sampler().summary(rows, 10.3, 10.35)
    assert s["window"].startswith("within 0.5 s") and s["samples"] == 1 and s["reasons"] == []
    assert _sampler().summary(rows, 11.0, 11.05)["reasons"] == ["no samples"]


def test_stop_fills_every_registered_region():
    c = bench.ClockSampler()  # no devices: a rank other than 0
    r1 = c.begin()
    bench.ClockSampler.end(r1)
    r2 = c.begin()
    c.stop()
    assert r1["reasons"] == ["nvidia-smi unavailable"] and r2["samples"] == 0
    assert "_t0" not in r1 and "_t1" not in r2


def test_tp_exchange_reads_consumer_launches():
    import numpy as np

    layers = 3
    rec = np.zeros((256, 1024, 8), np.uint64)
    # consumers: QKV of layers 1, 2 (launches 5, 10), gate/up (3, 8, 13), head (15)
    for launch, us in ((5, 2.0), (10, 2.0), (3, 1.0), (8, 3.0), (13, 3.0), (15, 2.0), (2, 50.0)):
        rec[launch, :4, 1] = 1000
        rec[launch, :4, 5] = 1000 + int(us * 1e3)
    out = bench.tp_exchange_us([rec], layers)
    assert out["us_per_allreduce"] == 2.0 and out["launches_sampled"] == 6 and out["allreduces_per_token"] == 6
