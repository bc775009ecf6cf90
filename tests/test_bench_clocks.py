"""bench.py's clock record: the samples inside the timed steps' wall-clock
window decide the median SM clock and the throttle reasons; a window too
short to hold a sample falls back to the loaded samples around it and says
so; no sample at all reads "unsampled"."""
import datetime
import pathlib
import sys

sys.path.insert(0, str(pathlib.Path(__file__).resolve().parents[1]))
import bench  # noqa: E402

T0 = datetime.datetime(2026, 12, 2, 11, 0, 0)


def row(sec, mhz, watts, cap="Not Active", thermal="Not Active"):
    ts = (T0 + datetime.timedelta(seconds=sec)).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return f"{ts}, 0, {mhz}, 1965, {watts}, 0x0, Not Active, Not Active, {thermal}, {cap}"


def at(sec):
    return (T0 + datetime.timedelta(seconds=sec)).timestamp()


def test_samples_inside_the_window_decide():
    text = "\n".join([
        row(0.0, 1965, 120),                           # idle, before
        row(0.1, 1900, 700),                           # warm-up
        row(0.2, 1600, 990, cap="Active"),             # timed
        row(0.3, 1620, 995, cap="Active"),             # timed
        row(0.4, 1500, 800, thermal="Active"),         # after the window
    ])
    c = bench.summarize_clocks(text, (at(0.15), at(0.35)))
    assert c["sm_mhz"] == 1610.0
    assert c["reasons"] == ["sw_power_cap"]
    assert c["samples"] == 2 and c["span"] == "timed steps"
    assert c["sm_max_mhz"] == 1965.0


def test_short_window_falls_back_to_loaded_samples():
    text = "\n".join([row(0.0, 1965, 100), row(0.1, 1800, 900), row(0.2, 1700, 950)])
    c = bench.summarize_clocks(text, (at(0.12), at(0.18)))
    assert c["sm_mhz"] == 1750.0 and c["samples"] == 2
    assert c["span"].startswith("loaded samples around the timed steps")


def test_no_samples_is_unsampled():
    assert bench.summarize_clocks("", (0.0, 1.0))["reasons"] == ["unsampled"]
    assert bench.summarize_clocks("garbage,line\n", None)["reasons"] == ["unsampled"]
