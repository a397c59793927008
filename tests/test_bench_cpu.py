"""bench.py's bookkeeping on the CPU: the roofline fractions it prints and the ncu traffic figures
it reads from profiles/. No GPU: the workloads here are stand-ins with a fixed algorithmic size."""
import bench

PEAKS = (6541.8, 1666.9, "measured", 1418.3)


class _Stand:
    """The roofline's view of a workload: its bound, name, kernel and work per launch."""

    def __init__(self, bound, name, work, peak_scale=1.0):
        self.bound, self.name, self.kernel = bound, name, "k"
        self._work = work
        if peak_scale != 1.0:
            self.peak_scale = peak_scale

    def algorithmic(self):
        return self._work


def test_hbm_roofline_is_bytes_over_time_against_the_copy_peak():
    r = bench.roofline(_Stand("hbm", "c3", 2.277e9), 0.35, PEAKS)
    assert r["unit"] == "GB/s" and r["peak"] == 6541.8
    assert abs(r["achieved"] - 2.277e9 / 0.35e-3 / 1e9) < 0.01
    assert abs(r["frac"] - r["achieved"] / 6541.8) < 1e-4
    assert "frac_sustained" not in r


def test_tensor_roofline_adds_the_sustained_fraction_only_under_the_power_cap():
    w = _Stand("tensor", "c5", 6.594e12)
    capped = bench.roofline(w, 5.77, PEAKS, {"reasons": ["sw_power_cap"]})
    free = bench.roofline(w, 5.77, PEAKS, {"reasons": []})
    unsampled = bench.roofline(w, 5.77, PEAKS)
    assert capped["peak"] == free["peak"] == 1666.9
    assert capped["frac"] == free["frac"]
    assert abs(capped["frac_sustained"] - capped["achieved"] / 1418.3) < 1e-4
    assert "frac_sustained" not in free and "frac_sustained" not in unsampled


def test_tf32_roofline_is_against_half_the_bf16_rates():
    w = _Stand("tensor", "prefill_f32", 5.498e11, peak_scale=0.5)
    r = bench.roofline(w, 1.4, PEAKS, {"reasons": ["sw_power_cap"]})
    assert r["peak"] == 1666.9 * 0.5
    assert abs(r["peak_sustained"] - 1418.3 * 0.5) < 0.01
    assert "tf32" in r["peak_source"]


def test_every_bandwidth_or_tensor_bound_line_has_a_committed_traffic_figure():
    # C1 and C2 are latency-bound (a megabyte, half a GFLOP): no DRAM figure is claimed for them
    for name in ("c3", "c3bf16", "decode256", "c4", "c5", "prefill", "prefill_f32", "qwen35",
                 "proj", "proj64", "prologue"):
        t = bench.profile_traffic(name)
        assert t is not None and t > 1e7, name
    assert bench.profile_traffic("c1") is None
