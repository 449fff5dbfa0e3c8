"""Host-side logic of bench.py that needs no GPU: the clock sampler's summary
(the clock-event reason bits it reports and the ones the measurement rules
reject) and the ffn_up algorithmic-byte count behind `roofline.achieved`."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_clock_summary_reasons(bench):
    s = bench.ClockSampler(0)
    s.max_mhz = 1965.0
    # (sm MHz, power W, clock-event reason mask): idle, power cap, HW slowdown,
    # HW power brake (reported as HW slowdown), SW and HW thermal slowdown.
    s.rows = [(1965.0, 700.0, 0x1), (1800.0, 990.0, 0x4), (1700.0, 990.0, 0x8),
              (1750.0, 980.0, 0x80), (1790.0, 985.0, 0x20), (1780.0, 985.0, 0x40)]
    out = s.summary()
    assert out["sm_max_mhz"] == 1965.0
    assert out["sm_mhz"] == pytest.approx(1785.0)
    assert out["samples"] == 6
    assert out["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_power_cap", "sw_thermal_slowdown"]


def test_clock_summary_power_cap_only_and_unsampled(bench):
    s = bench.ClockSampler(0)
    s.rows = [(1965.0, 900.0, 0x4), (1950.0, 990.0, 0x4 | 0x1)]
    assert s.summary()["reasons"] == ["sw_power_cap"]
    empty = bench.ClockSampler(0)
    assert empty.summary()["reasons"] == ["unsampled"]


def test_ffn_up_algorithmic_bytes(bench):
    # NVFP4 codes + swizzled scales of the 1760 x 3072 activation and the
    # 14336 x 3072 weight, the 1760 x 14336 NVFP4 output with its scales, and
    # the bf16 bias.
    m, n, k = 1760, 14336, 3072
    pad = lambda rows: (rows + 127) // 128 * 128
    expect = (m * k // 2 + pad(m) * k // 16 + n * k // 2 + pad(n) * k // 16
              + m * n // 2 + pad(m) * n // 16 + n * 2)
    assert bench.ffn_up_bytes() == expect
