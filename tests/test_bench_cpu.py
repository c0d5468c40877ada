"""Host-side logic of the benchmark line (no GPU): the data-parallel critical path and the clock
record built from sampled NVML readings."""
import importlib.util
from pathlib import Path

import pytest

_spec = importlib.util.spec_from_file_location("c3_bench", Path(__file__).resolve().parents[1] / "bench.py")
bench = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(bench)

KINDS = ("fwd", "prepass", "dw", "dx")


def test_allreduce_that_ends_after_dx_limits_the_step():
    # 8-GPU shape of the step: dX (100 us) runs beside an all-reduce of 126 us
    kt = {"fwd": 0.057, "prepass": 0.014, "dw": 0.054, "dx": 0.100, "allreduce": 0.126}
    cp = bench.critical_path(kt, KINDS, 0.265)
    assert cp["limiting"] == "allreduce"
    assert cp["ms"]["allreduce_exposed"] == pytest.approx(0.265 - 0.225)
    assert cp["allreduce_total_ms"] == 0.126


def test_longest_phase_limits_when_the_allreduce_is_hidden():
    # 2-GPU shape: the GEMMs dominate; an all-reduce shorter than dX does not limit
    kt = {"fwd": 0.177, "prepass": 0.029, "dw": 0.175, "dx": 0.193, "allreduce": 0.150}
    assert bench.critical_path(kt, KINDS, 0.600)["limiting"] == "dx"
    kt["fwd"] = 0.300
    assert bench.critical_path(kt, KINDS, 0.700)["limiting"] == "fwd"


def test_overlapped_dw_dx_counts_their_span_once():
    kt = {"fwd": 0.057, "prepass": 0.014, "dw": 0.054, "dx": 0.060, "dwdx": 0.080, "allreduce": 0.0}
    cp = bench.critical_path(kt, KINDS, 0.200)
    assert set(cp["ms"]) == {"fwd", "prepass", "dwdx", "allreduce_exposed"}
    assert cp["ms"]["allreduce_exposed"] == pytest.approx(0.200 - 0.151)
    assert cp["limiting"] == "dwdx"


def test_no_allreduce_time_and_a_step_shorter_than_its_phases():
    kt = {"fwd": 0.05, "prepass": 0.01, "dw": 0.05, "dx": 0.05}
    cp = bench.critical_path(kt, KINDS, 0.10)  # events overlap: nothing is exposed
    assert cp["ms"]["allreduce_exposed"] == 0.0
    assert cp["allreduce_total_ms"] is None
    assert cp["limiting"] in ("fwd", "dw", "dx")


def test_clock_record_uses_samples_under_load():
    cs = bench.ClockSampler(0, enabled=False)
    assert cs.record() is None
    cs.max_mhz = 1965
    # (MHz, NVML clock-event reason bits): two idle samples, three under load with sw_power_cap
    cs.samples = [(345, 0x1), (1965, 0x0), (1800, 0x4), (1700, 0x4), (300, 0x1)]
    rec = cs.record()
    assert rec["samples"] == 5 and rec["samples_under_load"] == 3
    assert rec["sm_mhz"] == 1800 and rec["sm_mhz_min_under_load"] == 1700
    assert rec["reasons"] == ["sw_power_cap"]
    assert rec["sm_max_mhz"] == 1965


def test_clock_record_falls_back_to_all_samples_when_every_one_is_idle():
    cs = bench.ClockSampler(0, enabled=False)
    cs.samples = [(345, 0x1), (400, 0x1 | 0x40)]
    rec = cs.record()
    assert rec["samples_under_load"] == 0
    assert rec["sm_mhz"] == pytest.approx(372.5)
    assert rec["reasons"] == ["hw_thermal_slowdown"]
