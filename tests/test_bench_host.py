"""Host-side pieces of bench.py (no GPU): the roofline's peak and DRAM-traffic inputs."""

import importlib.util
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_traffic_per_launch_from_profile_summary():
    # the committed ncu summary gives the step's DRAM traffic per layer; per launch it is that times
    # the layers over the step's launches (2 per layer plus the last side-output launch on one GPU)
    b = _bench()
    text = (ROOT / "profiles" / "gemv_w8_stack_decode_traffic.md").read_text()
    per_layer = int(next(l for l in text.splitlines() if l.startswith("traffic_bytes_per_step_layer:")).split(":")[1])
    assert b.traffic_per_launch(73, 36) == int(per_layer * 36 / 73)
    # the traffic is within 1 % of the algorithmic weight bytes of a layer (every byte read once)
    layer_bytes = 9059696640 // 36
    assert abs(per_layer - layer_bytes) / layer_bytes < 0.01


def test_peaks_are_the_measured_figures():
    b = _bench()
    pk = b.peaks()
    assert pk["hbm_gbs"] > 1000 and pk["source"] in ("measured", "fallback")
