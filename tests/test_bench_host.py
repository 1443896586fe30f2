"""Host-side logic of bench.py (no GPU): workload shapes and their scaling kinds, the algorithmic
byte counts the roofline divides by, the config block of the JSON line, and the CPU-baseline
sampler on a tiny budget."""
import pytest

import bench


def test_scan_workload_shapes():
    s = bench.scan_shape("scan", 4)  # north-star point: fixed batch 8 per GPU
    assert (s["b"], s["global_b"], s["d"], s["L"], s["n"], s["scaling"]) == (8, 32, 1536, 2048, 16, "weak")
    c4 = bench.scan_shape("scan-c4", 8)  # config 4: global batch 64 split over the GPUs
    assert (c4["b"], c4["global_b"], c4["d"], c4["scaling"]) == (8, 64, 5120, "strong")
    with pytest.raises(SystemExit):
        bench.scan_shape("scan-c4", 3)  # 64 rows do not split over 3 GPUs


def test_algorithmic_bytes_match_the_stated_per_unit_figures():
    fwd, bwd = bench.algorithmic_bytes(8, 1536, 2048, 16)
    elems, tokens = 8 * 1536 * 2048, 8 * 2048
    assert fwd == elems * 8 + tokens * 64          # 8 B / element, 64 B / token (bf16)
    assert bwd == elems * 14 + tokens * 192        # 14 B / element, 192 B / token
    assert abs((fwd + bwd) / 1e6 - 558.0) < 1.0    # the north-star step moves ~558 MB


def test_config_block_names_the_workload():
    for wl, world in (("scan", 1), ("scan", 8), ("scan-c4", 2)):
        s = bench.scan_shape(wl, world)
        cfg = bench.config_dict(world, s)
        assert cfg["global_batch"] == s["global_b"] and cfg["per_gpu_batch"] == s["b"]
        assert cfg["d_inner"] == s["d"] and cfg["seq_len"] == s["L"] and cfg["d_state"] == s["n"]
        assert "workload" in cfg and "l2" in cfg and f"x{world}" in cfg["parallelism"]


def test_cpu_baseline_sampler_reports_a_rate():
    s = bench.scan_shape("scan", 1)
    elems, tokens = s["b"] * s["d"] * s["L"], s["b"] * s["L"]
    value, threads, sample, seconds = bench.cpu_sample_rate(elems, tokens, 0.5, shape=s)
    assert value > 0 and threads >= 1 and seconds > 0
    assert "fwd+bwd" in sample


def test_compute_floor_is_a_fraction_of_the_step():
    f = bench.compute_floor(8, 1536, 2048, 16, ms_step=0.87, sm_mhz=1965.0)
    assert 0.2 < f["mufu_frac"] < 0.6 and f["mufu_floor_ms"] > 0
