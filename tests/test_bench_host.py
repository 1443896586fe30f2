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
    # the issue floor from the ncu instruction counts: 392.5M warp instructions per north-star step
    assert abs(f["issue_warp_inst_per_step"] - (124773888 + 267692544)) < 1
    assert 0.0 < f["issue_frac"] < 1.0
    assert "issue_floor_ms" not in bench.compute_floor(2, 1536, 2048, 16, 0.1, 1965.0, False, False, 4)


def test_reference_arm_line_and_other_ranks(capsys, monkeypatch):
    """`--impl reference`: rank 0 prints one line with the arm's keys and the median of the timed
    steps (warm-up steps dropped); other ranks print nothing and exit 0.  The sampler is faked so
    the test does not spend the arm's CPU budget."""
    import argparse
    import json

    monkeypatch.setattr(bench, "cpu_sample_rate",
                        lambda elems, tokens, budget, seed=0, shape=None: (1000.0 + seed, 8, "fake sample", 0.1))
    a = argparse.Namespace(workload="scan", steps=3, warmup=1)
    assert bench.reference_arm(a, 2, 1) == 0
    assert capsys.readouterr().out == ""
    assert bench.reference_arm(a, 2, 0) == 0
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["n_gpus"] == 2 and line["steps"] == 3
    assert line["value"] == 1002.0  # median of seeds 1..3; seed 0 was the warm-up
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] == 8
    assert line["e2e"] == {"value": 1002.0, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert line["metric"] == bench.METRIC and line["config"]["global_batch"] == 16


def test_config_workloads_0_1_2():
    c0, c1, c2 = (bench.scan_shape(w, 1) for w in ("scan-c0", "scan-c1", "scan-c2"))
    assert (c0["b"], c0["d"], c0["L"], c0["dtype"], c0["passes"], c0["z"], c0["last"]) == \
        (2, 1536, 2048, "f32", "fwd", False, True)
    assert (c1["b"], c1["dtype"], c1["passes"], c1["z"]) == (2, "bf16", "fwd+bwd", True)
    assert (c2["b"], c2["d"], c2["L"], c2["passes"], c2["last"]) == (1, 5120, 32768, "fwd", True)
    # per-GPU batch fixed: the job grows with the GPUs
    assert bench.scan_shape("scan-c2", 4)["global_b"] == 4
    # configs 0 and 1 fit in L2 and flush it between steps; the north star and config 2 do not
    assert bench.flushes_l2(c0) and bench.flushes_l2(c1)
    assert not bench.flushes_l2(bench.scan_shape("scan", 1)) and not bench.flushes_l2(c2)
    assert "flushed" in bench.config_dict(1, c0)["l2"]


def test_algorithmic_bytes_forward_only_and_fp32():
    # config 0: fp32, no gate: read u, delta, write out (12 B / element) + B, C (128 B / token) + final state
    fwd, _ = bench.algorithmic_bytes(2, 1536, 2048, 16, es=4, z=False, last=True)
    assert fwd == 2 * 1536 * 2048 * 12 + 2 * 2048 * 128 + 2 * 1536 * 16 * 4
    # config 2: bf16 with a gate: 8 B / element + 64 B / token + final state
    fwd, _ = bench.algorithmic_bytes(1, 5120, 32768, 16, es=2, z=True, last=True)
    assert fwd == 5120 * 32768 * 8 + 32768 * 64 + 5120 * 16 * 4
    assert bench.launches_per_step(1536, 16, True) == 2 and bench.launches_per_step(1536, 16, False) == 1
    assert bench.launches_per_step(1536, 64, True) == 4


def test_cpu_baseline_sampler_forward_only():
    s = bench.scan_shape("scan-c0", 1)
    elems, tokens = s["b"] * s["d"] * s["L"], s["b"] * s["L"]
    value, threads, sample, seconds = bench.cpu_sample_rate(elems, tokens, 0.3, shape=s)
    assert value > 0 and "(fwd," in sample


def test_parallelism_names_the_exchange():
    """N > 1 fwd+bwd steps carry one all-reduce of the partial parameter gradients; forward-only
    steps and single GPUs have no exchange."""
    ns, c2 = bench.scan_shape("scan", 2), bench.scan_shape("scan-c2", 2)
    assert "all-reduce" in bench.parallelism(2, ns) and "inside the step" in bench.parallelism(2, ns)
    assert "no exchange" in bench.parallelism(2, c2)
    assert bench.parallelism(1, ns) == "x1, no collective"


def test_launch_counter_reports_why_it_could_not_count():
    """Without a GPU the torch profiler cannot count kernels: the counter says so instead of
    claiming a number (the bench then falls back to its launch model and names the reason)."""
    n, why = bench.count_own_launches(lambda: None)
    if n is None:
        assert isinstance(why, str) and why
    else:  # a machine with a GPU: nothing of this library launched
        assert n == 0 and why is None
