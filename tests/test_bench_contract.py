"""bench.py's reference arm (the oracle port of the block on the host cores) keeps the one-JSON-line
contract: it runs without a GPU, so it is checked here on a small configuration."""

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_json_line():
    r = subprocess.run(
        [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--config", "c0_l2304", "--steps", "1",
         "--warmup", "0"],
        capture_output=True, text=True, timeout=600, cwd=REPO,
    )
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, lines
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["tokens"] == 2304
    # the line reports the blocks it actually timed and warmed up with (bench.py raises --warmup to 3)
    assert d["steps"] == 1 and d["warmup"] == 3


def test_reference_arm_stops_within_its_budget():
    """Asked for more blocks than fit in the wall-clock budget, the arm times fewer and says how many."""
    sys.path.insert(0, REPO)
    import time

    import bench

    calls = []

    def run():
        calls.append(time.perf_counter())
        time.sleep(0.05)

    times, warm = bench.time_cpu_steps(run, steps=100, warmup=2, budget_s=0.4)
    assert warm == 2
    assert 1 <= len(times) < 100
    assert len(calls) == warm + len(times)
    assert calls[-1] - calls[0] < 0.4


def test_branch_reference_arms_keep_the_contract():
    """``--impl reference --branch ffn|text``: the oracle port of that branch, under the branch's own metric."""
    sys.path.insert(0, REPO)
    import bench

    for branch, metric in (("ffn", bench.FFN_METRIC), ("text", bench.TEXT_METRIC)):
        r = subprocess.run(
            [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--branch", branch, "--config",
             "c0_l2304", "--context-tokens", "256", "--steps", "1", "--warmup", "0"],
            capture_output=True, text=True, timeout=600, cwd=REPO,
        )
        assert r.returncode == 0, r.stderr[-2000:]
        lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
        assert len(lines) == 1, lines
        d = json.loads(lines[0])
        assert d["impl"] == "reference" and d["metric"] == metric and d["config"]["branch"] == branch
        assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["kind"] == "port"
        assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]
