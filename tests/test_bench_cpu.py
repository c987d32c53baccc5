"""bench.py's reference arm on the CPU (no GPU): every --config runs on shrunken
shapes (--tiny) through the reference's CPU code (oracle/_ref, else the
restatement) and prints one JSON line that keeps the driver's contract: the
metric, unit and config of our arm, "impl": "reference", a cpu_baseline and an
e2e entry with no host-device bytes."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _run(*args, env_extra=None):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env.update(env_extra or {})
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                         timeout=300, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-3000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    return lines


@pytest.mark.parametrize("config", [2, 3, 4, 5, 6, 7])
def test_reference_arm_line(config):
    lines = _run("--impl", "reference", "--config", str(config), "--tiny", "--steps", "2", "--warmup", "3",
                 "--ref-seconds", "0.2")
    assert len(lines) == 1
    line = json.loads(lines[0])
    import bench
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert line["scaling"] == bench.SCALING[config]
    assert line["config"]["workload"].startswith(f"config{config}:")
    assert line["config"]["global_batch"] == bench.global_batch(config, 1)
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_describes_our_workload():
    """The reference arm's config entry is the one our arm prints for the same shape."""
    import bench
    lines = _run("--impl", "reference", "--config", "2", "--tiny", "--steps", "2", "--warmup", "3",
                 "--ref-seconds", "0.1")
    line = json.loads(lines[0])
    ours = bench.describe_config2(**{"n_q": 32, "n_kv": 8, "hd": 128, **bench.TINY[2]})
    for k, v in ours.items():
        assert line["config"][k] == v


def test_reference_arm_other_ranks_exit_quietly():
    """Under torchrun only rank 0 runs the CPU reference; the others print nothing and exit 0."""
    lines = _run("--impl", "reference", "--config", "2", "--tiny", "--gpus", "2", "--steps", "2", "--warmup", "3",
                 env_extra={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert lines == []


def test_default_shapes_describe_the_baseline_configs():
    """The untouched default shapes are BASELINE.json's configs 2-5 (the byte and FLOP counts the
    roofline divides by)."""
    import bench
    assert bench.describe_config2(32, 32, 8, 128, 4096)["kv_bytes_per_token"] == 302_063_616
    assert bench.describe_config4(64, 8, 128, 131072)["kv_bytes_per_token"] == 301_989_888
    assert bench.prefill_flops(32, 128, 2048, 2048) == 103_095_992_320
    assert "n=4097" in bench.describe_config2(32, 32, 8, 128, 4096)["workload"]
