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


def test_both_arms_draw_the_same_inputs():
    """The reference arm draws its inputs with the reference's own normal_sample (oracle/_ref,
    sequential, state jumped in Python), our arm with tqk_fill_normal: the same floats for the
    same windows of the stream, and the same uniforms (config 3's lengths and outlier picks)."""
    import numpy as np
    import bench
    ref, lib = bench.reference_generator(), bench.LibGen()
    if not isinstance(ref, bench.RefGen):
        pytest.skip("oracle/_ref/libtqref_rng.so not built (needs the reference tree at build time)")
    for first, n in ((0, 1000), (123_456_789, 513), (2 * 8 * 4097 * 128 * 32, 4096)):
        assert np.array_equal(ref.normal(first, n).view(np.uint32), lib.normal(first, n).view(np.uint32))
        assert np.array_equal(ref.uniform(first, n).view(np.uint32), lib.uniform(first, n).view(np.uint32))
    assert np.array_equal(bench.ragged_lengths(ref, 64, 512, 8192), bench.ragged_lengths(lib, 64, 512, 8192))


def test_config_streams_tile_without_overlap():
    """Every config's input windows are disjoint and leave no gap: each input is its own part of
    the stream, and a rank's share of a partitioned config is the same floats as at N = 1."""
    import numpy as np
    import bench

    def check(windows):
        windows = sorted(windows)
        for (a0, n0), (a1, _) in zip(windows, windows[1:]):
            assert a0 + n0 == a1, (a0, n0, a1)
        assert windows[0][0] == 0

    L, nq, nkv, hd, mt = 3, 8, 4, 64, 37
    o = bench.config2_stream(L, nq, nkv, hd, mt)
    w = [(o["kv"](l, p, h), mt * hd) for l in range(L) for p in (0, 1) for h in range(nkv)]
    w += [(o["step"] + l * (nq + 2 * nkv) * hd, (nq + 2 * nkv) * hd) for l in range(L)]
    w += [(o["norms"], 2 * L * hd)]
    check(w)
    n = 50
    check([(bench.config4_stream(nkv, n, hd, p, h), n * hd) for p in (0, 1) for h in range(nkv)] +
          [(bench.config4_stream(nkv, n, hd, 2, 0), 16 * hd)])
    lens = np.array([5, 9, 1], np.int32)
    o = bench.config3_stream(lens, nq, nkv, hd)
    w = [(o["kv"](b, p), nkv * int(lens[b]) * hd) for b in range(3) for p in (0, 1)]
    w += [(o["q"](b), nq * hd) for b in range(3)]
    check(w)
    pos0, nn = 6, 4
    o = bench.config5_stream(nq, nkv, hd, pos0, nn)
    check([(o["kv"](p, h), pos0 * hd) for p in (0, 1) for h in range(nkv)] +
          [(o["q"], nn * nq * hd), (o["k"], nn * nkv * hd), (o["v"], nn * nkv * hd)])
    hidden = 96
    o = bench.config6_stream(L, nkv, hd, mt, hidden)
    check([(o["kv"](l, p, h), mt * hd) for l in range(L) for p in (0, 1) for h in range(nkv)] +
          [(o["x"], hidden), (o["norms"], 2 * L * hd)])
    o = bench.config7_stream(L, nkv, hd, mt, hidden)
    check([(o["kv"](l, p, h), mt * hd) for l in range(L) for p in (0, 1) for h in range(nkv)] +
          [(o["norms"](l), 2 * hidden + 2 * hd) for l in range(L)] + [(o["final_norm"], hidden)])
