"""bench.py's reference arm (`--impl reference`) on the CPU, with the one-block timing replaced by a
fixed figure: the line carries the GPU arm's config, declares its extrapolation, reports the timed
sample as ms_per_step and stays silent on ranks other than 0."""
import types

import bench


def test_reference_arm_line(monkeypatch):
    monkeypatch.setattr(bench, "cpu_block_seconds", lambda reps=1: 0.5)
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    args = types.SimpleNamespace(warmup=3, steps=2, gpus=1, batch=1)
    out = bench.run_reference(args)
    assert out["impl"] == "reference"
    assert out["config"] == bench.cfg2_config(1, 1)          # the GPU arm's config, key for key
    assert out["metric"] == bench.METRIC and out["unit"] == "images/s" and out["higher_is_better"] is True
    assert out["steps"] == 2 and out["warmup"] == 3
    assert out["ms_per_step"] == 500.0                       # one timed block a step
    assert out["timed_s"] == 1.0
    assert out["extrapolated"] is True and out["timed_unit"] == "one DiT block"
    picture_s = bench.cpu_picture_seconds(0.5)
    assert abs(out["ms_per_picture_estimate"] - picture_s * 1e3) < 0.1
    assert abs(out["value"] - 1.0 / picture_s) < 1e-6
    assert out["e2e"] == {"value": out["value"], "unit": "images/s", "h2d_bytes_per_step": 0,
                          "d2h_bytes_per_step": 0}
    assert out["cpu_baseline"]["kind"] == "port" and out["cpu_baseline"]["value"] == out["value"]


def test_reference_arm_other_ranks_print_nothing(monkeypatch):
    monkeypatch.setattr(bench, "cpu_block_seconds", lambda reps=1: 0.5)
    monkeypatch.setenv("RANK", "1")
    monkeypatch.setenv("WORLD_SIZE", "2")
    assert bench.run_reference(types.SimpleNamespace(warmup=3, steps=1, gpus=2, batch=1)) is None


def test_picture_estimate_counts_every_block_pass():
    # 8 steps x 32 blocks, the first step's blocks over 128 more rows than the 4096 image rows
    assert abs(bench.cpu_picture_seconds(1.0) - 32 * (7 + 4224 / 4096)) < 1e-9
