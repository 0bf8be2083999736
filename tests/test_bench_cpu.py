"""CPU checks of bench.py's driver-facing pieces: the reference arm (the CPU oracle timed on the
host cores) and the algorithmic byte counts behind the roofline figures."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402

CFG_500M = dict(d_model=768, n_layers=16, n_dense=1, n_heads=12, n_kv_heads=3, head_dim=128, dense_ffn=2304,
                expert_ffn=320, n_experts=36, top_k=6, n_shared=1, vocab_size=50304)


def test_bs1_bytes_per_token_match_the_hot_path_figures():
    """500M: 189,609,984 B of Q8 weights a token touches (int8 + one f32 scale per 32) plus the
    1,658,880 B f32 router of the 15 MoE layers; 49,152 B of K + V per context position."""
    assert bench.weight_bytes_per_token(CFG_500M) == 189_609_984 + 1_658_880
    assert bench.kv_bytes_per_pos(CFG_500M) == 49_152


def test_metric_is_the_baseline_metric():
    with open(os.path.join(ROOT, "BASELINE.json")) as f:
        assert json.load(f)["metric"] == bench.METRIC


def _run(args, env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=900)


def test_reference_arm_prints_one_json_line():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "1"], {"RANK": "0", "WORLD_SIZE": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC and d["unit"] == "tok/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["steps"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_output():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "1", "--gpus", "2"], {"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


@pytest.mark.parametrize("n,world", [(256, 1), (256, 2), (256, 8), (5, 3), (0, 2)])
def test_sequence_shards_partition_the_batch(n, world):
    lengths = [(i * 7919) % 1000 + 1 for i in range(n)]
    parts = [bench.shard(lengths, r, world) for r in range(world)]
    assert sorted(i for p in parts for i in p) == list(range(n))
    assert max(map(len, parts)) - min(map(len, parts)) <= 1


def test_diffusion_cpu_sample_reports_the_oracle(model130):
    """bench.py --diffusion's CPU leg: one 32-id block of the oracle's generate_diffusion."""
    from hobbylm_b200 import synth

    base, ids = bench.diffusion_cpu_sample(model130, synth.prompt_ids(16, 6))
    assert base["kind"] == "port" and base["unit"] == "tok/s" and base["value"] > 0 and base["cores"] >= 1
    assert len(ids) == 32 and all(t < bench.VALID for t in ids)
