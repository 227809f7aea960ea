"""CPU tests of bench.py's host side: the algorithmic bytes of a decode step, the clock-record summary
and the reference arm's JSON line (the oracle timed on the host cores), whose keys are the bench
contract."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_step_bytes_llama8b():
    cfg = bench.l8_config()
    d, F, V, B, ctx = 4096, 14336, 128256, 16, 600
    per_layer = d * (32 + 2 * 8) * 128 + 32 * 128 * d + 3 * d * F + 2 * d
    weights = 2 * (32 * per_layer + d + d * V + B * d)
    kv = 32 * B * ctx * 2 * 8 * 128 * 2
    tot, w, k = bench.step_bytes(cfg, B, ctx)
    assert w == weights and k == kv and tot == weights + kv
    # tensor parallelism splits the projections, the LM head and the K / V heads, not the norms or the
    # embedding rows
    tot2, w2, k2 = bench.step_bytes(cfg, B, ctx, tp=2)
    assert w2 == 2 * (32 * (per_layer - 2 * d) / 2 + 32 * 2 * d + d + d * V / 2 + B * d)
    assert k2 == kv / 2


def test_step_bytes_gemma_local_layers_read_their_window():
    cfg = bench.g12_config(num_layers=12)
    B, ctx = 8, 5000
    _, _, kv = bench.step_bytes(cfg, B, ctx, family="gemma3")
    per_key = B * 2 * 8 * 256 * 2
    # layers 6 and 12 (every sliding_window_pattern-th) are global, the other ten read 1024 keys
    assert kv == per_key * (2 * ctx + 10 * 1024)


def test_step_bytes_neox_mlp_has_two_matrices():
    cfg = bench.nx_config()
    d, F = 512, 2048
    _, w, _ = bench.step_bytes(cfg, 1, 32, family="neox", elem=4)
    per_layer = d * 3 * 8 * 64 + 8 * 64 * d + 2 * d * F + 2 * d
    assert w == 4 * (6 * per_layer + d + d * 50304 + d)


def test_clock_summary_parses_reasons():
    s = bench.ClockSampler(0)
    s.lines = [
        "0, 1965, 1965, 700.1, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1950, 1965, 990.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1905, 1965, 1001.2, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "garbage",
    ]
    out = s.summary()
    assert out == {"sm_mhz": 1950.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 3}
    s.lines = []
    assert bench.ClockSampler(0).summary()["samples"] == 0


def _run_bench(args, env_extra=None, timeout=300):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, env=env, cwd=ROOT)


def test_reference_arm_prints_the_contract_line():
    r = _run_bench(["--impl", "reference", "--config", "nx", "--steps", "2", "--warmup", "1"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e", "extrapolated"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["metric"] == bench.metric_of(bench.CONFIGS["nx"])
    assert d["value"] > 0 and d["steps"] == 2 and d["n_gpus"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # one decoder layer of the 6 per sample, scaled by the layer count
    assert d["extrapolated"]["scale"] == 6
    assert abs(d["extrapolated"]["full_step_ms"] - 6 * d["ms_per_step"]) < 1e-6 * d["extrapolated"]["full_step_ms"]
    assert d["config"]["global_batch"] == 1 and d["config"]["seq_len"] == 32


def test_reference_arm_other_ranks_print_nothing():
    r = _run_bench(["--impl", "reference", "--config", "nx", "--steps", "1", "--warmup", "1"], {"RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


@pytest.mark.parametrize("name", sorted(bench.CONFIGS))
def test_configs_name_their_shapes(name):
    conf = bench.CONFIGS[name]
    cfg = conf["make"]()
    assert conf["family"] in ("llama", "neox", "gemma3") and conf["dtype"] in ("bf16", "f32")
    assert cfg.num_heads % cfg.num_key_value_heads == 0
    assert conf["B"] > 0 and conf["P"] > 0 and conf["new"] > 0
