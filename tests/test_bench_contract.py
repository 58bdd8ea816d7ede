"""CPU check of the benchmark's reference arm: `bench.py --impl reference` runs
the eager QLoRA step on the host cores (no GPU) and prints one JSON line with
the keys the harness reads, the metric and unit of the B200 arm, and a
cpu_baseline / e2e block; plus the FLOP-per-token formula it normalises by."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.strip().splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "QLoRA train tokens/s" and d["unit"] == "tokens/s"
    assert d["config"]["same_config"] is False
    assert d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["steps"] == 1 and d["warmup"] == 1
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["dtype"] == "bf16" and d["data"].startswith("synthetic")
    assert "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_flop_per_token_formula():
    """4 x (base + head params) + 3 x causal attention + 6 r (in + out) per LoRA projection."""
    from oracle.qlora_step import train_flop_per_token

    base = 1536 * (1536 + 256 + 256 + 1536) + 3 * 1536 * 8960
    lora = 16 * ((1536 + 1536) * 2 + (1536 + 256) * 2 + 3 * (1536 + 8960))
    attn = 4.0 * 12 * 128 * (2048 + 1) / 2
    expect = 28 * (4 * base + 3 * attn + 6 * lora) + 4 * 151936 * 1536
    assert abs(train_flop_per_token(2048) - expect) < 1.0
    assert 6.7e9 < train_flop_per_token(2048) < 6.9e9
