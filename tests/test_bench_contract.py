"""bench.py's JSON contract on the CPU: the reference arm's line (the oracle
port timed on host cores) carries every key the driver reads, the metric is
BASELINE.json's, engine-level scenarios print an `unavailable` line for the
reference arm, and the B200 arm fails loudly without a GPU."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def run(*args, timeout=300):
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=timeout, cwd=ROOT)


def last_json(out: str) -> dict:
    return json.loads(out.strip().splitlines()[-1])


def test_reference_arm_line_has_the_contract_keys():
    p = run("--impl", "reference", "--workload", "gpt2", "--steps", "2", "--warmup", "1")
    assert p.returncode == 0, p.stderr
    line = last_json(p.stdout)
    baseline = json.loads((ROOT / "BASELINE.json").read_text())
    assert line["impl"] == "reference" and line["metric"] == baseline["metric"]
    assert line["value"] > 0 and line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 2, 1)
    assert line["ms_per_step"] > 0 and line["scaling"] == "weak" and line["vs_baseline"] is None
    assert line["dtype"] == "u8" and "synthetic" in line["data"]
    assert line["config"]["workload"] == "gpt2"
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == "GB/s"
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


@pytest.mark.parametrize("workload", ["qwen3_pd", "llama8b_fp8_evict", "llama8b_duplex", "llama70b_tp_one_engine",
                                      "server_e2e"])
def test_engine_scenarios_report_the_reference_arm_unavailable(workload):
    p = run("--impl", "reference", "--workload", workload)
    assert p.returncode == 0, p.stderr
    line = last_json(p.stdout)
    assert line["impl"] == "reference" and line["unavailable"]


def test_b200_arm_fails_loudly_without_a_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = run("--steps", "1", "--warmup", "0", "--no-cpu", "--no-refcopy")
    assert p.returncode != 0
    assert not p.stdout.strip()  # no JSON line from a run that did not happen


def test_reference_arm_covers_every_tp_shard_of_the_default_workload():
    """The default workload is configs[3] at TP=N; the reference arm times the
    whole job on the host cores (all N head shards), like the b200 arm's value."""
    p = run("--impl", "reference", "--gpus", "2", "--steps", "2", "--warmup", "1", "--layers", "2")
    assert p.returncode == 0, p.stderr
    line = last_json(p.stdout)
    assert line["config"]["workload"] == "llama70b_tp"
    assert line["config"]["tp"] == 2 and line["config"]["heads_per_rank"] == 4
    assert line["n_gpus"] == 2 and line["value"] > 0
    assert line["cpu_baseline"]["sample"].startswith("2 TP shards x 2 of 2 layers x 2048 blocks")
