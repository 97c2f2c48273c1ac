"""The bench's output contract, on CPU: the reference arm prints one JSON
line with the metric, config and baseline keys the GPU arm uses; under a
multi-rank launch only rank 0 works and prints; and the GPU arm without a GPU
fails with a non-zero status instead of printing a number."""
import json
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench(*args, **env):
    e = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    e.update(env)
    return subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, env=e,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    r = _bench("--impl", "reference", "--steps", "3", "--warmup", "3")
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "I2_S matvec HBM GB/s" and d["unit"] == "GB/s"
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["ms_per_step"] > 0 and d["higher_is_better"] is True
    assert d["scaling"] == "weak" and d["vs_baseline"] is None
    assert d["config"]["workload"] == "bitnet2b_decode_bitlinear_sweep"
    assert not {"model", "global_batch", "seq_len"} & set(d["config"])
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_0_only():
    r = _bench("--impl", "reference", "--steps", "3", "--warmup", "3",
               RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


def test_gpu_arm_without_gpu_is_an_error():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the no-GPU failure cannot be observed here")
    r = _bench("--steps", "3", "--warmup", "3")
    assert r.returncode != 0
    assert any(w in r.stderr for w in ("NVIDIA", "CUDA", "cuda", "device")), r.stderr[-2000:]
    assert not any(ln.lstrip().startswith("{") for ln in r.stdout.splitlines()), r.stdout
