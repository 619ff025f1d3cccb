"""bench.py's reference arm (the CPU restatement timed on the host cores) and
its output contract, on the CPU: one JSON line with the driver's keys, the
reference arm's cpu_baseline and e2e blocks.  Our arm needs a GPU: without one
it must fail loudly (no CPU fallback)."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, timeout):
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), *args],
                          capture_output=True, text=True, timeout=timeout, cwd=REPO)


def test_reference_arm_prints_contract_line():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"], timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "weights/s"
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["h2d_bytes_per_step"] == 0


def test_our_arm_needs_the_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: the GPU tests and the bench cover this arm")
    r = _run(["--steps", "1", "--warmup", "0", "--no-e2e", "--no-cpu-baseline"], timeout=300)
    assert r.returncode != 0
    assert not r.stdout.strip() or "value" not in r.stdout.strip().splitlines()[-1]
