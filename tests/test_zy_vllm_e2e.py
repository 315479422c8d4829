"""Real vLLM (offline LLM engine) with TuttiConnectorV1: a prompt's KV persisted by one engine
is found and loaded by a fresh engine; the loaded run generates the same tokens as a full
recompute. Three vLLM processes (engine core in-process), a small random-init Llama, no
tokenizer; each phase is bounded and killed with its session if it overruns."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_vllm_reloads_persisted_prefix_and_matches_recompute(tmp_path):
    pytest.importorskip("vllm")
    env = dict(os.environ, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-m", "tutti_b200.benchmarks.vllm_e2e", "--root", str(tmp_path / "kv"),
                        "--engine-core", "inproc", "--phase-timeout", "420"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=1500)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert lines, r.stdout[-2000:] + r.stderr[-2000:]
    res = json.loads(lines[-1])
    assert res["ok"], res
    assert res["reload_cached_tokens"] == res["expected_cached_tokens"] == 1792
    assert res["first_token_agrees"]
