"""vLLM end to end: persist a long prompt's KV through TuttiConnectorV1, reload it in a new engine.

    python -m tutti_b200.benchmarks.vllm_e2e [--model DIR] [--prompt-tokens 2048] [--engine-core inproc|mp]

Three fresh vLLM processes share one store (vLLM's own prefix cache is off); the
connector is named by the same module path and store schema as a Tutti
deployment (``tutti.integration.vllm.connector``, ``store.type: tutti_nvme``):
  1. ``store``: the prompt is prefilled and its full chunks are saved;
  2. ``reload``: the scheduler's cold start finds the chunks, the worker loads
     them layer by layer, and only the tail is computed
     (``num_cached_tokens`` counts the loaded tokens);
  3. ``recompute``: the same prompt without the connector, as a reference.
Without ``--model`` a small random-init Llama is written to a temporary
directory (no tokenizer: prompts are token ids). Prints one JSON line.

``--engine-core``: ``inproc`` (default) runs vLLM's engine core, and with it
the connector's scheduler and worker sides, in the phase's own process
(``VLLM_ENABLE_V1_MULTIPROCESSING=0``); ``mp`` is vLLM's multiprocess engine
core (a forked child). Each phase runs in a session of its own with its
output in files: after the phase exits, whatever it left running is killed
with the session, and a phase that overruns ``--phase-timeout`` first gets
SIGUSR1 (every process of the phase dumps its Python stacks, which are
reported) and is then killed.
"""
from __future__ import annotations

import argparse
import json
import faulthandler
import os
import signal
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def make_tiny_llama(path: str, seed: int = 0) -> None:
    import torch
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=4,
                      num_attention_heads=8, num_key_value_heads=4, head_dim=64, max_position_embeddings=8192,
                      initializer_range=0.1, torch_dtype="bfloat16", tie_word_embeddings=False)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16)
    model.save_pretrained(path, safe_serialization=True)


def run_phase(args) -> dict:
    # the engine core child (mp) inherits this handler: SIGUSR1 dumps every thread's stack
    faulthandler.register(signal.SIGUSR1, all_threads=True)
    from vllm import LLM, SamplingParams
    from vllm.config import KVTransferConfig
    from vllm.inputs import TokensPrompt

    kw = dict(model=args.model, dtype="bfloat16", enforce_eager=True, gpu_memory_utilization=args.gpu_mem,
              max_model_len=args.prompt_tokens + 64, enable_prefix_caching=False, skip_tokenizer_init=True,
              block_size=16)
    if args.phase != "recompute":
        # configured exactly as a Tutti deployment is (module path and store schema)
        kw["kv_transfer_config"] = KVTransferConfig(
            kv_connector="TuttiConnectorV1", kv_connector_module_path="tutti.integration.vllm.connector",
            kv_role="kv_both",
            kv_connector_extra_config={"chunk_tokens": 256, "store": {"type": "tutti_nvme", "options": {
                "root": args.root, "capacity_chunks": 256, "segment_file_slots": 32}}})
    llm = LLM(**kw)
    import numpy as np

    ids = np.random.default_rng(1).integers(0, 2048, args.prompt_tokens).tolist()
    sp = SamplingParams(temperature=0.0, max_tokens=16)
    t0 = time.perf_counter()
    out = llm.generate([TokensPrompt(prompt_token_ids=ids)], sp, use_tqdm=False)[0]
    wall = time.perf_counter() - t0
    return {"phase": args.phase, "tokens": list(out.outputs[0].token_ids),
            "num_cached_tokens": int(getattr(out, "num_cached_tokens", 0) or 0), "wall_s": round(wall, 3)}


def _run_phase_process(cmd, env, timeout_s: float, log_dir: str, phase: str) -> tuple[int | None, str, str]:
    """Run one phase in its own session, output in files; returns (rc or None on timeout, stdout, stderr)."""
    out_path = os.path.join(log_dir, f"{phase}.out")
    err_path = os.path.join(log_dir, f"{phase}.err")
    with open(out_path, "w") as out, open(err_path, "w") as err:
        proc = subprocess.Popen(cmd, cwd=ROOT, env=env, stdout=out, stderr=err, start_new_session=True)
        try:
            rc = proc.wait(timeout=timeout_s)
        except subprocess.TimeoutExpired:
            rc = None
            try:
                os.killpg(proc.pid, signal.SIGUSR1)  # stacks of every process of the phase
                time.sleep(5)
            except ProcessLookupError:
                pass
        try:
            os.killpg(proc.pid, signal.SIGKILL)  # the phase's session: its leader and anything it left
        except ProcessLookupError:
            pass
        proc.wait()
    with open(out_path) as f:
        stdout = f.read()
    with open(err_path) as f:
        stderr = f.read()
    return rc, stdout, stderr


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--model", default="")
    p.add_argument("--prompt-tokens", type=int, default=2048)
    p.add_argument("--root", default="")
    p.add_argument("--gpu-mem", type=float, default=0.15)
    p.add_argument("--phase", default="", choices=["", "store", "reload", "recompute"])
    p.add_argument("--engine-core", default="inproc", choices=["inproc", "mp"])
    p.add_argument("--phase-timeout", type=float, default=600.0, help="seconds per phase")
    p.add_argument("--phases", default="store,reload,recompute",
                   help="phases to run (store,reload: persist and reload without the recompute reference)")
    args = p.parse_args(argv)
    if args.phase:
        print("RESULT " + json.dumps(run_phase(args)), flush=True)
        return 0
    work = tempfile.mkdtemp(prefix="tutti_vllm_")
    model = args.model or os.path.join(work, "tiny-llama")
    if not args.model:
        make_tiny_llama(model)
    root = args.root or os.path.join(work, "kv")
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    env["VLLM_ENABLE_V1_MULTIPROCESSING"] = "1" if args.engine_core == "mp" else "0"
    phases = [x for x in args.phases.split(",") if x]
    if not {"store", "reload"} <= set(phases) or not set(phases) <= {"store", "reload", "recompute"}:
        raise SystemExit("--phases must include store and reload (and may add recompute)")
    res = {}
    for phase in ("store", "reload", "recompute"):
        if phase not in phases:
            continue
        cmd = [sys.executable, "-m", "tutti_b200.benchmarks.vllm_e2e", "--phase", phase, "--model", model,
               "--root", root, "--prompt-tokens", str(args.prompt_tokens), "--gpu-mem", str(args.gpu_mem)]
        t0 = time.perf_counter()
        rc, stdout, stderr = _run_phase_process(cmd, env, args.phase_timeout, work, phase)
        line = [ln for ln in stdout.splitlines() if ln.startswith("RESULT ")]
        if rc is None or rc or not line:
            why = f"timed out after {args.phase_timeout:.0f} s" if rc is None else f"exit code {rc}"
            print(json.dumps({"bench": "vllm_e2e", "ok": False, "phase": phase, "engine_core": args.engine_core,
                              "why": why, "result_printed": bool(line),
                              "elapsed_s": round(time.perf_counter() - t0, 1),
                              "tail": (stdout[-1500:] + stderr[-6000:])}))
            return 1
        res[phase] = json.loads(line[-1][7:])
    expect = (args.prompt_tokens - 1) // 256 * 256
    ref = res.get("recompute", {}).get("tokens")
    agree = sum(a == b for a, b in zip(res["reload"]["tokens"], ref)) if ref is not None else None
    out = {"bench": "vllm_e2e", "prompt_tokens": args.prompt_tokens, "engine_core": args.engine_core,
           "reload_cached_tokens": res["reload"]["num_cached_tokens"], "expected_cached_tokens": expect,
           "store_cached_tokens": res["store"]["num_cached_tokens"],
           "tokens_agree_with_recompute": None if ref is None else f"{agree}/{len(ref)}",
           "first_token_agrees": None if ref is None else res["reload"]["tokens"][:1] == ref[:1],
           "wall_s": {k: v["wall_s"] for k, v in res.items()},
           "ok": res["reload"]["num_cached_tokens"] == expect and res["store"]["num_cached_tokens"] == 0}
    print(json.dumps(out))
    return 0 if out["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
