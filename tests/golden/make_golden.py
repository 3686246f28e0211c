"""Generate the committed golden fixtures of tests/golden/.

For every configuration this writes the synthetic model (strasgpt_b200.synth,
seed 0), runs the CPU checker and stores what the GPU parity tests compare
against:
  - the sha256 of model.safetensors (pins the synthetic generator, so the
    GPU box rebuilds bit-identical weights),
  - the prompt ids, the greedy ids (prefill + S steps),
  - small shapes (`t_*`): every step's full fp32 logits (<name>.npz);
  - benchmark shapes (`c*`): per step the top-16 (id, logit), the logit
    mean/std/max, the top-1 minus top-2 margin, and the dot of the logits
    with 4 fixed random unit vectors (<name>.json); plus the full fp32
    logits of the prefill row and of FULL_ROWS evenly spaced decode steps
    (<name>_logits.npz: `steps`, `logits` [n][V]), for the full-vocabulary
    max-abs and cosine checks.
Checker: the reference's own forward pass compiled from its sources
(oracle.Reference) for dense models; this project's restatement
(oracle.Restatement) for the MoE models the reference does not have.

Run: python tests/golden/make_golden.py [names...]  (default: all t_* shapes)
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from strasgpt_b200 import configs, synth  # noqa: E402
import oracle  # noqa: E402

CACHE = os.environ.get("STRASGPT_MODEL_CACHE", "/tmp/strasgpt_models")
PROJECTIONS = 4
FULL_ROWS = 8


def file_sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(1 << 24)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def projection_vectors(vocab: int) -> np.ndarray:
    rng = np.random.default_rng(12345)
    v = rng.standard_normal((PROJECTIONS, vocab))
    return (v / np.linalg.norm(v, axis=1, keepdims=True)).astype(np.float64)


def step_summary(logits: np.ndarray, proj: np.ndarray) -> dict:
    top = np.argsort(-logits, kind="stable")[:16]
    s = np.sort(logits)[::-1]
    return {
        "top_ids": [int(i) for i in top],
        "top_vals": [float(logits[i]) for i in top],
        "mean": float(logits.mean(dtype=np.float64)),
        "std": float(logits.std(dtype=np.float64)),
        "max": float(s[0]),
        "margin": float(s[0] - s[1]),
        "proj": [float(x) for x in proj @ logits.astype(np.float64)],
    }


def full_rows(steps: int) -> list:
    """Step 0 (the prefill row) and FULL_ROWS decode steps spread evenly
    over 1..steps."""
    picks = np.linspace(1, steps, min(FULL_ROWS, steps)).round().astype(int)
    return [0] + sorted({int(s) for s in picks})


def make(name: str) -> None:
    cfg = configs.get(name)
    d = synth.write_model(os.path.join(CACHE, f"{cfg.name}_s0"), cfg, seed=0)
    prompt = synth.prompt_tokens(cfg, seed=0)
    checker = oracle.Restatement if cfg.experts else oracle.Reference
    t0 = time.time()
    m = checker(d)
    gaps = [] if cfg.experts else None
    if cfg.experts:
        toks, logits = m.generate_greedy(prompt, cfg.steps, gaps=gaps)
    else:
        toks, logits = m.generate_greedy(prompt, cfg.steps)
    dt = time.time() - t0
    sha = file_sha256(os.path.join(d, "model.safetensors"))
    meta = {"config": name, "seed": 0, "checker": checker.__name__,
            "model_sha256": sha, "prompt": [int(x) for x in prompt],
            "tokens": [int(x) for x in toks], "seconds": round(dt, 1),
            "threads": os.cpu_count()}
    if name.startswith("t_"):
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), logits=logits,
                            prompt=prompt, tokens=toks)
        with open(os.path.join(HERE, f"{name}.json"), "w") as f:
            json.dump(meta, f, indent=1)
    else:
        proj = projection_vectors(cfg.vocab)
        meta["steps"] = [step_summary(l, proj) for l in logits]
        rows = full_rows(cfg.steps)
        meta["full_rows"] = rows
        np.savez_compressed(os.path.join(HERE, f"{name}_logits.npz"),
                            steps=np.array(rows, dtype=np.int32),
                            logits=np.stack([logits[s] for s in rows]).astype(np.float32))
        if gaps is not None:
            # Smallest top-k router margin over the layers (and, for the
            # prompt, its tokens) of each step.
            for st, g in zip(meta["steps"], gaps):
                st["router_gap"] = g
        with open(os.path.join(HERE, f"{name}.json"), "w") as f:
            json.dump(meta, f)
    print(f"{name}: {checker.__name__} {dt:.1f}s tokens {toks[:8]}...", flush=True)
    m.free()


if __name__ == "__main__":
    names = sys.argv[1:] or sorted(configs.TINY)
    for n in names:
        make(n)
