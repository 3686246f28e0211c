"""Full-size parity on the benchmark configurations (C1-C4, and C5's
width and 8192-token prompt on 4 layers) against the committed outputs of
the reference's own forward pass (C4: this project's restatement, the
reference has no MoE), made by tests/golden/make_golden.py.

Per configuration: the synthetic model is rebuilt on the GPU box and
pinned by its sha256; the greedy ids of transformer_generate_greedy must
equal the reference's bit for bit; for every step of the predict path
(host logits, as strasgpt.c reads them) the logits of the reference's
top-16 ids, the maximum, mean and standard deviation must be within the
north-star max-abs bound 1e-2, and the dot products with 4 fixed random
unit vectors within 1e-2 * sqrt(V) (what a max-abs error of 1e-2 allows);
and on the committed full-vocabulary rows (the prefill row and 8 decode
steps) the whole logits vector must be within max-abs 1e-2 and cosine
0.9999 of the reference's.

MoE (C4): a top-k router choice whose k-th and (k+1)-th router logits lie
within ROUTER_TIE of each other depends on the fp32 summation order (the
two implementations agree to ~1e-6 on router logits), so a step whose
smallest router margin (recorded by the restatement, `router_gap`) is
below ROUTER_TIE is numerically undecidable: its logits are not compared,
and the greedy ids are compared up to that step (later ids follow from a
different token). In the committed C4 fixture this is step 57 (margin
3.1e-5), where the GPU indeed picks another expert."""
import hashlib
import json
import os

import numpy as np
import pytest

from conftest import model_dir
from strasgpt_b200 import configs, synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
MAX_ABS = 1e-2
MIN_COS = 0.9999
ROUTER_TIE = 1e-4
NAMES = [n for n in ("c1_llama1b", "c2_qwen3_0p6b", "c4_moe_mxfp4", "c3_llama8b",
                     "c5_mistral24b_l4")
         if os.path.exists(os.path.join(GOLDEN, f"{n}.json"))]


def projection_vectors(vocab: int) -> np.ndarray:
    """The 4 unit vectors of tests/golden/make_golden.py."""
    rng = np.random.default_rng(12345)
    v = rng.standard_normal((4, vocab))
    return v / np.linalg.norm(v, axis=1, keepdims=True)


def cosine(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def _sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(1 << 24)
            if not b:
                return h.hexdigest()
            h.update(b)


@pytest.mark.gpu
@pytest.mark.parametrize("name", NAMES)
def test_full_size_matches_reference(cuda, name):
    from strasgpt_b200 import Transformer
    cfg = configs.get(name)
    meta = json.load(open(os.path.join(GOLDEN, f"{name}.json")))
    d = model_dir(cfg)
    assert _sha256(os.path.join(d, "model.safetensors")) == meta["model_sha256"]
    prompt = synth.prompt_tokens(cfg)
    assert [int(x) for x in prompt] == meta["prompt"]
    # Decode steps only: the prompt's margin is the minimum over all of its
    # tokens, where a flipped choice moves one cache row, not the output.
    ties = [s for s, st in enumerate(meta["steps"])
            if s > 0 and st.get("router_gap", 1.0) < ROUTER_TIE]
    upto = ties[0] if ties else len(meta["tokens"])
    m = Transformer(d)
    toks, _ = m.generate_greedy(prompt, cfg.steps)
    assert [int(t) for t in toks][:upto] == meta["tokens"][:upto], f"{name}: greedy ids differ"
    m.reset()
    full = np.load(os.path.join(GOLDEN, f"{name}_logits.npz"))
    full_rows = {int(st): row for st, row in zip(full["steps"], full["logits"])}
    proj = projection_vectors(cfg.vocab)
    proj_bound = MAX_ABS * np.sqrt(cfg.vocab)
    logits = m.predict(prompt, 1)[0]
    worst = 0.0
    checked_full = 0
    for s, want in enumerate(meta["steps"]):
        if s > 0:
            logits = m.predict([meta["tokens"][s - 1]], 1)[0]
        if s in ties:
            continue
        got = logits.astype(np.float64)
        ids = want["top_ids"]
        errs = [abs(got[i] - v) for i, v in zip(ids, want["top_vals"])]
        errs += [abs(got.max() - want["max"]), abs(got.mean() - want["mean"]),
                 abs(got.std() - want["std"])]
        worst = max(worst, max(errs))
        assert max(errs) <= MAX_ABS, f"{name} step {s}: logit error {max(errs):.3e}"
        perr = np.abs(proj @ got - np.asarray(want["proj"])).max()
        assert perr <= proj_bound, f"{name} step {s}: projection error {perr:.3e}"
        assert int(np.argmax(got)) == meta["tokens"][s], f"{name} step {s}: argmax"
        if s in full_rows:
            ref = full_rows[s].astype(np.float64)
            err = float(np.abs(got - ref).max())
            cos = cosine(got, ref)
            assert err <= MAX_ABS, f"{name} step {s}: full-vocabulary max-abs {err:.3e}"
            assert cos >= MIN_COS, f"{name} step {s}: cosine {cos:.8f}"
            checked_full += 1
    assert checked_full >= len(full_rows) - len(ties)
    m.free()
