"""The committed full-vocabulary logits rows (tests/golden/c*_logits.npz)
agree with the per-step summaries written beside them from the same
reference run (top id, maximum, mean, projections): a CPU check that the
two files of a configuration belong together."""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NAMES = sorted(n[:-len("_logits.npz")] for n in os.listdir(GOLDEN) if n.endswith("_logits.npz"))


def projection_vectors(vocab: int) -> np.ndarray:
    rng = np.random.default_rng(12345)
    v = rng.standard_normal((4, vocab))
    return v / np.linalg.norm(v, axis=1, keepdims=True)


@pytest.mark.parametrize("name", NAMES)
def test_full_rows_match_summaries(name):
    meta = json.load(open(os.path.join(GOLDEN, f"{name}.json")))
    full = np.load(os.path.join(GOLDEN, f"{name}_logits.npz"))
    steps, rows = full["steps"], full["logits"]
    assert list(steps) == meta["full_rows"]
    assert steps[0] == 0 and steps[-1] == len(meta["steps"]) - 1
    proj = projection_vectors(rows.shape[1])
    for s, row in zip(steps, rows):
        want = meta["steps"][int(s)]
        r = row.astype(np.float64)
        assert int(np.argmax(r)) == want["top_ids"][0] == meta["tokens"][int(s)]
        assert r.max() == pytest.approx(want["max"], abs=1e-6)
        assert r.mean() == pytest.approx(want["mean"], abs=1e-6)
        np.testing.assert_allclose(proj @ r, want["proj"], atol=1e-5)
