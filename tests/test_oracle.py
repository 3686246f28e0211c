"""Pinning the oracle (CPU, no GPU).

1. The project's C restatement equals the reference's own forward pass
   (compiled from its sources into oracle/_ref/) on every dense small shape.
2. Both reproduce the committed golden fixtures (which the reference made).
3. The MoE path, which has no reference, equals a float64 numpy restatement
   written independently here.
4. The synthetic generator reproduces the fixtures' exact model bytes.
"""
import json
import os

import numpy as np
import pytest

from conftest import model_dir
from strasgpt_b200 import configs, synth
import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DENSE = sorted(n for n, c in configs.TINY.items() if not c.experts)


def golden(name):
    return (json.load(open(os.path.join(GOLDEN, f"{name}.json"))),
            np.load(os.path.join(GOLDEN, f"{name}.npz")))


@pytest.mark.parametrize("name", sorted(configs.TINY))
def test_generator_reproduces_fixture_model(name):
    import hashlib
    meta, _ = golden(name)
    d = model_dir(configs.get(name))
    h = hashlib.sha256(open(os.path.join(d, "model.safetensors"), "rb").read())
    assert h.hexdigest() == meta["model_sha256"]


@pytest.mark.parametrize("name", DENSE)
def test_restatement_equals_reference(name):
    if not oracle.reference_available():
        pytest.skip("reference build not present")
    cfg = configs.get(name)
    d = model_dir(cfg)
    p = synth.prompt_tokens(cfg)
    t1, l1 = oracle.Restatement(d).generate_greedy(p, cfg.steps)
    t2, l2 = oracle.Reference(d).generate_greedy(p, cfg.steps)
    assert (t1 == t2).all()
    assert np.abs(l1 - l2).max() <= 1e-5


@pytest.mark.parametrize("name", sorted(configs.TINY))
def test_checkers_reproduce_golden(name):
    cfg = configs.get(name)
    meta, g = golden(name)
    d = model_dir(cfg)
    checkers = [oracle.Restatement]
    if not cfg.experts and oracle.reference_available():
        checkers.append(oracle.Reference)
    for C in checkers:
        toks, logits = C(d).generate_greedy(np.array(meta["prompt"], np.int32), cfg.steps)
        assert list(toks) == meta["tokens"], C.__name__
        assert np.abs(logits - g["logits"]).max() <= 1e-5, C.__name__


def _moe_numpy(cfg, d, prompt, steps):
    """Independent float64 restatement of the MoE model (greedy)."""
    import struct
    raw = open(os.path.join(d, "model.safetensors"), "rb").read()
    hlen = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + hlen])
    base = 8 + hlen

    def T(name):
        i = hdr[name]
        b, e = i["data_offsets"]
        buf = np.frombuffer(raw[base + b:base + e], dtype=np.uint8)
        if i["dtype"] == "BF16":
            u = buf.view(np.uint16).astype(np.uint32) << 16
            return u.view(np.float32).astype(np.float64).reshape(i["shape"])
        return buf.reshape(i["shape"])

    e2m1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0., -.5, -1, -1.5, -2, -3, -4, -6])

    def mx(codes, scales):  # [E][R][K/32][16], [E][R][K/32] -> [E][R][K]
        lo = e2m1[codes & 15]
        hi = e2m1[codes >> 4]
        v = np.stack([lo, hi], axis=-1).reshape(*codes.shape[:-1], 32)
        v = v * np.ldexp(1.0, scales.astype(np.int64) - 127)[..., None]
        return v.reshape(*codes.shape[:-2], -1)

    D, HD, QH, KH, L = cfg.dim, cfg.head_dim, cfg.q_heads, cfg.kv_heads, cfg.layers
    G = QH // KH
    emb, out = T("model.embed_tokens.weight"), T("lm_head.weight")
    def rms(x, w): return x / np.sqrt((x * x).mean(-1, keepdims=True) + cfg.eps) * w
    inv = 1.0 / cfg.rope_theta ** (np.arange(0, HD // 2) * 2.0 / HD)
    def rope(v, pos):
        a = pos * inv
        c, s = np.cos(a), np.sin(a)
        v0, v1 = v[..., :HD // 2], v[..., HD // 2:]
        return np.concatenate([v0 * c - v1 * s, v0 * s + v1 * c], -1)
    layers = []
    for l in range(L):
        p = f"model.layers.{l}."
        layers.append({k: T(p + n) for k, n in [
            ("an", "input_layernorm.weight"), ("q", "self_attn.q_proj.weight"),
            ("k", "self_attn.k_proj.weight"), ("v", "self_attn.v_proj.weight"),
            ("o", "self_attn.o_proj.weight"), ("fn", "post_attention_layernorm.weight"),
            ("r", "mlp.router.weight")]})
        for proj in ("gate_proj", "up_proj", "down_proj"):
            layers[-1][proj] = mx(T(p + f"mlp.experts.{proj}_blocks"),
                                  T(p + f"mlp.experts.{proj}_scales"))
    kc = [np.zeros((0, KH, HD)) for _ in range(L)]
    vc = [np.zeros((0, KH, HD)) for _ in range(L)]
    def step(tok, pos):
        x = emb[tok].copy()
        for l, y in enumerate(layers):
            h = rms(x, y["an"])
            q = (y["q"] @ h).reshape(QH, HD)
            k = (y["k"] @ h).reshape(KH, HD)
            v = (y["v"] @ h).reshape(KH, HD)
            q, k = rope(q, pos), rope(k, pos)
            kc[l] = np.concatenate([kc[l], k[None]])
            vc[l] = np.concatenate([vc[l], v[None]])
            att = np.zeros((QH, HD))
            for hh in range(QH):
                s = kc[l][:, hh // G] @ q[hh] / np.sqrt(HD)
                pr = np.exp(s - s.max())
                pr /= pr.sum()
                att[hh] = pr @ vc[l][:, hh // G]
            x = x + y["o"] @ att.ravel()
            h = rms(x, y["fn"])
            r = y["r"] @ h
            sel = sorted(range(cfg.experts), key=lambda e: (-r[e], e))[:cfg.top_k]
            w = np.exp(r[sel] - r[sel].max())
            w /= w.sum()
            acc = np.zeros(D)
            for wj, e in zip(w, sel):
                g = y["gate_proj"][e] @ h
                u = y["up_proj"][e] @ h
                acc += wj * (y["down_proj"][e] @ (g / (1 + np.exp(-g)) * u))
            x = x + acc
        return out @ rms(x, T("model.norm.weight"))
    logits = [None]
    for i, t in enumerate(prompt):
        logits[0] = step(int(t), i)
    toks = [int(np.argmax(logits[0]))]
    for s in range(steps):
        logits.append(step(toks[-1], len(prompt) + s))
        toks.append(int(np.argmax(logits[-1])))
    return np.array(toks), np.stack(logits)


def test_moe_restatement_equals_float64_numpy():
    cfg = configs.T_MOE
    d = model_dir(cfg)
    p = synth.prompt_tokens(cfg)
    t_np, l_np = _moe_numpy(cfg, d, p, cfg.steps)
    t_c, l_c = oracle.Restatement(d).generate_greedy(p, cfg.steps)
    assert (t_np == t_c).all()
    assert np.abs(l_np - l_c).max() <= 1e-4
