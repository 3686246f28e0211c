"""The synthetic-model generator: deterministic and distributed as the
benchmark description says (N(0, 0.02) bf16 weights, unit norm gains,
uniform MXFP4 codes, e8m0 scale bytes in [119, 127])."""
import ctypes
import json
import os
import struct

import numpy as np

from conftest import model_dir
from strasgpt_b200 import configs, synth


def tensors(d):
    raw = open(os.path.join(d, "model.safetensors"), "rb").read()
    hlen = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + hlen])
    hdr.pop("__metadata__")
    out = {}
    for n, i in hdr.items():
        b, e = i["data_offsets"]
        out[n] = (i["dtype"], np.frombuffer(raw[8 + hlen + b:8 + hlen + e], np.uint8))
    return out, hlen


def bf16(u8):
    return (u8.view(np.uint16).astype(np.uint32) << 16).view(np.float32)


def test_header_is_aligned_and_contiguous():
    d = model_dir(configs.T_MOE)
    t, hlen = tensors(d)
    assert (8 + hlen) % 8 == 0
    total = sum(len(v) for _, v in t.values())
    assert os.path.getsize(os.path.join(d, "model.safetensors")) == 8 + hlen + total


def test_distributions():
    d = model_dir(configs.T_MOE)
    t, _ = tensors(d)
    w = bf16(t["model.embed_tokens.weight"][1])
    assert abs(w.mean()) < 1e-3 and abs(w.std() - 0.02) < 1e-3
    assert (bf16(t["model.norm.weight"][1]) == 1.0).all()
    codes = t["model.layers.0.mlp.experts.gate_proj_blocks"][1]
    lo, hi = np.bincount(codes & 15, minlength=16), np.bincount(codes >> 4, minlength=16)
    assert lo.min() > 0.8 * lo.mean() and hi.min() > 0.8 * hi.mean()
    sc = t["model.layers.0.mlp.experts.gate_proj_scales"][1]
    assert sc.min() == 119 and sc.max() == 127


def test_fill_is_order_independent():
    lib = synth._lib()
    a = np.empty(1001, np.uint16)
    b = np.empty(2000, np.uint16)
    sid = lib.synth_stream_id(b"x")
    lib.synth_normal_bf16(a.ctypes.data_as(ctypes.c_void_p), a.size, 7, sid, 0.02)
    lib.synth_normal_bf16(b.ctypes.data_as(ctypes.c_void_p), b.size, 7, sid, 0.02)
    assert (a[:1000] == b[:1000]).all()
    c = np.empty(1001, np.uint16)
    lib.synth_normal_bf16(c.ctypes.data_as(ctypes.c_void_p), c.size, 8, sid, 0.02)
    assert (a != c).mean() > 0.9


def test_prompt_is_seeded():
    cfg = configs.C1
    p = synth.prompt_tokens(cfg)
    assert p.shape == (8,) and p.min() >= 0 and p.max() < cfg.vocab
    assert (p == synth.prompt_tokens(cfg)).all()
