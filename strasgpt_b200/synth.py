"""Write a synthetic, random-init model directory for a ModelConfig.

The directory holds what the reference's loader reads: config.json,
model.safetensors (tensors in sorted-name order, contiguous, header padded
to 8 bytes) and a synthetic tokenizer.json (byte-level vocabulary) so that
the stock strasgpt.c driver can start on it. Tensor values come from the
counter-based generator in csrc/synth/synth.c, so they are identical on
every machine for the same (config, seed).
"""
from __future__ import annotations

import ctypes
import json
import os
import struct

import numpy as np

from . import _paths
from .configs import ModelConfig

_synth = None


def _lib():
    global _synth
    if _synth is None:
        path = _paths.synth_lib()
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is missing: build it with strasgpt_b200.build.build()")
        lib = ctypes.CDLL(path)
        lib.synth_stream_id.restype = ctypes.c_uint64
        lib.synth_stream_id.argtypes = [ctypes.c_char_p]
        lib.synth_normal_bf16.argtypes = [ctypes.c_void_p, ctypes.c_size_t,
                                          ctypes.c_uint64, ctypes.c_uint64,
                                          ctypes.c_float]
        lib.synth_const_bf16.argtypes = [ctypes.c_void_p, ctypes.c_size_t,
                                         ctypes.c_float]
        lib.synth_uniform_u8.argtypes = [ctypes.c_void_p, ctypes.c_size_t,
                                         ctypes.c_uint64, ctypes.c_uint64,
                                         ctypes.c_uint32, ctypes.c_uint32]
        _synth = lib
    return _synth


def tensor_specs(cfg: ModelConfig):
    """(name, dtype, shape, init) for every tensor of the model."""
    D, F, HD = cfg.dim, cfg.hidden, cfg.head_dim
    qd, kd = cfg.q_heads * HD, cfg.kv_heads * HD
    specs = [("model.embed_tokens.weight", "BF16", [cfg.vocab, D], "normal"),
             ("model.norm.weight", "BF16", [D], "one")]
    if not cfg.tied:
        specs.append(("lm_head.weight", "BF16", [cfg.vocab, D], "normal"))
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        specs += [
            (p + "input_layernorm.weight", "BF16", [D], "one"),
            (p + "self_attn.q_proj.weight", "BF16", [qd, D], "normal"),
            (p + "self_attn.k_proj.weight", "BF16", [kd, D], "normal"),
            (p + "self_attn.v_proj.weight", "BF16", [kd, D], "normal"),
            (p + "self_attn.o_proj.weight", "BF16", [D, qd], "normal"),
            (p + "post_attention_layernorm.weight", "BF16", [D], "one"),
        ]
        if cfg.qk_norm:
            specs += [(p + "self_attn.q_norm.weight", "BF16", [HD], "one"),
                      (p + "self_attn.k_norm.weight", "BF16", [HD], "one")]
        if cfg.experts:
            E = cfg.experts
            specs.append((p + "mlp.router.weight", "BF16", [E, D], "normal"))
            for proj, rows, k in (("gate_proj", F, D), ("up_proj", F, D),
                                  ("down_proj", D, F)):
                specs += [
                    (p + f"mlp.experts.{proj}_blocks", "U8",
                     [E, rows, k // 32, 16], "codes"),
                    (p + f"mlp.experts.{proj}_scales", "U8",
                     [E, rows, k // 32], "scales"),
                ]
        else:
            specs += [
                (p + "mlp.gate_proj.weight", "BF16", [F, D], "normal"),
                (p + "mlp.up_proj.weight", "BF16", [F, D], "normal"),
                (p + "mlp.down_proj.weight", "BF16", [D, F], "normal"),
            ]
    specs.sort(key=lambda s: s[0])
    return specs


def config_json(cfg: ModelConfig) -> dict:
    c = {
        "architectures": ["SyntheticForCausalLM"],
        "model_type": cfg.model_type,
        "hidden_size": cfg.dim,
        "intermediate_size": cfg.hidden,
        "num_hidden_layers": cfg.layers,
        "num_attention_heads": cfg.q_heads,
        "num_key_value_heads": cfg.kv_heads,
        "head_dim": cfg.head_dim,
        "vocab_size": cfg.vocab,
        "max_position_embeddings": cfg.context_len,
        "rms_norm_eps": cfg.eps,
        "rope_theta": cfg.rope_theta,
        "tie_word_embeddings": cfg.tied,
        "bos_token_id": cfg.bos_token_id,
        "eos_token_id": cfg.eos_token_id,
        "torch_dtype": "bfloat16",
    }
    if cfg.rope_interleaved:
        c["rope_scaling"] = {"rope_type": "default", "mrope_interleaved": True}
    else:
        c["rope_scaling"] = None
    if cfg.experts:
        c["num_local_experts"] = cfg.experts
        c["num_experts_per_tok"] = cfg.top_k
    return c


def _byte_level_vocab(vocab: int) -> dict:
    # GPT-2 style printable mapping for the 256 byte tokens, then unique
    # placeholder strings; the forward pass never reads this file.
    bs = list(range(ord("!"), ord("~") + 1)) + \
        list(range(ord("¡"), ord("¬") + 1)) + list(range(ord("®"), ord("ÿ") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    table = {b: chr(c) for b, c in zip(bs, cs)}
    v = {}
    for b in range(min(256, vocab)):
        v[table[b]] = b
    for i in range(256, vocab):
        v[f"<|tok_{i}|>"] = i
    return v


def write_model(path: str, cfg: ModelConfig, seed: int = 0,
                tokenizer: bool = True) -> str:
    """Create `path` with config.json, model.safetensors (and tokenizer.json).

    Skips the work when a stamp file shows the same (config, seed) is already
    there.
    """
    os.makedirs(path, exist_ok=True)
    stamp = os.path.join(path, ".synth_stamp")
    key = json.dumps({"cfg": dataclass_dict(cfg), "seed": seed}, sort_keys=True)
    if os.path.exists(stamp) and open(stamp).read() == key:
        return path
    if os.path.exists(stamp):
        os.remove(stamp)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(config_json(cfg), f, indent=2)
    if tokenizer:
        with open(os.path.join(path, "tokenizer.json"), "w") as f:
            json.dump({"version": "1.0",
                       "model": {"type": "BPE",
                                 "vocab": _byte_level_vocab(cfg.vocab),
                                 "merges": []}}, f)
    specs = tensor_specs(cfg)
    header = {}
    offset = 0
    sizes = []
    for name, dtype, shape, _ in specs:
        n = int(np.prod(shape))
        size = n * (2 if dtype == "BF16" else 1)
        header[name] = {"dtype": dtype, "shape": shape,
                        "data_offsets": [offset, offset + size]}
        sizes.append(size)
        offset += size
    header["__metadata__"] = {"format": "pt", "generator": "strasgpt_b200.synth",
                              "seed": str(seed)}
    hjson = json.dumps(header, separators=(",", ":")).encode()
    hjson += b" " * ((8 - len(hjson) % 8) % 8)
    data_start = 8 + len(hjson)
    fpath = os.path.join(path, "model.safetensors")
    with open(fpath, "wb") as f:
        f.write(struct.pack("<Q", len(hjson)))
        f.write(hjson)
        f.truncate(data_start + offset)
    lib = _lib()
    mm = np.memmap(fpath, dtype=np.uint8, mode="r+", offset=data_start,
                   shape=(offset,))
    base = mm.ctypes.data
    off = 0
    for (name, dtype, shape, init), size in zip(specs, sizes):
        ptr = ctypes.c_void_p(base + off)
        stream = lib.synth_stream_id(name.encode())
        n = size // (2 if dtype == "BF16" else 1)
        if init == "normal":
            lib.synth_normal_bf16(ptr, n, seed, stream, 0.02)
        elif init == "one":
            lib.synth_const_bf16(ptr, n, 1.0)
        elif init == "codes":
            lib.synth_uniform_u8(ptr, n, seed, stream, 0, 255)
        elif init == "scales":
            lib.synth_uniform_u8(ptr, n, seed, stream, 119, 127)
        else:
            raise ValueError(init)
        off += size
    mm.flush()
    del mm
    with open(stamp, "w") as f:
        f.write(key)
    return path


def dataclass_dict(cfg: ModelConfig) -> dict:
    import dataclasses
    return dataclasses.asdict(cfg)


def prompt_tokens(cfg: ModelConfig, seed: int = 0) -> np.ndarray:
    """The seeded prompt: P ids uniform in [0, V)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, cfg.vocab, cfg.prompt_len).astype(np.int32)
