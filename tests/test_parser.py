"""The model-directory reader (parser_parse_safetensors / tokenizer) against
Python's json on the same files, plus its error behaviour (exit with a
"[StrasGPT] Error" message, like the reference's yyerror/UTIL_DIE)."""
import ctypes
import json
import os
import struct
import subprocess
import sys

import pytest

from conftest import ROOT, model_dir
from strasgpt_b200 import _paths, configs

MAX_TENSORS = 65536


class Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_int),
                ("dim_count", ctypes.c_size_t), ("dim", ctypes.c_size_t * 8),
                ("size", ctypes.c_size_t), ("file", ctypes.c_size_t),
                ("offset", ctypes.c_size_t)]


class Safetensors(ctypes.Structure):
    _fields_ = [("model_type", ctypes.c_char_p),
                ("embedding_dim", ctypes.c_size_t), ("head_dim", ctypes.c_size_t),
                ("hidden_dim", ctypes.c_size_t), ("layer_count", ctypes.c_size_t),
                ("q_head_count", ctypes.c_size_t), ("kv_head_count", ctypes.c_size_t),
                ("vocabulary_len", ctypes.c_size_t), ("context_len", ctypes.c_size_t),
                ("epsilon", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("rope_interleaved", ctypes.c_bool),
                ("mrope_section_count", ctypes.c_size_t),
                ("mrope_section", ctypes.c_size_t * 8),
                ("bos_token_id", ctypes.c_int), ("eos_token_id", ctypes.c_int),
                ("file_count", ctypes.c_size_t), ("file", ctypes.c_char_p * 64),
                ("tensor_count", ctypes.c_size_t), ("tensor", Tensor * MAX_TENSORS),
                ("expert_count", ctypes.c_size_t), ("expert_top_k", ctypes.c_size_t)]


def parse(path):
    lib = ctypes.CDLL(_paths.main_lib())
    lib.parser_parse_safetensors.restype = ctypes.POINTER(Safetensors)
    lib.parser_parse_safetensors.argtypes = [ctypes.c_char_p]
    return lib, lib.parser_parse_safetensors(path.encode())


@pytest.mark.parametrize("name", ["t_qwen", "t_moe", "t_interleaved", "t_untied"])
def test_parse_matches_python_json(name):
    cfg = configs.get(name)
    d = model_dir(cfg)
    lib, p = parse(d)
    s = p.contents
    c = json.load(open(os.path.join(d, "config.json")))
    assert s.model_type.decode() == c["model_type"]
    assert s.embedding_dim == c["hidden_size"]
    assert s.hidden_dim == c["intermediate_size"]
    assert s.layer_count == c["num_hidden_layers"]
    assert s.q_head_count == c["num_attention_heads"]
    assert s.kv_head_count == c["num_key_value_heads"]
    assert s.head_dim == c["head_dim"]
    assert s.vocabulary_len == c["vocab_size"]
    assert s.context_len == c["max_position_embeddings"]
    assert s.epsilon == pytest.approx(c["rms_norm_eps"], rel=1e-6)
    assert s.rope_theta == pytest.approx(c["rope_theta"], rel=1e-6)
    assert s.rope_interleaved == cfg.rope_interleaved
    assert s.expert_count == c.get("num_local_experts", 0)
    assert s.expert_top_k == c.get("num_experts_per_tok", 0)
    assert s.bos_token_id == c["bos_token_id"] and s.eos_token_id == c["eos_token_id"]
    assert s.file_count == 1
    assert s.file[0].decode() == os.path.join(d, "model.safetensors")
    raw = open(os.path.join(d, "model.safetensors"), "rb").read(1 << 20)
    hlen = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + hlen])
    header.pop("__metadata__")
    assert s.tensor_count == len(header)
    for i, (tname, info) in enumerate(header.items()):
        t = s.tensor[i]
        assert t.name.decode() == tname
        assert ["F16", "BF16", "F32", "U8"][t.type] == info["dtype"]
        assert list(t.dim[:t.dim_count]) == info["shape"]
        b, e = info["data_offsets"]
        assert t.size == e - b and t.offset == 8 + hlen + b
    lib.safetensors_free.argtypes = [ctypes.c_void_p]
    lib.safetensors_free(ctypes.cast(p, ctypes.c_void_p))


def test_head_dim_default_and_text_config(tmp_path):
    # head_dim absent -> hidden_size / heads (source/json_parser.y:614-619);
    # keys inside "text_config" are read like top-level keys.
    src = model_dir(configs.T_LLAMA)
    c = json.load(open(os.path.join(src, "config.json")))
    del c["head_dim"]
    inner = {k: c.pop(k) for k in ("hidden_size", "num_attention_heads")}
    c["text_config"] = inner
    c["eos_token_id"] = [7, 9]  # list form: first id
    c["quantization_config"] = {"model": "x", "hidden_size": 1}  # ignored
    (tmp_path / "config.json").write_text(json.dumps(c))
    os.symlink(os.path.join(src, "model.safetensors"), tmp_path / "model.safetensors")
    lib, p = parse(str(tmp_path))
    assert p.contents.embedding_dim == 256
    assert p.contents.head_dim == 256 // 8
    assert p.contents.eos_token_id == 7


def test_index_file_lists_shards_in_order(tmp_path):
    src = model_dir(configs.T_LLAMA)
    (tmp_path / "config.json").write_text(open(os.path.join(src, "config.json")).read())
    os.symlink(os.path.join(src, "model.safetensors"), tmp_path / "a.safetensors")
    os.symlink(os.path.join(src, "model.safetensors"), tmp_path / "b.safetensors")
    idx = {"metadata": {"total_size": 1},
           "weight_map": {"x": "b.safetensors", "y": "a.safetensors", "z": "b.safetensors"}}
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(idx))
    lib, p = parse(str(tmp_path))
    assert p.contents.file_count == 2
    assert p.contents.file[0].decode().endswith("/b.safetensors")
    assert p.contents.file[1].decode().endswith("/a.safetensors")
    n = p.contents.tensor_count
    assert n % 2 == 0 and p.contents.tensor[n - 1].file == 1


def _run_parse_in_child(path):
    code = ("import ctypes,sys; l=ctypes.CDLL(sys.argv[1]); "
            "l.parser_parse_safetensors.argtypes=[ctypes.c_char_p]; "
            "l.parser_parse_safetensors(sys.argv[2].encode())")
    return subprocess.run([sys.executable, "-c", code, _paths.main_lib(), path],
                          capture_output=True, text=True, timeout=60)


def test_non_integer_dimension_is_an_error(tmp_path):
    src = model_dir(configs.T_LLAMA)
    c = json.load(open(os.path.join(src, "config.json")))
    c["hidden_size"] = 256.5
    (tmp_path / "config.json").write_text(json.dumps(c))
    r = _run_parse_in_child(str(tmp_path))
    assert r.returncode != 0
    assert "[StrasGPT] Error" in r.stderr and "non integer" in r.stderr


def test_missing_config_is_an_error(tmp_path):
    r = _run_parse_in_child(str(tmp_path))
    assert r.returncode != 0 and "failed to open file" in r.stderr


def test_unknown_dtype_is_an_error(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"hidden_size": 32}))
    h = json.dumps({"w": {"dtype": "I64", "shape": [1], "data_offsets": [0, 8]}}).encode()
    with open(tmp_path / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    r = _run_parse_in_child(str(tmp_path))
    assert r.returncode != 0 and "unknown data type" in r.stderr


def test_tokenizer_vocab_raw_strings_and_scores(tmp_path):
    vocab = {"a": 0, "\\u0120b": 1, "\\\"q\\\"": 2, "model": 3, "zz": 4}
    body = '{"model": {"type": "BPE", "vocab": {' + ", ".join(
        f'"{k}": {v}' for k, v in vocab.items()) + '}, "merges": []}, "added": 1}'
    (tmp_path / "tokenizer.json").write_text(body)
    lib = ctypes.CDLL(_paths.main_lib())
    lib.parser_parse_tokenizer.restype = ctypes.c_void_p
    lib.parser_parse_tokenizer.argtypes = [ctypes.c_char_p]
    p = lib.parser_parse_tokenizer(str(tmp_path).encode())
    count = ctypes.c_size_t.from_address(p).value
    strings = (ctypes.c_char_p * 262144).from_address(p + 8)
    scores = (ctypes.c_float * 262144).from_address(p + 8 + 8 * 262144)
    assert count == len(vocab)
    for i, (k, v) in enumerate(vocab.items()):
        assert strings[i].decode() == k  # escapes kept, quotes stripped
        assert scores[i] == float(v)
