"""The C-ABI library loads without a GPU and exports every function that
include/*.h declares (no compute calls here)."""
import ctypes
import os
import re
import subprocess

from strasgpt_b200 import _paths

INCLUDE = _paths.include_dir()


def declared_functions():
    names = {}
    for h in sorted(os.listdir(INCLUDE)):
        if not h.endswith(".h"):
            continue
        text = open(os.path.join(INCLUDE, h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = re.sub(r"#[^\n]*", "", text)
        # a declaration: type name(args); at file scope
        for m in re.finditer(r"\b([A-Za-z_][A-Za-z_0-9]*)\s*\(([^;{}]*)\)\s*;", text):
            name = m.group(1)
            if name in ("if", "while", "for", "return", "sizeof"):
                continue
            names[name] = h
    return names


def test_headers_declare_the_reference_api():
    names = declared_functions()
    for f in ("transformer_from_safetensors", "transformer_free",
              "transformer_print", "transformer_logits_malloc",
              "transformer_predict", "parser_parse_safetensors",
              "safetensors_read", "safetensors_free"):
        assert f in names, f


def test_library_exports_every_declared_function():
    lib = ctypes.CDLL(_paths.main_lib())
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_library_exports_tokenizer_reader_and_scanner_stub():
    # Needed by the reference's tokenizer.c / strasgpt.c at link time.
    lib = ctypes.CDLL(_paths.main_lib())
    assert hasattr(lib, "parser_parse_tokenizer")
    assert hasattr(lib, "json_scanner_lex_destroy")


def test_library_is_built_for_sm100a():
    out = subprocess.run(["cuobjdump", "--list-elf", _paths.main_lib()],
                         capture_output=True, text=True)
    if out.returncode != 0:
        return  # tool unavailable: nothing to check
    assert "sm_100a" in out.stdout
