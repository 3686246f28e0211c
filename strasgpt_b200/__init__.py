"""strasgpt-b200: StrasGPT's transformer forward pass, B200-native.

The compute path is libstrasgpt.so (hand-written CUDA for sm_100a behind the
reference's transformer C ABI). This package holds the Python bindings of
that ABI (`runtime`), the benchmark/test model shapes (`configs`) and the
deterministic synthetic-model writer (`synth`).
"""
from . import configs  # noqa: F401
from .runtime import Transformer, lib  # noqa: F401

__all__ = ["Transformer", "lib", "configs"]
