"""ORACLE — test infrastructure only.

Python bindings of the two CPU checkers built by oracle/Makefile:
  - `Reference`: the reference's own forward pass compiled from its sources
    (oracle/_ref/libstrasgpt_ref.so);
  - `Restatement`: this project's C restatement (oracle/_build/liboracle.so),
    which also covers the mixture-of-experts models the reference lacks.
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this package, and only as the checker / CPU baseline.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "libstrasgpt_ref.so")
ORACLE_LIB = os.path.join(HERE, "_build", "liboracle.so")


def build(verbose: bool = False) -> None:
    """Build the restatement (and the reference when its sources exist)."""
    out = subprocess.run(["make", "-C", HERE, "-j4"], capture_output=not verbose,
                         text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + (out.stdout or "") +
                           (out.stderr or ""))


def reference_available() -> bool:
    return os.path.exists(REF_LIB)


class _Base:
    _prefix = ""
    _path = ""

    def __init__(self, model_dir: str):
        if not os.path.exists(self._path):
            raise RuntimeError(f"{self._path} missing: run oracle.build()")
        L = ctypes.CDLL(self._path)
        p = self._prefix
        vp, sz = ctypes.c_void_p, ctypes.c_size_t
        getattr(L, p + "load").restype = vp
        getattr(L, p + "load").argtypes = [ctypes.c_char_p]
        getattr(L, p + "vocab").restype = ctypes.c_int
        getattr(L, p + "vocab").argtypes = [vp]
        getattr(L, p + "cached").restype = sz
        getattr(L, p + "cached").argtypes = [vp]
        getattr(L, p + "reset").argtypes = [vp]
        getattr(L, p + "predict").argtypes = [vp, sz, ctypes.POINTER(ctypes.c_int),
                                              sz, ctypes.POINTER(ctypes.c_float)]
        getattr(L, p + "free").argtypes = [vp]
        self._L = L
        self._h = getattr(L, p + "load")(model_dir.encode())
        self.vocab = getattr(L, p + "vocab")(self._h)

    def predict(self, tokens, logits_count: int = 1) -> np.ndarray:
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        n = min(int(logits_count), tok.size)
        out = np.empty((n, self.vocab), dtype=np.float32)
        getattr(self._L, self._prefix + "predict")(
            self._h, tok.size, tok.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), n,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
        return out

    def reset(self) -> None:
        getattr(self._L, self._prefix + "reset")(self._h)

    @property
    def cached_count(self) -> int:
        return int(getattr(self._L, self._prefix + "cached")(self._h))

    def generate_greedy(self, prompt, steps: int):
        """Prefill + `steps` greedy steps; returns (tokens, logits[steps+1][V])."""
        logits = [self.predict(prompt, 1)[0]]
        toks = [int(np.argmax(logits[-1]))]
        for _ in range(steps):
            logits.append(self.predict([toks[-1]], 1)[0])
            toks.append(int(np.argmax(logits[-1])))
        return np.array(toks, dtype=np.int32), np.stack(logits)

    def free(self) -> None:
        if getattr(self, "_h", None):
            getattr(self._L, self._prefix + "free")(self._h)
            self._h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Reference(_Base):
    """The reference forward pass (its own C sources), OpenMP-parallel."""
    _prefix = "ref_"
    _path = REF_LIB


class Restatement(_Base):
    """This project's CPU restatement (dense + MXFP4 MoE)."""
    _prefix = "oracle_"
    _path = ORACLE_LIB

    def min_router_gap(self) -> float:
        """Smallest margin of a top-k expert choice in the last predict
        (inf for dense models)."""
        f = self._L.oracle_min_router_gap
        f.restype = ctypes.c_float
        f.argtypes = [ctypes.c_void_p]
        return float(f(self._h))

    def generate_greedy(self, prompt, steps: int, gaps=None):
        """As _Base.generate_greedy; appends each step's min_router_gap()
        to `gaps` when a list is given."""
        logits = [self.predict(prompt, 1)[0]]
        if gaps is not None:
            gaps.append(self.min_router_gap())
        toks = [int(np.argmax(logits[-1]))]
        for _ in range(steps):
            logits.append(self.predict([toks[-1]], 1)[0])
            if gaps is not None:
                gaps.append(self.min_router_gap())
            toks.append(int(np.argmax(logits[-1])))
        return np.array(toks, dtype=np.int32), np.stack(logits)
