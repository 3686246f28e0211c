"""ctypes bindings of libstrasgpt.so: the reference's transformer API.

`Transformer` mirrors include/transformer.h (the reference's
transformer_from_safetensors / transformer_predict / transformer_free,
include/transformer.h:87-99 there) plus the extensions of include/strasgpt.h.
The library is the only compute path: if it is missing, loading fails.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import _paths

_lib = None


class _Config(ctypes.Structure):
    # transformer_configuration_t (include/transformer.h)
    _fields_ = [
        ("embedding_dim", ctypes.c_size_t),
        ("head_dim", ctypes.c_size_t),
        ("hidden_dim", ctypes.c_size_t),
        ("layer_count", ctypes.c_size_t),
        ("q_head_count", ctypes.c_size_t),
        ("kv_head_count", ctypes.c_size_t),
        ("vocabulary_len", ctypes.c_size_t),
        ("context_len", ctypes.c_size_t),
        ("epsilon", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("rope_pair_bound", ctypes.c_size_t),
        ("rope_pair_offset", ctypes.c_size_t),
        ("rope_pair_stride", ctypes.c_size_t),
        ("mrope_section_count", ctypes.c_size_t),
        ("mrope_section", ctypes.POINTER(ctypes.c_size_t)),
        ("aliased_out_weight", ctypes.c_bool),
    ]


class _Transformer(ctypes.Structure):
    _fields_ = [("config", ctypes.POINTER(_Config)),
                ("weights", ctypes.c_void_p),
                ("state", ctypes.c_void_p)]


class Timing(ctypes.Structure):
    _fields_ = [("prefill_ms", ctypes.c_double), ("decode_ms", ctypes.c_double),
                ("prefill_tokens", ctypes.c_size_t),
                ("decode_steps", ctypes.c_size_t),
                ("kernel_launches", ctypes.c_size_t),
                ("decode_launches", ctypes.c_size_t)]


KERNEL_FAMILIES = ("matvec", "attention", "qkv_post", "lm_head", "argmax", "other")
TP_HANDLE_BYTES = 64  # STRASGPT_TP_HANDLE_BYTES (include/strasgpt.h)


class KernelProfile(ctypes.Structure):
    _fields_ = [("launches", ctypes.c_int * 6), ("ms", ctypes.c_double * 6),
                ("bytes", ctypes.c_double * 6)]


def lib() -> ctypes.CDLL:
    """Load libstrasgpt.so (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    path = _paths.main_lib()
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: the CUDA library is the only compute path; "
            "build it with `python -m strasgpt_b200.build`")
    L = ctypes.CDLL(path)
    vp, sz, i32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    L.parser_parse_safetensors.restype = vp
    L.parser_parse_safetensors.argtypes = [ctypes.c_char_p]
    L.safetensors_free.argtypes = [vp]
    L.transformer_from_safetensors.restype = ctypes.POINTER(_Transformer)
    L.transformer_from_safetensors.argtypes = [vp]
    L.transformer_free.argtypes = [ctypes.POINTER(_Transformer)]
    L.transformer_predict.argtypes = [ctypes.POINTER(_Transformer), sz,
                                      ctypes.POINTER(i32), sz,
                                      ctypes.POINTER(ctypes.c_float)]
    L.transformer_generate_greedy.restype = i32
    L.transformer_generate_greedy.argtypes = [ctypes.POINTER(_Transformer), sz,
                                              ctypes.POINTER(i32), sz,
                                              ctypes.POINTER(i32),
                                              ctypes.POINTER(Timing)]
    L.transformer_reset.argtypes = [ctypes.POINTER(_Transformer)]
    L.transformer_cached_count.restype = sz
    L.transformer_cached_count.argtypes = [ctypes.POINTER(_Transformer)]
    L.strasgpt_set_placement.restype = i32
    L.strasgpt_set_placement.argtypes = [i32, i32, i32]
    L.strasgpt_tp_handle.restype = i32
    L.strasgpt_tp_handle.argtypes = [ctypes.POINTER(_Transformer), ctypes.c_char_p]
    L.strasgpt_tp_connect.restype = i32
    L.strasgpt_tp_connect.argtypes = [ctypes.POINTER(_Transformer), ctypes.c_char_p]
    L.strasgpt_profile_decode.restype = i32
    L.strasgpt_profile_decode.argtypes = [ctypes.POINTER(_Transformer), i32, sz,
                                          ctypes.POINTER(KernelProfile)]
    for name in ("strasgpt_k_matvec",):
        f = getattr(L, name)
        f.restype = i32
        f.argtypes = [vp, vp, ctypes.c_float, vp, i32, i32, vp, i32, vp]
    L.strasgpt_k_gemm_simt.restype = i32
    L.strasgpt_k_gemm_simt.argtypes = [vp, i32, vp, i32, i32, i32, vp, i32, i32, vp]
    L.strasgpt_k_attn_prefill.restype = i32
    L.strasgpt_k_attn_prefill.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, i32, vp, vp]
    L.strasgpt_k_gemm_tc.restype = i32
    L.strasgpt_k_gemm_tc.argtypes = [vp, i32, vp, vp, vp, i32, i32, i32, vp, i32, i32,
                                     vp, vp]
    L.strasgpt_k_rmsnorm_rows.restype = i32
    L.strasgpt_k_rmsnorm_rows.argtypes = [vp, i32, i32, vp, ctypes.c_float, vp, vp]
    _lib = L
    return L


def _iptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int))


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


class Transformer:
    """A model resident on one GPU (or one tensor-parallel shard of it)."""

    def __init__(self, model_dir: str, rank: int = 0, world: int = 1,
                 device: int = 0, group=None, ngpu: int = 1):
        """With world > 1 this is rank `rank`'s tensor-parallel shard; the
        ranks' exchange handles are all-gathered over the torch.distributed
        process group `group` (any backend, e.g. gloo) and connected.
        With ngpu > 1 (and world 1) the library builds a tensor-parallel
        group of `ngpu` GPUs inside this process (STRASGPT_NGPU)."""
        L = lib()
        if ngpu > 1:
            if world != 1:
                raise ValueError("ngpu > 1 is a single-process group: world must be 1")
            L.strasgpt_set_placement(0, 0, 0)
            os.environ["STRASGPT_NGPU"] = str(ngpu)
        elif L.strasgpt_set_placement(rank, world, device) != 0:
            raise ValueError(f"invalid placement rank={rank} world={world}")
        st = L.parser_parse_safetensors(model_dir.encode())
        try:
            self._t = L.transformer_from_safetensors(st)
        finally:
            L.safetensors_free(st)
            if ngpu > 1:
                os.environ.pop("STRASGPT_NGPU", None)
        cfg = self._t.contents.config.contents
        self.vocab = int(cfg.vocabulary_len)
        self.context_len = int(cfg.context_len)
        self.dim = int(cfg.embedding_dim)
        self.rank, self.world = rank, world
        if world > 1:
            import torch.distributed as dist
            handles = [None] * world
            dist.all_gather_object(handles, self.tp_handle(), group=group)
            self.tp_connect(handles)

    def tp_handle(self) -> bytes:
        """strasgpt_tp_handle: this rank's exchange-buffer handle."""
        buf = ctypes.create_string_buffer(TP_HANDLE_BYTES)
        if lib().strasgpt_tp_handle(self._t, buf) != 0:
            raise RuntimeError("strasgpt_tp_handle failed (world 1?)")
        return buf.raw

    def tp_connect(self, handles) -> None:
        """strasgpt_tp_connect with every rank's handle in rank order."""
        blob = b"".join(handles)
        if len(blob) != TP_HANDLE_BYTES * self.world:
            raise ValueError("one handle per rank expected")
        if lib().strasgpt_tp_connect(self._t, blob) != 0:
            raise RuntimeError("strasgpt_tp_connect failed")

    from_safetensors = classmethod(lambda cls, d, **kw: cls(d, **kw))

    def predict(self, tokens, logits_count: int = 1) -> np.ndarray:
        """transformer_predict: logits [min(logits_count, T)][V] (fp32)."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        n = min(int(logits_count), tok.size)
        out = np.empty((n, self.vocab), dtype=np.float32)
        lib().transformer_predict(self._t, tok.size, _iptr(tok), n, _fptr(out))
        return out

    def generate_greedy(self, prompt, steps: int):
        """Prompt + `steps` greedy decode steps on the device.

        Returns (tokens[steps + 1], Timing)."""
        tok = np.ascontiguousarray(np.asarray(prompt, dtype=np.int32))
        out = np.empty(steps + 1, dtype=np.int32)
        tm = Timing()
        lib().transformer_generate_greedy(self._t, tok.size, _iptr(tok), steps,
                                          _iptr(out), ctypes.byref(tm))
        return out, tm

    def profile_decode(self, first_token: int, steps: int) -> dict:
        p = KernelProfile()
        lib().strasgpt_profile_decode(self._t, int(first_token), steps,
                                      ctypes.byref(p))
        return {name: {"launches": p.launches[i], "ms": p.ms[i],
                       "bytes": p.bytes[i]}
                for i, name in enumerate(KERNEL_FAMILIES)}

    def reset(self) -> None:
        lib().transformer_reset(self._t)

    @property
    def cached_count(self) -> int:
        return int(lib().transformer_cached_count(self._t))

    def free(self) -> None:
        if getattr(self, "_t", None):
            lib().transformer_free(self._t)
            self._t = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
