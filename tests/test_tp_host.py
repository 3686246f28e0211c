"""Host side of tensor parallelism on CPU, as world-2 gloo process groups:

1. runtime.Transformer's handle exchange: every rank publishes its
   exchange-buffer handle, the handles are all-gathered and every rank
   connects with all of them in rank order (a fake library stands in for
   libstrasgpt.so, which needs a GPU for these calls).
2. The partition the loader applies (strasgpt_b200/csrc/transformer.cu,
   load_weights): with kv heads, their q heads, o_proj columns, FFN rows /
   down columns and vocabulary rows sliced per rank, the per-rank partial
   sums all-reduced over gloo equal the unsliced layer (float64), and the
   gathered vocabulary slices equal the full LM head.
"""
import ctypes
import os
import socket

import numpy as np
import pytest

WORLD = 2


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _FakeLib:
    """The calls runtime.Transformer makes, without a GPU."""

    def __init__(self, rank, out):
        self.rank, self.out = rank, out

    def strasgpt_set_placement(self, rank, world, device):
        return 0

    def parser_parse_safetensors(self, path):
        return 1

    def safetensors_free(self, st):
        pass

    def transformer_from_safetensors(self, st):
        cfg = type("Cfg", (), {"vocabulary_len": 16, "context_len": 8, "embedding_dim": 4})()
        conf = type("P", (), {"contents": cfg})()
        return type("T", (), {"contents": type("TT", (), {"config": conf})()})()

    def strasgpt_tp_handle(self, t, buf):
        h = (b"rank%d" % self.rank).ljust(64, b"\0")
        ctypes.memmove(buf, h, 64)
        return 0

    def strasgpt_tp_connect(self, t, blob):
        self.out.put((self.rank, bytes(blob)))
        return 0


def _handles_rank(rank, port, out):
    import datetime
    import torch.distributed as dist
    from strasgpt_b200 import runtime
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    fake = _FakeLib(rank, out)
    runtime.lib = lambda: fake
    runtime.Transformer("unused", rank=rank, world=WORLD, device=rank)
    dist.destroy_process_group()


def test_handles_are_all_gathered_in_rank_order():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_handles_rank, args=(r, port, out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = dict(out.get(timeout=120) for _ in range(WORLD))
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    want = b"".join((b"rank%d" % r).ljust(64, b"\0") for r in range(WORLD))
    assert got == {r: want for r in range(WORLD)}


def _layer(seed=0, D=64, KH=4, G=2, HD=8, F=96, V=40):
    rng = np.random.default_rng(seed)
    QH = KH * G
    return {
        "D": D, "KH": KH, "G": G, "HD": HD, "F": F, "V": V,
        # q rows ordered [kv head][q in group][hd], then k, then v (as the
        # reference's Wq[kv][q][hd][D], Wk[kv][hd][D], Wv[kv][hd][D]).
        "wq": rng.standard_normal((QH * HD, D)), "wk": rng.standard_normal((KH * HD, D)),
        "wv": rng.standard_normal((KH * HD, D)), "wo": rng.standard_normal((D, QH * HD)),
        "wg": rng.standard_normal((F, D)), "wu": rng.standard_normal((F, D)),
        "wd": rng.standard_normal((D, F)), "wout": rng.standard_normal((V, D)),
        "x": rng.standard_normal(D), "att": rng.standard_normal(QH * HD),
    }


def _rank_slices(L, g, N):
    D, KH, G, HD, F, V = L["D"], L["KH"], L["G"], L["HD"], L["F"], L["V"]
    khl, fl, vl = KH // N, F // N, V // N
    q = slice(g * khl * G * HD, (g + 1) * khl * G * HD)
    kv = slice(g * khl * HD, (g + 1) * khl * HD)
    f = slice(g * fl, (g + 1) * fl)
    v = slice(g * vl, (g + 1) * vl)
    return q, kv, f, v


def _partition_rank(rank, port, out):
    import datetime
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    L = _layer()
    q, kv, f, v = _rank_slices(L, rank, WORLD)
    # o_proj: this rank's heads' attention columns -> partial residual update
    o_part = L["wo"][:, q] @ L["att"][q]
    # FFN: this rank's gate/up rows, SwiGLU, down columns -> partial
    xg, xu = L["wg"][f] @ L["x"], L["wu"][f] @ L["x"]
    h = xg / (1 + np.exp(-xg)) * xu
    ffn_part = L["wd"][:, f] @ h
    parts = torch.tensor(np.concatenate([o_part, ffn_part]))
    dist.all_reduce(parts)
    # vocabulary slice of the LM head, gathered in rank order
    logits = torch.tensor(L["wout"][v] @ L["x"])
    gathered = [torch.zeros_like(logits) for _ in range(WORLD)]
    dist.all_gather(gathered, logits)
    # each rank's q rows are the q heads of its kv heads
    heads_ok = (L["wq"][q].shape[0] == (L["KH"] // WORLD) * L["G"] * L["HD"]
                and L["wk"][kv].shape[0] == (L["KH"] // WORLD) * L["HD"])
    out.put((rank, parts.numpy(), torch.cat(gathered).numpy(), heads_ok))
    dist.destroy_process_group()


def test_partition_partials_sum_to_the_full_layer():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_partition_rank, args=(r, port, out)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [out.get(timeout=120) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    L = _layer()
    o_full = L["wo"] @ L["att"]
    xg, xu = L["wg"] @ L["x"], L["wu"] @ L["x"]
    ffn_full = L["wd"] @ (xg / (1 + np.exp(-xg)) * xu)
    logits_full = L["wout"] @ L["x"]
    for rank, parts, logits, heads_ok in res:
        assert heads_ok
        np.testing.assert_allclose(parts[:L["D"]], o_full, rtol=1e-12, atol=1e-9)
        np.testing.assert_allclose(parts[L["D"]:], ffn_full, rtol=1e-12, atol=1e-9)
        np.testing.assert_allclose(logits, logits_full, rtol=1e-12, atol=1e-9)
