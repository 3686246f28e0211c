"""strasgpt_k_matvec_noalloc (include/strasgpt_kernels.h) against
strasgpt_k_matvec and against the float64 torch product on the same inputs,
through the C ABI. The allocation-free entry point computes the same
projection split-K into a fixed device array, so it agrees with both to fp32
summation order: relative 1e-5 of the output scale, the tolerance of the
kernel tests. Kept in a file of its own that runs last,
so it is exercised both after every other test and alone in a fresh
process."""
import ctypes

import pytest

from strasgpt_b200 import runtime

STORE, ADD, SWIGLU = 0, 1, 2
SCRATCH_BYTES = 4 << 20
MAX_WEIGHT_ROWS = SCRATCH_BYTES // 4 - 64


def _noalloc():
    L = runtime.lib()
    f = L.strasgpt_k_matvec_noalloc
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    f.argtypes = [vp, vp, ctypes.c_float, vp, i32, i32, vp, i32, vp]
    f.restype = i32
    return L, f


def _close(got, want, what):
    scale = want.abs().max().item() + 1e-30
    err = (got - want).abs().max().item()
    assert err <= 1e-5 * scale + 1e-6, f"{what}: err {err:.3e} scale {scale:.3e}"


def test_noalloc_rejects_shapes_beyond_its_scratch(capfd):
    # Host-side checks only: these calls return before touching any device.
    _, f = _noalloc()
    fake = ctypes.c_void_p(1 << 20)  # 16-byte aligned, never dereferenced
    assert f(fake, None, 1e-5, fake, 64, MAX_WEIGHT_ROWS + 1, fake, STORE, None) == -1
    assert f(fake, None, 1e-5, fake, 64, MAX_WEIGHT_ROWS // 2 + 1, fake, SWIGLU, None) == -1
    assert f(fake, None, 1e-5, fake, 12, 16, fake, STORE, None) == -1
    err = capfd.readouterr().err
    assert "exceed the 4194304-byte scratch" in err
    assert "multiple of 8" in err


def _float64_product(x, nw, w, epi, base, eps=1e-5):
    """The projection in float64 torch: rmsnorm(x) * nw (when nw is given,
    source/transformer.c:978-999 of the reference), times the bf16 rows,
    then the epilogue (gate row 2i and up row 2i + 1 for SwiGLU)."""
    import torch
    xd = x.double()
    if nw is not None:
        inv = 1.0 / torch.sqrt((xd * xd).mean() + eps)
        xd = xd * inv * nw.view(torch.bfloat16).double()
    y = w.view(torch.bfloat16).double() @ xd
    if epi == SWIGLU:
        g, u = y[0::2], y[1::2]
        return g / (1.0 + torch.exp(-g)) * u
    if epi == ADD:
        return base.double() + y
    return y


@pytest.mark.gpu
def test_noalloc_matches_matvec_on_two_calls_in_a_row(cuda):
    torch = cuda
    L, f = _noalloc()
    g = torch.Generator(device="cuda").manual_seed(2024)
    cases = [
        # (rows, k, epi, norm): the first fills the scratch with many splits,
        # the second reads fewer, smaller partials than the first left there;
        # then the residual-add epilogue on a preset output and a projection
        # without the RMSNorm prologue.
        (4096, 2048, STORE, True),
        (1536, 1024, SWIGLU, True),
        (2048, 4096, ADD, False),
        (1000, 640, STORE, False),
    ]
    runs = []
    for rows, k, epi, norm in cases:
        wrows = 2 * rows if epi == SWIGLU else rows
        x = torch.randn(k, device="cuda", generator=g)
        w = (torch.randn(wrows, k, device="cuda", generator=g) * 0.02).to(
            torch.bfloat16).view(torch.int16)
        nw = (1 + 0.1 * torch.randn(k, device="cuda", generator=g)).to(
            torch.bfloat16).view(torch.int16)
        base = torch.randn(rows, device="cuda", generator=g)
        want = base.clone()
        args = (x.data_ptr(), nw.data_ptr() if norm else None, 1e-5, w.data_ptr(), k, rows)
        assert L.strasgpt_k_matvec(*args, want.data_ptr(), epi, None) == 0
        exact = _float64_product(x, nw if norm else None, w, epi, base)
        runs.append((args, base, want, exact, epi, (x, w, nw)))
    torch.cuda.synchronize()
    # The allocation-free calls back to back on one stream, twice over: the
    # second round starts from what the first left in the shared scratch.
    for rnd in range(2):
        outs = []
        for args, base, _, _, epi, _ in runs:
            out = base.clone()
            assert f(*args, out.data_ptr(), epi, None) == 0
            outs.append(out)
        torch.cuda.synchronize()
        for i, ((args, _, want, exact, epi, _), out) in enumerate(zip(runs, outs)):
            what = f"round {rnd + 1} call {i + 1}: rows={args[5]} k={args[4]} epi={epi}"
            _close(out, want, what + " vs strasgpt_k_matvec")
            _close(out.double(), exact, what + " vs float64")
