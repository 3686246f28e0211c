"""strasgpt_k_matvec_noalloc (include/strasgpt_kernels.h) against
strasgpt_k_matvec on the same inputs, through the C ABI. The allocation-free
entry point computes the same projection split-K into a fixed device array,
so the two agree to fp32 summation order: relative 1e-5 of the output scale,
the tolerance of the kernel tests. Kept in a file of its own that runs last,
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


@pytest.mark.gpu
def test_noalloc_matches_matvec_on_two_calls_in_a_row(cuda):
    torch = cuda
    L, f = _noalloc()
    g = torch.Generator(device="cuda").manual_seed(2024)
    cases = [
        # (rows, k, epi, norm): the first fills the scratch with many splits,
        # the second reads fewer, smaller partials than the first left there.
        (4096, 2048, STORE, True),
        (1536, 1024, SWIGLU, True),
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
        want, got = base.clone(), base.clone()
        args = (x.data_ptr(), nw.data_ptr() if norm else None, 1e-5, w.data_ptr(), k, rows)
        assert L.strasgpt_k_matvec(*args, want.data_ptr(), epi, None) == 0
        runs.append((args, got, want, epi, (x, w, nw)))
    torch.cuda.synchronize()
    # The two allocation-free calls back to back on one stream.
    for args, got, _, epi, _ in runs:
        assert f(*args, got.data_ptr(), epi, None) == 0
    torch.cuda.synchronize()
    for i, (args, got, want, epi, _) in enumerate(runs):
        _close(got, want, f"call {i + 1}: rows={args[5]} k={args[4]} epi={epi}")
