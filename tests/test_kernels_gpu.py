"""Kernel-level numerics through the C entry points of
include/strasgpt_kernels.h, against a float64 torch reference of the same op
(the reference's fp32 matvec/rmsnorm math, source/transformer.c:978-999,
1038-1180). Tolerance: relative 1e-5 of the output scale (fp32 accumulation
in a different order)."""
import numpy as np
import pytest

from strasgpt_b200 import runtime

STORE, ADD, SWIGLU = 0, 1, 2


def bf16_from_f32(t):
    import torch
    return t.to(torch.bfloat16).view(torch.int16)


def f32_from_bf16(w):
    import torch
    return w.view(torch.bfloat16).to(torch.float64)


def ref_rmsnorm(x, w, eps):
    import torch
    x = x.to(torch.float64)
    ss = (x * x).mean(dim=-1, keepdim=True)
    return x / torch.sqrt(ss + eps) * f32_from_bf16(w)


def ref_swiglu(g, u):
    import torch
    return g * torch.sigmoid(g) * u


def interleave_gate_up(gate, up):
    """[F][K] gate and up -> [2F][K] row by row (g0, u0, g1, u1, ...)."""
    import torch
    F, K = gate.shape
    return torch.stack([gate, up], dim=1).reshape(2 * F, K).contiguous()


def close(got, want, what, rel=1e-5):
    got = got.to(want.dtype)
    scale = want.abs().max().item() + 1e-30
    err = (got - want).abs().max().item()
    assert err <= rel * scale + 1e-6, f"{what}: err {err:.3e} scale {scale:.3e}"


# The tensor-core projections carry each fp32 activation as two bf16 halves
# (about 17 significant bits): their products are exact, but the split
# leaves a relative error of up to 2^-17 per activation, which SwiGLU's
# product of two projections amplifies. Relative 3e-5 of the output scale.
TC_REL = 3e-5


@pytest.mark.gpu
@pytest.mark.parametrize("rows,k", [(1, 32), (7, 256), (4096, 1024), (1024, 2048),
                                    (130, 8200), (3, 49152)])
@pytest.mark.parametrize("epi", [STORE, ADD])
@pytest.mark.parametrize("norm", [False, True])
def test_matvec(cuda, rows, k, epi, norm):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(rows * 31 + k)
    x = torch.randn(k, device="cuda", generator=g)
    w = bf16_from_f32(torch.randn(rows, k, device="cuda", generator=g) * 0.02)
    nw = bf16_from_f32(1 + 0.1 * torch.randn(k, device="cuda", generator=g))
    out = torch.randn(rows, device="cuda", generator=g)
    base = out.clone().to(torch.float64)
    L = runtime.lib()
    L.strasgpt_k_matvec(x.data_ptr(), nw.data_ptr() if norm else None, 1e-5,
                        w.data_ptr(), k, rows, out.data_ptr(), epi, None)
    torch.cuda.synchronize()
    xin = ref_rmsnorm(x, nw, 1e-5) if norm else x.to(torch.float64)
    want = f32_from_bf16(w) @ xin
    if epi == ADD:
        want = want + base
    close(out, want, f"matvec rows={rows} k={k}")


@pytest.mark.gpu
@pytest.mark.parametrize("f,k", [(16, 64), (3072, 1024), (1792, 4096)])
def test_matvec_swiglu(cuda, f, k):
    torch = cuda
    g = torch.Generator(device="cuda").manual_seed(f + k)
    x = torch.randn(k, device="cuda", generator=g)
    gate = torch.randn(f, k, device="cuda", generator=g) * 0.02
    up = torch.randn(f, k, device="cuda", generator=g) * 0.02
    w = bf16_from_f32(interleave_gate_up(gate, up))
    out = torch.empty(f, device="cuda")
    runtime.lib().strasgpt_k_matvec(x.data_ptr(), None, 0.0, w.data_ptr(), k, f,
                                    out.data_ptr(), SWIGLU, None)
    torch.cuda.synchronize()
    gb = f32_from_bf16(bf16_from_f32(gate))
    ub = f32_from_bf16(bf16_from_f32(up))
    want = ref_swiglu(gb @ x.double(), ub @ x.double())
    close(out, want, "swiglu matvec")


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(1, 64, 32), (5, 100, 96), (64, 64, 64),
                                   (130, 300, 512), (512, 1024, 1024)])
@pytest.mark.parametrize("epi", [STORE, ADD, SWIGLU])
def test_gemm_simt(cuda, m, n, k, epi):
    torch = cuda
    if epi == SWIGLU and n % 64:
        n = (n + 63) // 64 * 64
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, device="cuda", generator=g)
    wf = torch.randn(n, k, device="cuda", generator=g) * 0.02
    w = bf16_from_f32(wf)
    ncol = n // 2 if epi == SWIGLU else n
    c = torch.randn(m, ncol, device="cuda", generator=g)
    base = c.clone().to(torch.float64)
    runtime.lib().strasgpt_k_gemm_simt(a.data_ptr(), k, w.data_ptr(), k, m, n,
                                       c.data_ptr(), ncol, epi, None)
    torch.cuda.synchronize()
    full = a.double() @ f32_from_bf16(w).T
    if epi == STORE:
        want = full
    elif epi == ADD:
        want = full + base
    else:
        v = full.view(m, n // 2, 2)
        want = ref_swiglu(v[:, :, 0], v[:, :, 1])
    close(c, want, f"gemm {m}x{n}x{k} epi {epi}")


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (1, 64, 32), (77, 300, 200),
                                   (512, 4096, 1024), (300, 1024, 3072),
                                   (129, 6144, 1024)])
@pytest.mark.parametrize("epi", [STORE, ADD, SWIGLU])
def test_gemm_tc(cuda, m, n, k, epi):
    """tcgen05 prefill projection (bf16 hi/lo activation split, fp32
    accumulation in tensor memory) against float64."""
    torch = cuda
    if epi == SWIGLU and n % 2:
        n += 1
    g = torch.Generator(device="cuda").manual_seed(m * 13 + n + k)
    a = torch.randn(m, k, device="cuda", generator=g)
    w = bf16_from_f32(torch.randn(n, k, device="cuda", generator=g) * 0.02)
    ncol = n // 2 if epi == SWIGLU else n
    c = torch.randn(m, ncol, device="cuda", generator=g)
    base = c.clone().to(torch.float64)
    hi = torch.empty(m, k, dtype=torch.int16, device="cuda")
    lo = torch.empty_like(hi)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    runtime.lib().strasgpt_k_gemm_tc(a.data_ptr(), k, hi.data_ptr(), lo.data_ptr(),
                                     w.data_ptr(), k, m, n, c.data_ptr(), ncol, epi,
                                     err.data_ptr(), None)
    torch.cuda.synchronize()
    assert err.item() == 0, "tensor-core GEMM pipeline wait timed out"
    full = a.double() @ f32_from_bf16(w).T
    if epi == STORE:
        want = full
    elif epi == ADD:
        want = full + base
    else:
        v = full.view(m, n // 2, 2)
        want = ref_swiglu(v[:, :, 0], v[:, :, 1])
    close(c, want, f"gemm_tc {m}x{n}x{k} epi {epi}", rel=TC_REL)


@pytest.mark.gpu
@pytest.mark.parametrize("t,kh,g,hd,ctx,pos0", [
    (24, 2, 2, 64, 64, 0), (77, 2, 8, 32, 128, 10), (512, 8, 2, 128, 640, 0),
    (100, 1, 4, 128, 800, 600), (40, 2, 16, 64, 64, 3), (2, 1, 1, 128, 16, 5),
    (130, 2, 64, 64, 192, 0)])
@pytest.mark.parametrize("tc", [True, False])
def test_attn_prefill(cuda, t, kh, g, hd, ctx, pos0, tc, monkeypatch):
    """Causal GQA attention of a chunk against a float64 softmax
    (source/transformer.c:1375-1422), on the tensor cores (operands split
    into bf16 hi/lo halves: the projections' TC_REL bound) and on the CUDA
    cores (STRASGPT_ATTN_TC=0)."""
    torch = cuda
    monkeypatch.setenv("STRASGPT_ATTN_TC", "1" if tc else "0")
    gen = torch.Generator(device="cuda").manual_seed(t * 7 + g + hd + pos0)
    q = torch.randn(t, kh * g, hd, device="cuda", generator=gen)
    kc = torch.randn(kh, ctx, hd, device="cuda", generator=gen)
    vc = torch.randn(kh, ctx, hd, device="cuda", generator=gen)
    att = torch.full((t, kh * g, hd), float("nan"), device="cuda")
    runtime.lib().strasgpt_k_attn_prefill(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), t, kh,
                                          g, hd, ctx, pos0, att.data_ptr(), None)
    torch.cuda.synchronize()
    n = pos0 + t
    qd = q.double().view(t, kh, g, hd)
    k = kc[:, :n].double()
    v = vc[:, :n].double()
    s = torch.einsum("tkgd,knd->tkgn", qd, k) / hd ** 0.5
    pos = pos0 + torch.arange(t, device="cuda").view(t, 1, 1, 1)
    s = s.masked_fill(torch.arange(n, device="cuda").view(1, 1, 1, n) > pos, float("-inf"))
    want = torch.einsum("tkgn,knd->tkgd", torch.softmax(s, dim=-1), v).reshape(t, kh * g, hd)
    close(att, want, f"attn_prefill tc={tc} t={t} kh={kh} g={g} hd={hd} pos0={pos0}",
          rel=TC_REL if tc else 1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("t,d", [(1, 256), (3, 2048), (17, 5120)])
def test_rmsnorm_rows(cuda, t, d):
    torch = cuda
    x = torch.randn(t, d, device="cuda") * 3
    w = bf16_from_f32(1 + 0.1 * torch.randn(d, device="cuda"))
    y = torch.empty_like(x)
    runtime.lib().strasgpt_k_rmsnorm_rows(x.data_ptr(), t, d, w.data_ptr(), 1e-6,
                                          y.data_ptr(), None)
    torch.cuda.synchronize()
    close(y, ref_rmsnorm(x, w, 1e-6), "rmsnorm")
