"""Numerics of the sm_100a kernels against PyTorch fp32 definitions."""

import math

import pytest
import torch
import torch.nn.functional as F

from minispeed_b200.ops import _ext, kernels
from minispeed_b200.ops import nn as ops

pytestmark = pytest.mark.gpu
DT = [torch.float16, torch.bfloat16]


def _tol(dtype):
    return {torch.float16: (2e-3, 2e-3), torch.bfloat16: (1.6e-2, 1.6e-2),
            torch.float32: (1e-5, 1e-5)}[dtype]


def test_extension_is_native():
    mod = _ext.get()
    assert mod.__file__.endswith(".so")
    before = _ext.launch_count()
    kernels.grad_stats([torch.ones(10, device="cuda")])
    assert _ext.launch_count() > before


@pytest.mark.parametrize("dtype", [torch.float32] + DT)
@pytest.mark.parametrize("n,offset", [(1, 0), (1000, 0), (4097, 3), (1 << 20, 1)])
def test_grad_stats_matches_torch(dtype, n, offset):
    g = torch.Generator(device="cuda").manual_seed(n)
    base = torch.randn(n + offset, device="cuda", generator=g).to(dtype)
    x = base[offset:]
    flag, ss = kernels.grad_stats([x], inv_scale=0.25)
    ref = (x.float() * 0.25).pow(2).sum().double()
    assert float(flag) == 0.0
    assert float(ss) == pytest.approx(float(ref), rel=1e-5)
    x[n // 2] = float("inf")
    flag, _ = kernels.grad_stats([x])
    assert float(flag) == 1.0
    x[n // 2] = float("nan")
    assert float(kernels.grad_stats([x])[0]) == 1.0


def test_stats_finalize_clip_coefficient_and_determinism():
    st = kernels.StepStats(torch.device("cuda"))
    a = torch.randn(3_000_001, device="cuda")
    b = torch.randn(77, device="cuda", dtype=torch.float16)
    outs = []
    for _ in range(2):
        st.reset()
        st.accumulate(a, 2.0)
        st.accumulate(b, 0.5)
        outs.append(st.finalize(1.0).clone())
    assert torch.equal(outs[0], outs[1])
    ref = (a.double() * 2).pow(2).sum() + (b.double() * 0.5).pow(2).sum()
    out = outs[0].cpu()
    assert out[1].item() == pytest.approx(ref.item(), rel=1e-6)
    norm = math.sqrt(ref.item())
    assert out[2].item() == pytest.approx(norm, rel=1e-6)
    assert out[3].item() == pytest.approx(1.0 / (norm + 1e-6), rel=1e-6)


@pytest.mark.parametrize("gdtype", [torch.float32] + DT)
@pytest.mark.parametrize("pdtype", [None] + DT)
@pytest.mark.parametrize("n,off", [(4096, 0), (1001, 1)])
def test_adamw_kernel_matches_reference(gdtype, pdtype, n, off):
    torch.manual_seed(0)
    p0 = torch.randn(n + off, device="cuda")
    m0 = torch.randn(n, device="cuda").abs() * 1e-2
    v0 = torch.randn(n, device="cuda").abs() * 1e-3
    gr = (torch.randn(n + off, device="cuda") * 8).to(gdtype)
    stats = torch.tensor([0.0, 4.0, 2.0, 0.5, 0, 0, 0, 0], device="cuda")
    hp = dict(lr=1e-3, beta1=0.9, beta2=0.95, eps=1e-8, wd=0.1, bc1=1 - 0.9 ** 3,
              bc2=1 - 0.95 ** 3, grad_mul=0.125)
    outs = []
    for fn in (kernels.adamw_step, kernels.adamw_reference):
        p, m, v = p0.clone()[off:], m0.clone(), v0.clone()
        po = None if pdtype is None else torch.empty(n + off, device="cuda", dtype=pdtype)[off:]
        fn(p, m, v, gr[off:], stats=stats, param_out=po, **hp)
        outs.append((p, m, v, po))
    (p, m, v, po), (rp, rm, rv, rpo) = outs
    torch.testing.assert_close(p, rp, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(m, rm, rtol=1e-6, atol=1e-9)
    torch.testing.assert_close(v, rv, rtol=1e-6, atol=1e-10)
    if po is not None:
        torch.testing.assert_close(po, p.to(pdtype), rtol=0, atol=0)


def test_adamw_kernel_skips_on_overflow_flag():
    p = torch.randn(1000, device="cuda")
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    before = p.clone()
    stats = torch.tensor([1.0, float("inf"), float("inf"), 1.0, 0, 0, 0, 0], device="cuda")
    kernels.adamw_step(p, m, v, torch.ones_like(p), lr=1.0, beta1=0.9, beta2=0.99, eps=1e-8,
                       wd=0.1, bc1=0.1, bc2=0.01, stats=stats)
    assert torch.equal(p, before) and not m.any()


@pytest.mark.parametrize("dtype", DT)
def test_cast_scale(dtype):
    src = torch.randn(12345, device="cuda").to(dtype)
    dst = torch.empty(12345, device="cuda")
    kernels.cast_scale(src, dst, 0.5)
    torch.testing.assert_close(dst, src.float() * 0.5, rtol=0, atol=0)


# ------------------------------------------------------------- nn kernels
@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("rms", [False, True])
@pytest.mark.parametrize("C", [768, 1600])
def test_add_norm_fwd_bwd(dtype, rms, C):
    torch.manual_seed(1)
    M = 300
    x = torch.randn(M, C, device="cuda", dtype=dtype, requires_grad=True)
    d = torch.randn(M, C, device="cuda", dtype=dtype, requires_grad=True)
    w = (1 + 0.1 * torch.randn(C, device="cuda")).to(dtype).requires_grad_()
    b = None if rms else (0.1 * torch.randn(C, device="cuda")).to(dtype).requires_grad_()
    s, y = ops.add_norm(x, d, w, b, 1e-5, rms)
    (y.float().pow(2).sum() + (s.float() * 0.3).sum()).backward()
    grads = [t.grad.clone() for t in (x, d, w) + ((b,) if b is not None else ())]
    # fp32 oracle on the same (rounded) inputs
    xs = [t.detach().float().requires_grad_() for t in (x, d, w) + ((b,) if b is not None else ())]
    sr = (xs[0] + xs[1]).to(dtype).float()
    sr.retain_grad()
    yr = ops._norm_torch(sr, xs[2], xs[3] if b is not None else None, 1e-5, rms)
    if rms:
        yr = sr * torch.rsqrt(sr.pow(2).mean(-1, keepdim=True) + 1e-5) * xs[2]
    else:
        yr = F.layer_norm(sr, (C,), xs[2], xs[3], 1e-5)
    (yr.pow(2).sum() + (sr * 0.3).sum()).backward()
    rt, at = _tol(dtype)
    torch.testing.assert_close(s.float(), sr.detach(), rtol=0, atol=0)
    torch.testing.assert_close(y.float(), yr.detach(), rtol=rt, atol=at * 4)
    scale_dx = float(sr.grad.abs().max())
    torch.testing.assert_close(grads[0].float(), sr.grad, rtol=rt * 4, atol=at * scale_dx)
    torch.testing.assert_close(grads[1].float(), sr.grad, rtol=rt * 4, atol=at * scale_dx)
    gw = xs[2].grad
    torch.testing.assert_close(grads[2].float(), gw, rtol=rt * 4, atol=at * float(gw.abs().max()))
    if b is not None:
        gb = xs[3].grad
        torch.testing.assert_close(grads[3].float(), gb, rtol=rt * 4,
                                   atol=at * float(gb.abs().max()))


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("rms,C", [(False, 1600), (True, 1600), (True, 4096), (False, 768)])
@pytest.mark.parametrize("with_delta", [True, False])
@pytest.mark.parametrize("offset", [0, 1])
def test_norm_row_kernels(dtype, rms, C, with_delta, offset):
    """The row-looping norm kernels (all of a row's loads issued first; the
    weight and bias staged in shared memory) on 5000 rows, so every block
    loops over several row groups; offset 1 misaligns the rows (the
    per-vector kernels run instead); width 4096 uses 16 vectors per lane."""
    torch.manual_seed(C + offset)
    M = 5000

    def rows(scale=1.0):
        buf = (torch.randn(M * C + offset, device="cuda") * scale).to(dtype)
        return buf[offset:].view(M, C).requires_grad_()

    x = rows()
    d = rows() if with_delta else None
    w = (1 + 0.1 * torch.randn(C, device="cuda")).to(dtype).requires_grad_()
    b = None if rms else (0.1 * torch.randn(C, device="cuda")).to(dtype).requires_grad_()
    if with_delta:
        s, y = ops.add_norm(x, d, w, b, 1e-5, rms)
    else:
        s, y = x, ops.norm(x, w, b, 1e-5, rms)
    gy = torch.randn(M, C, device="cuda").to(dtype)
    y.backward(gy)
    leaves = [t for t in (x, d, w, b) if t is not None]
    xs = [t.detach().float().requires_grad_() for t in leaves]
    sr = (xs[0] + xs[1]).to(dtype).float() if with_delta else xs[0]
    wi = 2 if with_delta else 1
    if rms:
        yr = sr * torch.rsqrt(sr.pow(2).mean(-1, keepdim=True) + 1e-5) * xs[wi]
    else:
        yr = F.layer_norm(sr, (C,), xs[wi], xs[wi + 1], 1e-5)
    yr.backward(gy.float())
    rt, at = _tol(dtype)
    if with_delta:
        torch.testing.assert_close(s.float(), sr.detach(), rtol=0, atol=0)
    torch.testing.assert_close(y.float(), yr.detach(), rtol=rt, atol=at * 4)
    for got, ref in zip(leaves, xs):
        scale = float(ref.grad.abs().max())
        torch.testing.assert_close(got.grad.float(), ref.grad, rtol=rt * 4,
                                   atol=at * 2 * scale)


@pytest.mark.parametrize("dtype", DT)
def test_linear_gelu_and_linear(dtype):
    torch.manual_seed(2)
    x = torch.randn(256, 128, device="cuda", dtype=dtype, requires_grad=True)
    w = (torch.randn(384, 128, device="cuda") * 0.05).to(dtype).requires_grad_()
    b = (torch.randn(384, device="cuda") * 0.1).to(dtype).requires_grad_()
    out = ops.linear_gelu(x, w, b)
    g = torch.randn_like(out)
    out.backward(g)
    xf, wf, bf = (t.detach().float().requires_grad_() for t in (x, w, b))
    ref = F.gelu(xf @ wf.t() + bf)
    ref.backward(g.float())
    rt, at = _tol(dtype)
    torch.testing.assert_close(out.float(), ref, rtol=rt * 4, atol=at * 4)
    for got, exp in ((x.grad, xf.grad), (w.grad, wf.grad), (b.grad, bf.grad)):
        torch.testing.assert_close(got.float(), exp, rtol=rt * 8,
                                   atol=at * 8 * float(exp.abs().max()))


@pytest.mark.parametrize("dtype", DT)
def test_swiglu(dtype):
    gu = torch.randn(64, 2 * 256, device="cuda", dtype=dtype, requires_grad=True)
    h = ops.swiglu(gu)
    dh = torch.randn_like(h)
    h.backward(dh)
    ref_in = gu.detach().float().requires_grad_()
    g, u = ref_in.chunk(2, dim=-1)
    ref = F.silu(g) * u
    ref.backward(dh.float())
    rt, at = _tol(dtype)
    torch.testing.assert_close(h.float(), ref, rtol=rt * 2, atol=at * 2)
    torch.testing.assert_close(gu.grad.float(), ref_in.grad, rtol=rt * 4, atol=at * 4)


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("V,ld", [(50257, 50257), (1000, 1000), (50257, 50304), (1003, 1008)])
def test_cross_entropy(dtype, V, ld):
    """ld > V: rows padded to a multiple of 8 (the vectorized forward path)."""
    torch.manual_seed(3)
    M = 129
    logits = (torch.randn(M, ld, device="cuda") * 3).to(dtype)[:, :V]
    tgt = torch.randint(0, V, (M,), device="cuda")
    tgt[5] = -100
    ref_l = logits.detach().float().requires_grad_()
    ref = F.cross_entropy(ref_l, tgt)
    (ref * 7).backward()
    if ld == V:
        lg = logits.clone().requires_grad_()
        loss = ops.cross_entropy(lg * 1, tgt)  # autograd path (non-leaf logits)
    else:
        # the padded view itself (rows ld apart); its storage becomes the gradient
        lg = logits.requires_grad_()
        loss = ops.cross_entropy(lg, tgt)
    (loss * 7).backward()
    assert float(loss) == pytest.approx(float(ref), rel=1e-5, abs=1e-5)
    rt, at = _tol(dtype)
    torch.testing.assert_close(lg.grad.float(), ref_l.grad, rtol=rt, atol=at * 0.05)


@pytest.mark.parametrize("dtype", DT)
def test_embedding(dtype):
    V, C, B, T = 97, 64, 3, 40
    wte = torch.randn(V, C, device="cuda", dtype=dtype, requires_grad=True)
    wpe = torch.randn(T + 5, C, device="cuda", dtype=dtype, requires_grad=True)
    idx = torch.randint(0, V, (B, T), device="cuda")
    out = ops.embedding(idx, wte, wpe)
    g = torch.randn_like(out)
    out.backward(g)
    wf, pf = wte.detach().float().requires_grad_(), wpe.detach().float().requires_grad_()
    ref = F.embedding(idx, wf) + pf[:T]
    ref.backward(g.float())
    rt, at = _tol(dtype)
    torch.testing.assert_close(out.float(), ref, rtol=rt, atol=at)
    torch.testing.assert_close(wte.grad.float(), wf.grad, rtol=rt * 4, atol=at * 8)
    torch.testing.assert_close(wpe.grad.float(), pf.grad, rtol=rt * 4, atol=at * 8)


@pytest.mark.parametrize("dtype", DT)
def test_rope(dtype):
    B, T, H, D = 2, 33, 4, 64
    x = torch.randn(B, T, H, D, device="cuda", dtype=dtype, requires_grad=True)
    cos, sin = ops.rope_tables(T, D, 10000.0, "cuda")
    y = ops.rope(x, cos, sin)
    g = torch.randn_like(y)
    y.backward(g)
    xf = x.detach().float().requires_grad_()
    ref = ops.rope(xf.cpu(), cos.cpu(), sin.cpu()).cuda()
    rt, at = _tol(dtype)
    torch.testing.assert_close(y.float(), ref, rtol=rt, atol=at * 2)
    # rotation is orthogonal: the backward is the inverse rotation
    back = ops.rope(g.float().cpu(), cos.cpu(), -sin.cpu()).cuda()
    torch.testing.assert_close(x.grad.float(), back, rtol=rt, atol=at * 2)


@pytest.mark.parametrize("dtype", DT)
def test_embedding_backward_into_sink_twice(dtype):
    """Parameters whose ``.grad`` is bound (the engine's arena views) get the
    token and position gradients added in place; the persistent fp32
    accumulator is clean again for the second backward (other tokens)."""
    V, C, B, T = 211, 128, 4, 48
    wte = torch.nn.Parameter(torch.randn(V, C, device="cuda", dtype=dtype))
    wpe = torch.nn.Parameter(torch.randn(T + 3, C, device="cuda", dtype=dtype))
    wte.grad = torch.randn_like(wte) * 0.1
    wpe.grad = torch.randn_like(wpe) * 0.1
    want_te, want_pe = wte.grad.float().clone(), wpe.grad.float().clone()
    for seed in (1, 2):
        gen = torch.Generator(device="cuda").manual_seed(seed)
        idx = torch.randint(0, V // seed, (B, T), device="cuda", generator=gen)
        out = ops.embedding(idx, wte, wpe)
        g = torch.randn(out.shape, device="cuda", generator=gen).to(dtype)
        out.backward(g)
        want_te.index_add_(0, idx.reshape(-1), g.float().reshape(-1, C))
        want_pe[:T] += g.float().sum(0)
        rt, at = _tol(dtype)
        torch.testing.assert_close(wte.grad.float(), want_te, rtol=rt * 4, atol=at * 8)
        torch.testing.assert_close(wpe.grad.float(), want_pe, rtol=rt * 4, atol=at * 8)
        want_te, want_pe = wte.grad.float().clone(), wpe.grad.float().clone()


@pytest.mark.parametrize("dtype", DT)
@pytest.mark.parametrize("mult", [7.0, 3.0])
@pytest.mark.parametrize("V,ld", [(50257, 50304), (1003, 1008)])
def test_cross_entropy_gradient_in_forward(dtype, mult, V, ld):
    """Inside ``expected_loss_grad(seed)`` the forward writes the gradient for
    upstream gradient ``seed`` (here 7); a backward with that gradient leaves
    it as is, one with another (3) rescales it.  Both match the fp32 oracle,
    ignored targets included."""
    torch.manual_seed(4)
    M = 133
    logits = (torch.randn(M, ld, device="cuda") * 3).to(dtype)[:, :V]
    tgt = torch.randint(0, V, (M,), device="cuda")
    tgt[7] = -100
    ref_l = logits.detach().float().requires_grad_()
    ref = F.cross_entropy(ref_l, tgt)
    (ref * mult).backward()
    lg = logits.requires_grad_()
    seed = torch.full((1,), 7.0, device="cuda")
    with ops.expected_loss_grad(seed):
        loss = ops.cross_entropy(lg, tgt)
    assert float(loss) == pytest.approx(float(ref), rel=1e-5, abs=1e-5)
    (loss * mult).backward()
    rt, at = _tol(dtype)
    torch.testing.assert_close(lg.grad.float(), ref_l.grad, rtol=rt, atol=at * 0.05)
