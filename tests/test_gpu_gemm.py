"""tcgen05 GEMM numerics against an fp32 PyTorch product."""

import pytest
import torch

from minispeed_b200.ops import _ext, gemm

pytestmark = pytest.mark.gpu


def _ref(A, B, bias=None):
    r = A.float() @ B.float().t()
    if bias is not None:
        r = r + bias.float()
    return r


def _check(out, ref, K):
    # fp32 accumulation; the only rounding is the final 16-bit cast
    scale = ref.abs().max().item() + 1e-6
    err = (out.float() - ref).abs().max().item()
    assert err <= 1e-2 * scale + 1e-3, (err, scale, K)


@pytest.fixture(autouse=True, params=["auto", "1cta", "2cta"])
def _variant(request, monkeypatch):
    monkeypatch.setenv("MSB_GEMM_VARIANT", request.param)
    yield request.param


@pytest.fixture(autouse=True)
def _native():
    assert gemm.native_enabled(), "tcgen05 gemm must be built"
    yield
    gemm.check()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("a_k,b_k", [(True, True), (True, False), (False, False), (False, True)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 192), (300, 200, 130),
                                   (1000, 768, 768)])
def test_gemm_majors(dtype, a_k, b_k, M, N, K):
    torch.manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda").to(dtype)
    B = torch.randn(N, K, device="cuda").to(dtype)
    a = A if a_k else A.t().contiguous()
    b = B if b_k else B.t().contiguous()
    out = gemm.gemm(a, b, a_kmajor=a_k, b_kmajor=b_k)
    torch.cuda.synchronize()
    _check(out, _ref(A, B), K)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gemm_bias_and_padded_output(dtype):
    M, N, K = 513, 1001, 256
    A = torch.randn(M, K, device="cuda").to(dtype)
    B = torch.randn(N, K, device="cuda").to(dtype)
    bias = torch.randn(N, device="cuda").to(dtype)
    buf = torch.full((M, 1024), 7.0, device="cuda", dtype=dtype)
    out = buf[:, :N]
    gemm.gemm(A, B, a_kmajor=True, b_kmajor=True, bias=bias, out=out)
    _check(out, _ref(A, B, bias), K)
    assert torch.all(buf[:, N:] == 7.0)  # padding untouched


@pytest.mark.parametrize("M,N,K", [(2304, 768, 16384), (768, 3072, 4096), (64, 64, 8192)])
def test_gemm_wgrad_shapes_split_k(M, N, K):
    """dW = dY^T X with both operands M-major and a long reduction (split-K)."""
    dy = (torch.randn(K, M, device="cuda") * 0.1).half()
    x = (torch.randn(K, N, device="cuda") * 0.1).half()
    plan = _ext.get().gemm_plan(M, N, K)
    out = gemm.gemm(dy, x, a_kmajor=False, b_kmajor=False)
    _check(out, dy.float().t() @ x.float(), K)
    assert plan[0] in (128, 256, 512)


def test_gemm_accumulate():
    M, N, K = 640, 384, 512
    A = torch.randn(M, K, device="cuda").half()
    B = torch.randn(N, K, device="cuda").half()
    C0 = torch.randn(M, N, device="cuda").half()
    out = C0.clone()
    gemm.gemm(A, B, a_kmajor=True, b_kmajor=True, out=out, accumulate=True)
    _check(out, _ref(A, B) + C0.float(), K)


def test_gemm_unaligned_operand_is_copied():
    W = torch.randn(777 * 65 + 3, device="cuda").half()
    w = W[3:].view(777, 65)[:, :64]   # odd base offset and odd row stride
    x = torch.randn(200, 64, device="cuda").half()
    out = gemm.gemm(x, w, a_kmajor=True, b_kmajor=True)
    _check(out, _ref(x, w), 64)


def test_gpt2_shapes_match_library():
    """The GPT-2-small training shapes, fwd/dgrad/wgrad, against fp32."""
    Mt, C = 4096, 768
    for N, K in ((2304, C), (C, C), (4 * C, C), (C, 4 * C)):
        x = (torch.randn(Mt, K, device="cuda") * 0.5).half()
        w = (torch.randn(N, K, device="cuda") * 0.05).half()
        dy = (torch.randn(Mt, N, device="cuda") * 0.5).half()
        _check(gemm.linear_fwd(x, w, None), _ref(x, w), K)
        _check(gemm.linear_dgrad(dy, w), dy.float() @ w.float(), N)
        _check(gemm.linear_wgrad(dy, x), dy.float().t() @ x.float(), Mt)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_epilogue_bias_gelu_and_dgelu(dtype):
    from minispeed_b200.ops.nn import gelu_grad_reference

    M, N, K = 1000, 3072, 768
    A = (torch.randn(M, K, device="cuda") * 0.5).to(dtype)
    B = (torch.randn(N, K, device="cuda") * 0.05).to(dtype)
    bias = (torch.randn(N, device="cuda") * 0.1).to(dtype)
    u = torch.empty(M, N, device="cuda", dtype=dtype)
    h = torch.empty_like(u)
    gemm.gemm(A, B, a_kmajor=True, b_kmajor=True, bias=bias, out=u, mode=gemm.EPI_BIAS_GELU,
              aux=h)
    ref_u = _ref(A, B, bias)
    _check(u, ref_u, K)
    _check(h, torch.nn.functional.gelu(u.float()), K)
    # dgrad with gelu' fused: du = (dY @ W) * gelu'(u)
    dY = torch.randn(M, 768, device="cuda").to(dtype)
    W = (torch.randn(768, N, device="cuda") * 0.05).to(dtype)
    du = torch.empty(M, N, device="cuda", dtype=dtype)
    gemm.gemm(dY, W, a_kmajor=True, b_kmajor=False, out=du, mode=gemm.EPI_DGELU, aux=u)
    ref = (dY.float() @ W.float()).to(dtype).float() * gelu_grad_reference(u.float())
    _check(du, ref, 768)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_mlp_gelu_op_and_grad_sinks(dtype):
    from minispeed_b200.ops import nn as ops

    torch.manual_seed(5)
    C, F = 256, 1024
    fc = torch.nn.Linear(C, F).cuda().to(dtype)
    fc2 = torch.nn.Linear(F, C).cuda().to(dtype)
    x = (torch.randn(4, 64, C, device="cuda")).to(dtype).requires_grad_()
    params = list(fc.parameters()) + list(fc2.parameters())
    # pre-bound gradient buffers holding earlier contributions (engine arenas)
    for p in params:
        p.grad = torch.full_like(p, 0.25)
    out = ops.mlp_gelu(x, fc.weight, fc.bias, fc2.weight, fc2.bias)
    g = torch.randn_like(out)
    out.backward(g)
    ref_params = [p.detach().float().requires_grad_() for p in params]
    xf = x.detach().float().requires_grad_()
    rf = torch.nn.functional.linear(torch.nn.functional.gelu(
        torch.nn.functional.linear(xf, ref_params[0], ref_params[1])), ref_params[2], ref_params[3])
    rf.backward(g.float())
    _check(out, rf.detach(), F)
    _check(x.grad, xf.grad, F)
    for p, r in zip(params, ref_params):
        _check(p.grad, r.grad + 0.25, 4 * 64)


SK = (512, -1)   # the 2-CTA pair kernel with stream-K


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("a_k,b_k", [(True, True), (True, False), (False, False)])
@pytest.mark.parametrize("M,N,K", [(16384, 768, 3072), (2304, 768, 16384), (300, 200, 4160),
                                   (1000, 768, 768), (512, 512, 64)])
def test_stream_k(dtype, a_k, b_k, M, N, K, _variant):
    """Stream-K cuts tiles x K-slices evenly over the resident pairs; a tile
    split between pairs is finished by the pair holding its first slice.
    Two launches in a row: the tile counters must be back at zero."""
    if _variant != "auto":
        pytest.skip("forced plan; one variant is enough")
    torch.manual_seed(M + N + K)
    A = (torch.randn(M, K, device="cuda") * 0.1).to(dtype)
    B = (torch.randn(N, K, device="cuda") * 0.1).to(dtype)
    a = A if a_k else A.t().contiguous()
    b = B if b_k else B.t().contiguous()
    ref = _ref(A, B)
    for _ in range(2):
        out = gemm.gemm(a, b, a_kmajor=a_k, b_kmajor=b_k, plan=SK)
        torch.cuda.synchronize()
        _check(out, ref, K)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_stream_k_epilogues(dtype, _variant):
    """Bias, accumulate and the GELU modes are applied once, by the pair that
    finishes each tile."""
    if _variant != "auto":
        pytest.skip("forced plan; one variant is enough")
    M, N, K = 2000, 1000, 2112
    torch.manual_seed(5)
    A = (torch.randn(M, K, device="cuda") * 0.05).to(dtype)
    B = (torch.randn(N, K, device="cuda") * 0.05).to(dtype)
    bias = torch.randn(N, device="cuda").to(dtype)
    out = gemm.gemm(A, B, a_kmajor=True, b_kmajor=True, bias=bias, plan=SK)
    _check(out, _ref(A, B, bias), K)
    C0 = torch.randn(M, N, device="cuda").to(dtype)
    C = C0.clone()
    gemm.gemm(A, B, a_kmajor=True, b_kmajor=True, out=C, accumulate=True, plan=SK)
    _check(C, C0.float() + _ref(A, B), K)
    u = torch.empty(M, N, device="cuda", dtype=dtype)
    h = torch.empty_like(u)
    gemm.gemm(A, B, a_kmajor=True, b_kmajor=True, bias=bias, out=u, mode=gemm.EPI_BIAS_GELU,
              aux=h, plan=SK)
    uref = _ref(A, B, bias)
    _check(u, uref, K)
    _check(h, torch.nn.functional.gelu(u.float()), K)
    dY = (torch.randn(M, K, device="cuda") * 0.05).to(dtype)
    W = (torch.randn(K, N, device="cuda") * 0.05).to(dtype)
    du = torch.empty(M, N, device="cuda", dtype=dtype)
    gemm.gemm(dY, W, a_kmajor=True, b_kmajor=False, out=du, mode=gemm.EPI_DGELU, aux=u,
              plan=SK)
    from minispeed_b200.ops.nn import gelu_grad_reference
    want = (dY.float() @ W.float()).to(dtype).float() * gelu_grad_reference(u.float())
    _check(du, want, K)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(4096, 3072, 768), (1000, 520, 256)])
def test_dgelu_epilogue_column_sums(dtype, M, N, K, _variant):
    """The dGELU epilogue also writes the column sums of its stored output,
    one fp32 partial row per 32 rows (ragged last group included); their
    finished sum is the bias gradient of the column sums of du itself."""
    torch.manual_seed(M + N)
    dY = (torch.randn(M, K, device="cuda") * 0.05).to(dtype)
    W = (torch.randn(K, N, device="cuda") * 0.05).to(dtype)
    u = torch.randn(M, N, device="cuda").to(dtype)
    du = torch.empty(M, N, device="cuda", dtype=dtype)
    groups = -(-M // 32)
    part = torch.full((groups * N,), float("nan"), device="cuda")
    gemm.gemm(dY, W, a_kmajor=True, b_kmajor=False, out=du, mode=gemm.EPI_DGELU, aux=u,
              colsum=part)
    torch.cuda.synchronize()
    want = du.float().sum(0)
    got = part.view(groups, N).sum(0)
    torch.testing.assert_close(got, want, rtol=1e-3, atol=1e-3 * K ** 0.5)
    out = torch.zeros(N, device="cuda", dtype=dtype)
    _ext.get().colsum_finish(part, groups, out, False)
    torch.testing.assert_close(out.float(), want, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("splits", [2, 4])
@pytest.mark.parametrize("M,N,K", [(3072, 768, 16384), (2304, 768, 16384), (700, 300, 4096)])
def test_pair_split_k_fixup(dtype, splits, M, N, K, _variant):
    """Split-K on the pair kernel with every unit resident: the last split of
    each tile adds the others' fp32 partials and finishes it (bias and
    accumulation applied once); two launches in a row (counters reset)."""
    if _variant != "auto":
        pytest.skip("forced plan; one variant is enough")
    torch.manual_seed(M + splits)
    dy = (torch.randn(K, M, device="cuda") * 0.05).to(dtype)
    x = (torch.randn(K, N, device="cuda") * 0.05).to(dtype)
    bias = torch.randn(N, device="cuda").to(dtype)
    ref = dy.float().t() @ x.float()
    for _ in range(2):
        out = gemm.gemm(dy, x, a_kmajor=False, b_kmajor=False, bias=bias, plan=(512, splits))
        torch.cuda.synchronize()
        _check(out, ref + bias.float(), K)
    C0 = torch.randn(M, N, device="cuda").to(dtype)
    C = C0.clone()
    gemm.gemm(dy, x, a_kmajor=False, b_kmajor=False, out=C, accumulate=True, plan=(512, splits))
    _check(C, C0.float() + ref, K)
