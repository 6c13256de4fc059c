"""Native tcgen05 causal flash attention against an fp32 PyTorch reference."""

import math

import pytest
import torch

from minispeed_b200.ops import attention as A

pytestmark = pytest.mark.gpu


def _ref(qkv, H, Hkv):
    """fp32 causal attention of a [B, T, H + 2Hkv, D] projection -> (out, lse2)."""
    x = qkv.float()
    B, T, _, D = x.shape
    q, k, v = x[:, :, :H], x[:, :, H:H + Hkv], x[:, :, H + Hkv:]
    rep = H // Hkv
    k = k.repeat_interleave(rep, dim=2)
    v = v.repeat_interleave(rep, dim=2)
    s = torch.einsum("bthd,bshd->bhts", q, k) / math.sqrt(D)
    mask = torch.ones(T, T, dtype=torch.bool, device=x.device).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    lse2 = torch.logsumexp(s, dim=-1) / math.log(2.0)
    o = torch.einsum("bhts,bshd->bthd", s.softmax(-1), v)
    return o.reshape(B, T, H * D), lse2


SHAPES = [(2, 256, 4, 4, 64), (1, 200, 2, 2, 64), (2, 384, 8, 2, 64), (1, 1024, 2, 2, 64),
          (1, 256, 4, 2, 128)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("B,T,H,Hkv,D", SHAPES)
def test_forward_matches_reference(B, T, H, Hkv, D, dtype):
    torch.manual_seed(0)
    qkv = torch.randn(B, T, H + 2 * Hkv, D, device="cuda").to(dtype)
    out = A.attention_gqa(qkv, H, Hkv)
    ref, _ = _ref(qkv, H, Hkv)
    tol = 2e-2 if dtype == torch.bfloat16 else 4e-3
    torch.testing.assert_close(out.float(), ref, atol=tol, rtol=tol)


@pytest.mark.parametrize("B,T,H,Hkv,D", SHAPES[:3])
def test_lse_matches_reference(B, T, H, Hkv, D):
    torch.manual_seed(1)
    qkv = torch.randn(B, T, H + 2 * Hkv, D, device="cuda").half()
    from minispeed_b200.ops import _ext, gemm
    out = torch.empty(B * T, H * D, device="cuda", dtype=torch.half)
    lse = torch.empty(B * H, T, device="cuda", dtype=torch.float32)
    _ext.get().attention_fwd(qkv.view(B * T, -1), 0, H * D, (H + Hkv) * D, out, lse, B, T, H, Hkv,
                             D, 1.0 / math.sqrt(D), gemm.error_word(qkv.device), gemm.TIMEOUT_S)
    _, ref = _ref(qkv, H, Hkv)
    torch.testing.assert_close(lse.view(B, H, T), ref, atol=2e-3, rtol=1e-4)
    gemm.check()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
# the last two launch more key blocks than the GPU has SMs, so the persistent
# backward kernel walks several work items per CTA (GQA and a ragged length)
@pytest.mark.parametrize("B,T,H,Hkv,D", SHAPES + [(1, 384, 4, 1, 128), (4, 1024, 12, 6, 64),
                                                  (20, 200, 8, 8, 64)])
def test_backward_matches_reference(B, T, H, Hkv, D, dtype):
    torch.manual_seed(2)
    qkv = torch.randn(B, T, H + 2 * Hkv, D, device="cuda").to(dtype).requires_grad_()
    dout = torch.randn(B, T, H * D, device="cuda").to(dtype)
    out = A.attention_gqa(qkv, H, Hkv)
    (g,) = torch.autograd.grad(out, (qkv,), dout)
    x = qkv.detach().float().requires_grad_()
    ref, _ = _ref(x, H, Hkv)
    (gr,) = torch.autograd.grad(ref, (x,), dout.float())
    scale = gr.abs().amax().item()
    tol = (3e-2 if dtype == torch.bfloat16 else 6e-3) * max(scale, 1.0)
    torch.testing.assert_close(g.float(), gr, atol=tol, rtol=0.0)


def test_gpt_qkv_layout_matches_sdpa(monkeypatch):
    torch.manual_seed(3)
    qkv = torch.randn(2, 512, 3, 6, 64, device="cuda").half().requires_grad_()
    dout = torch.randn(2, 512, 6 * 64, device="cuda").half()
    out = A.attention_qkv(qkv)
    (g,) = torch.autograd.grad(out, (qkv,), dout)
    monkeypatch.setenv("MSB_ATTN", "sdpa")
    out2 = A.attention_qkv(qkv)
    (g2,) = torch.autograd.grad(out2, (qkv,), dout)
    torch.testing.assert_close(out, out2, atol=4e-3, rtol=1e-2)
    torch.testing.assert_close(g.float(), g2.float(), atol=2e-2, rtol=2e-2)
