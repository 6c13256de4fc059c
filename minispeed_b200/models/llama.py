"""Llama-3 family decoder on the fused sm_100a ops.

RMSNorm pre-norm blocks, rotary position embeddings (theta 500000 for
Llama 3), grouped-query attention (``n_kv_head`` < ``n_head``), a SwiGLU
feed-forward network and an untied output head.  The projections are fused
for the GEMM kernels: ``attn.qkv`` is [(H + 2*Hkv) * D, C] (q heads, then k,
then v) and ``mlp.gate_up`` is [2F, C] (gate rows, then up rows).  As in the
GPT model, every residual add is fused into the following RMSNorm kernel.

There is no reference counterpart: the reference trains only the example
GPT of ``examples/train_lm.py:97-115``.  The Llama-3-8B shape is the
largest model configuration of the benchmark set this library is measured on.

:func:`llama3_8b` is the Llama-3-8B shape (32 layers, d_model 4096, 32/8
heads, FFN 14336, vocab 128256).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from ..activation_checkpointing import checkpoint
from ..ops import nn as ops


@dataclass
class LlamaConfig:
    vocab_size: int = 128256
    block_size: int = 4096
    n_layer: int = 32
    n_head: int = 32
    n_kv_head: int = 8
    n_embd: int = 4096
    ffn_hidden: int = 14336
    rope_theta: float = 500000.0
    norm_eps: float = 1e-5
    activation_checkpointing: bool = False


def llama3_8b(**kw) -> LlamaConfig:
    return LlamaConfig(**kw)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))


class Attention(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.n_head, self.n_kv_head = cfg.n_head, cfg.n_kv_head
        self.head_dim = cfg.n_embd // cfg.n_head
        qkv_out = (cfg.n_head + 2 * cfg.n_kv_head) * self.head_dim
        self.qkv = nn.Linear(cfg.n_embd, qkv_out, bias=False)
        self.proj = nn.Linear(cfg.n_head * self.head_dim, cfg.n_embd, bias=False)

    def forward(self, h, cos, sin):
        B, T, _ = h.shape
        qkv = ops.linear(h, self.qkv.weight).view(B, T, -1, self.head_dim)
        qkv = ops.rope_qk(qkv, cos, sin, self.n_head, self.n_kv_head)
        att = ops.attention_gqa(qkv, self.n_head, self.n_kv_head)
        return ops.linear(att, self.proj.weight)


class FeedForward(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.gate_up = nn.Linear(cfg.n_embd, 2 * cfg.ffn_hidden, bias=False)
        self.down = nn.Linear(cfg.ffn_hidden, cfg.n_embd, bias=False)

    def forward(self, h):
        return ops.linear(ops.swiglu(ops.linear(h, self.gate_up.weight)), self.down.weight)


class LlamaBlock(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.eps = cfg.norm_eps
        self.attn_norm = RMSNorm(cfg.n_embd, cfg.norm_eps)
        self.attn = Attention(cfg)
        self.ffn_norm = RMSNorm(cfg.n_embd, cfg.norm_eps)
        self.mlp = FeedForward(cfg)

    def forward(self, x, delta: Optional[torch.Tensor], cos, sin):
        if delta is None:
            h = ops.norm(x, self.attn_norm.weight, None, self.eps, rms=True)
        else:
            x, h = ops.add_norm(x, delta, self.attn_norm.weight, None, self.eps, rms=True)
        a = self.attn(h, cos, sin)
        x, h = ops.add_norm(x, a, self.ffn_norm.weight, None, self.eps, rms=True)
        return x, self.mlp(h)


class Llama(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.config = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.n_embd)
        self.blocks = nn.ModuleList(LlamaBlock(cfg) for _ in range(cfg.n_layer))
        self.norm = RMSNorm(cfg.n_embd, cfg.norm_eps)
        self.head = nn.Linear(cfg.n_embd, cfg.vocab_size, bias=False)
        self._rope = None

    def _tables(self, T: int, device):
        hd = self.config.n_embd // self.config.n_head
        if self._rope is None or self._rope[0].shape[0] < T or self._rope[0].device != device:
            self._rope = ops.rope_tables(max(T, self.config.block_size), hd,
                                         self.config.rope_theta, device)
        return self._rope

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None):
        B, T = idx.shape
        cos, sin = self._tables(T, idx.device)
        x = ops.embedding(idx, self.embed.weight)
        delta = None
        for blk in self.blocks:
            if self.config.activation_checkpointing and self.training and torch.is_grad_enabled():
                x, delta = checkpoint(blk, x, delta, cos, sin)
            else:
                x, delta = blk(x, delta, cos, sin)
        _, h = ops.add_norm(x, delta, self.norm.weight, None, self.config.norm_eps, rms=True)
        logits = ops.linear(h, self.head.weight, pad_out=64)
        if targets is None:
            return logits
        return ops.cross_entropy(logits, targets)


@torch.no_grad()
def init_llama_(model: nn.Module, std: float = 0.02) -> nn.Module:
    for m in model.modules():
        if isinstance(m, (nn.Linear, nn.Embedding)):
            m.weight.normal_(0.0, std)
        elif isinstance(m, RMSNorm):
            m.weight.fill_(1.0)
    return model
