"""GPT (GPT-2 family) decoder on the fused sm_100a ops.

Architecture = the reference example's ``TinyGPT`` scaled to any size
(``examples/train_lm.py:62-115``): learned token + position embeddings,
pre-LayerNorm blocks with a fused qkv projection, causal attention, an
output projection, a 4x GELU MLP, a final LayerNorm and a head tied to the
token embedding.  Module and parameter names are the same (``wte``, ``wpe``,
``blocks.i.ln1``, ``blocks.i.attn.qkv``, ``blocks.i.attn.proj``,
``blocks.i.ln2``, ``blocks.i.mlp.0``, ``blocks.i.mlp.2``, ``ln_f``, ``head``),
so state dicts move between the two.

Execution differs: every residual add is fused into the LayerNorm that
follows it (``ops.add_norm``), bias+GELU is one pass that also keeps the
pre-activation for backward, and with ``targets`` the loss is the fused
cross-entropy over the model-dtype logits (no fp32 logits are ever
materialized).  GPT-2 sizes: :func:`gpt2_small` (124M), :func:`gpt2_xl`.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from ..activation_checkpointing import checkpoint
from ..ops import nn as ops


@dataclass
class GPTConfig:
    vocab_size: int = 50257
    block_size: int = 1024
    n_layer: int = 12
    n_head: int = 12
    n_embd: int = 768
    activation_checkpointing: bool = False
    ln_eps: float = 1e-5


def gpt2_small(**kw) -> GPTConfig:
    return GPTConfig(n_layer=12, n_head=12, n_embd=768, **kw)


def gpt2_xl(**kw) -> GPTConfig:
    return GPTConfig(n_layer=48, n_head=25, n_embd=1600, **kw)


class CausalSelfAttention(nn.Module):
    def __init__(self, n_embd: int, n_head: int):
        super().__init__()
        self.n_head = n_head
        self.head_dim = n_embd // n_head
        self.qkv = nn.Linear(n_embd, 3 * n_embd)
        self.proj = nn.Linear(n_embd, n_embd)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        B, T, C = h.shape
        qkv = ops.linear(h, self.qkv.weight, self.qkv.bias).view(B, T, 3, self.n_head,
                                                                 self.head_dim)
        att = ops.attention_qkv(qkv)
        return ops.linear(att, self.proj.weight, self.proj.bias)


class Block(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        C = cfg.n_embd
        self.eps = cfg.ln_eps
        self.ln1 = nn.LayerNorm(C, eps=cfg.ln_eps)
        self.attn = CausalSelfAttention(C, cfg.n_head)
        self.ln2 = nn.LayerNorm(C, eps=cfg.ln_eps)
        self.mlp = nn.Sequential(nn.Linear(C, 4 * C), nn.GELU(), nn.Linear(4 * C, C))

    def forward(self, x: torch.Tensor, delta: Optional[torch.Tensor]):
        """(residual stream, pending residual delta) -> the same after this block.

        The pending delta (the previous block's MLP output) is added inside
        this block's first LayerNorm kernel."""
        if delta is None:
            h = ops.norm(x, self.ln1.weight, self.ln1.bias, self.eps)
        else:
            x, h = ops.add_norm(x, delta, self.ln1.weight, self.ln1.bias, self.eps)
        a = self.attn(h)
        x, h = ops.add_norm(x, a, self.ln2.weight, self.ln2.bias, self.eps)
        fc, fc2 = self.mlp[0], self.mlp[2]
        m = ops.mlp_gelu(h, fc.weight, fc.bias, fc2.weight, fc2.bias)
        return x, m


class GPT(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.config = cfg
        self.block_size = cfg.block_size
        self.wte = nn.Embedding(cfg.vocab_size, cfg.n_embd)
        self.wpe = nn.Embedding(cfg.block_size, cfg.n_embd)
        self.blocks = nn.ModuleList(Block(cfg) for _ in range(cfg.n_layer))
        self.ln_f = nn.LayerNorm(cfg.n_embd, eps=cfg.ln_eps)
        self.head = nn.Linear(cfg.n_embd, cfg.vocab_size, bias=False)
        self.head.weight = self.wte.weight

    def forward(self, idx: torch.Tensor, targets: Optional[torch.Tensor] = None):
        """Logits [B, T, V] or, with ``targets``, the mean cross-entropy loss."""
        B, T = idx.shape
        if T > self.block_size:
            raise ValueError(f"sequence length {T} > block_size {self.block_size}")
        x = ops.embedding(idx, self.wte.weight, self.wpe.weight[:T] if not idx.is_cuda
                          else self.wpe.weight)
        delta = None
        for blk in self.blocks:
            if self.config.activation_checkpointing and self.training and torch.is_grad_enabled():
                x, delta = checkpoint(blk, x, delta)
            else:
                x, delta = blk(x, delta)
        _, h = ops.add_norm(x, delta, self.ln_f.weight, self.ln_f.bias, self.config.ln_eps)
        logits = ops.linear(h, self.head.weight, pad_out=64)
        if targets is None:
            return logits
        return ops.cross_entropy(logits, targets)

    def num_params(self) -> int:
        return sum(p.numel() for p in self.parameters())


@torch.no_grad()
def init_gpt2_(model: nn.Module, std: float = 0.02) -> nn.Module:
    """GPT-2 initialisation: N(0, std) weights for linears and embeddings,
    zero biases, unit LayerNorm scales."""
    for m in model.modules():
        if isinstance(m, (nn.Linear, nn.Embedding)):
            m.weight.normal_(0.0, std)
            if getattr(m, "bias", None) is not None:
                m.bias.zero_()
        elif isinstance(m, nn.LayerNorm):
            m.weight.fill_(1.0)
            m.bias.zero_()
    return model
