"""Shared models, data and loops for the tests.

The data layout mirrors how data parallelism splits a batch: tensors are
``[steps, gas, world*micro, features]`` and rank ``r`` takes columns
``r*micro:(r+1)*micro``, so the ranks' shards union to the batch a single
process would train on.
"""

from __future__ import annotations

import os
import socket

import torch
import torch.nn as nn
import torch.nn.functional as F

IN_DIM = 8


class TinyNet(nn.Module):
    """8 -> 32 -> 32 -> 1 regression net (Tanh, ReLU, LayerNorm)."""

    def __init__(self):
        super().__init__()
        self.l1 = nn.Linear(IN_DIM, 32)
        self.l2 = nn.Linear(32, 32)
        self.norm = nn.LayerNorm(32)
        self.out = nn.Linear(32, 1)

    def forward(self, x):
        h = torch.tanh(self.l1(x))
        h = self.norm(torch.relu(self.l2(h)))
        return self.out(h)


def make_net(seed: int = 1234, device="cpu") -> TinyNet:
    torch.manual_seed(seed)
    return TinyNet().to(device)


def make_data(steps: int, gas: int, world: int, micro: int, seed: int = 7, device="cpu"):
    gen = torch.Generator().manual_seed(seed)
    rows = steps * gas * world * micro
    x = torch.randn(rows, IN_DIM, generator=gen).view(steps, gas, world * micro, IN_DIM)
    y = torch.randn(rows, 1, generator=gen).view(steps, gas, world * micro, 1)
    return x.to(device), y.to(device)


def rank_slice(t: torch.Tensor, rank: int, micro: int) -> torch.Tensor:
    return t[:, :, rank * micro:(rank + 1) * micro]


def mse(pred, target):
    return F.mse_loss(pred.float(), target.float())


def config(micro=4, gas=2, lr=1e-3, wd=0.01, clip=1.0, dtype="fp32", stage=0,
           warmup=0, total=None, scheduler="WarmupLR", scale_power=8, window=100,
           **extra) -> dict:
    sched = {"warmup_min_lr": 0.0, "warmup_max_lr": lr, "warmup_num_steps": warmup}
    if total is not None:
        sched["total_num_steps"] = total
    cfg = {
        "train_micro_batch_size_per_gpu": micro,
        "gradient_accumulation_steps": gas,
        "gradient_clipping": clip,
        "dtype": dtype,
        "optimizer": {"type": "AdamW", "params": {"lr": lr, "betas": [0.9, 0.999],
                                                  "eps": 1e-8, "weight_decay": wd}},
        "scheduler": {"type": scheduler, "params": sched},
        "zero_optimization": {"stage": stage},
        "steps_per_print": 1000,
    }
    if dtype == "fp16":
        cfg["fp16"] = {"enabled": True, "loss_scale": 0, "initial_scale_power": scale_power,
                       "loss_scale_window": window}
    elif dtype == "bf16":
        cfg["bf16"] = {"enabled": True}
    cfg.update(extra)
    return cfg


def run(engine, x, y, steps: int, gas: int, device="cpu"):
    """forward/backward every micro-batch, step() after each; returns losses."""
    losses = []
    engine.train()
    for s in range(steps):
        for m in range(gas):
            loss = mse(engine(x[s, m].to(device)), y[s, m].to(device))
            losses.append(float(loss.detach()))
            engine.backward(loss)
            engine.step()
    return losses


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return int(s.getsockname()[1])


def set_rank_env(rank: int, world: int, port: int, backend: str, device: str) -> None:
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "MINISPEED_BACKEND": backend, "MINISPEED_DEVICE": device,
                       "MINISPEED_PG_TIMEOUT_S": "120"})
