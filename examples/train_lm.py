"""Train a small character-level GPT with minispeed_b200.

The whole training surface in one script: DeepSpeed-style JSON config (or
flags), fp16 loss scaling / bf16, ZeRO stages 0-3, gradient accumulation,
WarmupDecayLR, periodic and final checkpoints, resume, rank-0 logging of
loss / perplexity / lr / grad norm / loss scale / tokens per second / phase
timers, and a short sample at the end (capabilities of the reference
example, ``examples/train_lm.py``).

    python examples/train_lm.py --dtype fp16 --zero 2
    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 examples/train_lm.py --zero 3
    python examples/train_lm.py --resume out            # continue from out/latest
    python examples/train_lm.py --resume out/global_step150   # a given tag
    python examples/train_lm.py --config examples/ds_config_tiny.json --steps 50
    python examples/train_lm.py --arch llama --zero 3     # Llama-3 family block
"""

from __future__ import annotations

import argparse
import math
import os
import sys
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import minispeed_b200 as ms  # noqa: E402
from minispeed_b200 import comm  # noqa: E402
from minispeed_b200.models import GPT, GPTConfig, Llama, LlamaConfig  # noqa: E402

TEXT = """
a flat buffer holds every weight of a group in one piece, so one kernel can
update it and one collective can move it. each rank keeps a slice of the
optimizer state, adds the gradients of its peers for its own slice, steps
its slice, and hands the new weights back to everyone. when the loss scale
is too high an infinity appears, the step is skipped and the scale halves.
when many steps go well the scale doubles again. the learning rate climbs
during warm up and then falls in a straight line to its floor. a checkpoint
keeps the shards, the scaler and the schedule, so training picks up where it
stopped. the small model reads these lines over and over and learns which
letter comes next.
"""


def encode():
    vocab = sorted(set(TEXT))
    stoi = {c: i for i, c in enumerate(vocab)}
    return torch.tensor([stoi[c] for c in TEXT]), vocab, stoi


def batch(ids, block, size, offset, device):
    span = max(1, ids.numel() - block - 1)
    starts = [(offset + 13 * i) % span for i in range(size)]
    x = torch.stack([ids[s:s + block] for s in starts])
    y = torch.stack([ids[s + 1:s + block + 1] for s in starts])
    return x.to(device), y.to(device)


def make_config(a) -> dict:
    if a.config:
        return a.config
    cfg = {
        "train_micro_batch_size_per_gpu": a.batch_size,
        "gradient_accumulation_steps": a.gas,
        "gradient_clipping": 1.0,
        "dtype": a.dtype,
        "optimizer": {"type": "AdamW", "params": {"lr": a.lr, "betas": [0.9, 0.95],
                                                  "eps": 1e-8, "weight_decay": 0.1}},
        "scheduler": {"type": "WarmupDecayLR", "params": {
            "warmup_min_lr": a.lr * 0.1, "warmup_max_lr": a.lr,
            "warmup_num_steps": a.warmup, "total_num_steps": a.steps}},
        "zero_optimization": {"stage": a.zero},
        "steps_per_print": a.log_every,
    }
    if a.dtype == "fp16":
        cfg["fp16"] = {"enabled": True, "loss_scale": 0, "initial_scale_power": 16,
                       "loss_scale_window": 200}
    elif a.dtype == "bf16":
        cfg["bf16"] = {"enabled": True}
    return cfg


def gpu_times(engine) -> str:
    """GPU time per phase when ``"b200": {"device_timers": true}`` is set."""
    ms_ = engine.device_time_ms()
    return "".join(f" | gpu {k}: {v:.1f}ms" for k, v in ms_.items())


def resume(engine, path: str) -> None:
    """``path`` is a save dir (follow its ``latest`` file), a ``dir/tag``
    checkpoint directory, or the ``dir/latest`` file itself."""
    path = os.path.normpath(path)
    if os.path.isfile(os.path.join(path, "latest")):
        engine.load_checkpoint(path)
        return
    parent, tag = os.path.split(path)
    engine.load_checkpoint(parent, tag=None if tag == "latest" else tag)


def main():
    p = argparse.ArgumentParser(description="minispeed_b200 character LM example")
    p.add_argument("--steps", type=int, default=300)
    p.add_argument("--batch-size", type=int, default=8)
    p.add_argument("--gas", type=int, default=2)
    p.add_argument("--dtype", default="fp16", choices=["fp32", "fp16", "bf16"])
    p.add_argument("--zero", type=int, default=2, choices=[0, 1, 2, 3])
    p.add_argument("--lr", type=float, default=3e-3)
    p.add_argument("--warmup", type=int, default=30)
    p.add_argument("--block-size", type=int, default=64)
    p.add_argument("--n-embd", type=int, default=128)
    p.add_argument("--n-layer", type=int, default=2)
    p.add_argument("--n-head", type=int, default=4)
    p.add_argument("--arch", default="gpt", choices=["gpt", "llama"],
                   help="gpt: the reference example's TinyGPT; llama: RMSNorm, RoPE, GQA, SwiGLU")
    p.add_argument("--n-kv-head", type=int, default=2, help="llama: key/value heads")
    p.add_argument("--log-every", type=int, default=25)
    p.add_argument("--ckpt-dir", default="out")
    p.add_argument("--save-every", type=int, default=150)
    p.add_argument("--resume", default=None, help="checkpoint dir (uses latest) or dir/tag")
    p.add_argument("--config", default=None, help="DeepSpeed-style JSON config path")
    a = p.parse_args()

    comm.init_distributed()
    rank, world = comm.get_rank(), comm.get_world_size()
    device = comm.resolve_device()
    ms.set_seed(1337)
    ids, vocab, stoi = encode()
    if a.arch == "llama":
        model = Llama(LlamaConfig(vocab_size=len(vocab), block_size=a.block_size,
                                  n_layer=a.n_layer, n_head=a.n_head, n_kv_head=a.n_kv_head,
                                  n_embd=a.n_embd, ffn_hidden=4 * a.n_embd, rope_theta=10000.0))
    else:
        model = GPT(GPTConfig(vocab_size=len(vocab), block_size=a.block_size, n_layer=a.n_layer,
                              n_head=a.n_head, n_embd=a.n_embd))
    engine, _, _, sched = ms.initialize(model=model, model_parameters=model.parameters(),
                                        config=make_config(a))
    if a.resume:
        resume(engine, a.resume)
        if rank == 0:
            print(f"resumed {a.resume} at step {engine.global_steps}")
    if rank == 0:
        print(f"minispeed_b200 {ms.__version__} world={world} device={device} "
              f"dtype={engine.config.dtype} zero={engine.config.zero_stage} "
              f"params={sum(t.numel() for t in model.parameters()) / 1e3:.1f}K "
              f"batch={engine.config.train_batch_size} collectives={engine.collectives}")

    tokens = engine.config.train_batch_size * a.block_size
    t0, loss = time.time(), None
    while engine.global_steps < a.steps:
        base = engine.global_steps * engine.gas * a.batch_size * world
        for m in range(engine.gas):
            x, y = batch(ids, a.block_size, a.batch_size,
                         base + (m * world + rank) * a.batch_size, device)
            loss = engine(x, targets=y)
            engine.backward(loss)
            applied = engine.step()
        if not applied:
            continue
        step = engine.global_steps
        if rank == 0 and (step % a.log_every == 0 or step == 1):
            dt = max(time.time() - t0, 1e-9)
            lv = float(loss.detach())
            n = a.log_every if step > 1 else 1
            print(f"step {step:5d}/{a.steps} | loss {lv:.4f} | ppl {math.exp(min(lv, 20)):8.2f}"
                  f" | lr {sched.get_last_lr():.2e} | norm {engine.grad_norm:.3f}"
                  f" | scale {engine.get_loss_scale():.0f} | tok/s {n * tokens / dt:,.0f}"
                  f" | {engine.timers.log()}{gpu_times(engine)}", flush=True)
            engine.timers.reset()
            engine.device_timers.reset()
            t0 = time.time()
        if a.save_every and step % a.save_every == 0:
            engine.save_checkpoint(a.ckpt_dir)
    engine.save_checkpoint(a.ckpt_dir)

    # the sample reads whole parameters; at ZeRO-3 gathering them is a
    # collective, so every rank takes part before rank 0 samples alone
    engine.eval()
    engine.optimizer.gather_parameters()
    if rank == 0:
        print(f"done: loss {float(loss.detach()):.4f}, skipped {engine.skipped_steps}, "
              f"checkpoint in {a.ckpt_dir}")
        ctx = torch.tensor([[stoi[c] for c in "the "]], device=device)
        with torch.no_grad():
            for _ in range(60):
                logits = engine(ctx[:, -a.block_size:])
                probs = torch.softmax(logits[:, -1].float() / 0.8, dim=-1)
                ctx = torch.cat([ctx, torch.multinomial(probs, 1)], dim=1)
        print("sample:", repr("".join(vocab[int(i)] for i in ctx[0].tolist())))
    comm.barrier()
    engine.close()
    comm.destroy()


if __name__ == "__main__":
    main()
