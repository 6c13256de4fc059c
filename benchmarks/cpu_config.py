"""The CPU benchmark configuration, both engines, wall-clock tokens/s.

    python benchmarks/cpu_config.py [--steps K] [--warmup W] [--threads T]

The first benchmark configuration runs on CPU: two gloo ranks, ZeRO-2,
fp32, a 4-layer decoder-only GPT (d_model 128, 4 heads, MLP 512 with GELU,
learned position embeddings, vocab 256, seq 64), micro-batch 8 per rank,
gas 2, AdamW lr 1e-3 wd 0.01, clipping 1.0, uniform-random tokens with
targets the inputs shifted by one.  Each rank trains this library's GPT
through ``minispeed_b200`` and the same weights in a stock-PyTorch module of
the reference example's architecture through the reference engine in
``baseline/_ref`` (when installed).  W untimed steps, then K steps between
barriers; the reported time is the slowest rank's.  Each engine runs twice
(order A B B A, same initial weights) and keeps its faster run.  Prints one JSON line
per engine.  With no GPU the CUDA kernels are not involved: this measures
the engine's host-side pipeline and PyTorch's CPU operators.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
import time

import torch
import torch.multiprocessing as mp
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
WORLD, GAS, MICRO, VOCAB, SEQ = 2, 2, 8, 256, 64
SPEC = dict(vocab=VOCAB, seq=SEQ, layers=4, heads=4, embd=128, mlp=512, ckpt=False)


def _config() -> dict:
    return {"train_micro_batch_size_per_gpu": MICRO, "gradient_accumulation_steps": GAS,
            "gradient_clipping": 1.0, "dtype": "fp32",
            "optimizer": {"type": "AdamW", "params": {"lr": 1e-3, "weight_decay": 0.01}},
            "zero_optimization": {"stage": 2}, "steps_per_print": 10 ** 6}


def _worker(rank, port, steps, warmup, threads, out_dir):
    sys.path.insert(0, ROOT)
    torch.set_num_threads(threads)
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(WORLD), "LOCAL_RANK": str(rank),
                       "MINISPEED_BACKEND": "gloo", "MINISPEED_DEVICE": "cpu"})
    import minispeed_b200 as ours
    from bench import RefGPT
    from minispeed_b200.models import GPT, GPTConfig, init_gpt2_

    ours.comm.init_distributed()
    torch.manual_seed(0)
    mine = init_gpt2_(GPT(GPTConfig(vocab_size=VOCAB, block_size=SEQ, n_layer=4, n_head=4,
                                    n_embd=128)))
    arms = [("minispeed_b200", ours, mine, lambda e, x, y: e(x, targets=y))]
    if os.path.isdir(os.path.join(REF, "minispeed")):
        sys.path.insert(0, REF)
        ref = importlib.import_module("minispeed")
        stock = RefGPT(SPEC)
        stock.load_state_dict(mine.state_dict())
        arms.append(("reference", ref, stock, lambda e, x, y: F.cross_entropy(
            e(x).float().view(-1, VOCAB), y.reshape(-1))))
    g = torch.Generator().manual_seed(1000 + rank)
    tokens = torch.randint(0, VOCAB, (warmup + steps, GAS, MICRO, SEQ + 1), generator=g)
    results = {}
    # each engine runs twice, in the order A B B A, from the same initial
    # weights; the faster of its two runs is kept
    order = arms + arms[::-1]
    inits = {name: {k: v.clone() for k, v in model.state_dict().items()}
             for name, _, model, _ in arms}
    for name, lib, model, loss_fn in order:
        model.load_state_dict(inits[name])
        eng = lib.initialize(model=model, config=_config())

        def step(s):
            loss = None
            for m in range(GAS):
                t = tokens[s, m]
                loss = loss_fn(eng, t[:, :-1], t[:, 1:])
                eng.backward(loss)
                eng.step()
            return float(loss.detach())

        for s in range(warmup):
            step(s)
        torch.distributed.barrier()
        t0 = time.perf_counter()
        last = None
        for s in range(warmup, warmup + steps):
            last = step(s)
        torch.distributed.barrier()
        dt = torch.tensor([time.perf_counter() - t0], dtype=torch.float64)
        torch.distributed.all_reduce(dt, op=torch.distributed.ReduceOp.MAX)
        if name not in results or float(dt) < results[name][0]:
            results[name] = (float(dt), last)
    if rank == 0:
        with open(os.path.join(out_dir, "result.json"), "w") as fh:
            json.dump(results, fh)
    ours.comm.destroy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--threads", type=int, default=max(1, (os.cpu_count() or 2) // WORLD))
    a = ap.parse_args()
    import socket
    import tempfile
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as out:
        mp.spawn(_worker, args=(port, a.steps, a.warmup, a.threads, out), nprocs=WORLD, join=True)
        with open(os.path.join(out, "result.json")) as fh:
            results = json.load(fh)
    tokens_per_step = WORLD * GAS * MICRO * SEQ
    for name, (secs, last_loss) in results.items():
        print(json.dumps({
            "impl": name, "metric": "tokens/sec whole job (max over ranks), CPU gloo",
            "value": round(tokens_per_step * a.steps / secs, 1), "unit": "tokens/s",
            "n_ranks": WORLD, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(1000 * secs / a.steps, 2), "dtype": "fp32",
            "data": "synthetic uniform-random token ids", "threads_per_rank": a.threads,
            "final_loss": round(last_loss, 4),
            "config": {"model": "GPT 4L d128 4H MLP512 vocab256", "seq_len": SEQ,
                       "micro_batch": MICRO, "gas": GAS, "parallelism": "dp2 ZeRO-2 (gloo)"}}))


if __name__ == "__main__":
    main()
