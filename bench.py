"""Headline benchmark: training throughput of the BASELINE.json configs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--model gpt2-small|gpt2-xl|llama3-8b]

Default (the headline): GPT-2 small shape (12 layers,
d_model 768, 12 heads, MLP 3072, vocab 50257, seq 1024), fp16 with fp32
masters and dynamic loss scaling (initial_scale_power 16, window 1000), ZeRO
stage 2, micro-batch 16 per GPU, gas 1, AdamW, WarmupDecayLR, gradient
clipping 1.0.  ``--model gpt2-xl`` (config 3): 48 layers, d 1600, 25 heads,
MLP 6400, bf16, ZeRO-1, micro-batch 4, gas 4, clipping 1.0, activation
checkpointing on every block.  ``--model llama3-8b`` (config 4): 32 layers,
d 4096, 32 q / 8 kv heads, SwiGLU 14336, RMSNorm, RoPE theta 500000, vocab
128256, seq 4096, bf16, ZeRO-3, micro-batch 1, gas 8, AdamW.  Synthetic
uniform-random token ids, random init (std 0.02) for both arms.

``--impl ours`` runs minispeed_b200 (fused sm_100a kernels) through
``engine.train_batch`` with ``b200.cuda_graph`` on: after two eager warm-up
micro-steps the forward + backward is replayed as one captured CUDA graph and
the optimizer step runs eagerly after it (one host read per step; ZeRO-3
runs eagerly).  ``--impl reference`` runs the unmodified reference engine
installed in ``baseline/_ref`` through its public API with stock-PyTorch
models of the same architectures (nn.Linear / nn.LayerNorm / nn.GELU / SDPA
GPT-2 as in the reference example; a stock RMSNorm / RoPE / GQA-SDPA / SwiGLU
Llama) and the reference example's fp32-upcast cross-entropy.

Timing: W untimed warm-up steps, then K steps bracketed by barrier +
synchronize, timed with CUDA events on the launching stream; the reported
time is the max over ranks.  Each step streams > 2 GB (fp32 masters + Adam
moments alone are 1.5 GB for GPT-2 small) so its inputs are larger than L2.
A second loop ("e2e") times K more steps end to end through the public API
including the pinned host->device copy of each step's tokens and the
device->host read of its loss.  Prints one JSON line on rank 0.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch
import torch.nn as nn
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "tokens/sec whole box (max over ranks), ZeRO-2/3, 1/2/4/8 B200; exposed comm ms"

SPECS = {
    "gpt2-small": dict(kind="gpt", vocab=50257, seq=1024, layers=12, heads=12, embd=768,
                       mlp=3072, dtype="fp16", stage=2, micro=16, gas=1, clip=1.0, ckpt=False,
                       label="GPT-2 small (12L, d768, 12H, MLP 3072, vocab 50257)"),
    "gpt2-xl": dict(kind="gpt", vocab=50257, seq=1024, layers=48, heads=25, embd=1600,
                    mlp=6400, dtype="bf16", stage=1, micro=4, gas=4, clip=1.0, ckpt=True,
                    label="GPT-2 XL (48L, d1600, 25H, MLP 6400, vocab 50257), act-ckpt"),
    "llama3-8b": dict(kind="llama", vocab=128256, seq=4096, layers=32, heads=32, kv_heads=8,
                      embd=4096, mlp=14336, rope_theta=500000.0, dtype="bf16", stage=3,
                      micro=1, gas=8, clip=None, ckpt=False,
                      label="Llama-3-8B shape (32L, d4096, 32/8 heads, SwiGLU 14336, "
                            "vocab 128256)"),
}


def ds_config(spec: dict, world: int, total_steps: int) -> dict:
    cfg = {
        "train_micro_batch_size_per_gpu": spec["micro"],
        "gradient_accumulation_steps": spec["gas"],
        "dtype": spec["dtype"],
        "optimizer": {"type": "AdamW", "params": {"lr": 6e-4, "betas": [0.9, 0.95],
                                                  "eps": 1e-8, "weight_decay": 0.1}},
        "scheduler": {"type": "WarmupDecayLR", "params": {
            "warmup_min_lr": 6e-5, "warmup_max_lr": 6e-4, "warmup_num_steps": 10,
            "total_num_steps": max(total_steps, 20)}},
        "zero_optimization": {"stage": spec["stage"]},
        "steps_per_print": 1000000,
    }
    if spec["clip"]:
        cfg["gradient_clipping"] = spec["clip"]
    if spec["dtype"] == "fp16":
        cfg["fp16"] = {"enabled": True, "loss_scale": 0, "initial_scale_power": 16,
                       "loss_scale_window": 1000}
    else:
        cfg["bf16"] = {"enabled": True}
    return cfg


# ------------------------------------------------- stock PyTorch GPT-2
class _RefAttn(nn.Module):
    def __init__(self, embd, heads):
        super().__init__()
        self.heads = heads
        self.qkv = nn.Linear(embd, 3 * embd)
        self.proj = nn.Linear(embd, embd)

    def forward(self, x):
        b, t, c = x.shape
        q, k, v = self.qkv(x).chunk(3, dim=-1)
        q, k, v = (z.view(b, t, self.heads, c // self.heads).transpose(1, 2) for z in (q, k, v))
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.proj(y.transpose(1, 2).contiguous().view(b, t, c))


class _RefBlock(nn.Module):
    def __init__(self, embd, heads, mlp):
        super().__init__()
        self.ln1 = nn.LayerNorm(embd)
        self.attn = _RefAttn(embd, heads)
        self.ln2 = nn.LayerNorm(embd)
        self.mlp = nn.Sequential(nn.Linear(embd, mlp), nn.GELU(), nn.Linear(mlp, embd))

    def forward(self, x):
        x = x + self.attn(self.ln1(x))
        return x + self.mlp(self.ln2(x))


class RefGPT(nn.Module):
    """The reference example's TinyGPT architecture at GPT-2 sizes."""

    def __init__(self, spec):
        super().__init__()
        self.ckpt = spec["ckpt"]
        self.wte = nn.Embedding(spec["vocab"], spec["embd"])
        self.wpe = nn.Embedding(spec["seq"], spec["embd"])
        self.blocks = nn.ModuleList(_RefBlock(spec["embd"], spec["heads"], spec["mlp"])
                                    for _ in range(spec["layers"]))
        self.ln_f = nn.LayerNorm(spec["embd"])
        self.head = nn.Linear(spec["embd"], spec["vocab"], bias=False)
        self.head.weight = self.wte.weight

    def forward(self, idx):
        t = idx.shape[1]
        x = self.wte(idx) + self.wpe(torch.arange(t, device=idx.device))
        for blk in self.blocks:
            if self.ckpt and self.training:
                x = torch.utils.checkpoint.checkpoint(blk, x, use_reentrant=False)
            else:
                x = blk(x)
        return self.head(self.ln_f(x))


class _RefRMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return xf.to(x.dtype) * self.weight


def _ref_rope(x, cos, sin):
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
    return x * cos + torch.cat((-x2, x1), dim=-1) * sin


class _RefLlamaBlock(nn.Module):
    def __init__(self, spec):
        super().__init__()
        d, h, hk = spec["embd"], spec["heads"], spec["kv_heads"]
        self.h, self.hk, self.hd = h, hk, d // h
        self.attention_norm = _RefRMSNorm(d)
        self.wq = nn.Linear(d, d, bias=False)
        self.wk = nn.Linear(d, hk * self.hd, bias=False)
        self.wv = nn.Linear(d, hk * self.hd, bias=False)
        self.wo = nn.Linear(d, d, bias=False)
        self.ffn_norm = _RefRMSNorm(d)
        self.w1 = nn.Linear(d, spec["mlp"], bias=False)
        self.w3 = nn.Linear(d, spec["mlp"], bias=False)
        self.w2 = nn.Linear(spec["mlp"], d, bias=False)

    def forward(self, x, cos, sin):
        b, t, _ = x.shape
        hN = self.attention_norm(x)
        q = self.wq(hN).view(b, t, self.h, self.hd).transpose(1, 2)
        k = self.wk(hN).view(b, t, self.hk, self.hd).transpose(1, 2)
        v = self.wv(hN).view(b, t, self.hk, self.hd).transpose(1, 2)
        q, k = _ref_rope(q, cos, sin), _ref_rope(k, cos, sin)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        x = x + self.wo(y.transpose(1, 2).reshape(b, t, -1))
        hN = self.ffn_norm(x)
        return x + self.w2(F.silu(self.w1(hN)) * self.w3(hN))


class RefLlama(nn.Module):
    """A stock-PyTorch Llama-3 architecture (RMSNorm, RoPE, GQA SDPA, SwiGLU)."""

    def __init__(self, spec):
        super().__init__()
        self.spec = spec
        self.tok_embeddings = nn.Embedding(spec["vocab"], spec["embd"])
        self.layers = nn.ModuleList(_RefLlamaBlock(spec) for _ in range(spec["layers"]))
        self.norm = _RefRMSNorm(spec["embd"])
        self.output = nn.Linear(spec["embd"], spec["vocab"], bias=False)

    def forward(self, idx):
        t = idx.shape[1]
        hd = self.spec["embd"] // self.spec["heads"]
        inv = 1.0 / (self.spec["rope_theta"] ** (torch.arange(0, hd, 2, device=idx.device,
                                                              dtype=torch.float32) / hd))
        ang = torch.outer(torch.arange(t, device=idx.device, dtype=torch.float32), inv)
        emb = torch.cat((ang, ang), dim=-1)
        x = self.tok_embeddings(idx)
        cos, sin = emb.cos().to(x.dtype), emb.sin().to(x.dtype)
        for blk in self.layers:
            x = blk(x, cos, sin)
        return self.output(self.norm(x))


# ------------------------------------------------------------ clocks
class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons in a thread, one query every
    100 ms after the previous one returns (the timed region of the headline
    run lasts well under a second)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.gpus = gpu_indices
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(
                    ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-i", ",".join(str(g) for g in self.gpus)],
                    capture_output=True, text=True, timeout=5).stdout
                for line in out.strip().splitlines():
                    self.rows.append([c.strip() for c in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.1)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# -------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", choices=sorted(SPECS), default="gpt2-small")
    args = ap.parse_args()
    spec = SPECS[args.model]
    MICRO, GAS, SEQ, VOCAB = spec["micro"], spec["gas"], spec["seq"], spec["vocab"]
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch with torchrun")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    os.environ.setdefault("MINISPEED_DEVICE", f"cuda:{local}")
    os.environ.setdefault("MINISPEED_PG_TIMEOUT_S", "300")

    if args.impl == "reference":
        ref_dir = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_dir, "minispeed")):
            if rank == 0:
                print(json.dumps({"impl": "reference",
                                  "unavailable": "baseline/_ref is not installed"}))
            return
        sys.path.insert(0, ref_dir)
        import minispeed as lib  # the unmodified reference engine
        from minispeed import comm as lcomm
        torch.manual_seed(1234)
        with torch.device(device):   # build and initialize on the GPU (8B params)
            model = RefGPT(spec) if spec["kind"] == "gpt" else RefLlama(spec)
            _init(model)

        def micro_step(eng, x, y):
            logits = eng(x)
            loss = F.cross_entropy(logits.reshape(-1, logits.size(-1)).float(), y.reshape(-1))
            eng.backward(loss)
            eng.step()
            return loss
    else:
        sys.path.insert(0, ROOT)
        import minispeed_b200 as lib
        from minispeed_b200 import comm as lcomm
        from minispeed_b200.models import GPT, GPTConfig, Llama, LlamaConfig
        torch.manual_seed(1234)
        with torch.device(device):
            model = _build_ours(spec, GPT, GPTConfig, Llama, LlamaConfig)
            _init(model)

        def micro_step(eng, x, y):
            # forward + backward replayed as one CUDA graph, then the step
            return eng.train_batch(x, targets=y)

    lcomm.init_distributed()
    cfg = ds_config(spec, world, args.warmup + 2 * args.steps)
    if args.impl == "ours":
        cfg["b200"] = {"cuda_graph": os.environ.get("MINISPEED_CUDA_GRAPH", "1") == "1"}
    engine, _, _, _ = lib.initialize(model=model, model_parameters=model.parameters(),
                                     config=cfg)
    dist = torch.distributed
    distributed = dist.is_available() and dist.is_initialized() and world > 1

    gen = torch.Generator(device="cpu").manual_seed(1000 + rank)
    n_pool = 4
    pool = [torch.randint(0, VOCAB, (MICRO, SEQ + 1), generator=gen) for _ in range(n_pool)]
    dev_pool = [t.to(device) for t in pool]
    pin_pool = [t.pin_memory() for t in pool]

    def step_device(i):
        t = dev_pool[i % n_pool]
        loss = None
        for _ in range(GAS):
            loss = micro_step(engine, t[:, :-1], t[:, 1:])
        return loss

    def sync_all():
        torch.cuda.synchronize()
        if distributed:
            dist.barrier()
        torch.cuda.synchronize()

    def launches():
        if args.impl != "ours":
            return 0
        from minispeed_b200.ops import _ext
        return _ext.launch_count()

    for i in range(args.warmup):
        step_device(i)
    skipped_before = engine.skipped_steps
    # communication phases of the step (ours): reduce-scatter + statistics
    # exchange, and the parameter all-gather tail, device-timed per step
    opt = getattr(engine, "optimizer", None)
    if args.impl == "ours" and world > 1 and hasattr(opt, "phase_log"):
        opt.phase_log = []

    # -------- device-timed region
    sync_all()
    sampler = ClockSampler([local] if not distributed else list(range(world)))
    l0 = launches()
    with sampler if rank == 0 else _Null():
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(args.steps):
            step_device(i)
        end.record()
        sync_all()
    l1 = launches()
    ms_local = start.elapsed_time(end)
    ms_total = _max_over_ranks(ms_local, distributed, device)
    comm_ms, phases = None, None
    if args.impl == "ours" and world > 1 and getattr(opt, "phase_log", None):
        # the optimizer step's phases, device-timed per step (mean over the
        # timed steps, max over ranks); the exposed communication is the step
        # tail outside the AdamW kernel: peer barriers, the fused
        # reduce-scatter + statistics, the statistics exchange, the gather
        log = opt.phase_log
        names = sorted({k for r in log for k in r})
        phases = {k: round(_max_over_ranks(sum(r.get(k, 0.0) for r in log) / len(log),
                                           distributed, device), 4) for k in names}
        comm_ms = sum(v for k, v in phases.items() if k != "adamw")
        opt.phase_log = None
    skipped_timed = engine.skipped_steps - skipped_before

    # -------- end-to-end region (pinned H2D copy + loss D2H every step)
    sync_all()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record()
    losses = []
    for i in range(args.steps):
        t = pin_pool[i % n_pool].to(device, non_blocking=True)
        x, y = t[:, :-1], t[:, 1:]
        loss = None
        for _ in range(GAS):
            loss = micro_step(engine, x, y)
        losses.append(float(loss.item()))
    e1.record()
    sync_all()
    wall_e2e = time.perf_counter() - w0
    ms_e2e = _max_over_ranks(e0.elapsed_time(e1), distributed, device)

    tokens_per_step = world * MICRO * GAS * SEQ
    ms_step = ms_total / args.steps
    value = tokens_per_step / (ms_step / 1000.0)
    e2e_value = tokens_per_step / (ms_e2e / args.steps / 1000.0)
    if rank == 0:
        out = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": spec["dtype"],
            "data": "synthetic uniform-random token ids, random-init weights (std 0.02)",
            "config": {"model": spec["label"],
                       "global_batch": world * MICRO * GAS, "micro_batch": MICRO, "gas": GAS,
                       "seq_len": SEQ, "parallelism": f"dp{world} ZeRO-{spec['stage']}",
                       "zero_stage": spec["stage"],
                       "precision": ("fp16 + fp32 masters, dynamic loss scale 2^16"
                                     if spec["dtype"] == "fp16" else "bf16 + fp32 masters"),
                       "optimizer": "AdamW + WarmupDecayLR" + (
                           f", clip {spec['clip']}" if spec["clip"] else ""),
                       "l2": "per-step working set > L2 (fp32 optimizer state streamed)"},
            "impl": args.impl,
            "collectives": getattr(engine, "collectives", "reference comm"),
            "exposed_comm_ms": 0.0 if world == 1 else (
                round(comm_ms, 4) if comm_ms is not None else None),
            "step_phases_ms": phases,
            "skipped_steps_timed": skipped_timed,
            "clocks": sampler.summary(),
            "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(pin_pool[0].numel() * pin_pool[0].element_size()),
                    "d2h_bytes_per_step": 4, "wall_s": round(wall_e2e, 3),
                    "final_loss": losses[-1] if losses else None},
            "gpu_launches": int(l1 - l0),
        }
        print(json.dumps(out), flush=True)
    if hasattr(engine, "close"):
        engine.close()
    if distributed:
        dist.barrier()
        dist.destroy_process_group()


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _build_ours(spec, GPT, GPTConfig, Llama, LlamaConfig):
    if spec["kind"] == "gpt":
        return GPT(GPTConfig(vocab_size=spec["vocab"], block_size=spec["seq"],
                             n_layer=spec["layers"], n_head=spec["heads"], n_embd=spec["embd"],
                             activation_checkpointing=spec["ckpt"]))
    return Llama(LlamaConfig(vocab_size=spec["vocab"], block_size=spec["seq"],
                             n_layer=spec["layers"], n_head=spec["heads"],
                             n_kv_head=spec["kv_heads"], n_embd=spec["embd"],
                             ffn_hidden=spec["mlp"], rope_theta=spec["rope_theta"],
                             activation_checkpointing=spec["ckpt"]))


def _init(model):
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                m.weight.normal_(0.0, 0.02)
                if getattr(m, "bias", None) is not None:
                    m.bias.zero_()
            elif isinstance(m, nn.LayerNorm):
                m.weight.fill_(1.0)
                m.bias.zero_()


def _max_over_ranks(v: float, distributed: bool, device) -> float:
    if not distributed:
        return v
    t = torch.tensor([v], dtype=torch.float64, device=device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


if __name__ == "__main__":
    try:
        main()
    except torch.cuda.OutOfMemoryError as e:
        # a config that does not fit (e.g. the reference's full fp32 buffers
        # for an 8B model on few GPUs) reports itself instead of a number
        if int(os.environ.get("RANK", "0")) == 0:
            impl = "reference" if "--impl" in sys.argv and "reference" in sys.argv else "ours"
            print(json.dumps({"impl": impl, "unavailable": "CUDA out of memory: "
                              + str(e).splitlines()[0][:160]}), flush=True)
        sys.exit(0)
