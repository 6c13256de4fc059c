"""Child process of ``test_gpu_bounds_check.py``: the same work under the
build ``MSB_DEBUG_BUILD`` selects, one JSON line on stdout.

The work covers every checked site on valid inputs: GEMMs on the stream-K
plan, split-K finished inside the pair kernel, split-K with the reduce
launch (1-CTA), the dGELU column-sum epilogue, and three CUDA-graph
``train_batch`` steps of a small GPT (head dim 64: the tcgen05 attention
kernels, embedding, cross-entropy).  The engine reads the bounds records
after every step in the debug build; a failure raises there.  The parent
compares the numbers of both builds bit for bit: the checks change no
arithmetic.
"""

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

import minispeed_b200 as ms  # noqa: E402
from minispeed_b200.models import GPT, GPTConfig  # noqa: E402
from minispeed_b200.ops import _ext, gemm  # noqa: E402


def _digest(t: torch.Tensor) -> float:
    return float(t.double().sum().item())


def main() -> None:
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    out = {"module": _ext.module_name(), "debug": _ext.debug_build(), "gemm": {}}
    A = (torch.randn(2304, 16384, device=dev) * 0.05).half()
    B = (torch.randn(768, 16384, device=dev) * 0.05).half()
    for name, plan in [("stream_k", (512, -1)), ("fixup4", (512, 4)), ("reduce4", (256, 4))]:
        c = gemm.gemm(A, B, a_kmajor=True, b_kmajor=True, plan=plan)
        out["gemm"][name] = _digest(c)
    dY = (torch.randn(1000, 768, device=dev) * 0.05).half()
    W = (torch.randn(768, 520, device=dev) * 0.05).half()
    u = torch.randn(1000, 520, device=dev).half()
    du = torch.empty(1000, 520, device=dev, dtype=torch.float16)
    part = torch.zeros(-(-1000 // 32) * 520, device=dev)
    gemm.gemm(dY, W, a_kmajor=True, b_kmajor=False, out=du, mode=gemm.EPI_DGELU, aux=u,
              colsum=part)
    out["gemm"]["dgelu"] = _digest(du)
    out["gemm"]["dgelu_colsum"] = _digest(part)
    gemm.check()
    _ext.check_bounds()

    ms.set_seed(0)
    cfg = GPTConfig(vocab_size=1000, block_size=256, n_layer=2, n_head=4, n_embd=256)
    engine, _, _, _ = ms.initialize(model=GPT(cfg), config={
        "train_micro_batch_size_per_gpu": 4, "gradient_accumulation_steps": 1,
        "gradient_clipping": 1.0, "fp16": {"enabled": True, "initial_scale_power": 8},
        "zero_optimization": {"stage": 2},
        "optimizer": {"type": "AdamW", "params": {"lr": 1e-3, "weight_decay": 0.01}},
        "b200": {"cuda_graph": True},
    })
    g = torch.Generator().manual_seed(1)
    losses = []
    for _ in range(3):
        x = torch.randint(0, cfg.vocab_size, (4, cfg.block_size), generator=g)
        loss = engine.train_batch(x, targets=torch.roll(x, -1, dims=1))
        losses.append(float(loss.item()))
    out["losses"] = losses
    out["records"] = _ext.bounds_status(reset=True)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
