"""Loss curves against the reference engine on the CPU benchmark config.

The first benchmark configuration: two gloo ranks on CPU, ZeRO-2, fp32, a
4-layer decoder-only GPT (d_model 128, 4 heads, MLP 512 with GELU, learned
position embeddings, vocab 256, seq 64), micro-batch 8 per rank, gas 2,
AdamW lr 1e-3 wd 0.01, clipping 1.0, uniform-random tokens with targets the
inputs shifted by one.

Each rank trains the same initial weights twice: this library's GPT through
``minispeed_b200``, and a stock-PyTorch module of the reference example's
architecture (``examples/train_lm.py:62-115``, its fp32-upcast cross-entropy
at ``:246``) through the unmodified reference engine installed in
``baseline/_ref``.  The two must follow the same loss curve and end at the
same weights.  Skipped when the reference is not installed.
"""

import importlib
import os
import sys

import pytest
import torch
import torch.nn.functional as F

import minispeed_b200 as ours
from minispeed_b200.models import GPT, GPTConfig, init_gpt2_

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
WORLD, STEPS, GAS, MICRO = 2, 8, 2, 8
VOCAB, SEQ = 256, 64
SPEC = dict(vocab=VOCAB, seq=SEQ, layers=4, heads=4, embd=128, mlp=512, ckpt=False)


def _config(stage: int, clip: float = 1.0) -> dict:
    return {
        "train_micro_batch_size_per_gpu": MICRO,
        "gradient_accumulation_steps": GAS,
        "gradient_clipping": clip,
        "dtype": "fp32",
        "optimizer": {"type": "AdamW", "params": {"lr": 1e-3, "weight_decay": 0.01}},
        "zero_optimization": {"stage": stage},
        "steps_per_print": 10 ** 6,
    }


def _tokens(rank: int):
    g = torch.Generator().manual_seed(2024)
    t = torch.randint(0, VOCAB, (STEPS, GAS, WORLD * MICRO, SEQ + 1), generator=g)
    return t[:, :, rank * MICRO:(rank + 1) * MICRO]


def _train(engine, tokens, loss_fn):
    losses = []
    for s in range(STEPS):
        for m in range(GAS):
            t = tokens[s, m]
            loss = loss_fn(engine, t[:, :-1], t[:, 1:])
            losses.append(float(loss.detach()))
            engine.backward(loss)
            engine.step()
    return losses


def _ours_loss(engine, x, y):
    return engine(x, targets=y)


def _ref_loss(engine, x, y):
    logits = engine(x)
    return F.cross_entropy(logits.float().view(-1, logits.size(-1)), y.reshape(-1))


def _worker(rank, stage, clip, port, out_dir):
    sys.path.insert(0, ROOT)
    from bench import RefGPT
    from tests.helpers import set_rank_env
    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    sys.path.insert(0, REF)
    ref = importlib.import_module("minispeed")
    sys.path.remove(REF)

    torch.manual_seed(0)
    mine = init_gpt2_(GPT(GPTConfig(vocab_size=VOCAB, block_size=SEQ, n_layer=4, n_head=4,
                                    n_embd=128)))
    stock = RefGPT(SPEC)
    stock.load_state_dict(mine.state_dict())
    tokens = _tokens(rank)

    e_ours = ours.initialize(model=mine, config=_config(stage, clip))
    l_ours = _train(e_ours, tokens, _ours_loss)
    e_ref = ref.initialize(model=stock, config=_config(stage, clip))
    l_ref = _train(e_ref, tokens, _ref_loss)
    torch.save({"ours": torch.tensor(l_ours), "ref": torch.tensor(l_ref),
                "norms": (e_ours.grad_norm, e_ref.grad_norm),
                "p_ours": {k: v.clone() for k, v in e_ours.state_dict().items()},
                "p_ref": {k: v.clone() for k, v in e_ref.state_dict().items()}},
               os.path.join(out_dir, f"r{rank}.pt"))
    ours.comm.destroy()


@pytest.fixture(scope="module")
def have_ref():
    if not os.path.isdir(os.path.join(REF, "minispeed")):
        pytest.skip("reference not installed in baseline/_ref")


@pytest.mark.parametrize("stage,clip", [(2, 1.0), (3, 1.0), (0, 0.05)])
def test_loss_curve_matches_reference(have_ref, stage, clip, tmp_path):
    """Stage 2 is the benchmark config; stage 3 and a clip that binds on
    every step (stage 0, where the reference's norm is global) widen it."""
    import torch.multiprocessing as mp
    from tests.helpers import free_port
    mp.spawn(_worker, args=(stage, clip, free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    for rank in range(WORLD):
        r = torch.load(tmp_path / f"r{rank}.pt", weights_only=False)
        assert r["ours"].shape == (STEPS * GAS,)
        torch.testing.assert_close(r["ours"], r["ref"], rtol=2e-5, atol=2e-5)
        n_ours, n_ref = r["norms"]
        assert n_ours == pytest.approx(n_ref, rel=1e-4)
        if clip < 1.0:
            assert n_ours > clip                     # the clip was active
        for k, v in r["p_ref"].items():
            torch.testing.assert_close(r["p_ours"][k], v, rtol=1e-4, atol=1e-5)
