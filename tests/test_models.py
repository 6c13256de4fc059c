"""Model zoo through the engine on CPU."""

import pytest
import torch

import minispeed_b200 as ms
from minispeed_b200.models import GPT, GPTConfig, Llama, LlamaConfig, init_gpt2_, init_llama_


def _cfg(stage, gas=1, dtype="fp32"):
    return {"train_micro_batch_size_per_gpu": 2, "gradient_accumulation_steps": gas,
            "gradient_clipping": 1.0, "dtype": dtype, "zero_optimization": {"stage": stage},
            "optimizer": {"type": "AdamW", "params": {"lr": 3e-3, "weight_decay": 0.01}}}


def _tiny_llama():
    torch.manual_seed(0)
    return init_llama_(Llama(LlamaConfig(vocab_size=97, block_size=32, n_layer=2, n_head=4,
                                         n_kv_head=2, n_embd=64, ffn_hidden=128)))


def _tiny_gpt():
    torch.manual_seed(0)
    return init_gpt2_(GPT(GPTConfig(vocab_size=97, block_size=32, n_layer=2, n_head=4,
                                    n_embd=64)))


def _train(model, stage, steps=8, gas=1):
    engine = ms.initialize(model=model, config=_cfg(stage, gas))
    g = torch.Generator().manual_seed(3)
    data = torch.randint(0, 97, (2, 33), generator=g)
    losses = []
    for _ in range(steps):
        for _ in range(gas):
            loss = engine(data[:, :-1], targets=data[:, 1:])
            engine.backward(loss)
            engine.step()
        losses.append(float(loss.detach()))
    return engine, losses


@pytest.mark.parametrize("build", [_tiny_gpt, _tiny_llama])
def test_models_learn(build):
    _, losses = _train(build(), stage=2)
    assert losses[-1] < losses[0] - 0.5


def test_llama_stage3_matches_stage0():
    e0, l0 = _train(_tiny_llama(), 0, steps=4)
    e3, l3 = _train(_tiny_llama(), 3, steps=4)
    torch.testing.assert_close(torch.tensor(l3), torch.tensor(l0), rtol=1e-5, atol=1e-6)
    s0, s3 = e0.state_dict(), e3.state_dict()
    for k in s0:
        torch.testing.assert_close(s3[k], s0[k], rtol=1e-5, atol=1e-6)


def test_gpt_state_dict_names_match_reference_example():
    names = set(_tiny_gpt().state_dict())
    for must in ("wte.weight", "wpe.weight", "blocks.0.ln1.weight", "blocks.0.attn.qkv.weight",
                 "blocks.0.attn.proj.bias", "blocks.1.mlp.0.weight", "blocks.1.mlp.2.bias",
                 "ln_f.bias", "head.weight"):
        assert must in names


def test_gpt_activation_checkpointing_same_grads():
    a, b = _tiny_gpt(), _tiny_gpt()
    b.config.activation_checkpointing = True
    x = torch.randint(0, 97, (2, 32))
    for m in (a, b):
        m(x, targets=torch.roll(x, -1, 1)).backward()
    for p, q in zip(a.parameters(), b.parameters()):
        torch.testing.assert_close(p.grad, q.grad, rtol=1e-5, atol=1e-6)
