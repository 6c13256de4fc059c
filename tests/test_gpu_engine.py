"""Engine behaviour on one GPU: fp16 loss scaling, inf/nan skip, the fused
step pipeline against the CPU pipeline, and the GPT model."""

import pytest
import torch

import minispeed_b200 as ms
from minispeed_b200.models import GPT, GPTConfig, init_gpt2_
from tests.helpers import config, make_data, make_net, mse, run

pytestmark = pytest.mark.gpu
STEPS, GAS, MICRO = 6, 2, 4


def test_fp16_trains_and_scale_grows():
    x, y = make_data(STEPS, GAS, 1, MICRO, device="cuda")
    model = make_net(device="cuda")
    engine = ms.initialize(model=model, config=config(micro=MICRO, gas=GAS, dtype="fp16",
                                                      scale_power=4, window=3, lr=1e-2))
    losses = run(engine, x, y, STEPS, GAS, device="cuda")
    assert all(map(lambda v: v == v, losses)) and losses[-1] < losses[0]
    assert next(model.parameters()).dtype == torch.float16
    assert engine.flat_groups[0].data.dtype == torch.float32
    assert engine.get_loss_scale() > 16.0
    assert engine.loss_scaler.skipped_steps == 0
    assert engine.grad_norm is not None and engine.grad_norm > 0


def test_forced_inf_skips_step_everything_untouched():
    x, y = make_data(STEPS, GAS, 1, MICRO, device="cuda")
    model = make_net(device="cuda")
    engine = ms.initialize(model=model, config=config(
        micro=MICRO, gas=GAS, dtype="fp16", scale_power=6, lr=1e-2, warmup=5))
    run(engine, x, y, 1, GAS, device="cuda")
    for m in range(GAS):
        engine.backward(mse(engine(x[1, m]), y[1, m]))
    next(p for p in model.parameters()).grad.view(-1)[0] = float("inf")
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    masters = engine.flat_groups[0].data.clone()
    state = engine.optimizer.state[0]["exp_avg"].clone()
    steps, scale, lr = engine.global_steps, engine.get_loss_scale(), \
        engine.lr_scheduler.get_last_lr()
    assert engine.step() is False
    assert engine.global_steps == steps and engine.skipped_steps == 1
    assert engine.get_loss_scale() == scale / 2
    assert engine.lr_scheduler.get_last_lr() == lr
    for n, p in model.named_parameters():
        assert torch.equal(p, before[n])
    assert torch.equal(engine.flat_groups[0].data, masters)
    assert torch.equal(engine.optimizer.state[0]["exp_avg"], state)
    losses = run(engine, x[2:], y[2:], 2, GAS, device="cuda")
    assert all(v == v for v in losses) and engine.global_steps == steps + 2


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_gpu_pipeline_matches_cpu_pipeline(stage, dtype, monkeypatch):
    x, y = make_data(STEPS, GAS, 1, MICRO)
    cfg = config(micro=MICRO, gas=GAS, dtype=dtype, stage=stage, clip=0.05)
    monkeypatch.setenv("MINISPEED_DEVICE", "cpu")
    cpu = ms.initialize(model=make_net(), config=cfg)
    lc = run(cpu, x, y, STEPS, GAS)
    monkeypatch.setenv("MINISPEED_DEVICE", "cuda:0")
    gpu = ms.initialize(model=make_net(), config=cfg)
    lg = run(gpu, x, y, STEPS, GAS, device="cuda")
    tol = 1e-4 if dtype == "fp32" else 2e-2
    torch.testing.assert_close(torch.tensor(lg), torch.tensor(lc), rtol=tol, atol=tol)
    assert gpu.grad_norm == pytest.approx(cpu.grad_norm, rel=1e-3 if dtype == "fp32" else 5e-2)
    pc, pg = cpu.state_dict(), gpu.state_dict()
    for k in pc:
        torch.testing.assert_close(pg[k].cpu().float(), pc[k].float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_gpt_trains_on_gpu(dtype):
    torch.manual_seed(0)
    cfg = GPTConfig(vocab_size=1000, block_size=128, n_layer=2, n_head=4, n_embd=128)
    model = init_gpt2_(GPT(cfg))
    engine = ms.initialize(model=model, config={
        "train_micro_batch_size_per_gpu": 4, "gradient_accumulation_steps": 1,
        "gradient_clipping": 1.0, "dtype": dtype,
        "fp16": {"enabled": dtype == "fp16", "initial_scale_power": 12},
        "zero_optimization": {"stage": 2},
        "optimizer": {"type": "AdamW", "params": {"lr": 3e-3}}})
    data = torch.randint(0, 1000, (4, 129), device="cuda")
    losses = []
    for _ in range(15):
        loss = engine(data[:, :-1], targets=data[:, 1:])
        engine.backward(loss)
        engine.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0] - 1.0, losses


def test_gpt_matches_cpu_fp32_forward():
    torch.manual_seed(0)
    cfg = GPTConfig(vocab_size=512, block_size=64, n_layer=2, n_head=4, n_embd=128)
    cpu = init_gpt2_(GPT(cfg))
    gpu = GPT(cfg).cuda()
    gpu.load_state_dict(cpu.state_dict())
    gpu.half()
    idx = torch.randint(0, 512, (2, 64))
    tgt = torch.roll(idx, -1, 1)
    lc = cpu(idx, targets=tgt)
    lg = gpu(idx.cuda(), targets=tgt.cuda())
    assert float(lg) == pytest.approx(float(lc), rel=2e-3)


def test_peer_barrier_wait_times_out_with_status():
    """A device barrier whose peer never signals gives up and reports; the
    context stays usable (no trap, no endless wait)."""
    import time

    from minispeed_b200.ops import _ext

    C = _ext.get()
    a = C.peer_alloc(8192)
    b = C.peer_alloc(8192)   # stands in for a peer heap nobody writes
    try:
        heaps = torch.tensor([a, b], dtype=torch.int64, device="cuda")
        status = torch.zeros(4, dtype=torch.int32, device="cuda")
        t0 = time.time()
        ctr = torch.zeros(1, dtype=torch.int32, device="cuda")   # epoch counter
        C.peer_barrier(heaps, 0, 0, 2, ctr, 0.3, status)
        torch.cuda.synchronize()
        assert 0.2 < time.time() - t0 < 30
        assert int(status[0]) == 0x101          # waited on rank 1
        x = torch.ones(4, device="cuda") * 2    # context still healthy
        assert float(x.sum()) == 8.0
    finally:
        torch.cuda.synchronize()
        C.peer_free(a)
        C.peer_free(b)


def test_stats_exchange_times_out_and_blocks_the_update():
    from minispeed_b200.ops import _ext

    C = _ext.get()
    a = C.peer_alloc(8192)
    b = C.peer_alloc(8192)
    try:
        heaps = torch.tensor([a, b], dtype=torch.int64, device="cuda")
        status = torch.zeros(4, dtype=torch.int32, device="cuda")
        out = torch.tensor([0.0, 4.0, 0, 0, 0, 0, 0, 0], device="cuda")
        ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
        C.stats_exchange(heaps, 0, 0, 2, ctr, out, 1.0, 0.2, status)
        torch.cuda.synchronize()
        assert int(status[0]) == 0x201
        assert float(out[0]) == 1.0   # a timed-out step is flagged, never applied
    finally:
        torch.cuda.synchronize()
        C.peer_free(a)
        C.peer_free(b)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_llama_matches_cpu_fp32_and_trains(dtype):
    from minispeed_b200.models import Llama, LlamaConfig, init_llama_

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=512, block_size=64, n_layer=2, n_head=4, n_kv_head=2,
                      n_embd=128, ffn_hidden=256)
    cpu = init_llama_(Llama(cfg))
    gpu = Llama(cfg).cuda()
    gpu.load_state_dict(cpu.state_dict())
    gpu.to(torch.float16 if dtype == "fp16" else torch.bfloat16)
    idx = torch.randint(0, 512, (2, 64))
    tgt = torch.roll(idx, -1, 1)
    lc = cpu(idx, targets=tgt)
    lg = gpu(idx.cuda(), targets=tgt.cuda())
    assert float(lg) == pytest.approx(float(lc), rel=5e-3 if dtype == "fp16" else 2e-2)
    model = init_llama_(Llama(cfg))
    engine = ms.initialize(model=model, config={
        "train_micro_batch_size_per_gpu": 2, "dtype": dtype, "gradient_clipping": 1.0,
        "fp16": {"enabled": dtype == "fp16", "initial_scale_power": 12},
        "zero_optimization": {"stage": 3},
        "optimizer": {"type": "AdamW", "params": {"lr": 3e-3}}})
    data = torch.randint(0, 512, (2, 65), device="cuda")
    losses = []
    for _ in range(12):
        loss = engine(data[:, :-1], targets=data[:, 1:])
        engine.backward(loss)
        engine.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0] - 1.0, losses


def test_gqa_attention_and_rope_grads_match_fp32():
    from minispeed_b200.ops import nn as ops

    torch.manual_seed(1)
    B, T, H, Hkv, D = 2, 64, 4, 2, 64
    qkv = torch.randn(B, T, H + 2 * Hkv, D, device="cuda").half().requires_grad_()
    cos, sin = ops.rope_tables(T, D, 500000.0, "cuda")
    out = ops.attention_gqa(ops.rope_qk(qkv, cos, sin, H, Hkv), H, Hkv)
    g = torch.randn_like(out)
    out.backward(g)
    ref_in = qkv.detach().float().cpu().requires_grad_()
    ref = ops.attention_gqa(ops.rope_qk(ref_in, cos.cpu(), sin.cpu(), H, Hkv), H, Hkv)
    ref.backward(g.float().cpu())
    torch.testing.assert_close(out.float().cpu(), ref.detach(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(qkv.grad.float().cpu(), ref_in.grad, rtol=3e-2, atol=3e-2)
