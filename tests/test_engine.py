"""Single-process engine behaviour on CPU against plain PyTorch."""

import copy
import tempfile

import torch
import torch.nn.functional as F

import minispeed_b200 as ms
from tests.helpers import config, make_data, make_net, mse, run

STEPS, GAS, MICRO = 6, 2, 4


def plain_torch(x, y, lr, wd, clip):
    model = make_net()
    opt = torch.optim.AdamW(model.parameters(), lr=lr, betas=(0.9, 0.999), eps=1e-8,
                            weight_decay=wd)
    losses = []
    for s in range(STEPS):
        for m in range(GAS):
            loss = F.mse_loss(model(x[s, m]), y[s, m])
            losses.append(float(loss.detach()))
            (loss / GAS).backward()
        if clip:
            torch.nn.utils.clip_grad_norm_(model.parameters(), clip)
        opt.step()
        opt.zero_grad(set_to_none=True)
    return losses, model


def test_matches_torch_adamw_with_clipping():
    x, y = make_data(STEPS, GAS, 1, MICRO)
    ref_losses, ref = plain_torch(x, y, lr=1e-3, wd=0.01, clip=1.0)
    model = make_net()
    engine = ms.initialize(model=model, model_parameters=list(model.parameters()),
                           config=config(micro=MICRO, gas=GAS, clip=1.0))
    losses = run(engine, x, y, STEPS, GAS)
    assert engine.global_steps == STEPS
    torch.testing.assert_close(torch.tensor(losses), torch.tensor(ref_losses),
                               rtol=1e-4, atol=1e-6)
    for a, b in zip(model.parameters(), ref.parameters()):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-6)
    assert engine.get_gradient_norm() is not None and engine.get_gradient_norm() > 0


def test_accumulation_equals_big_batch():
    x, y = make_data(STEPS, GAS, 1, MICRO)
    big = ms.initialize(model=make_net(), config=config(micro=MICRO * GAS, gas=1, lr=5e-3,
                                                        wd=0.0, clip=None))
    run(big, x.reshape(STEPS, 1, GAS * MICRO, -1), y.reshape(STEPS, 1, GAS * MICRO, -1),
        STEPS, 1)
    acc = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=GAS, lr=5e-3, wd=0.0,
                                                        clip=None))
    run(acc, x, y, STEPS, GAS)
    for a, b in zip(acc.module.parameters(), big.module.parameters()):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-6)


def test_step_only_at_boundary_and_once():
    engine = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=3))
    x, y = make_data(1, 3, 1, MICRO)
    results = []
    for m in range(3):
        engine.backward(mse(engine(x[0, m]), y[0, m]))
        results.append(engine.step())
        assert engine.is_gradient_accumulation_boundary == (m == 2)
    assert results == [False, False, True]
    assert engine.step() is False
    assert engine.global_steps == 1 and engine.micro_steps == 3


def test_bf16_learns_with_fp32_masters():
    x, y = make_data(STEPS, GAS, 1, MICRO)
    model = make_net()
    engine = ms.initialize(model=model, config=config(micro=MICRO, gas=GAS, dtype="bf16",
                                                      lr=1e-2, clip=None))
    losses = run(engine, x, y, STEPS, GAS)
    assert all(map(torch.isfinite, torch.tensor(losses)))
    assert losses[-1] < losses[0]
    assert next(model.parameters()).dtype == torch.bfloat16
    assert engine.flat_groups[0].data.dtype == torch.float32
    assert engine.get_loss_scale() == 1.0


def test_fp16_on_cpu_runs_with_loss_scaling():
    x, y = make_data(STEPS, GAS, 1, MICRO)
    engine = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=GAS, dtype="fp16",
                                                           scale_power=4, window=2, lr=1e-2))
    losses = run(engine, x, y, STEPS, GAS)
    assert all(map(torch.isfinite, torch.tensor(losses)))
    assert engine.get_loss_scale() > 16.0


def test_params_and_grads_alias_the_arenas():
    model = make_net()
    engine = ms.initialize(model=model, config=config(micro=MICRO, gas=1, dtype="bf16"))
    g = engine.flat_groups[0]
    x, y = make_data(1, 1, 1, MICRO)
    engine.backward(mse(engine(x[0, 0]), y[0, 0]))
    base, gbase = g.param_arena.data_ptr(), g.grad_arena.data_ptr()
    esz = g.param_arena.element_size()
    for (start, _), p in zip(g.param_index_ranges(), model.parameters()):
        assert p.data_ptr() == base + start * esz
        assert p.grad.data_ptr() == gbase + start * esz
    assert engine.step() is True


def test_user_reset_grads_are_still_collected():
    x, y = make_data(1, 1, 1, MICRO)
    a = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=1))
    b = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=1))
    a.backward(mse(a(x[0, 0]), y[0, 0]))
    a.step()
    loss = mse(b(x[0, 0]), y[0, 0])
    b.module.zero_grad(set_to_none=True)   # detaches p.grad from the arena
    b.backward(loss)
    b.step()
    for p, q in zip(a.module.parameters(), b.module.parameters()):
        torch.testing.assert_close(p, q)


def test_checkpoint_replay_is_exact():
    x, y = make_data(STEPS, GAS, 1, MICRO)
    model = make_net()
    engine = ms.initialize(model=model, config=config(micro=MICRO, gas=GAS, warmup=4,
                                                      scheduler="WarmupDecayLR", total=40))
    run(engine, x, y, 2, GAS)
    with tempfile.TemporaryDirectory() as d:
        engine.save_checkpoint(d, tag="mid")
        expect = run(engine, x, y, 2, GAS)
        expect_steps = engine.global_steps
        expect_params = copy.deepcopy(model.state_dict())
        expect_lr = engine.lr_scheduler.get_last_lr()
        engine.load_checkpoint(d)   # follows `latest`
        assert engine.global_steps == expect_steps - 2
        replay = run(engine, x, y, 2, GAS)
        torch.testing.assert_close(torch.tensor(replay), torch.tensor(expect),
                                   rtol=1e-5, atol=1e-7)
        for k, v in model.state_dict().items():
            torch.testing.assert_close(v, expect_params[k], rtol=1e-5, atol=1e-7)
        assert engine.lr_scheduler.get_last_lr() == expect_lr


def test_tuple_unpacking_and_param_groups():
    model = make_net()
    groups = [{"params": list(model.l1.parameters()), "weight_decay": 0.0},
              {"params": [p for n, p in model.named_parameters() if not n.startswith("l1")]}]
    engine, opt, _, sched = ms.initialize(model=model, model_parameters=groups,
                                          config=config())
    assert isinstance(engine, ms.DeepSpeedEngine)
    assert opt is engine.optimizer and sched is engine.lr_scheduler
    assert len(engine.flat_groups) == 2
    assert opt.param_groups[0]["weight_decay"] == 0.0
    assert opt.param_groups[1]["weight_decay"] == 0.01
    assert engine.gas == 2


def test_no_trainable_params_raises():
    model = make_net()
    for p in model.parameters():
        p.requires_grad_(False)
    try:
        ms.initialize(model=model, config=config())
    except ValueError:
        return
    raise AssertionError("expected ValueError")


def test_activation_checkpointing_grads_match():
    from minispeed_b200.activation_checkpointing import checkpoint, checkpoint_sequential

    model = make_net()
    x, _ = make_data(1, 1, 1, MICRO)
    model(x[0, 0]).sum().backward()
    ref = [p.grad.clone() for p in model.parameters()]
    model.zero_grad(set_to_none=True)
    checkpoint(model, x[0, 0]).sum().backward()
    for p, g in zip(model.parameters(), ref):
        torch.testing.assert_close(p.grad, g, rtol=1e-5, atol=1e-7)
    seq = torch.nn.Sequential(torch.nn.Linear(8, 8), torch.nn.Tanh(), torch.nn.Linear(8, 1))
    inp = torch.randn(3, 8, requires_grad=True)
    checkpoint_sequential(seq, 2, inp).sum().backward()
    assert inp.grad is not None


def test_timers_log_format():
    engine = ms.initialize(model=make_net(), config=config(gas=1))
    x, y = make_data(1, 1, 1, 4)
    engine.backward(mse(engine(x[0, 0]), y[0, 0]))
    engine.step()
    text = engine.timers.log()
    assert "backward:" in text and "step:" in text
    engine.timers.reset()
    assert engine.timers("step").elapsed == 0.0


class _LossNet(torch.nn.Module):
    """TinyNet returning the loss, the module contract of train_batch."""

    def __init__(self):
        super().__init__()
        self.net = make_net()

    def forward(self, x, targets):
        return mse(self.net(x), targets)


def test_train_batch_equals_forward_backward_step():
    x, y = make_data(STEPS, GAS, 1, MICRO)
    torch.manual_seed(0)
    a, b = _LossNet(), _LossNet()
    b.load_state_dict(a.state_dict())
    cfg = config(micro=MICRO, gas=GAS, clip=0.5)
    ea = ms.initialize(model=a, config=cfg)
    eb = ms.initialize(model=b, config=dict(cfg, b200={"cuda_graph": True}))  # CPU: eager
    for s in range(STEPS):
        for m in range(GAS):
            la = ea(x[s, m], targets=y[s, m])
            ea.backward(la)
            ea.step()
            lb = eb.train_batch(x[s, m], targets=y[s, m])
            assert torch.equal(la.detach(), lb.detach())
    assert ea.global_steps == eb.global_steps == STEPS
    for pa, pb in zip(a.parameters(), b.parameters()):
        assert torch.equal(pa, pb)


def test_device_timers_option():
    """``b200.device_timers`` parses (config or env) and is a no-op off CUDA."""
    from minispeed_b200.config import DeepSpeedConfig
    assert DeepSpeedConfig({"b200": {"device_timers": True}}).b200.device_timers
    assert not DeepSpeedConfig({}).b200.device_timers
    engine = ms.initialize(model=make_net(), config=config(b200={"device_timers": True}))
    x, y = make_data(1, 2, 1, 4)
    run(engine, x, y, 1, 2)
    assert engine.device_time_ms() == {}
    assert "backward" in engine.timers.names() and "step" in engine.timers.names()
