"""ZeRO stage 3 on CPU: equivalence with stage 0 and the gather/free lifecycle."""

import copy
import tempfile

import torch

import minispeed_b200 as ms
from minispeed_b200.flat import FlatParamGroup
from tests.helpers import config, make_data, make_net, mse, run

STEPS, GAS, MICRO = 4, 2, 4


def _train(stage, **kw):
    x, y = make_data(STEPS, GAS, 1, MICRO)
    engine = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=GAS, stage=stage,
                                                           **kw))
    losses = run(engine, x, y, STEPS, GAS)
    return engine, torch.tensor(losses), engine.state_dict()


def test_stage3_matches_stage0():
    e0, l0, p0 = _train(0)
    e3, l3, p3 = _train(3)
    torch.testing.assert_close(l3, l0, rtol=1e-5, atol=1e-7)
    for k in p0:
        torch.testing.assert_close(p3[k], p0[k], rtol=1e-5, atol=1e-7)
    assert e0.global_steps == e3.global_steps == STEPS


def test_stage3_bf16_matches_stage0_bf16():
    _, l0, p0 = _train(0, dtype="bf16")
    _, l3, p3 = _train(3, dtype="bf16")
    torch.testing.assert_close(l3, l0, rtol=1e-5, atol=1e-7)
    for k in p0:
        torch.testing.assert_close(p3[k], p0[k])


def test_lifecycle_of_partitioned_params():
    model = make_net()
    reference_shapes = [p.shape for p in make_net().parameters()]
    engine = ms.initialize(model=model, config=config(micro=MICRO, gas=GAS, stage=3))
    g = engine.flat_groups[0]
    x, y = make_data(1, GAS, 1, MICRO)
    assert not engine.optimizer.params_gathered
    assert all(p.dim() == 1 for p in model.parameters())
    assert g.grad is None
    loss = mse(engine(x[0, 0]), y[0, 0])
    assert engine.optimizer.params_gathered
    assert [p.shape for p in model.parameters()] == reference_shapes
    engine.backward(loss)
    assert engine.step() is False and engine.optimizer.params_gathered
    engine.backward(mse(engine(x[0, 1]), y[0, 1]))
    assert engine.step() is True
    assert not engine.optimizer.params_gathered
    assert all(p.dim() == 1 for p in model.parameters())
    assert g.grad is None and g.grad_arena is None
    assert g.data.numel() == g.numel_shard()
    assert engine.optimizer.state[0]["exp_avg"].numel() == g.numel_shard()
    raw, full = model.state_dict(), engine.state_dict()
    for k in full:
        assert raw[k].dim() == 1 and raw[k].numel() == full[k].numel()


def test_partition_roundtrip_is_exact():
    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(6, 7)), torch.nn.Parameter(torch.randn(5)),
              torch.nn.Parameter(torch.randn(2, 2))]
    originals = [p.detach().clone() for p in params]
    g = FlatParamGroup(params, rank=1, world_size=3, zero_stage=3, device=torch.device("cpu"))
    g.copy_model_to_flat()
    g.partition_params()
    assert g.numel_padded == 51 and g.shard_size == 17 and g.shard_start == 17
    assert g.data.numel() == 17
    assert sum(p.numel() for p in params) == g.numel_shard()
    full = torch.cat([o.reshape(-1) for o in originals] + [torch.zeros(g.numel_padded - 51)])
    g.materialize_params()
    g.copy_flat_to_model(full)
    for p, o in zip(params, originals):
        assert p.shape == o.shape
        torch.testing.assert_close(p.data, o)
    g.dematerialize_params()
    g.copy_flat_to_model()
    for (start, end), p, o in zip(g.param_index_ranges(), params, originals):
        lo, hi = max(start, 17), min(end, 34)
        assert p.numel() == max(0, hi - lo)
        if hi > lo:
            torch.testing.assert_close(p.data, o.reshape(-1)[lo - start:hi - start])


def test_stage3_checkpoint_replay():
    x, y = make_data(STEPS + 2, GAS, 1, MICRO)
    engine = ms.initialize(model=make_net(), config=config(
        micro=MICRO, gas=GAS, stage=3, warmup=4, scheduler="WarmupDecayLR", total=40))
    run(engine, x, y, 2, GAS)
    with tempfile.TemporaryDirectory() as d:
        engine.save_checkpoint(d, tag="mid")
        assert not engine.optimizer.params_gathered
        expect = run(engine, x, y, 2, GAS)
        expect_params = copy.deepcopy(engine.state_dict())
        engine.load_checkpoint(d, tag="mid")
        replay = run(engine, x, y, 2, GAS)
        torch.testing.assert_close(torch.tensor(replay), torch.tensor(expect),
                                   rtol=1e-5, atol=1e-7)
        for k, v in engine.state_dict().items():
            torch.testing.assert_close(v, expect_params[k], rtol=1e-5, atol=1e-7)


def test_overflow_skip_frees_params_and_recovers():
    model = make_net()
    engine = ms.initialize(model=model, config=config(micro=MICRO, gas=1, stage=3,
                                                      dtype="fp16", scale_power=6))
    x, y = make_data(2, 1, 1, MICRO)
    engine.backward(mse(engine(x[0, 0]), y[0, 0]))
    next(p for p in model.parameters() if p.grad is not None).grad.view(-1)[0] = float("inf")
    before = engine.get_loss_scale()
    masters = engine.flat_groups[0].data.clone()
    assert engine.step() is False
    assert engine.skipped_steps == 1 and engine.global_steps == 0
    assert engine.get_loss_scale() == before / 2
    assert not engine.optimizer.params_gathered
    assert engine.flat_groups[0].grad is None
    torch.testing.assert_close(engine.flat_groups[0].data, masters, rtol=0, atol=0)
    losses = run(engine, x[1:], y[1:], 1, 1)
    assert all(map(torch.isfinite, torch.tensor(losses)))
    assert engine.global_steps == 1


def test_eval_forward_regathers():
    engine = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=GAS, stage=3))
    x, y = make_data(1, GAS, 1, MICRO)
    run(engine, x, y, 1, GAS)
    engine.eval()
    with torch.no_grad():
        out = engine(x[0, 0])
    assert out.shape == (MICRO, 1)
    assert engine.optimizer.params_gathered
