"""The reference-granular step API reproduces ``engine.step()``.

A caller of the reference can drive the optimizer step itself, in the order
of the reference engine's ``_take_optimizer_step`` (``engine.py:269-322``):
``flatten_grads`` -> ``has_overflow`` / ``global_overflow`` ->
``unscale_grads`` -> ``reduce_gradients`` -> ``clip_gradients`` -> ``step``
-> ``sync_parameters``.  The same names exist here; driven that way they
must give the same parameters as the fused pipeline behind
``engine.step()``.  One process (stages 0-3) and two gloo ranks.
"""

import os

import pytest
import torch
import torch.multiprocessing as mp

import minispeed_b200 as ms
from minispeed_b200.precision import global_overflow, has_overflow
from tests.helpers import config, free_port, make_data, make_net, mse, rank_slice, set_rank_env

STEPS, GAS, MICRO = 4, 2, 4


def _manual_step(engine, max_norm) -> bool:
    opt, groups = engine.optimizer, engine.flat_groups
    for g in groups:
        g.flatten_grads()
    if global_overflow(has_overflow(*[g.grad for g in groups])):
        engine.loss_scaler.update(overflow=True)
        engine.zero_grad()
        return False
    for g in groups:
        g.unscale_grads(engine.loss_scaler.loss_scale_factor)
    opt.reduce_gradients()
    norm = opt.clip_gradients(max_norm)
    opt.step()
    opt.sync_parameters()
    engine.grad_norm = norm
    engine.loss_scaler.update(overflow=False)
    engine.lr_scheduler.step()
    engine.zero_grad()
    engine.global_steps += 1
    return True


def _train(engine, x, y, manual: bool, clip):
    for s in range(STEPS):
        for m in range(GAS):
            engine.backward(mse(engine(x[s, m]), y[s, m]))
            if not manual:
                engine.step()
        if manual:
            assert engine.is_gradient_accumulation_boundary
            assert _manual_step(engine, clip)
    return {k: v.clone() for k, v in engine.state_dict().items()}, engine.grad_norm


def _pair(stage, x, y, clip):
    out = []
    for manual in (False, True):
        eng = ms.initialize(model=make_net(), config=config(
            micro=MICRO, gas=GAS, stage=stage, clip=clip, warmup=2))
        out.append(_train(eng, x, y, manual, clip))
    return out


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
def test_granular_steps_match_engine_step(stage):
    x, y = make_data(STEPS, GAS, 1, MICRO)
    (p_fused, n_fused), (p_manual, n_manual) = _pair(stage, x, y, clip=0.05)
    assert n_fused > 0.05                      # the clip was active
    assert n_manual == pytest.approx(n_fused, rel=1e-5)
    for k in p_fused:
        torch.testing.assert_close(p_manual[k], p_fused[k], rtol=1e-5, atol=1e-6)


WORLD = 2


def _worker(rank, stage, port, out_dir):
    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    x, y = make_data(STEPS, GAS, WORLD, MICRO)
    x, y = rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO)
    torch.save(_pair(stage, x, y, clip=0.05), os.path.join(out_dir, f"r{rank}.pt"))
    ms.comm.destroy()


@pytest.mark.parametrize("stage", [1, 2, 3])
def test_granular_steps_match_engine_step_two_ranks(stage, tmp_path):
    mp.spawn(_worker, args=(stage, free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    for rank in range(WORLD):
        (p_fused, n_fused), (p_manual, n_manual) = torch.load(tmp_path / f"r{rank}.pt",
                                                              weights_only=False)
        assert n_manual == pytest.approx(n_fused, rel=1e-5)
        for k in p_fused:
            torch.testing.assert_close(p_manual[k], p_fused[k], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("stage", [0, 2, 3])
def test_granular_overflow_skip_matches_engine_step(stage):
    """fp16 with an inf written into one gradient before the second boundary:
    both paths skip that step, halve the scale and end at the same weights."""
    x, y = make_data(STEPS, GAS, 1, MICRO)
    results = []
    for manual in (False, True):
        eng = ms.initialize(model=make_net(), config=config(
            micro=MICRO, gas=GAS, stage=stage, dtype="fp16", scale_power=8))
        skipped = 0
        for s in range(STEPS):
            for m in range(GAS):
                eng.backward(mse(eng(x[s, m]), y[s, m]))
                last = m == GAS - 1
                if last and s == 1:
                    p = next(eng.module.parameters())
                    p.grad.view(-1)[0] = float("inf")
                if not manual:
                    applied = eng.step()
                elif last:
                    applied = _manual_step(eng, 1.0)
                if last and not applied:
                    skipped += 1
        results.append(({k: v.float().clone() for k, v in eng.state_dict().items()},
                        skipped, eng.get_loss_scale(), eng.global_steps))
    (p0, s0, sc0, g0), (p1, s1, sc1, g1) = results
    assert s0 == s1 == 1 and sc0 == sc1 == 128.0 and g0 == g1 == STEPS - 1
    for k in p0:
        torch.testing.assert_close(p1[k], p0[k], rtol=1e-3, atol=1e-4)
