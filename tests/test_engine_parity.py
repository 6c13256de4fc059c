"""Whole-engine parity with the reference on generated configurations.

The same stock module, data and JSON config go through
``minispeed_b200.initialize`` and through the reference's ``initialize``
(``minispeed/engine.py:372-389``); for random ZeRO stages, micro-batch and
accumulation sizes, clipping thresholds, schedules and training dtypes the
losses, global steps, gradient norms, loss scales and final weights must
agree.  One process (the two-rank paths are covered elsewhere).  Skipped
when the reference is not installed in ``baseline/_ref``.
"""

import importlib
import os
import sys

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

import minispeed_b200 as ours
from tests.helpers import config, make_data, make_net, run

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "minispeed")):
        pytest.skip("reference not installed in baseline/_ref")
    sys.path.insert(0, REF)
    try:
        return importlib.import_module("minispeed")
    finally:
        sys.path.remove(REF)


TOL = {"fp32": (1e-5, 1e-6), "bf16": (2e-2, 2e-3), "fp16": (5e-3, 5e-4)}


@settings(max_examples=30, deadline=None,
          suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(stage=st.integers(0, 3), micro=st.integers(1, 6), gas=st.integers(1, 3),
       clip=st.sampled_from([0, 0.05, 1.0]), dtype=st.sampled_from(["fp32", "bf16", "fp16"]),
       sched=st.sampled_from(["WarmupLR", "WarmupDecayLR"]), warmup=st.integers(0, 3),
       steps=st.integers(1, 4), wd=st.sampled_from([0.0, 0.1]))
def test_engine_matches_reference(ref, stage, micro, gas, clip, dtype, sched, warmup, steps, wd):
    cfg = config(micro=micro, gas=gas, stage=stage, clip=clip, dtype=dtype, scheduler=sched,
                 warmup=warmup, total=steps + 2, wd=wd, lr=1e-2)
    x, y = make_data(steps, gas, 1, micro)
    out = []
    for lib in (ours, ref):
        eng = lib.initialize(model=make_net(), config=cfg)
        losses = run(eng, x, y, steps, gas)
        out.append((torch.tensor(losses), eng.global_steps, eng.skipped_steps,
                    eng.get_loss_scale(), eng.grad_norm, eng.lr_scheduler.get_last_lr(),
                    {k: v.float().clone() for k, v in eng.state_dict().items()}))
    (la, ga, sa, sca, na, lra, pa), (lb, gb, sb, scb, nb, lrb, pb) = out
    rtol, atol = TOL[dtype]
    assert (ga, sa, sca) == (gb, sb, scb)
    assert lra == pytest.approx(lrb, rel=1e-12)
    torch.testing.assert_close(la, lb, rtol=rtol, atol=atol)
    if na is None or nb is None:
        assert na is None and nb is None
    else:
        assert na == pytest.approx(nb, rel=max(rtol, 1e-4))
    for k in pa:
        torch.testing.assert_close(pa[k], pb[k], rtol=rtol, atol=atol)


@settings(max_examples=30, deadline=None,
          suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(stage=st.integers(0, 3), gas=st.integers(1, 2), window=st.integers(1, 3),
       inject=st.lists(st.booleans(), min_size=1, max_size=6))
def test_overflow_handling_matches_reference(ref, stage, gas, window, inject):
    """fp16 with inf written into a gradient before chosen boundaries: the
    same steps are skipped, and scale, counters and weights agree."""
    micro, steps = 4, len(inject)
    cfg = config(micro=micro, gas=gas, stage=stage, dtype="fp16", window=window, lr=1e-2)
    x, y = make_data(steps, gas, 1, micro)
    out = []
    for lib in (ours, ref):
        eng = lib.initialize(model=make_net(), config=cfg)
        scales, applied = [], []
        for s in range(steps):
            for m in range(gas):
                loss = ((eng(x[s, m]).float() - y[s, m]) ** 2).mean()
                eng.backward(loss)
                if m == gas - 1 and inject[s]:
                    p = next(eng.module.parameters())
                    if p.grad is None:      # stage 3 between gathers: inject into a live grad
                        p = [q for q in eng.module.parameters() if q.grad is not None][0]
                    p.grad.view(-1)[0] = float("inf")
                r = eng.step()
                if m == gas - 1:
                    applied.append(bool(r))
            scales.append(eng.get_loss_scale())
        out.append((applied, scales, eng.global_steps, eng.skipped_steps,
                    {k: v.float().clone() for k, v in eng.state_dict().items()}))
    (aa, sa, ga, ka, pa), (ab, sb, gb, kb, pb) = out
    assert aa == ab == [not i for i in inject]
    assert sa == sb and (ga, ka) == (gb, kb)
    for k in pa:
        torch.testing.assert_close(pa[k], pb[k], rtol=5e-3, atol=5e-4)
