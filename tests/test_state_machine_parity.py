"""Loss scaler and LR schedules against the reference on generated inputs.

The dynamic loss scaler (``minispeed/precision.py:10-76``) under random
overflow sequences, and the WarmupLR / WarmupDecayLR schedules
(``minispeed/optim/scheduler.py:12-114``) over random parameters, step
counts and ``state_dict`` round trips, must produce the reference's values
step for step.  Skipped when the reference is not installed in
``baseline/_ref``.
"""

import importlib
import os
import sys

import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from minispeed_b200.optim.scheduler import build_scheduler
from minispeed_b200.precision import DynamicLossScaler

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
SETTINGS = dict(max_examples=300, deadline=None,
                suppress_health_check=[HealthCheck.function_scoped_fixture])


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "minispeed")):
        pytest.skip("reference not installed in baseline/_ref")
    sys.path.insert(0, REF)
    try:
        return (importlib.import_module("minispeed.precision"),
                importlib.import_module("minispeed.optim.scheduler"))
    finally:
        sys.path.remove(REF)


class _Opt:
    def __init__(self, lrs):
        self.param_groups = [{"lr": lr} for lr in lrs]


@settings(**SETTINGS)
@given(enabled=st.booleans(), init=st.sampled_from([0.0, 1.0, 256.0, 3.0]),
       power=st.one_of(st.none(), st.integers(0, 30)), window=st.integers(0, 5),
       overflows=st.lists(st.booleans(), max_size=60))
def test_loss_scaler_matches_reference(ref, enabled, init, power, window, overflows):
    ref_prec, _ = ref
    a = DynamicLossScaler(enabled=enabled, init_scale=init, scale_window=window)
    b = ref_prec.DynamicLossScaler(enabled=enabled, init_scale=init, scale_window=window)
    if power is not None:
        a.set_scale_from_power(power)
        b.set_scale_from_power(power)
    for i, o in enumerate(overflows):
        a.update(o)
        b.update(o)
        assert (a.scale, a.good_steps, a.skipped_steps, a.loss_scale_factor) == \
               (b.scale, b.good_steps, b.skipped_steps, b.loss_scale_factor), i
        if i == len(overflows) // 2:
            a2 = DynamicLossScaler(enabled=enabled, init_scale=init, scale_window=window)
            a2.load_state_dict(b.state_dict())          # reference state -> ours
            assert a2.state_dict() == a.state_dict()


@settings(**SETTINGS)
@given(kind=st.sampled_from(["WarmupLR", "WarmupDecayLR", "WarmupLRConst", "ConstantLR"]),
       lo=st.sampled_from([0.0, 1e-5, 3e-4]), hi=st.sampled_from([None, 1e-3, 6e-4]),
       warm=st.integers(0, 12), total=st.integers(1, 40), steps=st.integers(0, 50),
       lrs=st.lists(st.sampled_from([1e-3, 2e-3, 5e-4]), min_size=1, max_size=3),
       resume_at=st.integers(0, 50))
def test_schedules_match_reference(ref, kind, lo, hi, warm, total, steps, lrs, resume_at):
    _, ref_sched = ref
    params = {"warmup_min_lr": lo, "warmup_num_steps": warm, "total_num_steps": total,
              "warmup_max_lr": hi if hi is not None else lrs[0]}
    oa, ob = _Opt(lrs), _Opt(lrs)
    a = build_scheduler(oa, kind, dict(params))
    b = ref_sched.build_scheduler(ob, kind, dict(params))
    for i in range(steps):
        if i == resume_at:                          # reference state -> a fresh scheduler
            a = build_scheduler(oa, kind, dict(params))
            a.load_state_dict(b.state_dict())
        a.step()
        b.step()
        assert a.last_epoch == b.last_epoch
        assert a.get_last_lr() == pytest.approx(b.get_last_lr(), rel=1e-12, abs=0)
        assert [g["lr"] for g in oa.param_groups] == \
               pytest.approx([g["lr"] for g in ob.param_groups], rel=1e-12, abs=0)
    assert a.state_dict() == b.state_dict()
