"""Flat-buffer layout against the reference's ``FlatParamGroup``.

For generated parameter shapes, world sizes, ranks and ZeRO stages, the
padded size, shard bounds, master range and master contents
(``minispeed/flat.py:36-193``) must equal the reference's, through
``copy_model_to_flat``, the stage-3 ``partition_params`` and the
``materialize`` / ``copy_flat_to_model`` / ``dematerialize`` cycle.  This
is the layout the checkpoint files carry.  Skipped when the reference is
not installed in ``baseline/_ref``.
"""

import importlib
import os
import sys

import pytest
import torch
import torch.nn as nn
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from minispeed_b200.flat import FlatParamGroup

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
CPU = torch.device("cpu")


@pytest.fixture(scope="module")
def ref_flat():
    if not os.path.isdir(os.path.join(REF, "minispeed")):
        pytest.skip("reference not installed in baseline/_ref")
    sys.path.insert(0, REF)
    try:
        return importlib.import_module("minispeed.flat")
    finally:
        sys.path.remove(REF)


def _params(shapes, seed):
    g = torch.Generator().manual_seed(seed)
    return [nn.Parameter(torch.randn(*s, generator=g)) for s in shapes]


def _layout(fg):
    return (fg.numel, fg.numel_padded, fg.shard_size, fg.shard_start, fg.shard_end,
            tuple(fg.master_range), fg.numel_shard())


shapes = st.lists(st.lists(st.integers(1, 7), min_size=1, max_size=3).map(tuple),
                  min_size=1, max_size=6)


@settings(max_examples=200, deadline=None,
          suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(shapes=shapes, world=st.integers(1, 8), stage=st.integers(0, 3), data=st.data())
def test_layout_and_masters_match_reference(ref_flat, shapes, world, stage, data):
    rank = data.draw(st.integers(0, world - 1))
    pa, pb = _params(shapes, 1), _params(shapes, 1)
    a = FlatParamGroup(pa, rank=rank, world_size=world, zero_stage=stage, device=CPU)
    b = ref_flat.FlatParamGroup(pb, rank=rank, world_size=world, zero_stage=stage, device=CPU)
    assert _layout(a) == _layout(b)
    a.copy_model_to_flat()
    b.copy_model_to_flat()
    assert torch.equal(a.data, b.data)
    if stage < 3:
        return
    a.partition_params()
    b.partition_params()
    assert _layout(a) == _layout(b)
    assert torch.equal(a.data, b.data)
    # gather cycle: a full buffer written back into the parameters
    full = torch.arange(a.numel_padded, dtype=torch.float32)
    for fg in (a, b):
        fg.materialize_params()
        fg.copy_flat_to_model(full)
    for p, q in zip(pa, pb):
        assert p.shape == q.shape and torch.equal(p.data, q.data)
    a.dematerialize_params()
    b.dematerialize_params()
    a.copy_flat_to_model()
    b.copy_flat_to_model()
    for p, q in zip(pa, pb):
        assert p.data.shape == q.data.shape and torch.equal(p.data, q.data)


@settings(max_examples=100, deadline=None,
          suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(shapes=shapes, world=st.integers(1, 4), stage=st.integers(0, 2), steps=st.integers(1, 4),
       lr=st.sampled_from([1e-3, 0.05]), wd=st.sampled_from([0.0, 0.1]),
       betas=st.sampled_from([(0.9, 0.999), (0.8, 0.95)]), data=st.data())
def test_adamw_shard_update_matches_reference(ref_flat, shapes, world, stage, steps, lr, wd,
                                               betas, data):
    """The AdamW update of a rank's shard (``minispeed/optim/adam.py:60-93``):
    same masters, moments and step counts after several steps."""
    from minispeed_b200.optim.adam import FlatAdam
    sys.path.insert(0, REF)
    try:
        ref_adam = importlib.import_module("minispeed.optim.adam")
    finally:
        sys.path.remove(REF)
    rank = data.draw(st.integers(0, world - 1))
    opts = [{"lr": lr, "betas": betas, "eps": 1e-8, "weight_decay": wd}]
    a = FlatParamGroup(_params(shapes, 2), rank=rank, world_size=world, zero_stage=stage,
                       device=CPU)
    b = ref_flat.FlatParamGroup(_params(shapes, 2), rank=rank, world_size=world,
                                zero_stage=stage, device=CPU)
    for fg in (a, b):
        fg.copy_model_to_flat()
    oa, ob = FlatAdam([a], opts, zero_stage=stage), ref_adam.FlatAdam([b], opts, zero_stage=stage)
    g = torch.Generator().manual_seed(9)
    for _ in range(steps):
        grad = torch.randn(a.numel_shard(), generator=g)
        for fg in (a, b):
            fg.grad_for_shard().copy_(grad)
        oa.step()
        ob.step()
    assert torch.equal(a.data, b.data)
    for sa, sb in zip(oa.state, ob.state):
        assert sa["step"] == sb["step"]
        assert torch.equal(sa["exp_avg"], sb["exp_avg"])
        assert torch.equal(sa["exp_avg_sq"], sb["exp_avg_sq"])
