"""Config parsing against the reference parser on generated configs.

Random DeepSpeed-subset dicts (valid and invalid: batch sizes that do not
divide, unknown dtypes and optimizers, ZeRO stage 4, offload, conflicting
fp16/bf16, falsy sections) must be accepted or rejected alike by
``minispeed_b200.config.DeepSpeedConfig`` and the reference's
(``minispeed/config.py:38-201``), and every resolved field must agree.
Skipped when the reference is not installed in ``baseline/_ref``.
"""

import importlib
import os
import sys

import pytest
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from minispeed_b200.config import ConfigError, DeepSpeedConfig

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")

FIELDS = ("micro_batch", "gas", "train_batch_size", "dtype", "fp16_enabled", "bf16_enabled",
          "loss_scale", "initial_scale_power", "loss_scale_window", "scale_wrt_gas",
          "gradient_clipping", "zero_stage", "optimizer_type", "optimizer_params",
          "scheduler_type", "scheduler_params", "steps_per_print", "seed", "drop_overflow")


@pytest.fixture(scope="module")
def ref_config():
    if not os.path.isdir(os.path.join(REF, "minispeed")):
        pytest.skip("reference not installed in baseline/_ref")
    sys.path.insert(0, REF)
    try:
        return importlib.import_module("minispeed.config")
    finally:
        sys.path.remove(REF)


def _maybe(strategy):
    return st.one_of(st.none(), strategy)


section = st.fixed_dictionaries({}, optional={
    "enabled": st.booleans(),
    "loss_scale": st.sampled_from([0, 0.0, 128, 1024.0]),
    "initial_scale_power": st.integers(0, 24),
    "loss_scale_window": st.integers(1, 2000),
})

zero = st.one_of(st.just(False), st.just({}), st.fixed_dictionaries(
    {"stage": st.integers(0, 4)},
    optional={"offload_optimizer": st.just({"device": "cpu"}),
              "offload_param": st.just({"device": "nvme"}),
              "stage3_gather_16bit_weights_on_model_save": st.booleans()}))

optimizer = st.fixed_dictionaries({}, optional={
    "type": st.sampled_from(["AdamW", "Adam", "SGD"]),
    "params": st.fixed_dictionaries({}, optional={
        "lr": st.sampled_from([1e-3, 3e-4, 0.1]),
        "betas": st.sampled_from([[0.9, 0.95], (0.8, 0.99)]),
        "eps": st.sampled_from([1e-8, 1e-6]),
        "weight_decay": st.sampled_from([0.0, 0.01, 0.1])}),
})

scheduler = st.fixed_dictionaries({}, optional={
    "type": st.sampled_from(["WarmupLR", "WarmupDecayLR", "WarmupLRConst", "ConstantLR",
                             "OneCycle"]),
    "params": st.fixed_dictionaries({}, optional={
        "warmup_min_lr": st.sampled_from([0.0, 1e-5]),
        "warmup_max_lr": st.sampled_from([1e-3, 6e-4]),
        "warmup_num_steps": st.integers(0, 100),
        "total_num_steps": st.integers(1, 1000)}),
})

configs = st.fixed_dictionaries({}, optional={
    "train_batch_size": st.integers(1, 128),
    "train_micro_batch_size_per_gpu": st.integers(1, 16),
    "gradient_accumulation_steps": st.integers(1, 8),
    "dtype": st.sampled_from(["fp32", "FP16", "bf16", "fp8"]),
    "fp16": st.one_of(st.just(None), section),
    "bf16": st.one_of(st.just(None), st.fixed_dictionaries({}, optional={
        "enabled": st.booleans()})),
    "gradient_clipping": st.sampled_from([0, 0.0, None, 1.0, 0.5]),
    "zero_optimization": zero,
    "optimizer": optimizer,
    "scheduler": scheduler,
    "steps_per_print": st.integers(1, 100),
    "seed": st.integers(0, 10 ** 6),
    "drop_overflow_on_loss": st.booleans(),
    "scale_wrt_gas": st.booleans(),
    "unknown_key": st.just({"ignored": True}),
})


def _parse(cls, err, raw, world):
    try:
        return cls(raw, world_size=world), None
    except err as e:
        return None, e


@settings(max_examples=400, deadline=None, suppress_health_check=[HealthCheck.function_scoped_fixture])
@given(raw=configs, world=st.sampled_from([1, 2, 4, 8]))
def test_same_verdict_and_fields_as_reference(ref_config, raw, world):
    ours, e_ours = _parse(DeepSpeedConfig, ConfigError, dict(raw), world)
    ref, e_ref = _parse(ref_config.DeepSpeedConfig, ref_config.ConfigError, dict(raw), world)
    assert (e_ours is None) == (e_ref is None), (raw, world, e_ours, e_ref)
    if ours is None:
        return
    for f in FIELDS:
        assert getattr(ours, f) == getattr(ref, f), (f, raw, world)
