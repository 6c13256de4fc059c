import json

import pytest

from minispeed_b200.config import ConfigError, DeepSpeedConfig


def test_gas_is_derived_from_global_batch():
    cfg = DeepSpeedConfig({"train_batch_size": 48, "train_micro_batch_size_per_gpu": 6},
                          world_size=4)
    assert cfg.gas == 2 and cfg.train_batch_size == 48


@pytest.mark.parametrize("raw,world", [
    ({"train_batch_size": 33, "train_micro_batch_size_per_gpu": 8}, 2),
    ({"train_batch_size": 64, "train_micro_batch_size_per_gpu": 8,
      "gradient_accumulation_steps": 3}, 2),
])
def test_batch_mismatch_raises(raw, world):
    with pytest.raises(ConfigError):
        DeepSpeedConfig(raw, world_size=world)


def test_dtype_resolution_order():
    assert DeepSpeedConfig({}).dtype == "fp32"
    assert DeepSpeedConfig({"fp16": {"enabled": True}}).dtype == "fp16"
    assert DeepSpeedConfig({"bf16": {"enabled": True}}).dtype == "bf16"
    assert DeepSpeedConfig({"dtype": "BF16"}).dtype == "bf16"
    assert DeepSpeedConfig({"dtype": "fp32", "fp16": {"enabled": True}}).dtype == "fp32"
    with pytest.raises(ConfigError):
        DeepSpeedConfig({"dtype": "fp8"})
    with pytest.raises(ConfigError):
        DeepSpeedConfig({"fp16": {"enabled": True}, "bf16": {"enabled": True}})


def test_zero_validation():
    assert DeepSpeedConfig({"zero_optimization": {"stage": 2}}).zero_stage == 2
    assert DeepSpeedConfig({"zero_optimization": False}).zero_stage == 0
    for bad in ({"stage": 4}, {"stage": 1, "offload_optimizer": {"device": "cpu"}},
                {"stage": 3, "offload_param": {"device": "nvme"}},
                {"stage": 3, "stage3_gather_16bit_weights_on_model_save": False}):
        with pytest.raises(ConfigError):
            DeepSpeedConfig({"zero_optimization": bad})
    ok = DeepSpeedConfig({"zero_optimization": {
        "stage": 3, "stage3_gather_16bit_weights_on_model_save": True}})
    assert ok.zero_stage == 3


def test_optimizer_and_scheduler_defaults():
    cfg = DeepSpeedConfig({"optimizer": {"type": "Adam", "params": {"lr": 3e-4}}})
    assert cfg.optimizer_params["betas"] == (0.9, 0.999)
    assert cfg.optimizer_params["weight_decay"] == 0.0
    assert cfg.scheduler_type == "WarmupLR"
    assert cfg.scheduler_params["warmup_max_lr"] == 3e-4
    assert cfg.scheduler_params["warmup_min_lr"] == 0.0
    with pytest.raises(ConfigError):
        DeepSpeedConfig({"optimizer": {"type": "SGD"}})
    with pytest.raises(ConfigError):
        DeepSpeedConfig({"scheduler": {"type": "OneCycle"}})


def test_fp16_fields_and_misc():
    cfg = DeepSpeedConfig({"fp16": {"enabled": True, "loss_scale": 128,
                                    "loss_scale_window": 50}, "gradient_clipping": 0})
    assert cfg.loss_scale == 128.0 and cfg.loss_scale_window == 50
    assert cfg.initial_scale_power == 16
    assert cfg.gradient_clipping is None
    assert cfg.steps_per_print == 10 and cfg.seed == 1234


def test_json_path_and_b200_section(tmp_path):
    p = tmp_path / "ds.json"
    p.write_text(json.dumps({"train_micro_batch_size_per_gpu": 2, "b200": {"comm": "nccl",
                                                                           "bucket_mb": 16}}))
    cfg = DeepSpeedConfig(str(p))
    assert cfg.micro_batch == 2
    assert cfg.b200.comm == "nccl" and cfg.b200.bucket_mb == 16
    with pytest.raises(ConfigError):
        DeepSpeedConfig({"b200": {"comm": "mpi"}})


def test_reference_example_config_parses():
    from pathlib import Path

    cfg = DeepSpeedConfig(str(Path(__file__).parent.parent / "examples" / "ds_config.json"))
    assert cfg.dtype == "fp16" and cfg.zero_stage == 2 and cfg.gas == 2
