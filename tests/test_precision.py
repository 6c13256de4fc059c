import torch

from minispeed_b200.optim.scheduler import WarmupDecayLR, WarmupLR, build_scheduler
from minispeed_b200.precision import DynamicLossScaler, has_overflow


class _Opt:
    def __init__(self, lr=0.0):
        self.param_groups = [{"lr": lr}, {"lr": lr}]


def test_scale_doubles_after_window_and_caps():
    s = DynamicLossScaler(init_scale=4.0, scale_window=2, max_scale=16.0)
    for _ in range(2):
        s.update(False)
    assert s.scale == 8.0
    for _ in range(10):
        s.update(False)
    assert s.scale == 16.0


def test_overflow_halves_resets_and_floors():
    s = DynamicLossScaler(init_scale=4.0, scale_window=2)
    s.update(False)
    s.update(True)
    assert (s.scale, s.good_steps, s.skipped_steps) == (2.0, 0, 1)
    s.update(True)
    s.update(True)
    assert s.scale == 1.0  # floor
    s.update(False)
    s.update(False)
    assert s.scale == 2.0


def test_disabled_scaler_is_constant_one():
    s = DynamicLossScaler(enabled=False, init_scale=1024.0)
    assert s.loss_scale_factor == 1.0
    s.update(True)
    assert s.scale == 1.0 and s.skipped_steps == 0


def test_static_scale_still_adapts():
    s = DynamicLossScaler(init_scale=256.0, scale_window=1)
    s.update(True)
    assert s.scale == 128.0


def test_power_and_state_roundtrip():
    s = DynamicLossScaler()
    s.set_scale_from_power(5)
    s.update(True)
    t = DynamicLossScaler()
    t.load_state_dict(s.state_dict())
    assert t.state_dict() == s.state_dict() == {"enabled": True, "scale": 16.0,
                                                "good_steps": 0, "skipped_steps": 1}


def test_has_overflow():
    assert not has_overflow(torch.ones(3), None, torch.empty(0))
    assert has_overflow(torch.tensor([0.0, float("-inf")]))
    assert has_overflow(torch.ones(2), torch.tensor([float("nan")], dtype=torch.float16))


def test_warmup_lr_sequence_and_all_groups():
    opt = _Opt()
    sch = WarmupLR(opt, warmup_min_lr=0.0, warmup_max_lr=1.0, warmup_num_steps=4)
    seq = []
    for _ in range(6):
        sch.step()
        seq.append(sch.get_last_lr())
    assert seq == [0.0, 0.25, 0.5, 0.75, 1.0, 1.0]
    assert opt.param_groups[1]["lr"] == 1.0


def test_warmup_decay_sequence():
    opt = _Opt()
    sch = WarmupDecayLR(opt, warmup_min_lr=0.0, warmup_max_lr=1.0, warmup_num_steps=2,
                        total_num_steps=6)
    seq = []
    for _ in range(8):
        sch.step()
        seq.append(round(sch.get_last_lr(), 6))
    assert seq == [0.0, 0.5, 1.0, 0.75, 0.5, 0.25, 0.0, 0.0]


def test_scheduler_state_and_factory():
    opt = _Opt(lr=0.1)
    sch = build_scheduler(opt, "WarmupDecayLR", {"warmup_min_lr": 0.0, "warmup_max_lr": 0.2,
                                                 "warmup_num_steps": 0, "total_num_steps": 10})
    for _ in range(3):
        sch.step()
    sd = sch.state_dict()
    assert sd["type"] == "WarmupDecayLR" and sd["last_epoch"] == 2
    other = build_scheduler(_Opt(), "ConstantLR", {"warmup_max_lr": 0.2})
    other.load_state_dict(sd)
    assert other.last_epoch == 2
    assert isinstance(other, WarmupLR)
