"""``import minispeed_b200.alias`` makes ``import minispeed`` code run here.

Each case runs in a fresh interpreter: the in-process suite may already
have imported the real reference package (checkpoint interop tests).
"""

import os
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _py(code: str) -> subprocess.CompletedProcess:
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE")}
    env.update(MINISPEED_DEVICE="cpu", PYTHONPATH=ROOT)
    return subprocess.run([sys.executable, "-c", textwrap.dedent(code)], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=300)


def test_reference_style_script_runs_unchanged():
    r = _py("""
        import minispeed_b200.alias
        import minispeed as ms
        import minispeed_b200
        import torch
        import torch.nn as nn
        from minispeed.config import ConfigError, DeepSpeedConfig
        from minispeed.flat import FlatParamGroup
        from minispeed.optim.scheduler import WarmupDecayLR, WarmupLR
        from minispeed.precision import DynamicLossScaler, has_overflow
        from minispeed.activation_checkpointing import checkpoint
        assert ms is minispeed_b200 and ms.DeepSpeedEngine is minispeed_b200.DeepSpeedEngine
        assert has_overflow is minispeed_b200.precision.has_overflow
        torch.manual_seed(0)
        model = nn.Sequential(nn.Linear(8, 16), nn.Tanh(), nn.Linear(16, 1))
        engine, opt, _, sched = ms.initialize(model=model, model_parameters=model.parameters(),
            config={"train_micro_batch_size_per_gpu": 4, "gradient_accumulation_steps": 1,
                    "optimizer": {"type": "AdamW", "params": {"lr": 1e-2}}})
        x, y = torch.randn(4, 8), torch.randn(4, 1)
        for _ in range(3):
            loss = ((engine(x) - y) ** 2).mean()
            engine.backward(loss)
            engine.step()
        assert engine.global_steps == 3 and isinstance(engine, minispeed_b200.DeepSpeedEngine)
        print("ok")
    """)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-3000:]


def test_refuses_when_another_minispeed_is_loaded():
    r = _py("""
        import sys, types
        sys.modules["minispeed"] = types.ModuleType("minispeed")
        try:
            import minispeed_b200.alias
        except RuntimeError as e:
            print("refused:", "already imported" in str(e))
    """)
    assert r.returncode == 0 and "refused: True" in r.stdout, r.stderr[-3000:]


def test_uninstall_removes_the_names():
    r = _py("""
        import sys
        import minispeed_b200.alias as a
        assert "minispeed.precision" in sys.modules
        a.uninstall()
        assert "minispeed" not in sys.modules and "minispeed.precision" not in sys.modules
        print("ok")
    """)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr[-3000:]
