"""minispeed_b200 - a ZeRO training engine built for NVIDIA B200 (sm_100a).

Drop-in API of lzwjava/minispeed::

    import minispeed_b200 as ms

    engine, optimizer, _, lr_scheduler = ms.initialize(
        model=model, model_parameters=model.parameters(), config="ds_config.json")
    loss = loss_fn(engine(x), y)
    engine.backward(loss)
    engine.step()

PyTorch is the framework layer; the optimizer step, the collectives fused
with it and the model hot ops run as hand-written sm_100a kernels
(``minispeed_b200._C``).

Reference: the package exports of ``minispeed/__init__.py:23-42``
(``initialize``, ``DeepSpeedEngine``, ``DeepSpeedConfig``, ``ConfigError``,
``ZeROOptimizer``, ``DynamicLossScaler``, ``WarmupLR``, ``WarmupDecayLR``,
``Timers``, ``set_seed``, ``comm``).
"""

from . import comm
from .config import ConfigError, DeepSpeedConfig
from .engine import DeepSpeedEngine, initialize
from .optim import WarmupDecayLR, WarmupLR
from .precision import DynamicLossScaler
from .utils import Timers, set_seed
from .zero import ZeROOptimizer

__version__ = "0.1.0"

__all__ = [
    "initialize",
    "DeepSpeedEngine",
    "DeepSpeedConfig",
    "ConfigError",
    "ZeROOptimizer",
    "DynamicLossScaler",
    "WarmupLR",
    "WarmupDecayLR",
    "Timers",
    "set_seed",
    "comm",
    "__version__",
]
