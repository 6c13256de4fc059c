"""DeepSpeed-subset JSON configuration with fail-fast validation.

The accepted schema, its defaults and every rejected combination follow the
reference parser (``minispeed/config.py:38-201``) so that an existing
``ds_config.json`` keeps working unchanged:

* batch math: ``train_batch_size == micro * gas * world`` (gas derived when
  omitted, ``config.py:61-83``);
* dtype: ``"dtype"`` key, else ``fp16.enabled``, else ``bf16.enabled``, else
  fp32; fp16 and bf16 both enabled is an error (``config.py:86-94,163-176``);
* ZeRO stage in {0,1,2,3}; offload and
  ``stage3_gather_16bit_weights_on_model_save: false`` are rejected
  (``config.py:105-123``);
* optimizer AdamW/Adam, scheduler WarmupDecayLR/WarmupLR/WarmupLRConst/
  ConstantLR with the reference defaults (``config.py:126-155``).

Unknown keys are ignored, as in the reference.  Knobs specific to this
implementation live under a namespaced ``"b200"`` section (see
:class:`B200Options`); they never change the training math, only how the
step pipeline is executed.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Any, Dict, Optional, Union

DTYPES = ("fp32", "fp16", "bf16")
OPTIMIZERS = ("AdamW", "Adam")
SCHEDULERS = ("WarmupDecayLR", "WarmupLR", "WarmupLRConst", "ConstantLR")


class ConfigError(ValueError):
    """Raised for a malformed or unsupported configuration."""


def _read(config: Union[dict, str, os.PathLike, None]) -> Dict[str, Any]:
    if config is None:
        return {}
    if isinstance(config, dict):
        return config
    if isinstance(config, (str, os.PathLike)):
        with open(config, "r", encoding="utf-8") as fh:
            return json.load(fh)
    raise ConfigError(f"config must be a dict, a JSON path or None, got {type(config)!r}")


def _section(raw: dict, key: str) -> dict:
    """A sub-dict that may be absent, null or ``false`` (all mean empty)."""
    value = raw.get(key)
    if not value:
        return {}
    if not isinstance(value, dict):
        raise ConfigError(f"'{key}' must be an object, got {value!r}")
    return value


@dataclass
class B200Options:
    """Execution knobs of the B200 step pipeline (``"b200": {...}`` in JSON).

    ``comm``: ``"auto"`` uses the fused in-kernel NVLink collectives when every
    rank owns a distinct GPU of one node and falls back to NCCL otherwise;
    ``"nccl"`` forces the library path; ``"fused"`` requires the fused path.
    ``bucket_mb``: gradient bucket size for backward/communication overlap.
    ``overlap``: move each model block's gradients (fused collectives) as
    soon as backward has produced them, on a second stream, instead of after
    backward (env ``MINISPEED_OVERLAP=1``).  At stages 1-2 the copy engines
    send each peer its part of the block (the step then reduces local
    copies); at stages 0 and 3 the reduction kernel runs per block.
    ``wait_timeout_ms``: bound on every cross-GPU spin inside fused kernels;
    past it the kernel reports an error status instead of waiting forever.
    ``cuda_graph``: ``engine.train_batch`` replays forward + backward as one
    captured CUDA graph (stages 0-2, CUDA) after ``graph_warmup`` eager
    micro-steps; env ``MINISPEED_CUDA_GRAPH=1`` turns it on.
    ``device_timers``: also time the engine's phases on the GPU with CUDA
    events (``engine.device_time_ms()``); env ``MINISPEED_DEVICE_TIMERS=1``.
    """

    comm: str = "auto"
    bucket_mb: float = 64.0
    overlap: bool = False
    wait_timeout_ms: float = 10000.0
    cuda_graph: bool = False
    graph_warmup: int = 2
    device_timers: bool = False

    @classmethod
    def parse(cls, raw: dict) -> "B200Options":
        sec = _section(raw, "b200")
        opts = cls(
            comm=str(sec.get("comm", os.environ.get("MINISPEED_COMM", "auto"))).lower(),
            bucket_mb=float(sec.get("bucket_mb", 64.0)),
            overlap=bool(sec.get("overlap", os.environ.get("MINISPEED_OVERLAP", "0") == "1")),
            wait_timeout_ms=float(sec.get("wait_timeout_ms", 10000.0)),
            cuda_graph=bool(sec.get("cuda_graph",
                                    os.environ.get("MINISPEED_CUDA_GRAPH", "0") == "1")),
            graph_warmup=int(sec.get("graph_warmup", 2)),
            device_timers=bool(sec.get("device_timers",
                                       os.environ.get("MINISPEED_DEVICE_TIMERS", "0") == "1")),
        )
        if opts.comm not in ("auto", "nccl", "fused"):
            raise ConfigError(f"b200.comm must be auto|nccl|fused, got {opts.comm!r}")
        if opts.bucket_mb <= 0:
            raise ConfigError("b200.bucket_mb must be positive")
        if opts.graph_warmup < 1:
            raise ConfigError("b200.graph_warmup must be at least 1")
        return opts


class DeepSpeedConfig:
    """Parsed and validated training configuration."""

    def __init__(self, config: Union[dict, str, None], world_size: int = 1):
        raw = _read(config)
        self.raw = raw
        self.world_size = int(world_size)
        self._parse_batch(raw)
        self._parse_precision(raw)
        clip = raw.get("gradient_clipping")
        self.gradient_clipping: Optional[float] = float(clip) if clip else None
        self._parse_zero(raw)
        self._parse_optimizer(raw)
        self._parse_scheduler(raw)
        self.steps_per_print = int(raw.get("steps_per_print", 10))
        # parsed for schema compatibility; the engine does not consume them
        self.seed = int(raw.get("seed", 1234))
        self.drop_overflow = bool(raw.get("drop_overflow_on_loss", True))
        self.b200 = B200Options.parse(raw)

    # ----------------------------------------------------------------- parts
    def _parse_batch(self, raw: dict) -> None:
        micro = int(raw.get("train_micro_batch_size_per_gpu", 1))
        total = raw.get("train_batch_size")
        gas = raw.get("gradient_accumulation_steps")
        per_step = micro * self.world_size
        if gas is None and total is not None:
            if int(total) % per_step:
                raise ConfigError(
                    f"train_batch_size={total} is not divisible by "
                    f"micro_batch*world_size={per_step}")
            gas = int(total) // per_step
        gas = 1 if gas is None else int(gas)
        derived = micro * gas * self.world_size
        if total is not None and int(total) != derived:
            raise ConfigError(
                f"train_batch_size={total} != micro_batch({micro}) * gas({gas}) "
                f"* world_size({self.world_size}) = {derived}")
        self.micro_batch = micro
        self.gas = gas
        self.train_batch_size = derived

    def _parse_precision(self, raw: dict) -> None:
        fp16 = _section(raw, "fp16")
        bf16 = _section(raw, "bf16")
        explicit = raw.get("dtype")
        if explicit is not None:
            dtype = str(explicit).lower()
            if dtype not in DTYPES:
                raise ConfigError(f"dtype must be one of {DTYPES}, got {explicit!r}")
        elif fp16.get("enabled"):
            dtype = "fp16"
        elif bf16.get("enabled"):
            dtype = "bf16"
        else:
            dtype = "fp32"
        if fp16.get("enabled") and bf16.get("enabled"):
            raise ConfigError("fp16 and bf16 cannot both be enabled")
        self.dtype = dtype
        self.fp16_enabled = dtype == "fp16"
        self.bf16_enabled = dtype == "bf16"
        self.loss_scale = float(fp16.get("loss_scale", 0.0))  # 0 => dynamic
        self.initial_scale_power = int(fp16.get("initial_scale_power", 16))
        self.loss_scale_window = int(fp16.get("loss_scale_window", 1000))
        # kept for schema parity: engine.backward takes its own flag
        self.scale_wrt_gas = bool(raw.get("scale_wrt_gas", True))

    def _parse_zero(self, raw: dict) -> None:
        zero = _section(raw, "zero_optimization")
        stage = int(zero.get("stage", 0))
        if stage not in (0, 1, 2, 3):
            raise ConfigError(f"Unsupported zero stage {stage}; stages 0, 1, 2 and 3 exist")
        if zero.get("offload_optimizer") or zero.get("offload_param"):
            raise ConfigError("CPU/NVMe offload is not supported")
        if zero.get("stage3_gather_16bit_weights_on_model_save") is False:
            raise ConfigError(
                "stage-3 checkpoints always store the full model state; "
                "stage3_gather_16bit_weights_on_model_save must be true or omitted")
        self.zero_stage = stage

    def _parse_optimizer(self, raw: dict) -> None:
        opt = _section(raw, "optimizer")
        kind = str(opt.get("type", "AdamW"))
        if kind not in OPTIMIZERS:
            raise ConfigError(f"Unsupported optimizer {kind!r}; expected one of {OPTIMIZERS}")
        params = dict(opt.get("params") or {})
        params.setdefault("lr", 1e-3)
        params.setdefault("betas", (0.9, 0.999))
        params.setdefault("eps", 1e-8)
        params.setdefault("weight_decay", 0.0)
        params["betas"] = tuple(float(b) for b in params["betas"])
        self.optimizer_type = kind
        self.optimizer_params = params

    def _parse_scheduler(self, raw: dict) -> None:
        sched = _section(raw, "scheduler")
        kind = str(sched.get("type", "WarmupLR"))
        if kind not in SCHEDULERS:
            raise ConfigError(f"Unsupported scheduler {kind!r}; expected one of {SCHEDULERS}")
        params = dict(sched.get("params") or {})
        params.setdefault("warmup_num_steps", 0)
        params.setdefault("warmup_max_lr", float(self.optimizer_params["lr"]))
        params.setdefault("warmup_min_lr", 0.0)
        self.scheduler_type = kind
        self.scheduler_params = params

    # --------------------------------------------------------------- helpers
    @property
    def torch_dtype(self):
        import torch

        return {"fp32": torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}[self.dtype]

    def __repr__(self) -> str:  # pragma: no cover - debug helper
        return (f"DeepSpeedConfig(dtype={self.dtype}, zero_stage={self.zero_stage}, "
                f"micro_batch={self.micro_batch}, gas={self.gas}, "
                f"world_size={self.world_size}, clip={self.gradient_clipping}, "
                f"comm={self.b200.comm})")


def load_config(config, world_size: int = 1) -> DeepSpeedConfig:
    """Accept a :class:`DeepSpeedConfig`, a dict, a JSON path or ``None``."""
    if isinstance(config, DeepSpeedConfig):
        return config
    return DeepSpeedConfig(config, world_size=world_size)
