"""Process-group bootstrap and host-level collectives.

``torch.distributed`` carries the plumbing: rendezvous (``env://``), the
rank/world bookkeeping, a key-value store for the peer-memory handshake of
the fused NVLink kernels (:mod:`minispeed_b200.parallel`) and the NCCL/gloo
collectives used on the fallback path and on CPU.  Every wrapper is a valid
no-op (or a local copy) for a single process, so the engine runs the same
code at world size 1.

Environment contract (reference ``minispeed/comm.py:22-91``):

* ``MINISPEED_BACKEND`` forces ``nccl`` or ``gloo``; otherwise NCCL when CUDA
  is present and ``WORLD_SIZE <= device_count``, else gloo (gloo can move CUDA
  tensors between ranks that share one GPU).
* ``MINISPEED_DEVICE`` forces the device; otherwise ``cuda:LOCAL_RANK``
  (clamped to the visible devices), else CPU.
* ``RANK``/``WORLD_SIZE``/``LOCAL_RANK``/``MASTER_ADDR``/``MASTER_PORT`` come
  from ``torchrun``.

Added here: ``MINISPEED_PG_TIMEOUT_S`` bounds every collective so that ranks
waiting for a peer that died end with an error instead of hanging.
"""

from __future__ import annotations

import datetime
import os
from typing import Iterable, List

import torch
import torch.distributed as dist

_OPS = {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}


def _env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def resolve_backend() -> str:
    """``MINISPEED_BACKEND`` if set, else NCCL when every rank can have its own
    visible GPU, else gloo."""
    forced = os.environ.get("MINISPEED_BACKEND")
    if forced:
        return forced
    if torch.cuda.is_available() and _env_int("WORLD_SIZE", 1) <= torch.cuda.device_count():
        return "nccl"
    return "gloo"


def get_local_rank() -> int:
    return _env_int("LOCAL_RANK", 0)


def resolve_device() -> torch.device:
    """``MINISPEED_DEVICE`` if set, else ``cuda:LOCAL_RANK`` (clamped to the visible
    GPUs), else the CPU."""
    forced = os.environ.get("MINISPEED_DEVICE")
    if forced:
        return torch.device(forced)
    if torch.cuda.is_available():
        return torch.device("cuda", min(get_local_rank(), torch.cuda.device_count() - 1))
    return torch.device("cpu")


def _initialized() -> bool:
    return dist.is_available() and dist.is_initialized()


def get_rank() -> int:
    return dist.get_rank() if _initialized() else _env_int("RANK", 0)


def get_world_size() -> int:
    return dist.get_world_size() if _initialized() else _env_int("WORLD_SIZE", 1)


def is_distributed() -> bool:
    """True when a process group with more than one rank exists."""
    return _initialized() and dist.get_world_size() > 1


def init_distributed(timeout_s: float | None = None) -> None:
    """Create the process group from ``env://`` if torchrun variables exist.

    A no-op for a plain single process or when a group already exists.
    """
    if _initialized() or "RANK" not in os.environ or "WORLD_SIZE" not in os.environ:
        return
    backend = resolve_backend()
    if backend == "nccl":
        dev = resolve_device()
        if dev.type != "cuda":
            torch.cuda.set_device(0)
        elif dev.index is not None:     # a bare "cuda" keeps the current device
            torch.cuda.set_device(dev)
    if timeout_s is None:
        timeout_s = float(os.environ.get("MINISPEED_PG_TIMEOUT_S", 600))
    kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if backend == "nccl":
        kwargs["device_id"] = torch.device("cuda", torch.cuda.current_device())
    dist.init_process_group(backend=backend, init_method="env://", **kwargs)


def barrier() -> None:
    if is_distributed():
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def all_reduce(tensor: torch.Tensor, op: str = "sum") -> torch.Tensor:
    if is_distributed():
        dist.all_reduce(tensor, op=_OPS[op])
    return tensor


def _flag_device() -> torch.device:
    if _initialized() and dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def all_reduce_flag(flag: bool) -> bool:
    """Logical OR of a host bool over all ranks."""
    if not is_distributed():
        return bool(flag)
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=_flag_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return bool(t.item())


_FORCE_STAGING = os.environ.get("MINISPEED_STAGE_COLLECTIVES", "0") == "1"
# how many reduce-scatters / all-gathers took the host-staged path (tests
# check that the path they force is the one that ran)
staged_calls = {"reduce_scatter": 0, "all_gather": 0}


def host_staged(*tensors: torch.Tensor) -> bool:
    """Whether a reduce-scatter or all-gather over these tensors goes through
    host copies: gloo (the backend of ranks that share a GPU) moves CUDA
    tensors for broadcast, all-reduce and barrier, not for these two.
    ``MINISPEED_STAGE_COLLECTIVES=1`` forces the host copies (tests)."""
    if not _initialized():
        return False
    return _FORCE_STAGING or (dist.get_backend() == "gloo" and any(t.is_cuda for t in tensors))


def reduce_scatter(output: torch.Tensor, input_: torch.Tensor) -> torch.Tensor:
    """SUM-reduce ``input_`` (world * output.numel()) and keep this rank's slice."""
    if is_distributed():
        if host_staged(output, input_):
            # the receive buffer is written whole: no need to copy output down
            out = torch.empty_like(output, device="cpu")
            dist.reduce_scatter_tensor(out, input_.to("cpu", copy=True))
            output.copy_(out)
            staged_calls["reduce_scatter"] += 1
        else:
            dist.reduce_scatter_tensor(output, input_)
    else:
        output.copy_(input_)
    return output


def all_gather_flat(output: torch.Tensor, local_shard: torch.Tensor) -> torch.Tensor:
    """Concatenate every rank's shard, in rank order, into ``output``."""
    if is_distributed():
        if host_staged(output, local_shard):
            out = torch.empty_like(output, device="cpu")
            dist.all_gather_into_tensor(out, local_shard.to("cpu", copy=True))
            output.copy_(out)
            staged_calls["all_gather"] += 1
        else:
            dist.all_gather_into_tensor(output, local_shard)
    else:
        output.copy_(local_shard)
    return output


def broadcast(tensor: torch.Tensor, src: int = 0) -> torch.Tensor:
    if is_distributed():
        dist.broadcast(tensor, src=src)
    return tensor


def broadcast_tensors(tensors: Iterable[torch.Tensor], src: int = 0) -> None:
    """Broadcast many tensors with one collective per dtype.

    The tensors are packed into one contiguous buffer per dtype, broadcast,
    and unpacked in place: one launch instead of one per tensor.
    """
    if not is_distributed():
        return
    by_dtype: dict = {}
    for t in tensors:
        by_dtype.setdefault((t.dtype, t.device), []).append(t)
    for (dtype, device), group in by_dtype.items():
        flat = torch.cat([t.detach().reshape(-1) for t in group]) if group else None
        if flat is None or flat.numel() == 0:
            continue
        dist.broadcast(flat, src=src)
        off = 0
        for t in group:
            n = t.numel()
            t.detach().copy_(flat[off:off + n].view_as(t))
            off += n


def all_gather_object(obj) -> List:
    """Every rank's picklable ``obj``, in rank order (``[obj]`` in one process)."""
    if not is_distributed():
        return [obj]
    out: List = [None] * dist.get_world_size()
    dist.all_gather_object(out, obj)
    return out


def destroy() -> None:
    if _initialized():
        dist.destroy_process_group()
