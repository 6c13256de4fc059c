"""Sharded checkpoints in the reference's on-disk format.

Layout (reference ``minispeed/checkpoint.py:1-125``)::

    save_dir/latest                                        text: newest tag
    save_dir/<tag>/mp_rank_00_model_states.pt              rank 0: {"module", "tag"}
    save_dir/<tag>/zero_pp_rank<r>_mp_rank_00_optim_states.pt   every rank

The per-rank file holds ``optimizer`` (param groups + shard Adam state),
``fp32_groups`` (the full padded fp32 master buffer at stages 0-2, this
rank's shard at stage 3), ``lr_scheduler``, ``loss_scaler``, the step
counters, ``rank`` and ``world_size``.  Files written here load in the
reference and vice versa.

Two robustness changes that keep the format:

* every file is written to ``<name>.tmp`` and renamed into place, and rank 0
  writes ``latest`` only after every rank has reported its shard written
  (one flag all-reduce), so a crash or a failed write never leaves
  ``latest`` naming an incomplete tag, and a rank whose write failed makes
  every rank raise at once instead of leaving them in a barrier (the
  reference writes ``latest`` before the shards, ``checkpoint.py:52-68``);
* a load reads and checks every rank's files, and the ranks agree on the
  outcome and the tag, before any state changes;
* the saved module tensors are detached copies, one per distinct storage
  (tied weights stay tied), so the file has the same structure as the
  reference's even though the live params are views into one arena.
"""

from __future__ import annotations

import os
from typing import Optional, Tuple

import torch

from . import comm

MODEL_STATES = "mp_rank_00_model_states.pt"
LATEST = "latest"


def optim_states_name(rank: int) -> str:
    return f"zero_pp_rank{rank}_mp_rank_00_optim_states.pt"


def _read_latest(save_dir: str) -> str:
    with open(os.path.join(save_dir, LATEST), "r", encoding="utf-8") as fh:
        return fh.read().strip()


def _atomic_save(obj, path: str) -> None:
    tmp = path + ".tmp"
    torch.save(obj, tmp)
    os.replace(tmp, path)


def _standalone_state_dict(module: torch.nn.Module) -> dict:
    """Module state with each distinct tensor storage copied once."""
    out, seen = {}, {}
    for k, v in module.state_dict().items():
        key = (v.data_ptr(), v.dtype, tuple(v.shape), v.stride())
        if key not in seen:
            seen[key] = v.detach().clone()
        out[k] = seen[key]
    return out


@torch.no_grad()
def save_checkpoint(engine, save_dir: str, tag: Optional[str] = None) -> str:
    """Write ``save_dir/<tag>/`` (rank 0: the module states; every rank: its optimizer
    shard) and then ``save_dir/latest``.  Collective: every rank calls it."""
    tag = tag or f"global_step{engine.global_steps}"
    ckpt_dir = os.path.join(save_dir, tag)
    os.makedirs(ckpt_dir, exist_ok=True)

    was_gathered = engine.optimizer.params_gathered
    engine.optimizer.gather_parameters()
    engine.optimizer.sync_master_weights()

    err: Optional[BaseException] = None
    try:
        if engine.rank == 0:
            _atomic_save({"module": _standalone_state_dict(engine.module), "tag": tag},
                         os.path.join(ckpt_dir, MODEL_STATES))
        state = {
            "optimizer": engine.optimizer.state_dict(),
            "fp32_groups": [g.data.clone() for g in engine.flat_groups],
            "lr_scheduler": engine.lr_scheduler.state_dict(),
            "loss_scaler": engine.loss_scaler.state_dict(),
            "global_steps": engine.global_steps,
            "micro_steps": engine.micro_steps,
            "grad_norm": engine.grad_norm,
            "rank": engine.rank,
            "world_size": engine.world_size,
        }
        _atomic_save(state, os.path.join(ckpt_dir, optim_states_name(engine.rank)))
    except Exception as e:  # e.g. a full disk: reported to every rank below
        err = e
    # every rank's files are written (or one failed) before ``latest`` moves
    failed = comm.all_reduce_flag(err is not None)
    if failed:
        if not was_gathered:
            engine.optimizer.free_parameters()
        if err is not None:
            raise err
        raise RuntimeError(f"checkpoint {ckpt_dir}: another rank failed to write its files; "
                           "latest still names the previous checkpoint")
    latest_err: Optional[BaseException] = None
    if engine.rank == 0:
        try:
            latest = os.path.join(save_dir, LATEST)
            with open(latest + ".tmp", "w", encoding="utf-8") as fh:
                fh.write(tag)
            os.replace(latest + ".tmp", latest)
        except Exception as e:  # reported to every rank by the flag below
            latest_err = e
    # the flag doubles as the final barrier: no rank waits on a rank 0 that
    # raised, and every rank frees stage-3 parameters on either outcome
    latest_failed = comm.all_reduce_flag(latest_err is not None)
    if not was_gathered:
        engine.optimizer.free_parameters()
    if latest_failed:
        if latest_err is not None:
            raise latest_err
        raise RuntimeError(f"checkpoint {ckpt_dir}: rank 0 failed to update {LATEST}; the "
                           "files are written but latest still names the previous checkpoint")
    return ckpt_dir


def _read_and_check(engine, ckpt_dir: str) -> Tuple[dict, dict]:
    """This rank's two files, checked against the engine before anything is
    changed: shard present, same world size, same groups and master sizes,
    same module keys and shapes."""
    optim_path = os.path.join(ckpt_dir, optim_states_name(engine.rank))
    if not os.path.exists(optim_path):
        raise FileNotFoundError(f"Missing optimizer shard for rank {engine.rank}: {optim_path}")
    model_state = torch.load(os.path.join(ckpt_dir, MODEL_STATES), map_location="cpu",
                             weights_only=True)
    state = torch.load(optim_path, map_location="cpu", weights_only=True)
    saved_world = int(state.get("world_size", engine.world_size))
    if saved_world != engine.world_size:
        raise RuntimeError(f"Checkpoint was saved with world_size={saved_world} but the "
                           f"current world_size={engine.world_size}; ZeRO shards do not "
                           "transfer between world sizes.")
    groups = state["fp32_groups"]
    if len(groups) != len(engine.flat_groups):
        raise RuntimeError(f"checkpoint has {len(groups)} parameter groups, engine has "
                           f"{len(engine.flat_groups)}")
    for g, buf in zip(engine.flat_groups, groups):
        if buf.numel() != g.data.numel():
            raise RuntimeError(f"fp32 master size mismatch: checkpoint {buf.numel()} vs "
                               f"engine {g.data.numel()}")
    live = engine.module.state_dict()
    saved = model_state["module"]
    if set(saved) != set(live):
        missing, extra = sorted(set(live) - set(saved)), sorted(set(saved) - set(live))
        raise RuntimeError(f"module keys differ: missing {missing[:5]}, unexpected {extra[:5]}")
    for k, v in saved.items():
        if torch.is_tensor(v) and torch.is_tensor(live[k]) and \
                tuple(v.shape) != tuple(live[k].shape):
            raise RuntimeError(f"module tensor {k}: checkpoint shape {tuple(v.shape)} vs "
                               f"engine {tuple(live[k].shape)}")
    return model_state, state


@torch.no_grad()
def load_checkpoint(engine, load_dir: str, tag: Optional[str] = None) -> Tuple[str, dict]:
    """Restore a checkpoint on every rank, or on none.

    Each rank reads and checks its files first; the ranks then agree (one
    flag all-reduce) before any state changes.  A rank whose files are bad
    raises its own error (``FileNotFoundError`` for a missing shard), the
    others a ``RuntimeError``, and no rank has changed anything, so no rank
    is left waiting in a collective the failed one never joins."""
    was_gathered = engine.optimizer.params_gathered
    engine.optimizer.gather_parameters()     # stage 3: full-shaped params to check and load

    err: Optional[BaseException] = None
    ckpt_dir = None
    try:
        tag = tag or _read_latest(load_dir)
        ckpt_dir = os.path.join(load_dir, tag)
        model_state, state = _read_and_check(engine, ckpt_dir)
    except Exception as e:  # re-raised below, after every rank has reported
        err = e
    # one collective: every rank's outcome and tag (a save directory that is
    # not shared can show the ranks different ``latest`` files)
    reports = comm.all_gather_object((err is not None, tag))
    if any(failed for failed, _ in reports) or len({t for _, t in reports}) > 1:
        if not was_gathered:
            engine.optimizer.free_parameters()
        if err is not None:
            raise err
        if len({t for _, t in reports}) > 1:
            raise RuntimeError(f"ranks would load different checkpoints: "
                               f"{[t for _, t in reports]}; nothing was changed")
        raise RuntimeError(f"checkpoint {ckpt_dir} failed to load on another rank; "
                           "nothing was changed")

    engine.module.load_state_dict(model_state["module"])
    for g, buf in zip(engine.flat_groups, state["fp32_groups"]):
        g.data.copy_(buf)
        g.copy_flat_to_model()
    engine.optimizer._masters_stale = False

    if engine.config.zero_stage >= 3:
        engine.optimizer.free_parameters()
        if was_gathered:
            engine.optimizer.gather_parameters()

    engine.optimizer.load_state_dict(state["optimizer"])
    engine.lr_scheduler.load_state_dict(state["lr_scheduler"])
    engine.loss_scaler.load_state_dict(state["loss_scaler"])
    engine.global_steps = int(state.get("global_steps", 0))
    engine.micro_steps = int(state.get("micro_steps", 0))
    engine.grad_norm = state.get("grad_norm")
    comm.barrier()
    return tag, state
