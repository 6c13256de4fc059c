"""Checkpoint failures are detected before anything changes, on every rank.

Host-side fault injection only: a missing or truncated shard, a shard from
another world size, a checkpoint of another model, a save that dies before
``latest`` is written, and two-rank cases where only one rank fails (a
missing shard, a full disk while saving, ranks that would load different
tags): every rank must fail promptly, change nothing, keep ``latest``, and
stay in lockstep for the collectives that follow.
"""

import os

import pytest
import torch
import torch.multiprocessing as mp

import minispeed_b200 as ms
from minispeed_b200 import checkpoint as ckpt
from tests.helpers import config, free_port, make_data, make_net, rank_slice, run, set_rank_env

GAS, MICRO = 2, 4


def _trained(tmp_path, stage=2, steps=2):
    x, y = make_data(steps + 2, GAS, 1, MICRO)
    eng = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=GAS, stage=stage))
    run(eng, x, y, steps, GAS)
    eng.save_checkpoint(str(tmp_path), tag="t")
    return eng, x, y


def _snapshot(eng):
    return ({k: v.clone() for k, v in eng.state_dict().items()},
            [g.data.clone() for g in eng.flat_groups], eng.global_steps,
            eng.lr_scheduler.last_epoch)


def _assert_unchanged(eng, snap):
    params, masters, steps, epoch = snap
    for k, v in eng.state_dict().items():
        assert torch.equal(v, params[k]), k
    for g, m in zip(eng.flat_groups, masters):
        assert torch.equal(g.data, m)
    assert eng.global_steps == steps and eng.lr_scheduler.last_epoch == epoch


def _fresh(stage=2):
    return ms.initialize(model=make_net(seed=5), config=config(micro=MICRO, gas=GAS, stage=stage))


@pytest.mark.parametrize("stage", [2, 3])
def test_missing_shard(stage, tmp_path):
    _trained(tmp_path, stage)
    os.remove(tmp_path / "t" / ckpt.optim_states_name(0))
    eng = _fresh(stage)
    snap = _snapshot(eng)
    if stage == 3:
        eng.optimizer.free_parameters()
    with pytest.raises(FileNotFoundError, match="rank 0"):
        eng.load_checkpoint(str(tmp_path))
    assert not eng.optimizer.params_gathered or stage < 3   # freed again
    _assert_unchanged(eng, snap)


def test_world_size_mismatch(tmp_path):
    _trained(tmp_path)
    path = tmp_path / "t" / ckpt.optim_states_name(0)
    state = torch.load(path, weights_only=True)
    state["world_size"] = 2
    torch.save(state, path)
    eng = _fresh()
    snap = _snapshot(eng)
    with pytest.raises(RuntimeError, match="world_size=2"):
        eng.load_checkpoint(str(tmp_path))
    _assert_unchanged(eng, snap)


def test_truncated_shard(tmp_path):
    _trained(tmp_path)
    path = tmp_path / "t" / ckpt.optim_states_name(0)
    data = path.read_bytes()
    path.write_bytes(data[: len(data) // 3])
    eng = _fresh()
    snap = _snapshot(eng)
    with pytest.raises(Exception):
        eng.load_checkpoint(str(tmp_path))
    _assert_unchanged(eng, snap)


class _Wrapped(torch.nn.Module):
    """The same network one level down: same sizes, other state-dict keys."""

    def __init__(self):
        super().__init__()
        self.net = make_net(seed=5)

    def forward(self, x):
        return self.net(x)


def test_checkpoint_of_another_model(tmp_path):
    _trained(tmp_path)
    wider = make_net(seed=5)
    wider.out = torch.nn.Linear(32, 2)                 # other sizes
    for model, match in ((wider, "size mismatch"), (_Wrapped(), "module keys differ")):
        eng = ms.initialize(model=model, config=config(micro=MICRO, gas=GAS, stage=2))
        snap = _snapshot(eng)
        with pytest.raises(RuntimeError, match=match):
            eng.load_checkpoint(str(tmp_path))
        _assert_unchanged(eng, snap)
    _fresh().load_checkpoint(str(tmp_path))           # the matching model still loads


def test_save_that_dies_before_latest_keeps_the_old_tag(tmp_path, monkeypatch):
    eng, x, y = _trained(tmp_path)
    eng.save_checkpoint(str(tmp_path), tag="good")
    assert (tmp_path / "latest").read_text() == "good"

    def dead(*a, **k):
        raise RuntimeError("rank died")

    monkeypatch.setattr(ckpt.comm, "all_reduce_flag", dead)
    with pytest.raises(RuntimeError, match="rank died"):
        eng.save_checkpoint(str(tmp_path), tag="partial")
    monkeypatch.undo()
    assert (tmp_path / "latest").read_text() == "good"
    assert not [n for n in os.listdir(tmp_path / "partial") if n.endswith(".tmp")]
    fresh = _fresh()
    tag, _ = fresh.load_checkpoint(str(tmp_path))
    assert tag == "good"


WORLD = 2


def _two_rank_worker(rank, port, out_dir):
    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    x, y = make_data(4, GAS, WORLD, MICRO)
    x, y = rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO)
    cfg = config(micro=MICRO, gas=GAS, stage=2)
    eng = ms.initialize(model=make_net(), config=cfg)
    run(eng, x, y, 2, GAS)
    eng.save_checkpoint(out_dir, tag="t")
    ms.comm.barrier()
    if rank == 1:
        os.remove(os.path.join(out_dir, "t", ckpt.optim_states_name(1)))
    ms.comm.barrier()
    fresh = ms.initialize(model=make_net(seed=5), config=cfg)
    snap = _snapshot(fresh)
    try:
        fresh.load_checkpoint(out_dir)
        outcome = "loaded"
    except FileNotFoundError:
        outcome = "missing"
    except RuntimeError as e:
        outcome = "other rank" if "another rank" in str(e) else repr(e)
    _assert_unchanged(fresh, snap)
    # the ranks are still in lockstep: training continues on both
    run(fresh, x[2:], y[2:], 2, GAS)
    torch.save({"outcome": outcome, "params": fresh.state_dict()},
               os.path.join(out_dir, f"r{rank}.pt"))
    ms.comm.destroy()


def test_one_rank_missing_shard_fails_both_and_keeps_lockstep(tmp_path):
    mp.spawn(_two_rank_worker, args=(free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    r0 = torch.load(tmp_path / "r0.pt", weights_only=False)
    r1 = torch.load(tmp_path / "r1.pt", weights_only=False)
    assert r0["outcome"] == "other rank" and r1["outcome"] == "missing"
    for k in r0["params"]:
        torch.testing.assert_close(r0["params"][k], r1["params"][k], rtol=0, atol=0)


def _diverging_tags_worker(rank, port, out_dir):
    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    x, y = make_data(2, GAS, WORLD, MICRO)
    x, y = rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO)
    cfg = config(micro=MICRO, gas=GAS, stage=1)
    eng = ms.initialize(model=make_net(), config=cfg)
    run(eng, x, y, 1, GAS)
    eng.save_checkpoint(out_dir, tag="t1")
    run(eng, x[1:], y[1:], 1, GAS)
    eng.save_checkpoint(out_dir, tag="t2")
    fresh = ms.initialize(model=make_net(seed=5), config=cfg)
    snap = _snapshot(fresh)
    try:      # as if each rank saw a different ``latest`` file
        fresh.load_checkpoint(out_dir, tag="t1" if rank == 0 else "t2")
        outcome = "loaded"
    except RuntimeError as e:
        outcome = "refused" if "different checkpoints" in str(e) else repr(e)
    _assert_unchanged(fresh, snap)
    torch.save(outcome, os.path.join(out_dir, f"o{rank}.pt"))
    ms.comm.destroy()


def test_ranks_refuse_to_load_different_tags(tmp_path):
    mp.spawn(_diverging_tags_worker, args=(free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    assert [torch.load(tmp_path / f"o{r}.pt") for r in range(WORLD)] == ["refused", "refused"]


def _failed_write_worker(rank, port, out_dir):
    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    x, y = make_data(2, GAS, WORLD, MICRO)
    x, y = rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO)
    eng = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=GAS, stage=2))
    run(eng, x, y, 1, GAS)
    eng.save_checkpoint(out_dir, tag="good")
    if rank == 1:
        def full_disk(*a, **k):
            raise OSError(28, "No space left on device")
        ckpt.torch.save = full_disk
    try:
        eng.save_checkpoint(out_dir, tag="bad")
        outcome = "saved"
    except OSError:
        outcome = "own error"
    except RuntimeError as e:
        outcome = "other rank" if "another rank" in str(e) else repr(e)
    ms.comm.barrier()      # still in lockstep
    with open(os.path.join(out_dir, f"w{rank}.txt"), "w") as fh:   # torch.save is patched
        fh.write(outcome)
    ms.comm.destroy()


def test_failed_write_on_one_rank_fails_all_and_keeps_latest(tmp_path):
    mp.spawn(_failed_write_worker, args=(free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    assert (tmp_path / "w0.txt").read_text() == "other rank"
    assert (tmp_path / "w1.txt").read_text() == "own error"
    assert (tmp_path / "latest").read_text() == "good"


def _failed_latest_worker(rank, port, out_dir):
    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    x, y = make_data(2, GAS, WORLD, MICRO)
    x, y = rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO)
    eng = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=GAS, stage=3))
    run(eng, x, y, 1, GAS)
    eng.save_checkpoint(out_dir, tag="good")
    if rank == 0:
        real_replace = ckpt.os.replace

        def failing_replace(src, dst):
            if os.path.basename(dst) == "latest":
                raise OSError(5, "Input/output error")
            return real_replace(src, dst)
        ckpt.os.replace = failing_replace
    try:
        eng.save_checkpoint(out_dir, tag="bad")
        outcome = "saved"
    except OSError:
        outcome = "own error"
    except RuntimeError as e:
        outcome = "other rank" if "failed to update latest" in str(e) else repr(e)
    gathered = eng.optimizer.params_gathered
    ms.comm.barrier()      # still in lockstep
    with open(os.path.join(out_dir, f"l{rank}.txt"), "w") as fh:
        fh.write(f"{outcome} gathered={gathered}")
    ms.comm.destroy()


def test_failed_latest_update_on_rank0_fails_all(tmp_path):
    """Rank 0 fails to move ``latest`` after every shard is written: every
    rank raises at once (none waits for a barrier rank 0 never reaches), and
    stage-3 parameters are freed again on every rank."""
    mp.spawn(_failed_latest_worker, args=(free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    assert (tmp_path / "l0.txt").read_text() == "own error gathered=False"
    assert (tmp_path / "l1.txt").read_text() == "other rank gathered=False"
    assert (tmp_path / "latest").read_text() == "good"
