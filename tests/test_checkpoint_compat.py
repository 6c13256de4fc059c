"""Checkpoints move between minispeed_b200 and the reference engine.

Writes a checkpoint with one framework, resumes it with the other, and checks
that the restored weights, optimizer shards and scheduler/scaler state agree
and that both continue along the same trajectory.  Needs the unmodified
reference installed in ``baseline/_ref`` (skipped otherwise).
"""

import importlib
import os
import sys

import pytest
import torch

import minispeed_b200 as ours
from tests.helpers import config, make_data, make_net, run

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
GAS, MICRO = 2, 4


@pytest.fixture(scope="module")
def ref():
    if not os.path.isdir(os.path.join(REF, "minispeed")):
        pytest.skip("reference not installed in baseline/_ref")
    sys.path.insert(0, REF)
    try:
        return importlib.import_module("minispeed")
    finally:
        sys.path.remove(REF)


def _pair(ref, stage, writer, tmp_path):
    x, y = make_data(6, GAS, 1, MICRO)
    cfg = config(micro=MICRO, gas=GAS, stage=stage, warmup=3, scheduler="WarmupDecayLR",
                 total=20, dtype="fp32")
    lib_w, lib_r = (ours, ref) if writer == "ours" else (ref, ours)
    w = lib_w.initialize(model=make_net(), config=cfg)
    run(w, x, y, 2, GAS)
    w.save_checkpoint(str(tmp_path), tag="mid")
    expect = run(w, x[2:], y[2:], 2, GAS)
    r = lib_r.initialize(model=make_net(seed=99), config=cfg)
    r.load_checkpoint(str(tmp_path))
    assert r.global_steps == 2
    assert r.lr_scheduler.last_epoch == 1
    got = run(r, x[2:], y[2:], 2, GAS)
    torch.testing.assert_close(torch.tensor(got), torch.tensor(expect), rtol=1e-5, atol=1e-6)
    sw, sr = w.state_dict(), r.state_dict()
    for k in sw:
        torch.testing.assert_close(sr[k].float(), sw[k].float(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("stage", [0, 2, 3])
@pytest.mark.parametrize("writer", ["ours", "reference"])
def test_checkpoint_crosses_frameworks(ref, stage, writer, tmp_path):
    _pair(ref, stage, writer, tmp_path)


def test_file_layout_matches(ref, tmp_path):
    cfg = config(micro=MICRO, gas=1, stage=2)
    x, y = make_data(1, 1, 1, MICRO)
    a = ours.initialize(model=make_net(), config=cfg)
    run(a, x, y, 1, 1)
    a.save_checkpoint(str(tmp_path / "a"))
    b = ref.initialize(model=make_net(), config=cfg)
    run(b, x, y, 1, 1)
    b.save_checkpoint(str(tmp_path / "b"))
    for root in ("a", "b"):
        assert (tmp_path / root / "latest").read_text() == "global_step1"
    ours_files = sorted(os.listdir(tmp_path / "a" / "global_step1"))
    ref_files = sorted(os.listdir(tmp_path / "b" / "global_step1"))
    assert ours_files == ref_files
    sa = torch.load(tmp_path / "a" / "global_step1" / ref_files[-1], weights_only=False)
    sb = torch.load(tmp_path / "b" / "global_step1" / ref_files[-1], weights_only=False)
    assert sorted(sa) == sorted(sb)
    assert sorted(sa["optimizer"]) == sorted(sb["optimizer"])
    assert [t.shape for t in sa["fp32_groups"]] == [t.shape for t in sb["fp32_groups"]]
    ma = torch.load(tmp_path / "a" / "global_step1" / ref_files[0], weights_only=False)
    mb = torch.load(tmp_path / "b" / "global_step1" / ref_files[0], weights_only=False)
    assert sorted(ma["module"]) == sorted(mb["module"])


WORLD = 2


def _import_ref():
    sys.path.insert(0, REF)
    try:
        return importlib.import_module("minispeed")
    finally:
        sys.path.remove(REF)


def _two_rank_worker(rank, stage, writer, port, out_dir):
    from tests.helpers import rank_slice, set_rank_env
    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    ref = _import_ref()
    lib_w, lib_r = (ours, ref) if writer == "ours" else (ref, ours)
    x, y = make_data(6, GAS, WORLD, MICRO)
    x, y = rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO)
    # no clipping: the reference's stage-1 norm covers only the local shard
    cfg = config(micro=MICRO, gas=GAS, stage=stage, clip=0, warmup=3,
                 scheduler="WarmupDecayLR", total=20, dtype="fp32")
    w = lib_w.initialize(model=make_net(), config=cfg)
    run(w, x, y, 2, GAS)
    w.save_checkpoint(out_dir, tag="mid")
    expect = run(w, x[2:], y[2:], 2, GAS)
    r = lib_r.initialize(model=make_net(seed=99), config=cfg)
    r.load_checkpoint(out_dir)
    got = run(r, x[2:], y[2:], 2, GAS)
    torch.save({"expect": torch.tensor(expect), "got": torch.tensor(got),
                "steps": r.global_steps, "w": w.state_dict(), "r": r.state_dict()},
               os.path.join(out_dir, f"result{rank}.pt"))
    ours.comm.destroy()


@pytest.mark.parametrize("stage", [1, 2, 3])
@pytest.mark.parametrize("writer", ["ours", "reference"])
def test_two_rank_checkpoint_crosses_frameworks(ref, stage, writer, tmp_path):
    """W=2 over gloo: the per-rank optimizer shards (and, at stage 3, the
    fp32 master shards) written by one framework resume in the other."""
    import torch.multiprocessing as mp
    from tests.helpers import free_port
    mp.spawn(_two_rank_worker, args=(stage, writer, free_port(), str(tmp_path)),
             nprocs=WORLD, join=True)
    names = sorted(os.listdir(tmp_path / "mid"))
    assert names == ["mp_rank_00_model_states.pt",
                     "zero_pp_rank0_mp_rank_00_optim_states.pt",
                     "zero_pp_rank1_mp_rank_00_optim_states.pt"]
    for rank in range(WORLD):
        res = torch.load(tmp_path / f"result{rank}.pt", weights_only=False)
        assert res["steps"] == 4
        torch.testing.assert_close(res["got"], res["expect"], rtol=1e-5, atol=1e-6)
        for k in res["w"]:
            torch.testing.assert_close(res["r"][k].float(), res["w"][k].float(),
                                       rtol=1e-5, atol=1e-6)
