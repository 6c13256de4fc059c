"""The process-group contract of ``minispeed_b200.comm``.

Backend and device choice follow the environment contract of the reference
(``minispeed/comm.py:22-48``), checked here against a faked CUDA inventory;
the collectives are checked as single-process no-ops / copies and on two
gloo ranks.
"""

import os

import pytest
import torch
import torch.multiprocessing as mp

from minispeed_b200 import comm
from tests.helpers import free_port, set_rank_env


@pytest.fixture
def fake_cuda(monkeypatch):
    def setup(available: bool, count: int):
        monkeypatch.setattr(torch.cuda, "is_available", lambda: available)
        monkeypatch.setattr(torch.cuda, "device_count", lambda: count)
    for k in ("MINISPEED_BACKEND", "MINISPEED_DEVICE", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(k, raising=False)
    return setup


def test_backend_choice(fake_cuda, monkeypatch):
    fake_cuda(True, 8)
    monkeypatch.setenv("WORLD_SIZE", "8")
    assert comm.resolve_backend() == "nccl"
    monkeypatch.setenv("WORLD_SIZE", "16")           # ranks share GPUs
    assert comm.resolve_backend() == "gloo"
    fake_cuda(False, 0)
    monkeypatch.setenv("WORLD_SIZE", "1")
    assert comm.resolve_backend() == "gloo"
    monkeypatch.setenv("MINISPEED_BACKEND", "nccl")  # forced wins
    assert comm.resolve_backend() == "nccl"


def test_device_choice(fake_cuda, monkeypatch):
    fake_cuda(True, 4)
    monkeypatch.setenv("LOCAL_RANK", "2")
    assert comm.resolve_device() == torch.device("cuda", 2)
    monkeypatch.setenv("LOCAL_RANK", "7")            # clamped to the visible devices
    assert comm.resolve_device() == torch.device("cuda", 3)
    monkeypatch.setenv("MINISPEED_DEVICE", "cpu")
    assert comm.resolve_device() == torch.device("cpu")
    monkeypatch.delenv("MINISPEED_DEVICE")
    fake_cuda(False, 0)
    assert comm.resolve_device() == torch.device("cpu")


def test_single_process_collectives_are_local(monkeypatch):
    for k in ("RANK", "WORLD_SIZE"):
        monkeypatch.delenv(k, raising=False)
    comm.init_distributed()                          # no torchrun variables: nothing
    assert not comm.is_distributed() and comm.get_rank() == 0 and comm.get_world_size() == 1
    comm.barrier()
    t = torch.arange(4.0)
    assert comm.all_reduce(t, "max") is t and torch.equal(t, torch.arange(4.0))
    assert comm.all_reduce_flag(True) is True and comm.all_reduce_flag(False) is False
    out = torch.zeros(4)
    comm.reduce_scatter(out, t)
    assert torch.equal(out, t)
    out = torch.zeros(4)
    comm.all_gather_flat(out, t)
    assert torch.equal(out, t)
    assert comm.broadcast(t) is t
    assert comm.all_gather_object({"a": 1}) == [{"a": 1}]


WORLD = 2


def _worker(rank, port, out_dir):
    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    comm.init_distributed()
    res = {"rank": comm.get_rank(), "world": comm.get_world_size(),
           "backend": torch.distributed.get_backend()}
    x = torch.tensor([1.0 + rank, 10.0 * (rank + 1)])
    res["sum"] = comm.all_reduce(x.clone(), "sum")
    res["max"] = comm.all_reduce(x.clone(), "max")
    res["min"] = comm.all_reduce(x.clone(), "min")
    res["flag_any"] = comm.all_reduce_flag(rank == 1)
    res["flag_none"] = comm.all_reduce_flag(False)
    full = torch.arange(4.0) + 100 * rank                # [0..3] and [100..103]
    shard = torch.zeros(2)
    res["rs"] = comm.reduce_scatter(shard, full).clone()
    gathered = torch.zeros(4)
    res["ag"] = comm.all_gather_flat(gathered, torch.full((2,), float(rank))).clone()
    b = torch.full((3,), float(rank))
    res["bcast"] = comm.broadcast(b, src=1).clone()
    ts = [torch.full((2,), float(rank)), torch.full((3,), float(rank), dtype=torch.float64)]
    comm.broadcast_tensors(ts, src=0)
    res["bcast_many"] = [t.clone() for t in ts]
    res["objs"] = comm.all_gather_object(rank * 7)
    comm.barrier()
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))
    comm.destroy()


def test_two_rank_collectives(tmp_path):
    mp.spawn(_worker, args=(free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    for rank in range(WORLD):
        r = torch.load(tmp_path / f"r{rank}.pt", weights_only=False)
        assert (r["rank"], r["world"], r["backend"]) == (rank, 2, "gloo")
        assert r["sum"].tolist() == [3.0, 30.0]
        assert r["max"].tolist() == [2.0, 20.0] and r["min"].tolist() == [1.0, 10.0]
        assert r["flag_any"] is True and r["flag_none"] is False
        assert r["rs"].tolist() == ([100.0, 102.0] if rank == 0 else [104.0, 106.0])
        assert r["ag"].tolist() == [0.0, 0.0, 1.0, 1.0]
        assert r["bcast"].tolist() == [1.0, 1.0, 1.0]
        assert [t.tolist() for t in r["bcast_many"]] == [[0.0, 0.0], [0.0, 0.0, 0.0]]
        assert r["objs"] == [0, 7]
