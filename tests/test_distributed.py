"""Two ranks on gloo/CPU must reproduce a single-process run on the union batch.

Each rank trains on its half of every micro-batch; the averaged gradient equals
the union-batch gradient, so trajectories agree up to fp32 summation order.
Covers stages 0-3, the exact global clipping norm (including stage 1) and the
partitioning of optimizer state.
"""

import os

import pytest
import torch
import torch.multiprocessing as mp

import minispeed_b200 as ms
from tests.helpers import config, free_port, make_data, make_net, mse, rank_slice, run, set_rank_env

WORLD, STEPS, GAS, MICRO = 2, 5, 2, 4


def _worker(rank, stage, port, out_dir, clip, dtype):
    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    engine = ms.initialize(model=make_net(), config=config(
        micro=MICRO, gas=GAS, stage=stage, clip=clip, dtype=dtype))
    x, y = make_data(STEPS, GAS, WORLD, MICRO)
    losses = run(engine, rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO), STEPS, GAS)
    params = {k: v.clone() for k, v in engine.state_dict().items()}
    engine.optimizer.sync_master_weights()
    torch.save({"losses": torch.tensor(losses), "params": params,
                "steps": engine.global_steps, "norm": engine.grad_norm,
                "exp_avg": [s["exp_avg"].clone() for s in engine.optimizer.state],
                "opt_step": engine.optimizer.state[0]["step"],
                "masters": engine.flat_groups[0].data.clone(),
                "coll": engine.collectives, "staged": dict(ms.comm.staged_calls)},
               os.path.join(out_dir, f"r{rank}.pt"))
    ms.comm.destroy()


def padded_total():
    total = sum(p.numel() for p in make_net().parameters())
    return -(-total // WORLD) * WORLD


def _single(clip, dtype):
    engine = ms.initialize(model=make_net(), config=config(
        micro=MICRO * WORLD, gas=GAS, stage=0, clip=clip, dtype=dtype))
    x, y = make_data(STEPS, GAS, WORLD, MICRO)
    losses = run(engine, x, y, STEPS, GAS)
    return torch.tensor(losses), engine.state_dict(), engine.grad_norm


def _spawn(stage, tmp_path, clip=1.0, dtype="fp32"):
    mp.spawn(_worker, args=(stage, free_port(), str(tmp_path), clip, dtype), nprocs=WORLD,
             join=True)
    return [torch.load(tmp_path / f"r{r}.pt", weights_only=False) for r in range(WORLD)]


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
def test_two_ranks_match_union_batch(stage, tmp_path):
    r0, r1 = _spawn(stage, tmp_path)
    ref_losses, ref_params, _ = _single(1.0, "fp32")
    assert r0["steps"] == r1["steps"] == STEPS
    assert r0["coll"] == "gloo"
    torch.testing.assert_close((r0["losses"] + r1["losses"]) / 2, ref_losses,
                               rtol=5e-3, atol=1e-4)
    num = den = 0.0
    for k, ref in ref_params.items():
        torch.testing.assert_close(r0["params"][k], r1["params"][k], rtol=0, atol=0)
        num += float((r0["params"][k] - ref).pow(2).sum())
        den += float(ref.pow(2).sum())
    assert (num / den) ** 0.5 < 1e-4
    if stage < 3:   # full fp32 masters agree across ranks once synced
        torch.testing.assert_close(r0["masters"], r1["masters"], rtol=0, atol=0)
    else:           # stage 3 keeps disjoint shards
        assert r0["masters"].numel() == r1["masters"].numel() == padded_total() // WORLD


@pytest.mark.parametrize("stage", [1, 2, 3])
def test_clipping_uses_exact_global_norm(stage, tmp_path):
    """Tiny clip threshold: every step clips, so the norm must be global."""
    r0, r1 = _spawn(stage, tmp_path, clip=0.01)
    _, ref_params, ref_norm = _single(0.01, "fp32")
    assert r0["norm"] == pytest.approx(r1["norm"], rel=0, abs=0)
    assert r0["norm"] == pytest.approx(ref_norm, rel=1e-3)
    num = den = 0.0
    for k, ref in ref_params.items():
        num += float((r0["params"][k] - ref).pow(2).sum())
        den += float(ref.pow(2).sum())
    assert (num / den) ** 0.5 < 1e-4


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
def test_optimizer_state_is_partitioned(stage, tmp_path):
    r0, r1 = _spawn(stage, tmp_path)
    total = sum(p.numel() for p in make_net().parameters())
    padded = -(-total // WORLD) * WORLD
    n0 = [t.numel() for t in r0["exp_avg"]]
    assert n0 == [t.numel() for t in r1["exp_avg"]]
    assert r0["opt_step"] == STEPS
    if stage == 0:
        assert n0 == [padded]
        torch.testing.assert_close(r0["exp_avg"][0], r1["exp_avg"][0])
    else:
        assert n0 == [padded // WORLD]
        assert not torch.equal(r0["exp_avg"][0], r1["exp_avg"][0])


def test_bf16_two_ranks_stage2(tmp_path):
    r0, r1 = _spawn(2, tmp_path, dtype="bf16")
    ref_losses, _, _ = _single(1.0, "bf16")
    torch.testing.assert_close((r0["losses"] + r1["losses"]) / 2, ref_losses,
                               rtol=3e-2, atol=3e-3)
    for k in r0["params"]:
        torch.testing.assert_close(r0["params"][k], r1["params"][k], rtol=0, atol=0)


def test_bucket_plan_covers_each_shard_exactly():
    """Overlapped buckets + the step's remainder reduce every element of the
    rank's shard once, on 16-byte boundaries."""
    import types

    from minispeed_b200.parallel.fused import FusedCollectives

    for stage in (0, 2):
        for rank in range(3):
            fc = FusedCollectives.__new__(FusedCollectives)
            fc.OVERLAP_MODE = "kernel"
            fc.rank, fc.world_size, fc.stage = rank, 3, stage
            g = types.SimpleNamespace(shard_size=1000, shard_start=1000 * rank,
                                      shard_end=1000 * (rank + 1))
            fc.groups = [g]
            buckets = [[(0, 5, 733)], [(0, 733, 1501)], [(0, 1501, 2999)]]
            slots = fc.plan_buckets(buckets)
            assert slots == 3 * FusedCollectives.BUCKET_SLOTS
            a, b = fc._shard_range(g)
            segs = [(s, e) for bk in fc.bucket_plan for (_, s, e) in bk] + fc.remaining[0]
            segs.sort()
            assert segs[0][0] == a and segs[-1][1] == b
            for (s0, e0), (s1, _) in zip(segs, segs[1:]):
                assert e0 == s1            # disjoint and gap-free
            for bk in fc.bucket_plan:
                for (_, s, e) in bk:
                    assert s % 8 == 0 and e % 8 == 0 and e > s


def _leaving_worker(rank, port, out_dir):
    import time

    set_rank_env(rank, WORLD, port, "gloo", "cpu")
    os.environ["MINISPEED_PG_TIMEOUT_S"] = "20"
    engine = ms.initialize(model=make_net(), config=config(micro=MICRO, gas=1, stage=2))
    x, y = make_data(2, 1, WORLD, MICRO)
    xs, ys = rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO)
    engine.backward(mse(engine(xs[0, 0]), ys[0, 0]))
    engine.step()
    if rank == 1:
        os._exit(0)          # leaves between steps, nothing of its own in flight
    t0 = time.time()
    try:
        engine.backward(mse(engine(xs[1, 0]), ys[1, 0]))
        engine.step()
        result = "no error"
    except Exception as e:   # the step's reduce-scatter finds the peer gone
        result = type(e).__name__
    torch.save({"result": result, "seconds": time.time() - t0},
               os.path.join(out_dir, "r0.pt"))
    os._exit(0)


@pytest.mark.timeout(180)
def test_surviving_rank_fails_cleanly_when_a_peer_leaves(tmp_path):
    """A rank that leaves mid-run makes the others' next collective raise
    (bounded by the process-group timeout) instead of hanging."""
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, port, str(tmp_path)))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=150)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung after its peer left")
    out = torch.load(tmp_path / "r0.pt", weights_only=False)
    assert out["result"] != "no error"
    assert out["seconds"] < 60


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
def test_host_staged_collectives_match(stage, tmp_path, monkeypatch):
    """Ranks that share a GPU use gloo, which does not reduce-scatter or
    all-gather CUDA tensors; those two then go through host copies.  Forced
    here on CPU ranks, the staged path gives the same results bit for bit."""
    (tmp_path / "a").mkdir()
    (tmp_path / "b").mkdir()
    plain = _spawn(stage, tmp_path / "a")
    monkeypatch.setenv("MINISPEED_STAGE_COLLECTIVES", "1")
    staged = _spawn(stage, tmp_path / "b")
    for p, s in zip(plain, staged):
        assert sum(p["staged"].values()) == 0
        # stage 0 only all-reduces; stages 1-3 reduce-scatter the gradient
        # and all-gather the parameters
        for kind in ("reduce_scatter", "all_gather"):
            assert (s["staged"][kind] > 0) == (stage >= 1), kind
        assert torch.equal(p["losses"], s["losses"])
        for k in p["params"]:
            assert torch.equal(p["params"][k], s["params"][k]), k
        assert torch.equal(p["masters"], s["masters"])


def test_dma_plan_sends_each_element_to_its_owner_once():
    """Copy-engine overlap: every bucket element outside this rank's shard is
    sent to exactly its owner, and the shard is split into the covered part
    (16-byte aligned) and the rest without gaps or overlaps."""
    from minispeed_b200.parallel.fused import dma_plan

    S, W, per = 1000, 3, 8
    buckets = [[(0, 5, 733)], [(0, 733, 1501)], [(0, 1501, 2999)]]
    for rank in range(W):
        sends, covered, remaining = dma_plan(buckets, [S], [per], W, rank)
        seen = []
        for k, bucket in enumerate(sends):
            for (i, q, e0, e1) in bucket:
                assert q != rank and q * S <= e0 < e1 <= (q + 1) * S
                lo, hi = buckets[k][0][1], buckets[k][0][2]
                assert lo <= e0 and e1 <= hi
                seen.append((e0, e1))
        seen.sort()
        total = sum(e1 - e0 for e0, e1 in seen)
        mine = max(0, min(2999, (rank + 1) * S) - max(5, rank * S))
        assert total == (2999 - 5) - mine
        segs = sorted(covered[0] + remaining[0])
        assert segs[0][0] == rank * S and segs[-1][1] == (rank + 1) * S
        for (s0, e0), (s1, _) in zip(segs, segs[1:]):
            assert e0 == s1
        for s0, e0 in covered[0]:
            assert s0 % per == 0 and e0 % per == 0


def test_peer_heap_view_refuses_an_overrun():
    """A view of a peer-heap region larger than the region is refused before
    any device call (every rank addresses the same layout, so an overrun
    would write into the next region of every peer)."""
    import torch

    from minispeed_b200.parallel.peer import PeerHeap

    heap = object.__new__(PeerHeap)          # the layout alone, no device memory
    heap.offsets = {"grad0": 0, "pshard0": 512}
    heap.sizes = {"grad0": 400, "pshard0": 100}
    heap.base, heap.device = 0, torch.device("cpu")
    with pytest.raises(ValueError, match="does not fit region 'grad0'"):
        heap.view("grad0", torch.float16, 201)
    with pytest.raises(ValueError, match="does not fit region 'pshard0'"):
        heap.view("pshard0", torch.float32, 26)
