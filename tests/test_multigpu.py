"""Two ranks on two GPUs: the fused NVLink collectives against the
single-process union-batch run and against the NCCL path (stages 0-3)."""

import os

import pytest
import torch
import torch.multiprocessing as mp

import minispeed_b200 as ms
from tests.helpers import config, free_port, make_data, make_net, rank_slice, run

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
WORLD, STEPS, GAS, MICRO = 2, 4, 2, 4


def _worker(rank, stage, dtype, comm_mode, port, out_dir):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "RANK": str(rank), "WORLD_SIZE": str(WORLD), "LOCAL_RANK": str(rank),
                       "LOCAL_WORLD_SIZE": str(WORLD), "MINISPEED_DEVICE": f"cuda:{rank}",
                       "MINISPEED_PG_TIMEOUT_S": "120", "NCCL_NVLS_ENABLE": "0"})
    os.environ.pop("MINISPEED_BACKEND", None)
    torch.cuda.set_device(rank)
    cfg = config(micro=MICRO, gas=GAS, stage=stage, dtype=dtype, clip=0.5,
                 b200={"comm": comm_mode, "wait_timeout_ms": 20000})
    engine = ms.initialize(model=make_net(), config=cfg)
    x, y = make_data(STEPS, GAS, WORLD, MICRO)
    losses = run(engine, rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO), STEPS, GAS,
                 device=f"cuda:{rank}")
    params = {k: v.detach().float().cpu() for k, v in engine.state_dict().items()}
    torch.save({"losses": torch.tensor(losses), "params": params, "coll": engine.collectives,
                "norm": engine.grad_norm, "steps": engine.global_steps},
               os.path.join(out_dir, f"r{rank}.pt"))
    engine.close()
    ms.comm.destroy()


def _spawn(tmp_path, stage, dtype, comm_mode):
    mp.spawn(_worker, args=(stage, dtype, comm_mode, free_port(), str(tmp_path)), nprocs=WORLD,
             join=True)
    return [torch.load(tmp_path / f"r{r}.pt", weights_only=False) for r in range(WORLD)]


@pytest.fixture(autouse=True)
def _two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


@pytest.mark.parametrize("stage", [0, 1, 2, 3])
def test_fused_nvlink_matches_single_process(stage, tmp_path, monkeypatch):
    r0, r1 = _spawn(tmp_path, stage, "fp32", "fused")
    assert r0["coll"] == "fused-nvlink"
    assert r0["steps"] == STEPS
    monkeypatch.setenv("MINISPEED_DEVICE", "cuda:0")
    ref = ms.initialize(model=make_net(), config=config(micro=MICRO * WORLD, gas=GAS, stage=0,
                                                        clip=0.5))
    x, y = make_data(STEPS, GAS, WORLD, MICRO)
    ref_losses = torch.tensor(run(ref, x, y, STEPS, GAS, device="cuda:0"))
    torch.testing.assert_close((r0["losses"] + r1["losses"]) / 2, ref_losses, rtol=2e-3,
                               atol=1e-4)
    assert r0["norm"] == r1["norm"]
    for k, v in ref.state_dict().items():
        torch.testing.assert_close(r0["params"][k], r1["params"][k], rtol=0, atol=0)
        torch.testing.assert_close(r0["params"][k], v.float().cpu(), rtol=2e-3, atol=2e-4)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_fused_matches_nccl_path(dtype, tmp_path):
    fused = _spawn(tmp_path / "f", 2, dtype, "fused") if (tmp_path / "f").mkdir() is None else None
    nccl = _spawn(tmp_path / "n", 2, dtype, "nccl") if (tmp_path / "n").mkdir() is None else None
    assert fused[0]["coll"] == "fused-nvlink" and nccl[0]["coll"] == "nccl"
    tol = 2e-2 if dtype == "bf16" else 2e-3
    torch.testing.assert_close(fused[0]["losses"], nccl[0]["losses"], rtol=tol, atol=tol)
    for k in fused[0]["params"]:
        torch.testing.assert_close(fused[0]["params"][k], nccl[0]["params"][k], rtol=tol,
                                   atol=tol)


def _gpt_worker(rank, stage, overlap, graph, port, out_dir, world=WORLD, comm_mode="fused"):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank),
                       "LOCAL_WORLD_SIZE": str(world), "MINISPEED_DEVICE": f"cuda:{rank}",
                       "MINISPEED_PG_TIMEOUT_S": "120", "NCCL_NVLS_ENABLE": "0"})
    os.environ.pop("MINISPEED_BACKEND", None)
    torch.cuda.set_device(rank)
    from minispeed_b200.models import GPT, GPTConfig, init_gpt2_
    torch.manual_seed(0)
    model = GPT(GPTConfig(vocab_size=512, block_size=64, n_layer=3, n_head=4, n_embd=128))
    init_gpt2_(model)
    cfg = {"train_micro_batch_size_per_gpu": 4, "gradient_accumulation_steps": 2,
           "gradient_clipping": 1.0, "dtype": "fp16",
           "fp16": {"enabled": True, "initial_scale_power": 10, "loss_scale_window": 3},
           "optimizer": {"type": "AdamW", "params": {"lr": 1e-3, "weight_decay": 0.1}},
           "zero_optimization": {"stage": stage},
           "b200": {"comm": comm_mode, "overlap": overlap, "cuda_graph": graph,
                    "wait_timeout_ms": 20000}}
    engine = ms.initialize(model=model, config=cfg)
    g = torch.Generator().manual_seed(11)
    data = [torch.randint(0, 512, (world * 4, 65), generator=g) for _ in range(12)]
    losses = []
    for t in data:
        t = t[rank * 4:(rank + 1) * 4].cuda()
        losses.append(float(engine.train_batch(t[:, :-1], targets=t[:, 1:])))
    params = {k: v.detach().float().cpu() for k, v in engine.state_dict().items()}
    torch.save({"losses": torch.tensor(losses), "params": params,
                "slots": engine.optimizer.overlap_slots,
                "planned": engine.optimizer.comm_stream is not None,
                "dma": bool(getattr(engine.optimizer.coll, "dma", False)),
                "steps": engine.global_steps,
                "scale": engine.get_loss_scale(), "coll": engine.collectives},
               os.path.join(out_dir, f"r{rank}.pt"))
    engine.close()
    ms.comm.destroy()


@pytest.mark.parametrize("stage,graph", [(0, False), (0, True), (1, False), (2, False),
                                         (2, True), (3, False)])
def test_overlapped_bucket_reduction_matches_step_reduction(stage, graph, tmp_path):
    """Buckets reduced during backward (stages 1-2: copied to their owners by
    the copy engines; stages 0 and 3: the reduction kernel on a second
    stream) give the same trajectory as the reduction at the step."""
    runs = {}
    for overlap in (False, True):
        d = tmp_path / f"o{int(overlap)}"
        d.mkdir()
        mp.spawn(_gpt_worker, args=(stage, overlap, graph, free_port(), str(d)), nprocs=WORLD,
                 join=True)
        runs[overlap] = [torch.load(d / f"r{r}.pt", weights_only=False) for r in range(WORLD)]
    off, on = runs[False], runs[True]
    assert not off[0]["planned"] and on[0]["planned"]       # the buckets were planned
    assert on[0]["dma"] == (stage in (1, 2))
    assert on[0]["steps"] == off[0]["steps"] == 6 and on[0]["scale"] == off[0]["scale"]
    torch.testing.assert_close(on[0]["losses"], off[0]["losses"], rtol=2e-3, atol=2e-3)
    for k in off[0]["params"]:
        torch.testing.assert_close(on[0]["params"][k], on[1]["params"][k], rtol=0, atol=0)
        torch.testing.assert_close(on[0]["params"][k], off[0]["params"][k], rtol=2e-3, atol=2e-4)


def test_stage3_layer_gather_matches_stage2(tmp_path):
    """ZeRO-3 gathers each block one block ahead of its forward over NVLink;
    the training trajectory equals ZeRO-2's."""
    runs = {}
    for stage in (2, 3):
        d = tmp_path / f"s{stage}"
        d.mkdir()
        mp.spawn(_gpt_worker, args=(stage, False, False, free_port(), str(d)), nprocs=WORLD,
                 join=True)
        runs[stage] = [torch.load(d / f"r{r}.pt", weights_only=False) for r in range(WORLD)]
    s2, s3 = runs[2], runs[3]
    assert s3[0]["steps"] == s2[0]["steps"] == 6
    torch.testing.assert_close(s3[0]["losses"], s2[0]["losses"], rtol=2e-3, atol=2e-3)
    # attention's dQ and the embedding gradient are summed by unordered atomics:
    # for parameters with near-zero gradients AdamW's m / sqrt(v) turns the
    # last-bit differences into sign flips worth up to ~lr per step
    for k in s2[0]["params"]:
        torch.testing.assert_close(s3[0]["params"][k], s2[0]["params"][k], rtol=2e-3, atol=6e-3)
        torch.testing.assert_close(s3[0]["params"][k], s3[1]["params"][k], rtol=0, atol=0)


@pytest.mark.parametrize("stage", [2, 3])
def test_all_gpus_fused_matches_nccl(stage, tmp_path):
    """Every visible GPU as one rank (8 on a full box): the fused NVLink step
    and the NCCL step give the same GPT training trajectory, and every rank
    holds the same parameters."""
    world = torch.cuda.device_count()
    if world <= 2:
        pytest.skip("covered by the two-GPU tests")
    runs = {}
    for mode in ("fused", "nccl"):
        d = tmp_path / mode
        d.mkdir()
        mp.spawn(_gpt_worker, args=(stage, False, stage < 3, free_port(), str(d), world, mode),
                 nprocs=world, join=True)
        runs[mode] = [torch.load(d / f"r{r}.pt", weights_only=False) for r in range(world)]
    fused, nccl = runs["fused"], runs["nccl"]
    assert fused[0]["coll"] == "fused-nvlink" and nccl[0]["coll"] == "nccl"
    assert fused[0]["steps"] == nccl[0]["steps"] == 6
    torch.testing.assert_close(fused[0]["losses"], nccl[0]["losses"], rtol=2e-3, atol=2e-3)
    for k in fused[0]["params"]:
        for r in range(1, world):
            torch.testing.assert_close(fused[r]["params"][k], fused[0]["params"][k], rtol=0,
                                       atol=0)
        torch.testing.assert_close(fused[0]["params"][k], nccl[0]["params"][k], rtol=2e-3,
                                   atol=6e-3)
