"""Two ranks sharing ONE GPU over gloo, stages 0-3, fp32 and fp16.

NCCL refuses two ranks on one GPU; gloo accepts them.  gloo moves CUDA
tensors for broadcast, all-reduce and barrier but not for reduce-scatter or
all-gather, so those two go through host copies (``comm.host_staged``); the
fused NVLink collectives are never chosen for such ranks (their kernels wait
on peers, and two waiting kernels from two processes on one GPU need not run
at the same time).  Each rank trains on its half of every micro-batch; the
mean of the two ranks' losses must follow one process training on the union
batch, and the ranks' parameters must agree.

Reference: ``tests/test_gpu.py:159-231`` (``test_two_ranks_one_gpu``).
"""

import os

import pytest
import torch
import torch.multiprocessing as mp

import minispeed_b200 as ms
from tests.helpers import config, free_port, make_data, make_net, rank_slice, run, set_rank_env

pytestmark = pytest.mark.gpu
WORLD, STEPS, GAS, MICRO = 2, 6, 2, 4


def _worker(rank, stage, dtype, port, out_dir):
    set_rank_env(rank, WORLD, port, "gloo", "cuda:0")
    torch.cuda.set_device(0)
    model = make_net(device="cuda")
    engine = ms.initialize(model=model, config=config(micro=MICRO, gas=GAS, stage=stage,
                                                      dtype=dtype, clip=1.0))
    x, y = make_data(STEPS, GAS, WORLD, MICRO, device="cuda")
    losses = run(engine, rank_slice(x, rank, MICRO), rank_slice(y, rank, MICRO), STEPS, GAS,
                 device="cuda")
    if stage >= 3:
        engine.optimizer.gather_parameters()
    torch.save({"losses": torch.tensor(losses), "steps": engine.global_steps,
                "coll": engine.collectives, "staged": dict(ms.comm.staged_calls),
                "params": {k: v.detach().cpu().clone() for k, v in model.state_dict().items()}},
               os.path.join(out_dir, f"r{rank}.pt"))
    ms.comm.destroy()


def _single(dtype):
    model = make_net(device="cuda")
    engine = ms.initialize(model=model, config=config(micro=MICRO * WORLD, gas=GAS, stage=0,
                                                      dtype=dtype, clip=1.0))
    x, y = make_data(STEPS, GAS, WORLD, MICRO, device="cuda")
    return torch.tensor(run(engine, x, y, STEPS, GAS, device="cuda"))


@pytest.mark.timeout(300)
@pytest.mark.parametrize("stage", [0, 1, 2, 3])
@pytest.mark.parametrize("dtype", ["fp32", "fp16"])
def test_two_ranks_share_one_gpu(stage, dtype, tmp_path):
    mp.spawn(_worker, args=(stage, dtype, free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    r0, r1 = (torch.load(tmp_path / f"r{r}.pt", weights_only=False) for r in range(WORLD))
    assert r0["steps"] == r1["steps"] == STEPS
    assert r0["coll"] == "gloo"            # not the fused NVLink collectives
    # stage 0 only all-reduces (gloo moves CUDA tensors); stages 1-3
    # reduce-scatter and all-gather through the host-staged path
    for kind in ("reduce_scatter", "all_gather"):
        assert (r0["staged"][kind] > 0) == (stage >= 1), kind
    ref = _single(dtype)
    torch.testing.assert_close((r0["losses"] + r1["losses"]) / 2, ref, rtol=5e-3, atol=1e-4)
    for k in r0["params"]:
        torch.testing.assert_close(r0["params"][k], r1["params"][k], rtol=1e-4, atol=1e-5)
