"""engine.train_batch with the forward + backward replayed from a CUDA graph
against the same micro-steps run eagerly."""

import pytest
import torch

import minispeed_b200 as ms
from minispeed_b200.models import GPT, GPTConfig, init_gpt2_
from minispeed_b200.ops import _ext

pytestmark = pytest.mark.gpu

CFG = dict(vocab_size=512, block_size=64, n_layer=2, n_head=4, n_embd=128)


def _engine(stage, gas, graph, dtype="fp16", window=2):
    torch.manual_seed(0)
    model = GPT(GPTConfig(**CFG))
    init_gpt2_(model)
    cfg = {
        "train_micro_batch_size_per_gpu": 4,
        "gradient_accumulation_steps": gas,
        "gradient_clipping": 1.0,
        "dtype": dtype,
        "optimizer": {"type": "AdamW", "params": {"lr": 1e-3, "weight_decay": 0.1}},
        "zero_optimization": {"stage": stage},
        "b200": {"cuda_graph": graph, "graph_warmup": 2},
        "steps_per_print": 10 ** 6,
    }
    if dtype == "fp16":
        cfg["fp16"] = {"enabled": True, "initial_scale_power": 8, "loss_scale_window": window}
    return ms.initialize(model=model, config=cfg), model


def _batches(n):
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, CFG["vocab_size"], (4, CFG["block_size"] + 1), generator=g)
            for _ in range(n)]


@pytest.mark.parametrize("stage", [0, 1, 2])
@pytest.mark.parametrize("gas", [1, 2])
def test_graph_matches_eager(stage, gas):
    data = _batches(8 * gas)
    results = []
    for graph in (False, True):
        eng, model = _engine(stage, gas, graph)
        losses = []
        for t in data:
            t = t.cuda()
            loss = eng.train_batch(t[:, :-1], targets=t[:, 1:])
            losses.append(float(loss))
        results.append((losses, [p.detach().float().clone() for p in model.parameters()],
                        eng.get_loss_scale(), eng.global_steps))
        if graph:
            assert eng._graph is not None and eng._graph.replays == len(data) - 2
            assert eng._graph.kernels > 0
        eng.close()
    (l0, p0, s0, g0), (l1, p1, s1, g1) = results
    assert g0 == g1 == 8 and s0 == s1 and s1 > 256.0   # the scale grew: the seed followed
    for a, b in zip(l0, l1):
        assert abs(a - b) <= 2e-3 * max(1.0, abs(a))
    for a, b in zip(p0, p1):
        torch.testing.assert_close(a, b, rtol=2e-2, atol=2e-3)


def test_graph_host_inputs_and_launch_count():
    eng, _ = _engine(2, 1, True, dtype="bf16")
    data = _batches(5)
    for t in data[:3]:
        eng.train_batch(t[:, :-1].pin_memory(), targets=t[:, 1:].pin_memory())
    n0 = _ext.launch_count()
    loss = eng.train_batch(data[3][:, :-1], targets=data[3][:, 1:])
    n1 = _ext.launch_count()
    assert torch.isfinite(loss) and n1 - n0 >= eng._graph.kernels > 0
    eng.close()


def test_graph_overflow_skips_and_recovers():
    eng, model = _engine(2, 1, True)
    data = [t.cuda() for t in _batches(8)]
    for t in data[:4]:
        eng.train_batch(t[:, :-1], targets=t[:, 1:])
    assert eng._graph is not None
    steps, skipped, scale = eng.global_steps, eng.skipped_steps, eng.get_loss_scale()
    w = model.ln_f.weight
    saved = w.detach().clone()
    with torch.no_grad():
        w.view(-1)[0] = float("inf")   # in the param arena: the graph reads it
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    eng.train_batch(data[4][:, :-1], targets=data[4][:, 1:])
    assert eng.skipped_steps == skipped + 1 and eng.global_steps == steps
    assert eng.get_loss_scale() == scale / 2
    for n, p in model.named_parameters():
        assert torch.equal(p, before[n])
    with torch.no_grad():
        w.copy_(saved)
    for t in data[5:]:
        loss = eng.train_batch(t[:, :-1], targets=t[:, 1:])
        assert torch.isfinite(loss)
    assert eng.global_steps == steps + 3
    eng.close()


def test_graph_is_captured_once():
    eng, _ = _engine(2, 1, True)
    data = [t.cuda() for t in _batches(8)]
    first = None
    for i, t in enumerate(data):
        eng.train_batch(t[:, :-1], targets=t[:, 1:])
        if i == 2:
            first = eng._graph
    assert eng._graph is first and first.replays == len(data) - 2
    eng.close()


@pytest.mark.parametrize("graph", [False, True])
def test_device_timers_on_gpu(graph):
    """``b200.device_timers``: CUDA-event phase times over a few
    ``train_batch`` steps are positive and add up to less than the wall
    time of those steps (eager, and with the micro-step replayed as a graph,
    where the replay is timed under ``backward``)."""
    import time

    import minispeed_b200 as ms
    from minispeed_b200.models import GPT, GPTConfig, init_gpt2_

    torch.manual_seed(0)
    model = init_gpt2_(GPT(GPTConfig(vocab_size=512, block_size=128, n_layer=2, n_head=4,
                                     n_embd=256))).cuda()
    engine = ms.initialize(model=model, config={
        "train_micro_batch_size_per_gpu": 4, "gradient_accumulation_steps": 1,
        "fp16": {"enabled": True, "initial_scale_power": 8},
        "zero_optimization": {"stage": 2},
        "optimizer": {"type": "AdamW", "params": {"lr": 1e-3}},
        "b200": {"device_timers": True, "cuda_graph": graph}})
    x = torch.randint(0, 512, (4, 129), device="cuda")
    for _ in range(4):                      # eager warm-up (and the capture)
        engine.train_batch(x[:, :-1], targets=x[:, 1:])
    engine.device_time_ms()
    engine.device_timers.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(5):
        engine.train_batch(x[:, :-1], targets=x[:, 1:])
    torch.cuda.synchronize()
    wall_ms = (time.perf_counter() - t0) * 1e3
    times = engine.device_time_ms()
    assert times.get("backward", 0) > 0 and times.get("step", 0) > 0, times
    if not graph:
        assert times.get("forward", 0) > 0, times
    assert sum(times.values()) < wall_ms, (times, wall_ms)


def test_alternating_signatures_keep_their_graphs():
    """Two input shapes used in turn: each gets its own captured graph once
    (after its eager warm-up micro-steps) and both are replayed from then on,
    with the same losses as the eager engine."""
    data = _batches(12)
    runs = []
    for graph in (False, True):
        eng, _ = _engine(2, 1, graph)
        losses = []
        for k, t in enumerate(data):
            t = t.cuda()
            if k % 2:
                t = t[:, : CFG["block_size"] // 2 + 1]     # the other signature
            losses.append(float(eng.train_batch(t[:, :-1], targets=t[:, 1:])))
        if graph:
            assert len(eng._graphs) == 2
            assert sorted(g.replays for g in eng._graphs.values()) == [4, 4]
        runs.append(torch.tensor(losses))
        eng.close()
    torch.testing.assert_close(runs[1], runs[0], rtol=2e-3, atol=2e-3)
