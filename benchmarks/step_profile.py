"""Per-kernel device time of one training step (torch.profiler, CUDA activity).

    python benchmarks/step_profile.py [--model gpt2-small|gpt2-xl|llama3-8b] [--impl ours|reference]
                                      [--host]

Builds the same model and config as ``bench.py`` (synthetic tokens, random
weights), runs three warm-up steps, profiles one step and prints the step's
span, the summed kernel time, the kernels sorted by total time, and the
device's idle gaps between them (count and time by length, the longest with
their neighbours).  Profiler
timings are for shares, not for the headline number (``bench.py`` times
without a profiler).

``--host`` profiles the host instead: cProfile over ten steps, the functions
by own time (the host's share of the step boundary: what runs between the
optimizer's device-to-host read and the next replay).
"""

import argparse
import collections
import os
import sys

import torch
import torch.nn.functional as F
from torch.profiler import ProfilerActivity, profile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def idle_gaps(intervals):
    """Idle stretches of the device between ``(start, end, name)`` intervals
    (any order, possibly overlapping across streams): a gap opens when every
    activity seen so far has ended.  Returns ``[(length, after_name,
    before_name)]``."""
    gaps, busy_until, last = [], None, None
    for start, end, name in sorted(intervals):
        if busy_until is not None and start > busy_until:
            gaps.append((start - busy_until, last, name))
        if busy_until is None or end > busy_until:
            busy_until, last = end, name
    return gaps


def gap_report(gaps, top=5):
    """Total idle time, a histogram by gap length and the longest gaps."""
    bins = [(2, "< 2 us"), (10, "2-10 us"), (100, "10-100 us"), (float("inf"), ">= 100 us")]
    hist = collections.OrderedDict((label, [0, 0.0]) for _, label in bins)
    for g, _, _ in gaps:
        label = next(lb for lim, lb in bins if g < lim)
        hist[label][0] += 1
        hist[label][1] += g
    lines = [f"idle {sum(g for g, _, _ in gaps) / 1000:.3f} ms in {len(gaps)} gaps: " +
             ", ".join(f"{lb} {n} ({t / 1000:.3f} ms)" for lb, (n, t) in hist.items())]
    for g, after, before in sorted(gaps, reverse=True)[:top]:
        lines.append(f"  {g:9.1f} us  after {after[:50]}  before {before[:50]}")
    return "\n".join(lines)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=sorted(bench.SPECS), default="gpt2-small")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--top", type=int, default=25)
    ap.add_argument("--host", action="store_true")
    a = ap.parse_args()
    spec = bench.SPECS[a.model]
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    os.environ.setdefault("MINISPEED_DEVICE", "cuda:0")
    if a.impl == "ours":
        import minispeed_b200 as lib
        from minispeed_b200.models import GPT, GPTConfig, Llama, LlamaConfig
        with torch.device(dev):
            model = bench._build_ours(spec, GPT, GPTConfig, Llama, LlamaConfig)
            bench._init(model)
        cfg = bench.ds_config(spec, 1, 100)
        cfg["b200"] = {"cuda_graph": True}
        eng = lib.initialize(model=model, config=cfg)

        def micro(x, y):
            eng.train_batch(x, targets=y)
    else:
        sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
        import minispeed as lib
        with torch.device(dev):
            model = bench.RefGPT(spec) if spec["kind"] == "gpt" else bench.RefLlama(spec)
            bench._init(model)
        eng = lib.initialize(model=model, config=bench.ds_config(spec, 1, 100))

        def micro(x, y):
            loss = F.cross_entropy(eng(x).reshape(-1, spec["vocab"]).float(), y.reshape(-1))
            eng.backward(loss)
            eng.step()
    t = torch.randint(0, spec["vocab"], (spec["micro"], spec["seq"] + 1), device=dev)

    def step():
        for _ in range(spec["gas"]):
            micro(t[:, :-1], t[:, 1:])
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    if a.host:
        import cProfile
        import pstats
        import time

        prof = cProfile.Profile()
        t0 = time.perf_counter()
        prof.enable()
        for _ in range(10):
            step()
        prof.disable()
        torch.cuda.synchronize()
        print(f"{a.model} {a.impl}: {(time.perf_counter() - t0) * 100:.2f} ms per step (wall, "
              "under cProfile)")
        st = pstats.Stats(prof)
        st.sort_stats("tottime").print_stats(a.top)
        st.sort_stats("cumulative").print_stats(a.top)
        return
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    evs = [e for e in prof.events()
           if e.device_type == torch.autograd.DeviceType.CUDA and e.time_range.elapsed_us() > 0]
    evs.sort(key=lambda e: e.time_range.start)
    span = evs[-1].time_range.end - evs[0].time_range.start
    tot, cnt = collections.defaultdict(float), collections.Counter()
    for e in evs:
        tot[e.name[:90]] += e.time_range.elapsed_us()
        cnt[e.name[:90]] += 1
    print(f"{a.model} {a.impl}: span {span / 1000:.2f} ms, kernel sum {sum(tot.values()) / 1000:.2f} ms")
    for k, v in sorted(tot.items(), key=lambda kv: -kv[1])[:a.top]:
        print(f"{v / 1000:9.3f} ms  {cnt[k]:5d}  {k}")
    print(gap_report(idle_gaps([(e.time_range.start, e.time_range.end, e.name) for e in evs])))


if __name__ == "__main__":
    main()
