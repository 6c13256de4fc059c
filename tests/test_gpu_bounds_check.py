"""The bounds-checked debug build and the batched column-sum finishes.

Debug build (``MSB_DEBUG_BUILD=1``, extension ``minispeed_b200._C_debug``):
a failed check is recorded on the device and its access skipped; these
tests make checks fail only where the skipped access would have stayed in
allocated memory anyway (an embedding table that is a view of a longer
one, a target inside the logits row's padding), so neither build can fault.
"""

import contextlib
import json
import os
import subprocess
import sys

import pytest
import torch

from minispeed_b200.ops import _ext
from minispeed_b200.ops import nn as nn_ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _debug_module():
    import importlib

    import torch  # noqa: F401

    return importlib.import_module("minispeed_b200._C_debug")


# ------------------------------------------------------------------ CPU
def test_build_flags():
    """The debug build reports its checks; the release build has none."""
    if not _ext.available():
        pytest.skip("extension not built")
    assert _ext.get().bounds_check_build() is False
    try:
        dbg = _debug_module()
    except ImportError:
        pytest.skip("debug build not built (MSB_DEBUG_BUILD=1 python setup.py build_ext --inplace)")
    assert dbg.bounds_check_build() is True


class _FakeBounds:
    """Stands in for an extension: records as bounds_status(reset) returns."""

    def __init__(self, records):
        self.records = records
        self.resets = 0

    def bounds_status(self, reset):
        out = list(self.records)
        if reset:
            self.resets += 1
            self.records = [(u, 0, 0, 0, 0) for u, *_ in self.records]
        return out


def test_check_bounds_names_the_first_failure_per_unit():
    """check_bounds raises with each failing unit's count, site and index,
    resets the records, and is silent when nothing failed."""
    fake = _FakeBounds([("nn", 3, 1, 102, 100), ("gemm", 0, 0, 0, 0),
                        ("attention", 1, 3, 13, 8)])
    with pytest.raises(_ext.BoundsError) as e:
        _ext.check_bounds(mod=fake)
    msg = str(e.value)
    assert "nn: 3 failed check(s), first: embedding token id" in msg
    assert "(index 102, limit 100)" in msg
    assert "attention: 1 failed check(s), first: TMA load x coordinate" in msg
    assert "gemm" not in msg
    assert fake.resets == 1
    _ext.check_bounds(mod=fake)          # reset: nothing left to report
    rows = _ext.bounds_status(reset=False, mod=fake)
    assert [r["unit"] for r in rows] == ["nn", "gemm", "attention"]
    assert all(r["count"] == 0 and r["what"] == "none" for r in rows)


class _FakeC:
    def __init__(self):
        self.single, self.batches = [], []

    def colsum_finish(self, part, nparts, out, accumulate):
        self.single.append((part, nparts, out, accumulate))

    def colsum_finish_many(self, parts, nparts, outs, accs):
        self.batches.append([(p, n, o, a) for p, n, o, a in zip(parts, nparts, outs, accs)])


@pytest.fixture
def fake_c(monkeypatch):
    fake = _FakeC()
    monkeypatch.setattr(nn_ops, "_C", lambda: fake)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: "s0")
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    nn_ops._finishes.clear()
    yield fake
    nn_ops._finishes.clear()
    nn_ops._finishes.depth = 0


def test_finish_queue_batches_and_flushes(fake_c):
    """Inside batched_colsums finishes into sinks wait for one batched launch
    (on exit, at the batch size, or before a second finish into the same
    sink); outside they launch at once; an exception drops the queue."""
    sinks = [torch.zeros(8) for _ in range(60)]
    part = torch.zeros(16)
    nn_ops._finish_into(part, 2, sinks[0])
    assert len(fake_c.single) == 1 and not fake_c.batches
    with nn_ops.batched_colsums():
        for s in sinks[:3]:
            nn_ops._finish_into(part, 2, s)
        assert not fake_c.batches
        nn_ops._finish_into(part, 2, sinks[1])          # same sink again: flush first
        assert [len(b) for b in fake_c.batches] == [3]
        with nn_ops.batched_colsums():                   # nests: no flush on inner exit
            nn_ops._finish_into(part, 2, sinks[4])
        assert [len(b) for b in fake_c.batches] == [3]
    assert [len(b) for b in fake_c.batches] == [3, 2]
    assert all(a is True for b in fake_c.batches for *_, a in b)
    fake_c.batches.clear()
    with nn_ops.batched_colsums():
        for s in sinks[:49]:
            nn_ops._finish_into(part, 2, s)
        assert [len(b) for b in fake_c.batches] == [nn_ops._FinishQueue._BATCH]
        nn_ops.flush_colsums()                           # a bucket is about to be read
        assert [len(b) for b in fake_c.batches] == [48, 1]
    assert [len(b) for b in fake_c.batches] == [48, 1]
    fake_c.batches.clear()
    with pytest.raises(ValueError):
        with nn_ops.batched_colsums():
            nn_ops._finish_into(part, 2, sinks[0])
            raise ValueError
    assert not fake_c.batches and not nn_ops._finishes.outs and nn_ops._finishes.depth == 0


# ------------------------------------------------------------------ GPU
@pytest.mark.gpu
def test_colsum_finish_many_matches_single_launches():
    """One batched launch per 48 jobs gives the same bits as one launch per
    job (same sums in the same order), accumulating or not, ragged widths."""
    C = _ext.get()
    torch.manual_seed(0)
    jobs = []
    for j in range(100):
        n = [1, 31, 32, 33, 768, 1600, 3072][j % 7]
        nparts = [1, 7, 256, 296][j % 4]
        part = torch.randn(nparts * n, device="cuda")
        base = torch.randn(n, device="cuda").half()
        jobs.append((part, nparts, base, j % 3 != 0))
    singles = []
    for part, nparts, base, acc in jobs:
        o = base.clone()
        C.colsum_finish(part, nparts, o, acc)
        singles.append(o)
    outs = [base.clone() for _, _, base, _ in jobs]
    C.colsum_finish_many([p for p, *_ in jobs], [n for _, n, _, _ in jobs], outs,
                         [a for *_, a in jobs])
    torch.cuda.synchronize()
    for a, b in zip(outs, singles):
        assert torch.equal(a, b)
    want = jobs[5][0].view(jobs[5][1], -1).sum(0)
    torch.testing.assert_close(outs[5].float(), (jobs[5][2].float() + want) if jobs[5][3] else want,
                               rtol=1e-2, atol=1e-2)


@pytest.mark.gpu
def test_debug_build_records_bad_token_and_target():
    """An out-of-range token id reads as a zero row in both builds; the
    debug build also records site, index and limit.  The same for a
    cross-entropy target outside the vocabulary (an ignored one is fine)."""
    dbg = _debug_module()
    _ext.bounds_status(reset=True, mod=dbg)
    V, C, T = 100, 64, 8
    full = torch.randn(V + 8, C, device="cuda").half()
    wte = full[:V]                       # row V + 2 exists in memory, not in the table
    wpe = torch.randn(T, C, device="cuda").half()
    idx = torch.arange(T, device="cuda", dtype=torch.long)
    idx[3] = V + 2
    out = torch.empty(T, C, device="cuda", dtype=torch.float16)
    dbg.embedding_fwd(idx, wte, wpe, out, T)
    rec = {r["unit"]: r for r in _ext.bounds_status(reset=True, mod=dbg)}
    assert rec["nn"]["count"] == 1, rec
    assert (rec["nn"]["site"], rec["nn"]["index"], rec["nn"]["limit"]) == (1, V + 2, V)
    assert torch.equal(out[3], wpe[3])
    assert torch.equal(out[2], (wte[2].float() + wpe[2].float()).half())
    with pytest.raises(_ext.BoundsError, match="embedding token id"):
        dbg.embedding_fwd(idx, wte, wpe, out, T)
        _ext.check_bounds(mod=dbg)

    M, Vp = 6, 128
    logits = torch.randn(M, Vp, device="cuda").half()[:, :V]   # row stride 128, V = 100
    tgt = torch.tensor([1, 5, V + 5, -100, 7, 9], device="cuda")
    lse = torch.empty(M, device="cuda")
    rows = torch.empty(M, device="cuda")
    loss = torch.empty(1, device="cuda")
    inv = torch.empty(1, device="cuda")
    dbg.cross_entropy_fwd(logits, tgt, lse, rows, loss, inv, -100)
    rec = {r["unit"]: r for r in _ext.bounds_status(reset=True, mod=dbg)}
    assert rec["nn"]["count"] == 1, rec
    assert (rec["nn"]["site"], rec["nn"]["index"], rec["nn"]["limit"]) == (2, V + 5, V)
    assert rows[2].item() == 0.0 and rows[3].item() == 0.0
    hint = torch.ones(1, device="cuda")
    dbg.cross_entropy_fwd_grad(logits, tgt, lse, rows, loss, inv, hint, -100)
    rec = {r["unit"]: r for r in _ext.bounds_status(reset=True, mod=dbg)}
    assert rec["nn"]["count"] == 1 and rec["nn"]["site"] == 2, rec


def _child(debug: bool) -> dict:
    env = dict(os.environ)
    env["MSB_DEBUG_BUILD"] = "1" if debug else "0"
    env.setdefault("MINISPEED_DEVICE", "cuda:0")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "bounds_check_child.py")],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-4000:]
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.gpu
def test_debug_build_is_clean_and_bitwise_equal_on_valid_work():
    """Valid work trips no check (stream-K, split-K fixup, split-K reduce,
    dGELU column sums, attention, CUDA-graph engine steps), and the debug
    build computes the same bits as the release build."""
    rel = _child(False)
    dbg = _child(True)
    assert rel["module"].endswith("._C") and not rel["debug"]
    assert dbg["module"].endswith("._C_debug") and dbg["debug"]
    assert all(r["count"] == 0 for r in dbg["records"]), dbg["records"]
    assert dbg["gemm"] == rel["gemm"]
    assert dbg["losses"] == rel["losses"]
