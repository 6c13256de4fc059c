"""Barrier protocols of the tcgen05 kernels, checked on the CPU: the
persistent head-dim-64 attention backward (``attn_bwd64_kernel``), the
head-dim-128 backward (``attn_bwd128_kernel``) and the attention forward's
event loop (``attn_fwd_kernel``), all in ``csrc/attention_tcgen05.cu``,
the 1-CTA and 2-CTA GEMMs (``csrc/gemm_tcgen05.cu``, including the
stream-K and split-K fixup tile hand-off between CTA pairs), and the
cross-GPU epoch protocol of the fused NVLink step (``csrc/collectives.cu``).

The kernel's roles (TMA warp, MMA warp, softmax warps, dQ warps) synchronise
only through mbarriers whose waits name a phase parity.  A wrong parity is a
hang (the barrier already ran two phases ahead) or a silent race (the wait
passes one phase early).  This test replays the roles' sequences of waits,
arrivals and asynchronous completions exactly as the kernel orders them --
the same cursor over work items and query tiles, the same ring slots and
parities -- under many random interleavings, with hardware parity semantics
(``try_wait.parity(P)`` passes while the current phase's parity differs from
P), and checks that every wait passes exactly at its intended completion,
that no barrier ever runs two phases ahead of a waiter, and that nothing
deadlocks.  Asynchronous work is modelled as the kernel relies on it: TMA
loads complete in any order, the tensor core retires its MMAs and commits in
issue order.
"""

import random

import pytest

STAGES = 5          # Q / dO ring (kStages64)
N_SOFTMAX = 8       # ds_ready / acc_free arrivals per phase
N_DQ = 4            # dq_free arrivals per phase


class Barrier:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.completed = name, count, count, 0

    def arrive(self):
        self.pending -= 1
        if self.pending == 0:
            self.completed += 1
            self.pending = self.count

    def passes(self, parity):
        # hardware: the phase with this parity has completed
        return (self.completed & 1) != parity


def items_of_cta(cta, grid, n_q, nbh, rep):
    """Tile counts of the work items CTA `cta` walks (key block j: 2 (n_q - j) tiles per head)."""
    out, k = [], 0
    while True:
        w = cta + k * grid
        if w >= n_q * nbh:
            return out
        j = w // nbh
        out.append(rep * 2 * (n_q - j))
        k += 1


def roles(items):
    """Each role as a list of ops: ('wait', bar, parity, intended_index),
    ('arrive', bar), ('async', kind, bar) for completions the hardware does
    later, ('poll_kv', k) for the TMA warp's non-blocking K/V prefetch."""
    total = sum(items)
    assert total % 2 == 0
    first, last = set(), set()
    t = 0
    item_of = []
    for k, n in enumerate(items):
        first.add(t)
        last.add(t + n - 1)
        item_of += [k] * n
        t += n

    tma = []
    kv_next = 0
    for t in range(total):
        k = item_of[t]
        if kv_next <= k:                      # this item's K / V (blocking)
            if k >= 2:
                tma.append(("wait", f"kv_empty{k & 1}", ((k - 2) >> 1) & 1, (k - 2) >> 1))
            tma.append(("async", "tma", f"kv_full{k & 1}"))
            kv_next = k + 1
        s, ph = t % STAGES, (t // STAGES) & 1
        if kv_next == k + 1 and k + 1 < len(items):
            tma.append(("poll_kv", k + 1))    # may load the next item's K / V now
        if t >= STAGES:
            tma.append(("wait", f"qo_empty{s}", ph ^ 1, t // STAGES - 1))
        tma.append(("async", "tma", f"qo_full{s}"))
        # after the load, one more chance for the next item's K / V
        if kv_next == k + 1 and k + 1 < len(items):
            tma.append(("poll_kv", k + 1))

    mma = []
    pr_count = 0
    for u in range(total + 2):
        if u >= 2:
            mma.append(("wait", f"ds_ready{u & 1}", ((u - 2) >> 1) & 1, (u - 2) >> 1))
        if u < total:
            k = item_of[u]
            if u in first:
                mma.append(("wait", f"kv_full{k & 1}", (k >> 1) & 1, k >> 1))
            mma.append(("wait", f"qo_full{u % STAGES}", (u // STAGES) & 1, u // STAGES))
            mma.append(("mma_op", (), (f"S{u & 1}",)))
            mma.append(("async", "mma", f"st_full{u & 1}"))
        if u >= 2:
            v = u - 2
            k = item_of[v]
            if v in first and k > 0:
                mma.append(("wait", "acc_free", (k - 1) & 1, k - 1))
            mma.append(("mma_op", (f"P{v & 1}", f"DS{(v >> 1) & 1}_{v & 1}"), ("ACC",)))
            mma.append(("async", "mma", f"qo_empty{v % STAGES}"))
            mma.append(("async", "mma", f"p_free{v & 1}"))
            if v & 1:
                pr = v >> 1
                if pr > 0:
                    mma.append(("wait", "dq_free", (pr - 1) & 1, pr - 1))
                mma.append(("mma_op", (f"DS{pr & 1}_0", f"DS{pr & 1}_1"), ("DQ",)))
                mma.append(("async", "mma", "dq_full"))
                pr_count += 1
            if v in last:
                mma.append(("async", "mma", "acc_full"))
                mma.append(("async", "mma", f"kv_empty{k & 1}"))
    mma.append(("async", "mma", "drain"))
    mma.append(("wait", "drain", 0, 0))

    sm = []
    ep = None
    for t in range(total):
        k = item_of[t]
        sm.append(("wait", f"st_full{t & 1}", (t >> 1) & 1, t >> 1))
        sm.append(("read_begin", f"S{t & 1}"))
        if t >= 2:
            sm.append(("wait", f"p_free{t & 1}", ((t - 2) >> 1) & 1, (t - 2) >> 1))
        sm.append(("write", f"P{t & 1}"))
        sm.append(("write", f"DS{(t >> 1) & 1}_{t & 1}"))
        sm.append(("read_end", f"S{t & 1}"))
        sm.append(("arrive", f"ds_ready{t & 1}"))
        if ep is not None:
            sm.append(("wait", "acc_full", ep & 1, ep))
            sm.append(("read_begin", "ACC"))
            sm.append(("read_end", "ACC"))
            sm.append(("arrive", "acc_free"))
            ep = None
        if t in last:
            ep = k
    if ep is not None:
        sm.append(("wait", "acc_full", ep & 1, ep))
        sm.append(("read_begin", "ACC"))
        sm.append(("read_end", "ACC"))
        sm.append(("arrive", "acc_free"))

    dq = []
    for pr in range(total // 2):
        dq.append(("wait", "dq_full", pr & 1, pr))
        dq.append(("read_begin", "DQ"))
        dq.append(("read_end", "DQ"))
        dq.append(("arrive", "dq_free"))
    return {"tma": tma, "mma": mma, "softmax": sm, "dq": dq}


def barriers():
    bars = {}
    for i in range(2):
        for n in ("kv_full", "kv_empty", "st_full", "p_free"):
            bars[f"{n}{i}"] = Barrier(f"{n}{i}", 1)
        bars[f"ds_ready{i}"] = Barrier(f"ds_ready{i}", 1)   # the 8 warps arrive as one here
    for s in range(STAGES):
        bars[f"qo_full{s}"] = Barrier(f"qo_full{s}", 1)
        bars[f"qo_empty{s}"] = Barrier(f"qo_empty{s}", 1)
    for n in ("dq_full", "dq_free", "acc_full", "acc_free", "drain"):
        bars[n] = Barrier(n, 1)
    return bars


def run(items, seed, progs=None, bars=None):
    """Random interleavings of the roles; a wait whose intended completion
    index is None only has to pass (no index check)."""
    rng = random.Random(seed)
    if progs is None:
        progs, bars = roles(items), barriers()
    pc = {r: 0 for r in progs}
    tma_async, mma_fifo = [], []
    readers = {}          # resource -> number of warps reading it (generic proxy)
    inflight = []         # (resource, 'r'|'w') of issued MMAs not yet retired, in issue order
    retire_mark = []      # per queued commit: how many in-flight entries it retires
    kv_loaded = set()
    kv_item_of_load = {}
    steps = 0
    while True:
        steps += 1
        assert steps < 1_000_000
        choices = []
        for r, ops in progs.items():
            if pc[r] >= len(ops):
                continue
            op = ops[pc[r]]
            if op[0] == "wait":
                _, b, parity, k = op
                bar = bars[b]
                if k is None:
                    if bar.passes(parity):
                        choices.append(("run", r))
                    continue
                # no barrier may run two phases ahead of a waiter
                assert bar.completed <= k + 1, (r, op, bar.completed)
                if bar.passes(parity):
                    assert bar.completed == k + 1, (r, op, bar.completed)
                    choices.append(("run", r))
            else:
                choices.append(("run", r))
        if tma_async:
            choices.append(("tma_done", None))
        if mma_fifo:
            choices.append(("mma_done", None))
        if not choices:
            unfinished = [r for r in progs if pc[r] < len(progs[r])]
            assert not unfinished, ("deadlock", {r: progs[r][pc[r]] for r in unfinished})
            return
        kind, r = rng.choice(choices)
        if kind == "tma_done":
            b = tma_async.pop(rng.randrange(len(tma_async)))
            bars[b].arrive()
            continue
        if kind == "mma_done":
            bars[mma_fifo.pop(0)].arrive()
            # a commit retires every MMA issued before it
            n = retire_mark.pop(0)
            del inflight[:n]
            retire_mark[:] = [m - n for m in retire_mark]
            continue
        op = progs[r][pc[r]]
        pc[r] += 1
        if op[0] == "arrive":
            bars[op[1]].arrive()
        elif op[0] == "async":
            if op[1] == "tma":
                tma_async.append(op[2])
            else:
                mma_fifo.append(op[2])
                retire_mark.append(len(inflight))
        elif op[0] == "mma_op":
            reads, writes = op[1], op[2]
            for res in writes:
                assert not readers.get(res), ("tensor core overwrites a buffer still read", res)
            inflight.extend([(res, "r") for res in reads] + [(res, "w") for res in writes])
        elif op[0] == "read_begin":
            readers.setdefault(op[1], set()).add(r)
        elif op[0] == "read_end":
            readers[op[1]].discard(r)
        elif op[0] == "write":
            assert all(res != op[1] for res, _ in inflight), ("write while an MMA uses it", op[1])
            assert not (readers.get(op[1], set()) - {r}), ("write while another role reads", op[1])
        elif op[0] == "poll_kv":
            k = op[1]
            if k in kv_loaded:
                continue
            ok = k < 2 or bars[f"kv_empty{k & 1}"].passes(((k - 2) >> 1) & 1)
            if ok:
                kv_loaded.add(k)
                tma_async.append(f"kv_full{k & 1}")
                # the blocking load for this item is then skipped
                ops = progs["tma"]
                for i in range(pc["tma"], len(ops)):
                    if ops[i] == ("async", "tma", f"kv_full{k & 1}"):
                        del ops[i]
                        if i > 0 and ops[i - 1][0] == "wait" and ops[i - 1][1] == f"kv_empty{k & 1}":
                            del ops[i - 1]
                        break
        # waits advance pc only; their pass was checked above


@pytest.mark.parametrize("B,T,H,Hkv,grid", [
    (1, 256, 2, 2, 148),      # 2 items: every CTA has at most one
    (16, 1024, 12, 12, 148),  # the GPT-2 layer: 10-11 items per CTA
    (4, 1024, 12, 6, 148),    # GQA, 2 heads per kv head
    (20, 200, 8, 8, 148),     # ragged length
    (1, 4096, 32, 8, 8),      # few CTAs, long items
])
def test_backward_barrier_protocol(B, T, H, Hkv, grid):
    n_q = (T + 127) // 128
    nbh = B * Hkv
    grid = min(grid, n_q * nbh)
    ctas = sorted({0, grid // 2, grid - 1})
    for cta in ctas:
        items = items_of_cta(cta, grid, n_q, nbh, H // Hkv)
        for seed in range(12):
            run(items, seed * 7919 + cta)


def test_work_items_cover_every_tile_once():
    B, T, H, Hkv = 3, 640, 6, 2
    n_q, nbh, rep = (T + 127) // 128, B * Hkv, H // Hkv
    seen = set()
    for grid in (1, 5, 148):
        seen.clear()
        g = min(grid, n_q * nbh)
        for cta in range(g):
            k = 0
            while True:
                w = cta + k * g
                if w >= n_q * nbh:
                    break
                j, bh = divmod(w, nbh)
                for hh in range(rep):
                    for ti in range(2 * (n_q - j)):
                        key = (bh, j, hh, ti)
                        assert key not in seen
                        seen.add(key)
                k += 1
        assert len(seen) == nbh * rep * sum(2 * (n_q - j) for j in range(n_q))


# ---------------------------------------------------------------- GEMM
def gemm_roles(units_kb, stages=4):
    """The persistent tcgen05 GEMM (``gemm_kernel`` in ``csrc/gemm_tcgen05.cu``)
    for one CTA: a TMA producer over a `stages`-deep operand ring, the MMA
    warp with two tensor-memory accumulators, the epilogue warps (one role
    here; the barrier counts them as one arrival per phase).  `units_kb`
    lists the k-blocks of each tile the CTA owns."""
    tma, mma, epi = [], [], []
    g = 0                                  # k-blocks so far: slot g % stages, use g // stages
    stage, phase = 0, 0
    for kbs in units_kb:
        for _ in range(kbs):
            tma.append(("wait", f"empty{stage}", phase ^ 1, g // stages - 1))
            tma.append(("async", "tma", f"full{stage}"))
            stage, phase = (0, phase ^ 1) if stage + 1 == stages else (stage + 1, phase)
            g += 1
    g = 0
    stage, phase = 0, 0
    for u, kbs in enumerate(units_kb):
        buf, tphase = u & 1, (u >> 1) & 1
        mma.append(("wait", f"tempty{buf}", tphase ^ 1, (u >> 1) - 1))
        for _ in range(kbs):
            mma.append(("wait", f"full{stage}", phase, g // stages))
            g += 1
            mma.append(("mma_op", (f"ring{stage}",), (f"ACC{buf}",)))
            mma.append(("async", "mma", f"empty{stage}"))
            stage, phase = (0, phase ^ 1) if stage + 1 == stages else (stage + 1, phase)
        mma.append(("async", "mma", f"tfull{buf}"))
        epi.append(("wait", f"tfull{buf}", tphase, u >> 1))
        epi.append(("read_begin", f"ACC{buf}"))
        epi.append(("read_end", f"ACC{buf}"))
        epi.append(("arrive", f"tempty{buf}"))
    mma.append(("async", "mma", "drain"))
    mma.append(("wait", "drain", 0, 0))
    return {"tma": tma, "mma": mma, "epilogue": epi}


def gemm_barriers(stages=4):
    bars = {}
    for s in range(stages):
        bars[f"full{s}"] = Barrier(f"full{s}", 1)
        bars[f"empty{s}"] = Barrier(f"empty{s}", 1)
    for b in range(2):
        bars[f"tfull{b}"] = Barrier(f"tfull{b}", 1)
        bars[f"tempty{b}"] = Barrier(f"tempty{b}", 1)
    bars["drain"] = Barrier("drain", 1)
    return bars


@pytest.mark.parametrize("units_kb", [[12] * 8, [3, 1, 7, 2, 5], [1] * 9, [256, 256, 1]])
def test_gemm_barrier_protocol(units_kb):
    for seed in range(10):
        run(None, seed, progs=gemm_roles(units_kb), bars=gemm_barriers())


def gemm2_roles(units_kb, stages=4):
    """The 2-CTA GEMM (``gemm2_kernel``): both CTAs' TMA warps load into
    their own operand rings and signal the leader's stage barrier (the
    leader's expect_tx is the one arrival, each CTA's loads complete the
    transaction bytes); the leader's MMA warp issues for the pair and its
    commits arrive on both CTAs' barriers; both epilogues release the
    leader's accumulator barrier."""
    progs = {"tma0": [], "tma1": [], "mma": [], "epi0": [], "epi1": []}
    for c in (0, 1):
        tma = progs[f"tma{c}"]
        g, stage, phase = 0, 0, 0
        for kbs in units_kb:
            for _ in range(kbs):
                tma.append(("wait", f"c{c}.empty{stage}", phase ^ 1, g // stages - 1))
                if c == 0:
                    tma.append(("arrive", f"c0.full{stage}"))     # expect_tx
                tma.append(("write", f"c{c}.ring{stage}"))
                tma.append(("async", "tma", f"c0.full{stage}"))   # complete_tx
                stage, phase = (0, phase ^ 1) if stage + 1 == stages else (stage + 1, phase)
                g += 1
    mma = progs["mma"]
    g, stage, phase = 0, 0, 0
    for u, kbs in enumerate(units_kb):
        buf, tphase = u & 1, (u >> 1) & 1
        mma.append(("wait", f"c0.tempty{buf}", tphase ^ 1, (u >> 1) - 1))
        for _ in range(kbs):
            mma.append(("wait", f"c0.full{stage}", phase, g // stages))
            mma.append(("mma_op", (f"c0.ring{stage}", f"c1.ring{stage}"), (f"c0.ACC{buf}", f"c1.ACC{buf}")))
            mma.append(("async", "mma", f"c0.empty{stage}"))
            mma.append(("async", "mma", f"c1.empty{stage}"))
            stage, phase = (0, phase ^ 1) if stage + 1 == stages else (stage + 1, phase)
            g += 1
        mma.append(("async", "mma", f"c0.tfull{buf}"))
        mma.append(("async", "mma", f"c1.tfull{buf}"))
        for c in (0, 1):
            epi = progs[f"epi{c}"]
            epi.append(("wait", f"c{c}.tfull{buf}", tphase, u >> 1))
            epi.append(("read_begin", f"c{c}.ACC{buf}"))
            epi.append(("read_end", f"c{c}.ACC{buf}"))
            epi.append(("arrive", f"c0.tempty{buf}"))
    mma.append(("async", "mma", "c0.drain"))
    mma.append(("wait", "c0.drain", 0, 0))
    return progs


def gemm2_barriers(stages=4):
    bars = {}
    for c in (0, 1):
        for s in range(stages):
            bars[f"c{c}.empty{s}"] = Barrier(f"c{c}.empty{s}", 1)
        for b in range(2):
            bars[f"c{c}.tfull{b}"] = Barrier(f"c{c}.tfull{b}", 1)
    for s in range(stages):
        bars[f"c0.full{s}"] = Barrier(f"c0.full{s}", 3)        # expect_tx + both CTAs' bytes
    for b in range(2):
        bars[f"c0.tempty{b}"] = Barrier(f"c0.tempty{b}", 2)    # both CTAs' epilogues
    bars["c0.drain"] = Barrier("c0.drain", 1)
    return bars


@pytest.mark.parametrize("units_kb", [[12] * 8, [3, 1, 7, 2, 5], [1] * 9])
def test_gemm2_barrier_protocol(units_kb):
    for seed in range(10):
        run(None, seed, progs=gemm2_roles(units_kb, stages=6), bars=gemm2_barriers(stages=6))


# ------------------------------------------------------- attention forward
def run_forward(nkv0, nkv1, sep_p, kv_stages, seed):
    """The attention forward (``attn_fwd_kernel``) for one CTA with query
    tiles needing nkv0 and nkv1 key tiles: the TMA warp's K / V ring, the MMA
    warp's event loop (issue S of a tile when its key tile landed and its
    score columns are free; issue P V when P is written and V landed; release
    ring slots once every tile that reads them has issued), and the two
    softmax groups.  Checks waits, parities and tensor-memory reuse as run()
    does, with the MMA warp's non-blocking probes taken from the live state."""
    rng = random.Random(seed)
    nk = [nkv0, nkv1]
    nkv = max(nkv0, nkv1)
    bars = {n: Barrier(n, 1) for n in ["q_full", "drain"]}
    for s in range(kv_stages):
        for n in ("k_full", "k_empty", "v_full", "v_empty"):
            bars[f"{n}{s}"] = Barrier(f"{n}{s}", 1)
    for t in range(2):
        for n in ("s_full", "s_free", "p_full", "pv_done"):
            bars[f"{n}{t}"] = Barrier(f"{n}{t}", 1)

    tma = [("async", "tma", "q_full")]
    for j in range(nkv):
        st, ph = j % kv_stages, (j // kv_stages) & 1
        tma += [("wait", f"k_empty{st}", ph ^ 1, j // kv_stages - 1),
                ("write", f"K{st}"), ("async", "tma", f"k_full{st}"),
                ("wait", f"v_empty{st}", ph ^ 1, j // kv_stages - 1),
                ("write", f"V{st}"), ("async", "tma", f"v_full{st}")]
    softmax = {}
    for t in range(2):
        ops = []
        for j in range(nk[t]):
            ops += [("wait", f"s_full{t}", j & 1, j), ("read_begin", f"S{t}")]
            if sep_p:
                ops += [("read_end", f"S{t}"), ("arrive", f"s_free{t}")]
                if j > 0:
                    ops.append(("wait", f"pv_done{t}", (j - 1) & 1, j - 1))
            ops += [("write", f"P{t}"), ("write", f"O{t}")]     # P, and O rescaled in place
            if not sep_p:
                ops.append(("read_end", f"S{t}"))
            ops.append(("arrive", f"p_full{t}"))
        if nk[t] > 0:
            ops += [("wait", f"pv_done{t}", (nk[t] - 1) & 1, nk[t] - 1), ("read_begin", f"O{t}"),
                    ("read_end", f"O{t}")]
        softmax[f"softmax{t}"] = ops
    progs = {"tma": tma, **softmax}
    pc = {r: 0 for r in progs}
    js, jp = [0, 0], [0, 0]
    kfree = vfree = 0
    q_ok = False
    mma_done = False
    tma_async, mma_fifo, retire_mark, inflight = [], [], [], []
    readers = {}

    def mma_issue(reads, writes, commits):
        for res in writes:
            assert not readers.get(res), ("tensor core overwrites a buffer still read", res)
        inflight.extend([(r, "r") for r in reads] + [(w, "w") for w in writes])
        for c in commits:
            mma_fifo.append(c)
            retire_mark.append(len(inflight))

    def mma_pass():
        """One pass of the event loop; returns True if it issued anything."""
        nonlocal kfree, vfree, q_ok
        if not q_ok:
            q_ok = bars["q_full"].passes(0)
            return q_ok
        progress = False
        for t in range(2):
            j = js[t]
            if j < nk[t]:
                st = j % kv_stages
                free = j == 0 or (bars[f"s_free{t}"].passes((j - 1) & 1) if sep_p
                                  else bars[f"pv_done{t}"].passes((j - 1) & 1))
                if free and bars[f"k_full{st}"].passes((j // kv_stages) & 1):
                    mma_issue((f"Q{t}", f"K{st}"), (f"S{t}",), [f"s_full{t}"])
                    js[t] += 1
                    progress = True
            jj = jp[t]
            if jj < nk[t]:
                st = jj % kv_stages
                if (jj < js[t] and bars[f"p_full{t}"].passes(jj & 1)
                        and bars[f"v_full{st}"].passes((jj // kv_stages) & 1)):
                    mma_issue((f"P{t}", f"V{st}"), (f"O{t}",), [f"pv_done{t}"])
                    jp[t] += 1
                    progress = True
        while kfree < nkv and (kfree < js[0] or kfree >= nk[0]) and (kfree < js[1] or kfree >= nk[1]):
            mma_issue((), (), [f"k_empty{kfree % kv_stages}"])
            kfree += 1
        while vfree < nkv and (vfree < jp[0] or vfree >= nk[0]) and (vfree < jp[1] or vfree >= nk[1]):
            mma_issue((), (), [f"v_empty{vfree % kv_stages}"])
            vfree += 1
        return progress

    steps = 0
    while True:
        steps += 1
        assert steps < 2_000_000
        choices = []
        for r, ops in progs.items():
            if pc[r] >= len(ops):
                continue
            op = ops[pc[r]]
            if op[0] == "wait":
                _, b, parity, k = op
                bar = bars[b]
                assert bar.completed <= k + 1, (r, op, bar.completed)
                if bar.passes(parity):
                    assert bar.completed == k + 1, (r, op, bar.completed)
                    choices.append(("run", r))
            else:
                choices.append(("run", r))
        pending_mma = js[0] < nk[0] or js[1] < nk[1] or jp[0] < nk[0] or jp[1] < nk[1] or not q_ok
        if pending_mma:
            choices.append(("mma", None))
        if tma_async:
            choices.append(("tma_done", None))
        if mma_fifo:
            choices.append(("mma_done", None))
        if not choices:
            unfinished = [r for r in progs if pc[r] < len(progs[r])]
            assert not unfinished and not pending_mma, ("deadlock", unfinished, js, jp)
            return
        kind, r = rng.choice(choices)
        if kind == "mma":
            if not mma_pass() and not tma_async and not mma_fifo:
                # the event loop can only make progress after another role acts
                others = [c for c in choices if c[0] == "run"]
                assert others, ("MMA event loop stuck", js, jp, {k: pc[k] for k in pc})
            continue
        if kind == "tma_done":
            bars[tma_async.pop(rng.randrange(len(tma_async)))].arrive()
            continue
        if kind == "mma_done":
            bars[mma_fifo.pop(0)].arrive()
            n = retire_mark.pop(0)
            del inflight[:n]
            retire_mark[:] = [m - n for m in retire_mark]
            continue
        op = progs[r][pc[r]]
        pc[r] += 1
        if op[0] == "arrive":
            bars[op[1]].arrive()
        elif op[0] == "async":
            tma_async.append(op[2])
        elif op[0] == "read_begin":
            readers.setdefault(op[1], set()).add(r)
        elif op[0] == "read_end":
            readers[op[1]].discard(r)
        elif op[0] == "write":
            assert all(res != op[1] for res, _ in inflight), ("write while an MMA uses it", op[1])
            assert not (readers.get(op[1], set()) - {r}), ("write while another role reads", op[1])


@pytest.mark.parametrize("sep_p,kv_stages", [(True, 3), (False, 2)])
@pytest.mark.parametrize("nkv0,nkv1", [(1, 2), (3, 4), (7, 8), (5, 0), (8, 8)])
def test_attention_forward_protocol(sep_p, kv_stages, nkv0, nkv1):
    for seed in range(15):
        run_forward(nkv0, nkv1, sep_p, kv_stages, seed)


# ------------------------------------------- attention backward, head dim 128
def bwd128_roles(nit):
    """``attn_bwd128_kernel`` for one CTA walking `nit` 128-row query tiles:
    one score buffer in tensor memory (P^T and dS^T packed in place, the dQ
    halves in the freed columns), the dS^T tile in shared memory doubling as
    the dQ staging of the reduce-adds.  The four softmax warps and the four
    dQ warps are one role each (one arrival per phase)."""
    tma = [("write", "K"), ("async", "tma", "kv_full")]
    for it in range(nit):
        st, ph = it & 1, (it >> 1) & 1
        if it >= 2:
            tma.append(("wait", f"qo_empty{st}", ph ^ 1, (it >> 1) - 1))
        tma += [("write", f"Q{st}"), ("async", "tma", f"qo_full{st}")]
    mma = [("wait", "kv_full", 0, 0)]
    for it in range(nit):
        st, ph = it & 1, (it >> 1) & 1
        mma.append(("wait", f"qo_full{st}", ph, it >> 1))
        if it > 0:
            mma += [("wait", "mma2_done", (it - 1) & 1, it - 1),
                    ("wait", "dq_free", (it - 1) & 1, it - 1)]
        mma += [("mma_op", ("K", f"Q{st}"), ("S", "DQ")), ("async", "mma", "st_full"),
                ("wait", "ds_ready", it & 1, it),
                ("mma_op", ("S", f"Q{st}", "DSB", "K"), ("ACC", "DQ")),
                ("async", "mma", f"qo_empty{st}"), ("async", "mma", "mma2_done"),
                ("async", "mma", "dq_full")]
    mma += [("async", "mma", "drain"), ("wait", "drain", 0, 0)]
    sm = []
    for it in range(nit):
        if it > 0:
            sm.append(("wait", "ds_ready", (it - 1) & 1, it - 1))
        sm += [("arrive", "lse_full"), ("wait", "lse_full", it & 1, it),
               ("wait", "st_full", it & 1, it)]
        if it > 0:
            sm.append(("wait", "stg_free", (it - 1) & 1, it - 1))
        sm += [("read_begin", "S"), ("write", "S"), ("write", "DSB"), ("read_end", "S"),
               ("arrive", "ds_ready")]
    if nit:
        sm += [("wait", "mma2_done", (nit - 1) & 1, nit - 1), ("read_begin", "ACC"),
               ("read_end", "ACC")]
    dq = []
    for it in range(nit):
        dq += [("wait", "dq_full", it & 1, it), ("read_begin", "DQ"), ("read_end", "DQ"),
               ("arrive", "dq_free"), ("write", "DSB"), ("read_begin", "DSB"),
               ("read_end", "DSB"), ("arrive", "stg_free")]
    progs = {"tma": tma, "mma": mma, "softmax": sm, "dq": dq}
    bars = {n: Barrier(n, 1) for n in ("kv_full", "st_full", "ds_ready", "mma2_done", "dq_full",
                                        "dq_free", "stg_free", "lse_full", "drain")}
    for s in range(2):
        bars[f"qo_full{s}"] = Barrier(f"qo_full{s}", 1)
        bars[f"qo_empty{s}"] = Barrier(f"qo_empty{s}", 1)
    return progs, bars


@pytest.mark.parametrize("nit", [1, 2, 5, 32])
def test_attention_backward128_protocol(nit):
    for seed in range(12):
        progs, bars = bwd128_roles(nit)
        run(None, seed, progs=progs, bars=bars)


# ------------------------------------------------- fused NVLink step pipeline
def run_fused_step(world, steps, seed, barrier_after=True):
    """The fused collective step (``minispeed_b200/parallel/fused.py``,
    ``csrc/collectives.cu``) across `world` ranks: backward writes the rank's
    gradient arena; ``peer_barrier``; ``rs_stats`` reads every peer's arena;
    ``stats_exchange`` posts (flag, sum of squares, epoch) on every peer's
    board and waits for every board slot to carry this epoch; ``adamw_fanout``
    stores into every peer's parameter arena; ``peer_barrier``.  Both barrier
    kinds take their epoch from the rank's one device counter.  Checks that
    no rank reads a peer's gradients while that peer writes them, that no
    parameter store lands while the owner computes with its parameters, that
    every exchange reads the values of its own epoch, and that nothing hangs."""
    rng = random.Random(seed)
    flags = [[0] * world for _ in range(world)]        # flags[owner][writer]
    board = [[(0, None) for _ in range(world)] for _ in range(world)]   # (epoch, value)
    busy = {}                                           # resource -> set of ranks using it
    progs = []
    for r in range(world):
        ops, e = [], 0
        for s in range(steps):
            ops += [("use", f"P{r}", f"G{r}", "begin"), ("use", f"P{r}", f"G{r}", "end")]
            e += 1
            ops += [("flag_post", e), ("flag_wait", e)]
            ops += [("read_peers", "G", "begin"), ("read_peers", "G", "end")]
            e += 1
            ops += [("board_post", e, (s, r)), ("board_wait", e, s)]
            ops += [("write_peers", "P", "begin"), ("write_peers", "P", "end")]
            if barrier_after:
                e += 1
                ops += [("flag_post", e), ("flag_wait", e)]
        progs.append(ops)
    pc = [0] * world
    n = 0
    while True:
        n += 1
        assert n < 2_000_000
        runnable = []
        for r in range(world):
            if pc[r] >= len(progs[r]):
                continue
            op = progs[r][pc[r]]
            if op[0] == "flag_wait":
                # signed difference, as the kernel compares epochs
                if all(flags[r][q] - op[1] >= 0 for q in range(world)):
                    runnable.append(r)
            elif op[0] == "board_wait":
                eps = [board[r][q][0] for q in range(world)]
                assert all(x <= op[1] for x in eps), ("a peer posted a later epoch", r, eps, op)
                if all(x == op[1] for x in eps):
                    runnable.append(r)
            else:
                runnable.append(r)
        if not runnable:
            assert all(pc[r] >= len(progs[r]) for r in range(world)), ("hang", pc)
            return
        r = rng.choice(runnable)
        op = progs[r][pc[r]]
        pc[r] += 1
        kind = op[0]
        if kind == "use":        # forward + backward: reads own params, writes own gradients
            _, p, g, phase = op
            if phase == "begin":
                assert not busy.get(p) and not busy.get(g), ("peers use this rank's arenas", r, busy)
                busy.setdefault(f"own{p}", set()).add(r)
                busy.setdefault(f"own{g}", set()).add(r)
            else:
                busy[f"own{p}"].discard(r)
                busy[f"own{g}"].discard(r)
        elif kind == "flag_post":
            for q in range(world):
                flags[q][r] = op[1]
        elif kind == "board_post":
            for q in range(world):
                board[q][r] = (op[1], op[2])
        elif kind == "board_wait":
            vals = [board[r][q][1] for q in range(world)]
            assert all(v == (op[2], q) for q, v in enumerate(vals)), ("stale board", r, vals)
        elif kind == "read_peers":
            for q in range(world):
                if op[2] == "begin":
                    assert not busy.get(f"ownG{q}"), ("reads gradients a peer is writing", r, q)
                    busy.setdefault(f"G{q}", set()).add(r)
                else:
                    busy[f"G{q}"].discard(r)
        elif kind == "write_peers":
            for q in range(world):
                if op[2] == "begin":
                    assert not busy.get(f"ownP{q}"), ("stores into parameters in use", r, q)
                    busy.setdefault(f"P{q}", set()).add(r)
                else:
                    busy[f"P{q}"].discard(r)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_step_protocol(world):
    for seed in range(20):
        run_fused_step(world, steps=4, seed=seed)


def test_fused_step_needs_the_closing_barrier():
    """Without the barrier after the parameter stores, some interleaving lets
    a rank start its next backward while a peer still stores into it."""
    failures = 0
    for seed in range(200):
        try:
            run_fused_step(2, steps=3, seed=seed, barrier_after=False)
        except AssertionError:
            failures += 1
    assert failures > 0


# ---------------------------------------------------------------------------
# Stream-K and split-K fixup of the pair GEMM (gemm2_kernel): which pair
# finishes which tile, the per-tile counters, and termination.  Mirrors
# sk_range / sk_pair_of / work_item and the epilogue's contrib / finish roles.

WARPS = 16          # epilogue warps of a CTA pair: each arrives once


def sk_range(pair, per, extra):
    b = pair * per + min(pair, extra)
    return b, b + per + (1 if pair < extra else 0)


def sk_pair_of(it, per, extra):
    big = extra * (per + 1)
    if it < big:
        return it // (per + 1)
    return extra + (it - big) // per


def sk_items(pair, kbt, per, extra):
    b, e = sk_range(pair, per, extra)
    k, out = 0, []
    while True:
        t = b // kbt + k
        lo, hi = max(b, t * kbt), min(e, (t + 1) * kbt)
        if lo >= hi:
            return out
        out.append((t, lo - t * kbt, hi - t * kbt))
        k += 1


def stream_k_plan(tiles, kbt, npairs):
    total = tiles * kbt
    per, extra = total // npairs, total % npairs
    plan = []
    for pair in range(npairs):
        items = []
        for (t, kb0, kb1) in sk_items(pair, kbt, per, extra):
            contrib = kb0 > 0
            finish = kb0 == 0 and kb1 < kbt
            n = sk_pair_of((t + 1) * kbt - 1, per, extra) - pair if finish else 0
            items.append(dict(tile=t, kb0=kb0, kb1=kb1, contrib=contrib, finish=finish,
                              wait=WARPS * n, slots=[pair + j for j in range(1, n + 1)],
                              slot=pair))
        plan.append(items)
    return plan


def fixup_plan(tiles, splits):
    """Split-K with every unit resident: unit = split * tiles + tile, one per pair."""
    plan = []
    for u in range(tiles * splits):
        split, t = divmod(u, tiles)
        last = split == splits - 1
        plan.append([dict(tile=t, kb0=split, kb1=split + 1, contrib=not last, finish=last,
                          wait=WARPS * (splits - 1) if last else 0,
                          slots=[s * tiles + t for s in range(splits - 1)] if last else [],
                          slot=split * tiles + t)])
    return plan


def run_tiles(plan, tiles, kbt, seed):
    """Execute every pair's items in order under a random interleaving of
    the pairs (warps of a pair step together); a finisher blocks until its
    counter reaches the target.  Returns the K slices each tile summed."""
    rng = random.Random(seed)
    ctr = [0] * tiles
    slots = {}
    summed = {t: [] for t in range(tiles)}
    pos = [0] * len(plan)
    while True:
        live = [p for p in range(len(plan)) if pos[p] < len(plan[p])]
        if not live:
            break
        ready = []
        for p in live:
            it = plan[p][pos[p]]
            if not it["finish"] or ctr[it["tile"]] >= it["wait"]:
                ready.append(p)
        assert ready, "deadlock: every live pair waits"
        p = rng.choice(ready)
        it = plan[p][pos[p]]
        rng_slices = list(range(it["kb0"], it["kb1"]))
        t = it["tile"]
        if it["contrib"]:
            assert it["slot"] not in slots          # a slot holds one partial at a time
            slots[it["slot"]] = (t, rng_slices)
            ctr[t] += WARPS
        elif it["finish"]:
            got = list(rng_slices)
            for s in it["slots"]:
                tt, sl = slots.pop(s)
                assert tt == t                      # the slot holds this tile's partial
                got += sl
            summed[t].append(sorted(got))
            # the 16 finishing warps count out; the last one clears the counter
            ctr[t] += WARPS
            assert ctr[t] == it["wait"] + WARPS
            ctr[t] = 0
        else:
            summed[t].append(rng_slices)
        pos[p] += 1
    assert all(c == 0 for c in ctr), "a counter was left raised"
    assert not slots, "a partial was never consumed"
    for t in range(tiles):
        assert summed[t] == [list(range(kbt))], (t, summed[t])


@pytest.mark.parametrize("tiles,kbt,npairs", [(36, 256, 74), (27, 256, 74), (2, 65, 74),
                                              (192, 48, 74), (9, 256, 74), (5, 7, 31)])
def test_stream_k_finishes_every_tile_once(tiles, kbt, npairs):
    if tiles * kbt < npairs:
        pytest.skip("the host falls back to units below one slice per pair")
    plan = stream_k_plan(tiles, kbt, npairs)
    # a finisher is always its pair's last item and waits only for later
    # pairs' first items, which never wait: no cycle is possible
    for p, items in enumerate(plan):
        for k, it in enumerate(items):
            if it["finish"]:
                assert k == len(items) - 1
                for q in it["slots"]:
                    assert q > p and plan[q][0]["contrib"] and plan[q][0]["tile"] == it["tile"]
            if it["contrib"]:
                assert k == 0
    for seed in range(20):
        run_tiles(plan, tiles, kbt, seed)


@pytest.mark.parametrize("tiles,splits", [(36, 2), (27, 2), (9, 8), (18, 4)])
def test_split_k_fixup_finishes_every_tile_once(tiles, splits):
    plan = fixup_plan(tiles, splits)
    for seed in range(20):
        run_tiles(plan, tiles, splits, seed)


# ------------------------------------------------- batched column-sum finishes
# colsum_finish_many (csrc/nn_kernels.cu): the host cuts the job list into
# launches of at most MAX_JOBS; a launch's job j owns the blocks
# first[j] .. first[j + 1] - 1 (ceil(N_j / 32) of them), and a block finds
# its job by scanning first[] upward from 0.
MAX_JOBS = 48


def colsum_launches(widths):
    """Host plan: per launch, (first[], block count), as colsum_finish_many."""
    launches = []
    for j0 in range(0, len(widths), MAX_JOBS):
        chunk = widths[j0:j0 + MAX_JOBS]
        first, blocks = [], 0
        for n in chunk:
            first.append(blocks)
            blocks += (n + 31) // 32
        first.append(blocks)
        launches.append((j0, first, blocks))
    return launches


def block_job(first, njobs, block):
    """Device scan: the job that owns `block` (the kernel's while loop)."""
    j = 0
    while j + 1 < njobs and block >= first[j + 1]:
        j += 1
    return j, block - first[j]


@pytest.mark.parametrize("seed", range(8))
def test_colsum_batches_cover_every_column_once(seed):
    """Every column of every job is finished by exactly one thread of one
    block, across launches, for ragged widths (including 1 and multiples
    of 32) and job counts around the per-launch limit."""
    import random

    rng = random.Random(seed)
    njobs = rng.choice([1, 47, 48, 49, 98, 100])
    widths = [rng.choice([1, 31, 32, 33, 768, 1600, 3072, 6400]) for _ in range(njobs)]
    seen = [[0] * n for n in widths]
    for j0, first, blocks in colsum_launches(widths):
        nj = len(first) - 1
        for b in range(blocks):
            j, cb = block_job(first, nj, b)
            for lane in range(32):
                c = cb * 32 + lane
                if c < widths[j0 + j]:          # the kernel's `c < N` guard
                    seen[j0 + j][c] += 1
    assert all(all(x == 1 for x in cols) for cols in seen)
    # one launch per MAX_JOBS jobs, as the GPU profile shows (98 -> 3)
    assert len(colsum_launches(widths)) == -(-njobs // MAX_JOBS)


# ----------------------------------------- partial-tile slot of the pair kernel
# gemm2_kernel's epilogue (csrc/gemm_tcgen05.cu): 8 epilogue warps per CTA
# (warps 2..9), quarter = warp & 3, half = (warp - 2) / 4; CTA `rank` of the
# pair owns tile rows 128 * rank + 32 * quarter + lane and 32-column chunks
# c = half, half + 2, ...; a partial is stored in register order, float4 q of
# lane l of (row block rb, chunk c) at ((rb * 8 + c) * 8 + q) * 32 + l.
PAIR_TM, PAIR_BN2, PAIR_HALF = 256, 256, 128


def test_pair_partial_slot_is_a_bijection():
    """Every fp32 value of a 256 x 256 partial tile has its own float4 slot
    entry inside the slot (65536 floats), so contributing pairs and splits
    never overwrite one another and never leave their slot."""
    seen = {}
    for rank in range(2):
        for warp in range(2, 10):
            quarter, half = warp & 3, (warp - 2) // 4
            for lane in range(32):
                row = PAIR_HALF * rank + quarter * 32 + lane
                for c in range(half, PAIR_BN2 // 32, 2):
                    slot_off = ((row >> 5) * (PAIR_BN2 // 32) + c) * 8 * 32 + lane
                    for q in range(8):
                        f4 = slot_off + q * 32
                        assert 0 <= f4 and f4 * 4 + 3 < PAIR_TM * PAIR_BN2
                        for k in range(4):          # the four floats of the float4
                            key = f4 * 4 + k
                            assert key not in seen, (rank, warp, lane, c, q)
                            seen[key] = (row, c * 32 + q * 4 + k)
    assert len(seen) == PAIR_TM * PAIR_BN2
    # every (row, column) of the tile appears once
    assert len(set(seen.values())) == PAIR_TM * PAIR_BN2
