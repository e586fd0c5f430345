"""Executable models of the mbarrier protocols of the persistent tensor-core
kernels, run under random schedules on the CPU.

Each role of a kernel (TMA producer, MMA issuers, softmax / elementwise
warpgroups) is a generator that yields the waits and arrivals it performs, in
the order the kernel performs them (fwd_bf16_sm100.cu, bwd_bf16_sm100.cu).  A
barrier completes a phase after `count` arrivals.  A wait "for completion n"
is what the kernels express as a parity wait, so two properties are checked on
every schedule:
  * no deadlock: some role can always run until all have finished;
  * no parity ambiguity: when a role starts waiting for completion n the
    barrier has completed at least n - 1 phases (else the parity test could
    pass on an older phase), and no barrier runs two phases past a role still
    blocked on it.
The models must follow the kernels: a change to a kernel's waits, arrivals or
their order goes into its model here too.
"""
import random

import pytest


class _Bar:
    def __init__(self, name, count=1):
        self.name, self.count, self.arr, self.done = name, count, 0, 0


def _run(make_roles, seed):
    rnd = random.Random(seed)
    bars, hazards = {}, []

    def bar(name, count=1):
        bars[name] = _Bar(name, count)

    def W(name, target):
        return ("wait", bars[name], target)

    def A(name):
        return ("arr", bars[name])

    gens = make_roles(bar, W, A)
    roles = [{"name": n, "gen": g, "wait": None, "done": False} for n, g in gens]

    def arrive(b):
        b.arr += 1
        if b.arr == b.count:
            b.arr, b.done = 0, b.done + 1
            for r in roles:
                w = r["wait"]
                if w and w[0] is b and b.done >= w[1] + 1:
                    hazards.append(("overshoot", b.name, w[1], b.done, r["name"]))

    def step(r):
        while True:
            if r["wait"] is not None:
                b, t = r["wait"]
                if b.done < t:
                    return
                r["wait"] = None
            try:
                op = next(r["gen"])
            except StopIteration:
                r["done"] = True
                return
            if op[0] == "wait":
                b, t = op[1], op[2]
                if b.done < t - 1:
                    hazards.append(("false-pass", b.name, t, b.done, r["name"]))
                r["wait"] = (b, t)
                if b.done < t or rnd.random() < 0.5:
                    return
            else:
                arrive(op[1])
                if rnd.random() < 0.3:
                    return

    while True:
        live = [r for r in roles if not r["done"]]
        if not live:
            return None, hazards
        ready = [r for r in live if r["wait"] is None or r["wait"][0].done >= r["wait"][1]]
        if not ready:
            return [(r["name"], r["wait"][0].name, r["wait"][1], r["wait"][0].done) for r in live], hazards
        step(rnd.choice(ready))


# ---------------------------------------------------------------------------
# fwd_bf16_sm100.cu: items of two query tiles (n0 and n1 key tiles, n1 = n0 + 1
# or 0), Q double buffer, 4-stage K/V ring with K and V on separate barriers;
# query tile i of item k goes to warpgroup i ^ swap(k)
# ---------------------------------------------------------------------------
def _fwd_roles(items, stages=4, alternate=True):
    def swap(k):
        return (k & 1) if alternate else 0

    def make(bar, W, A):
        for q in range(2):
            bar(("QF", q))
            bar(("QE", q))
        for s in range(stages):
            bar(("KF", s))
            bar(("VF", s))
            bar(("KVE", s), 3)
        for w in range(2):
            for n in ("SF", "SE", "PF", "OD", "OF"):
                bar((n, w))

        def producer():
            g = 0
            for k, (n0, n1, nkv) in enumerate(items):
                qb = k & 1
                if k >= 2:
                    yield W(("QE", qb), k >> 1)
                yield A(("QF", qb))
                for j in range(nkv):
                    st = g % stages
                    if g >= stages:
                        yield W(("KVE", st), g // stages)
                    yield A(("KF", st))
                    yield A(("VF", st))
                    g += 1

        def s_issuer():
            g, t = 0, [0, 0]
            for k, (n0, n1, nkv) in enumerate(items):
                qb = k & 1
                yield W(("QF", qb), (k >> 1) + 1)
                for j in range(nkv):
                    st = (g + j) % stages
                    yield W(("KF", st), (g + j) // stages + 1)
                    for i in range(2):
                        if j >= (n1 if i else n0):
                            continue
                        w = i ^ swap(k)
                        if t[w] > 0:
                            yield W(("SE", w), t[w])
                        yield A(("SF", w))
                        t[w] += 1
                    yield A(("KVE", st))
                    if j == nkv - 1:
                        yield A(("QE", qb))
                g += nkv

        def pv(i):
            g, t, kw = 0, 0, 0
            for k, (n0, n1, nkv) in enumerate(items):
                n = n1 if i ^ swap(k) else n0
                for j in range(nkv):
                    st = (g + j) % stages
                    yield W(("VF", st), (g + j) // stages + 1)
                    if j >= n:
                        yield A(("KVE", st))
                        continue
                    if j == 0 and kw > 0:
                        yield W(("OF", i), kw)
                    yield W(("PF", i), t + 1)
                    yield A(("OD", i))
                    yield A(("KVE", st))
                    t += 1
                if n > 0:
                    kw += 1
                g += nkv

        def softmax(w):
            t = 0
            for k, (n0, n1, nkv) in enumerate(items):
                n = n1 if w ^ swap(k) else n0
                if n == 0:
                    continue
                for j in range(n):
                    yield W(("SF", w), t + 1)
                    yield A(("SE", w))
                    if t > 0:
                        yield W(("OD", w), t)
                    yield A(("PF", w))
                    t += 1
                yield W(("OD", w), t)
                yield A(("OF", w))

        return [("producer", producer()), ("S", s_issuer()), ("PV0", pv(0)), ("PV1", pv(1)),
                ("softmax0", softmax(0)), ("softmax1", softmax(1))]
    return make


def _fwd_items(T, pairs):
    out = []
    for pair in pairs:
        q0 = pair * 256
        has_q1 = q0 + 128 < T
        n0 = q0 // 128 + 1
        n1 = n0 + 1 if has_q1 else 0
        out.append((n0, n1, n1 if has_q1 else n0))
    return out


@pytest.mark.parametrize("T", [128, 200, 300, 1024, 1100, 4096])
@pytest.mark.parametrize("alternate", [True, False])
def test_fwd_bf16_protocol(T, alternate):
    n_pairs = (T + 255) // 256
    for trial in range(40):
        rnd = random.Random(trial * 31 + T)
        pairs = sorted((rnd.randrange(n_pairs) for _ in range(rnd.randint(1, 6))), reverse=True)
        dead, hazards = _run(_fwd_roles(_fwd_items(T, pairs), alternate=alternate), trial)
        assert dead is None, (pairs, dead)
        assert not hazards, (pairs, hazards[:3])


# ---------------------------------------------------------------------------
# bwd_bf16_sm100.cu: persistent, units of `count` streamed tiles, fixed tiles
# in two buffers, 3-stage streamed ring, accumulators handed over per unit
# ---------------------------------------------------------------------------
def _bwd_roles(counts, kind, stages=3):
    def make(bar, W, A):
        for f in range(2):
            bar(("FIX", f))
            bar(("FE", f))
        for s in range(stages):
            bar(("SF", s))
            bar(("SE", s))
        bar("XY")
        bar("XYE", 2)
        bar("W", 2)
        bar("ACC")
        bar("ST", 2)
        bar("AF", 2)

        def producer():
            g = 0
            for k, cnt in enumerate(counts):
                fb = k & 1
                if k >= 2:
                    yield W(("FE", fb), k >> 1)
                yield A(("FIX", fb))
                for _ in range(cnt):
                    st = g % stages
                    if g >= stages:
                        yield W(("SE", st), g // stages)
                    yield A(("SF", st))
                    g += 1

        def xy():
            g = 0
            for k, cnt in enumerate(counts):
                fb = k & 1
                yield W(("FIX", fb), (k >> 1) + 1)
                for it in range(cnt):
                    yield W(("SF", g % stages), g // stages + 1)
                    if g > 0:
                        yield W("XYE", g)
                    yield A("XY")
                    if it == cnt - 1:
                        yield A(("FE", fb))
                    g += 1

        def acc():
            g = 0
            for k, cnt in enumerate(counts):
                for it in range(cnt):
                    if it == 0 and k > 0:
                        yield W("AF", k)
                    yield W("W", g + 1)
                    yield A("ACC")
                    yield A(("SE", g % stages))
                    g += 1

        def elementwise():
            g = 0
            for cnt in counts:
                for _ in range(cnt):
                    if kind == 0:
                        yield A("ST")
                        yield W("ST", g + 1)
                    yield W("XY", g + 1)
                    if g > 0:
                        yield W("ACC", g)
                    yield A("XYE")
                    yield A("W")
                    g += 1
                yield W("ACC", g)
                yield A("AF")

        return [("producer", producer()), ("xy", xy()), ("acc", acc()),
                ("elementwise0", elementwise()), ("elementwise1", elementwise())]
    return make


@pytest.mark.parametrize("kind", [0, 1])
def test_bwd_bf16_persistent_protocol(kind):
    for trial in range(300):
        rnd = random.Random(trial)
        counts = [rnd.randint(1, 7) for _ in range(rnd.randint(1, 7))]
        dead, hazards = _run(_bwd_roles(counts, kind), trial)
        assert dead is None, (counts, dead)
        assert not hazards, (counts, hazards[:3])


# ---------------------------------------------------------------------------
# bwd_tf32_sm100.cu: one unit of `count` streamed tiles through a 2-stage ring;
# X/Y (and the P/dS parts written over them) double-buffered in TMEM by tile
# parity, so tile it+1's X/Y products run while tile it is in the elementwise
# warpgroup; accumulators restart every `group` tiles once the elementwise
# warpgroup has folded them into its running sums
# ---------------------------------------------------------------------------
def _bwd_tf32_roles(count, kind, group):
    def make(bar, W, A):
        bar("FXF")
        bar("FX", 2)
        for s in range(2):
            bar(("SF", s))
            bar(("SS", s), 2)
            bar(("SE", s))
            bar(("XY", s))
            bar(("W", s), 2)
            bar(("ACC", s))
        bar("ST", 2)
        bar("AF", 2)

        def producer():
            yield A("FXF")
            for it in range(count):
                st = it & 1
                if it >= 2:
                    yield W(("SE", st), it >> 1)
                yield A(("SF", st))

        def splitter():
            yield W("FXF", 1)
            yield A("FX")
            for it in range(count):
                st = it & 1
                yield W(("SF", st), (it >> 1) + 1)
                yield A(("SS", st))

        def xy():
            yield W("FX", 1)
            for it in range(count):
                b = it & 1
                yield W(("SS", b), (it >> 1) + 1)
                if it >= 2:
                    yield W(("ACC", b), it >> 1)        # the buffer's previous tile was accumulated
                yield A(("XY", b))

        def acc():
            for it in range(count):
                b = it & 1
                yield W(("W", b), (it >> 1) + 1)
                if it >= group and it % group == 0:
                    yield W("AF", it // group)
                yield A(("ACC", b))
                yield A(("SE", b))

        def elementwise():
            for it in range(count):
                b = it & 1
                if kind == 0:
                    yield A("ST")
                    yield W("ST", it + 1)
                yield W(("XY", b), (it >> 1) + 1)
                yield A(("W", b))
                if it % group == group - 1 or it == count - 1:
                    yield W(("ACC", b), (it >> 1) + 1)
                    yield A("AF")

        return [("producer", producer()), ("splitter0", splitter()), ("splitter1", splitter()),
                ("xy", xy()), ("acc", acc()), ("elementwise0", elementwise()), ("elementwise1", elementwise())]
    return make


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("group", [1, 2, 3, 8])
def test_bwd_tf32_double_buffered_protocol(kind, group):
    for trial in range(150):
        rnd = random.Random(trial * 7 + group)
        count = rnd.randint(1, 40)
        dead, hazards = _run(_bwd_tf32_roles(count, kind, group), trial)
        assert dead is None, (count, dead)
        assert not hazards, (count, hazards[:3])


def test_models_catch_a_missing_wait():
    """The checker itself: without the producer's wait for a free fixed-tile
    buffer, the backward model must report a parity hazard."""
    def broken(bar, W, A):
        roles = _bwd_roles([2, 1, 7, 3, 3], 0)(bar, W, A)

        def producer():
            g = 0
            for k, cnt in enumerate([2, 1, 7, 3, 3]):
                yield A(("FIX", k & 1))
                for _ in range(cnt):
                    st = g % 3
                    if g >= 3:
                        yield W(("SE", st), g // 3)
                    yield A(("SF", st))
                    g += 1
        return [("producer", producer())] + roles[1:]
    found = False
    for trial in range(200):
        dead, hazards = _run(broken, trial)
        if hazards or dead:
            found = True
            break
    assert found

