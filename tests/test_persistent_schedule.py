"""The persistent schedule of the two-tile kernel, checked on the CPU
(attnprofile_b200/csrc/attn_kernel.cuh: ItemCursor, step_owner,
load_role_persistent, mma_role_persistent, softmax_role_persistent).

1. Items: CTA c of G first runs the whole units c, c + G, ... (R' rounds:
   R' = U // G when G divides U, else max(U // G - 1, 0)), then its share
   [base + c T_t / G, base + (c + 1) T_t / G) of the remaining T_t steps
   (base = R' G n_kv).  Over every CTA the items cover each step once; a
   unit cut between CTAs has exactly one kMerger piece (its first key tile,
   the last item of its CTA c0, peer = the last CTA c1 holding a piece) and
   its other pieces are kWriter items, the first tail items of CTAs
   c0 + 1 .. c1, each naming c0; with U >= G every unit has at most two
   pieces.  The host planner's grid and most pieces per unit
   (attn_plan_schedule) agree with this model.
2. Barrier protocol: a discrete-event model of one CTA -- the producer, the
   TMA engine, the MMA issuer, the tensor pipe (in order; a commit arrives
   once every earlier MMA has executed) and the two softmax warpgroups --
   written after the kernel's code, run under many random interleavings.
   mbarrier waits use the hardware's parity rule (a wait on parity P returns
   once the barrier's completed-phase count k has (k & 1) != P).  Checked:
   every wait returns at exactly the completion it means (k = i + 1 for the
   i-th completion; no parity aliasing, no deadlock), every shared-memory
   slot and TMEM region is rewritten only after its last reader ran, and every
   reader sees the data of its own item and step.
"""
import random

import pytest


# ---------------------------------------------------------------------------
# 1. items
# ---------------------------------------------------------------------------
def step_owner(x, T, G):
    return ((x + 1) * G - 1) // T


def rr_rounds(U, G):
    R, r = divmod(U, G)
    return R if r == 0 else max(R - 1, 0)


def items_of(c, U, nkv, G):
    rr = rr_rounds(U, G)
    out = [dict(u=k * G + c, lo=0, n=nkv, role="whole", peer=-1, tail=False) for k in range(rr)]
    base = rr * G * nkv
    Tt = (U - rr * G) * nkv
    cur, end = base + c * Tt // G, base + (c + 1) * Tt // G
    while cur < end:
        u, lo = divmod(cur, nkv)
        hi = min(nkv, lo + (end - cur))
        if lo == 0 and hi == nkv:
            role, peer = "whole", -1
        elif lo == 0:
            role, peer = "merger", step_owner((u + 1) * nkv - 1 - base, Tt, G)
        else:
            role, peer = "writer", step_owner(u * nkv - base, Tt, G)
        out.append(dict(u=u, lo=lo, n=hi - lo, role=role, peer=peer, tail=True))
        cur += hi - lo
    return out


CASES = [(256, 32, 148), (8192, 64, 148), (64, 64, 148), (2048, 256, 148), (16, 32, 148),
         (1, 7, 5), (3, 5, 7), (10, 3, 29), (100, 1, 37), (5, 40, 148), (7, 13, 90)]


@pytest.mark.parametrize("U,nkv,G", CASES)
def test_items_cover_every_step_once_with_one_merger_per_cut_unit(U, nkv, G):
    T = U * nkv
    G = min(G, T)
    seen = []
    pieces = {}
    for c in range(G):
        its = items_of(c, U, nkv, G)
        assert its, "every CTA has at least one step (G <= T)"
        for k, it in enumerate(its):
            seen += [it["u"] * nkv + it["lo"] + j for j in range(it["n"])]
            pieces.setdefault(it["u"], []).append((c, k, len(its), it))
    assert sorted(seen) == list(range(T))
    for u, ps in pieces.items():
        ps.sort(key=lambda p: p[3]["lo"])
        if len(ps) == 1:
            assert ps[0][3]["role"] == "whole"
            continue
        if U >= G:
            assert len(ps) == 2, "a unit is cut at most once when units >= CTAs"
        c0, k0, nk0, m = ps[0]
        assert m["role"] == "merger" and m["lo"] == 0 and k0 == nk0 - 1
        assert m["peer"] == ps[-1][0]
        assert [p[0] for p in ps] == list(range(c0, m["peer"] + 1))
        for c, k, nk, it in ps[1:]:
            first_tail = min(i for i, x in enumerate(items_of(c, U, nkv, G)) if x["tail"])
            assert it["role"] == "writer" and k == first_tail and it["peer"] == c0
    # one writer slot per CTA (its first tail item), one counter per merging CTA
    for c in range(G):
        its = items_of(c, U, nkv, G)
        assert sum(it["role"] == "writer" for it in its) <= 1
        assert sum(it["role"] == "merger" for it in its) <= 1
        assert all(x["tail"] for x in its[rr_rounds(U, G):])
    # the whole units that run round-robin are neighbours at every moment
    rr = rr_rounds(U, G)
    for k in range(rr):
        assert sorted(items_of(c, U, nkv, G)[k]["u"] for c in range(G)) == \
            list(range(k * G, (k + 1) * G))


@pytest.mark.parametrize("U,nkv,slots", [(256, 32, 148), (8192, 64, 148), (64, 64, 148),
                                         (2048, 256, 148), (16, 32, 148), (3, 5, 7)])
def test_host_planner_matches_the_model(engine, U, nkv, slots):
    plan = engine.plan_schedule(U, nkv, slots)
    G = plan["ctas"]
    assert 1 <= G <= min(slots, U * nkv)
    per_unit = {}
    for c in range(G):
        for it in items_of(c, U, nkv, G):
            per_unit[it["u"]] = per_unit.get(it["u"], 0) + 1
    assert plan["pieces"] == max(per_unit.values())
    # the automatic mode runs the classic schedule (measured no slower)
    assert plan["persistent"] is False
    assert plan["persistent_cost"] > 0 and plan["classic_cost"] > 0


# ---------------------------------------------------------------------------
# 2. barrier protocol of one CTA
# ---------------------------------------------------------------------------
class Bar:
    def __init__(self, name, count):
        self.name, self.count = name, count
        self.pending, self.tx, self.k = count, 0, 0

    def arrive(self, tx=0, expect=0):
        self.tx += expect - tx
        self.pending -= 1
        self._check()

    def complete_tx(self, b):
        self.tx -= b
        self._check()

    def _check(self):
        assert self.pending >= 0, self.name
        if self.pending == 0 and self.tx == 0:
            self.k += 1
            self.pending = self.count

    def ready(self, parity):
        return (self.k & 1) != parity


class Sim:
    """One CTA: NQ = 2 tiles, PHALVES = 2, STAGES ring slots, joint landing."""

    def __init__(self, items, stages, rng):
        self.items, self.S, self.rng = items, stages, rng
        self.bars = {}
        self.log = []
        for i in range(2):
            self.bar(f"Q{i}"), self.bar(f"S_FULL{i}"), self.bar(f"O_FINAL{i}"), self.bar(f"Q_FREE{i}")
            for h in range(2):
                self.bar(f"P{i}{h}")
        for s in range(stages):
            self.bar(f"FULL{s}"), self.bar(f"EMPTY{s}")
        self.bar("DRAIN")
        self.tma = []        # pending loads: (slot name, payload, barrier)
        self.pipe = []       # issued tensor ops, executed in order
        self.smem = {}       # slot -> payload currently written
        self.readers = {}    # slot -> number of issued-but-unexecuted MMAs reading it
        self.tmem = {}       # region -> payload
        self.done = set()

    def bar(self, n, c=1):
        self.bars[n] = Bar(n, c)

    # --- waits: generator helper --------------------------------------
    def wait(self, name, parity, idx):
        """Wait for the idx-th completion (0-based) with the kernel's parity."""
        b = self.bars[name]
        assert parity == idx & 1
        while not b.ready(parity):
            assert b.k <= idx, f"{name}: awaited completion {idx} was overtaken (k={b.k})"
            yield
        assert b.k == idx + 1, f"{name}: wait for completion {idx} returned at k={b.k}"

    # --- TMA and tensor pipe --------------------------------------------
    def tma_load(self, slot, payload, bar, nbytes):
        assert self.readers.get(slot, 0) == 0, f"{slot} reloaded while an MMA still reads it"
        self.tma.append((slot, payload, bar, nbytes))

    def mma(self, kind, reads, writes, payload_check):
        for r in reads:
            self.readers[r] = self.readers.get(r, 0) + 1
        self.pipe.append(("mma", kind, reads, writes, payload_check))

    def commit(self, bar):
        self.pipe.append(("commit", bar))

    def step_async(self):
        opts = []
        if self.tma:
            opts.append("tma")
        if self.pipe:
            opts.append("pipe")
        if not opts:
            return False
        if self.rng.choice(opts) == "tma":
            slot, payload, bar, nbytes = self.tma.pop(self.rng.randrange(len(self.tma)))
            self.smem[slot] = payload
            self.bars[bar].complete_tx(nbytes)
        else:
            op = self.pipe.pop(0)
            if op[0] == "commit":
                self.bars[op[1]].arrive()
            else:
                _, kind, reads, writes, check = op
                check(self)
                for r in reads:
                    self.readers[r] -= 1
                for w_, val in writes:
                    self.tmem[w_] = val
        return True

    # --- the roles, after the kernel -------------------------------------
    def producer(self):
        S, its = self.S, self.items
        t = 0
        last_k_commit = {}

        def produce(kind, it_idx, j, J, joint, k_bar):
            nonlocal t
            s = t % S
            if t >= S:
                period = S // 2 if S % 2 == 0 else S
                m = (t - S + 1) // 2
                yield from self.wait(f"EMPTY{(2 * m) % S}", (m // period) & 1, m // period)
            full = f"FULL{s}"
            payload = (kind, it_idx, j)
            if k_bar is not None:
                self.bars[full].arrive()
                full = f"FULL{k_bar}"
                self.tma_load(f"slot{s}", payload, full, 1)
            else:
                self.bars[full].arrive(expect=2 if joint else 1)
                self.tma_load(f"slot{s}", payload, full, 1)
            t += 1

        def load_q(it_idx):
            for i in range(2):
                self.bars[f"Q{i}"].arrive(expect=1)
                self.tma_load(f"q{i}", ("Q", it_idx), f"Q{i}", 1)

        load_q(0)
        yield from produce("K", 0, 0, 0, False, None)
        J = 0
        for k, it in enumerate(its):
            for j in range(it["n"]):
                last = j == it["n"] - 1
                joint = not last
                sv = t % S
                yield from produce("V", k, j, J, joint, None)
                if not last:
                    yield from produce("K", k, j + 1, J + 1, False, sv)
                elif k + 1 < len(its):
                    yield from produce("K", k + 1, 0, J + 1, False, None)
                    for i in range(2):
                        yield from self.wait(f"Q_FREE{i}", k & 1, k)
                    load_q(k + 1)
                J += 1
        self.done.add("producer")

    def mma_issuer(self):
        S, its = self.S, self.items
        t = 0

        def ring_wait():
            nonlocal t
            s = t % S
            yield from self.wait(f"FULL{s}", (t // S) & 1, t // S)
            t += 1
            return s

        def issue_s(i, slot, it_idx, j):
            def check(sim, i=i, slot=slot, it_idx=it_idx, j=j):
                assert sim.smem[f"q{i}"] == ("Q", it_idx), "S read another item's Q"
                assert sim.smem[f"slot{slot}"] == ("K", it_idx, j), "S read the wrong K"
            self.mma("S", [f"q{i}", f"slot{slot}"], [(f"S{i}", ("S", it_idx, j))], check)

        def issue_pv(i, slot, it_idx, j, h):
            def check(sim, i=i, slot=slot, it_idx=it_idx, j=j, h=h):
                assert sim.smem[f"slot{slot}"] == ("V", it_idx, j), "P V read the wrong V"
                assert sim.tmem.get(f"P{i}") == ("P", it_idx, j), "P V read a stale P"
                if h == 0 and j == 0:
                    assert sim.tmem.get(f"Oread{i}", it_idx - 1) == it_idx - 1, \
                        "O overwritten before its epilogue read it"
            self.mma("PV", [f"slot{slot}"], [(f"O{i}", ("O", it_idx, j, h))], check)

        for i in range(2):
            yield from self.wait(f"Q{i}", 0, 0)
        sk = yield from ring_wait()
        for i in range(2):
            issue_s(i, sk, 0, 0)
            self.commit(f"S_FULL{i}")
        self.commit(f"EMPTY{sk}")
        J = 0
        for k, it in enumerate(its):
            has_nx = k + 1 < len(its)
            n = it["n"]
            for j in range(n - 1):          # the item's steps but its last
                sv = yield from ring_wait()
                sk = -1
                for i in range(2):
                    for h in range(2):
                        if h == 1 and sk < 0:
                            sk = t % S   # K_{J+1} landed with V_J (joint landing)
                            t += 1
                        yield from self.wait(f"P{i}{h}", J & 1, J)
                        issue_pv(i, sv, k, j, h)
                    issue_s(i, sk, k, j + 1)
                    self.commit(f"S_FULL{i}")
                self.commit(f"EMPTY{sk}")
                J += 1
            # the item's last step
            for i in range(2):
                self.commit(f"Q_FREE{i}")
            sv = yield from ring_wait()
            sk = -1
            for i in range(2):
                for h in range(2):
                    yield from self.wait(f"P{i}{h}", J & 1, J)
                    issue_pv(i, sv, k, n - 1, h)
                self.commit(f"O_FINAL{i}")
                if has_nx:
                    if sk < 0:
                        sk = yield from ring_wait()
                    yield from self.wait(f"Q{i}", (k + 1) & 1, k + 1)
                    issue_s(i, sk, k + 1, 0)
                    self.commit(f"S_FULL{i}")
            if sk >= 0:
                self.commit(f"EMPTY{sk}")
            J += 1
        self.commit("DRAIN")
        yield from self.wait("DRAIN", 0, 0)
        self.done.add("mma")

    def softmax(self, i):
        J = 0
        for k, it in enumerate(self.items):
            for j in range(it["n"]):
                yield from self.wait(f"S_FULL{i}", J & 1, J)
                assert self.tmem[f"S{i}"] == ("S", k, j), "softmax read the wrong S"
                self.tmem[f"P{i}"] = ("P", k, j)
                for h in range(2):
                    self.bars[f"P{i}{h}"].arrive()
                    yield
                J += 1
            yield from self.wait(f"O_FINAL{i}", k & 1, k)
            assert self.tmem[f"O{i}"] == ("O", k, it["n"] - 1, 1), "epilogue read an unfinished O"
            self.tmem[f"Oread{i}"] = k
        self.done.add(f"softmax{i}")

    def run(self):
        gens = {"producer": self.producer(), "mma": self.mma_issuer(),
                "softmax0": self.softmax(0), "softmax1": self.softmax(1)}
        live = dict(gens)
        stalls = 0
        while live or self.tma or self.pipe:
            names = list(live) + (["async"] if (self.tma or self.pipe) else [])
            pick = self.rng.choice(names)
            if pick == "async":
                self.step_async()
                stalls = 0
                continue
            try:
                next(live[pick])
            except StopIteration:
                del live[pick]
            stalls += 1
            assert stalls < 100000, f"deadlock: {sorted(live)} waiting, nothing in flight"
        assert self.done == {"producer", "mma", "softmax0", "softmax1"}


@pytest.mark.parametrize("stages", [2, 3, 4, 5, 6, 8])
@pytest.mark.parametrize("U,nkv,G,cta", [(256, 32, 148, 0), (256, 32, 148, 1), (256, 32, 148, 147),
                                         (5, 3, 2, 1), (7, 1, 3, 2), (4, 6, 3, 1), (2, 5, 1, 0),
                                         (40, 4, 9, 3), (41, 3, 8, 7)])
def test_barrier_protocol_under_random_interleavings(stages, U, nkv, G, cta):
    its = items_of(cta, U, nkv, G)
    for seed in range(12):
        Sim(its, stages, random.Random(seed * 7919 + stages)).run()
