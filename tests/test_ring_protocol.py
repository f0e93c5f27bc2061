"""The K/V ring protocol of the one-S-buffer kernel variants, checked on the
CPU by simulation (attnprofile_b200/csrc/attn_kernel.cuh: load_role,
mma_role, AttnConfig::V_RELEASE_WITH_K / K_SLOT_PERIOD / KV_JOINT_FULL).

Ring items in producer order: K_0, then V_j, K_{j+1} for each step j (item
t in slot t mod STAGES).  Releases: K_0's slot by a commit after the first
S; at the end of step j one commit on K_{j+1}'s EMPTY barrier frees both
V_j's and K_{j+1}'s slots.  Before reloading slot t mod STAGES (t >= STAGES)
the producer waits for phase m // K_SLOT_PERIOD of EMPTY[2m mod STAGES] with
m = (t - STAGES + 1) // 2.  The model below replays every schedule shape
that matters -- all ring depths, short and long key ranges -- and checks
that (1) the awaited completion is exactly the one that frees the slot's
previous occupant, (2) that completion cannot be overtaken by a later one
on the same barrier before the producer has waited (no parity aliasing),
(3) no wait depends on a release that needs the awaited item itself
(no deadlock), and (4) with the joint landing every FULL barrier advances
one phase per item, so the MMA warp's parity (t // STAGES) & 1 holds.
"""
import pytest


def k_item(m):
    """Ring item index of K_m (K_0 is item 0, K_{j+1} follows V_j)."""
    return 2 * m


def v_item(j):
    return 2 * j + 1


def releasing_k(u):
    """The K index whose commit frees item u: K_m frees itself, V_j is
    freed with K_{j+1}."""
    return u // 2 if u % 2 == 0 else (u + 1) // 2


def kernel_wait(t, stages):
    """(barrier slot, phase index) that the producer waits on before item t,
    as the kernel computes it."""
    period = stages // 2 if stages % 2 == 0 else stages
    m = (t - stages + 1) // 2
    return (2 * m) % stages, m // period


def commit_phases(n, stages):
    """Phase index of each K_m's commit on its EMPTY barrier: the number of
    earlier K items whose slot is the same."""
    seen, ph = {}, {}
    for m in range(n):
        s = k_item(m) % stages
        ph[m] = seen.get(s, 0)
        seen[s] = ph[m] + 1
    return ph


@pytest.mark.parametrize("stages", range(2, 13))
@pytest.mark.parametrize("n", [1, 2, 3, 5, 32, 257])
def test_slot_reuse_waits_for_the_right_release(stages, n):
    items = [k_item(0)] + [x for j in range(n) for x in
                           ([v_item(j)] + ([k_item(j + 1)] if j + 1 < n else []))]
    assert items == list(range(len(items)))
    ph = commit_phases(n, stages)
    period = stages // 2 if stages % 2 == 0 else stages
    for t in items:
        if t < stages:
            continue
        u = t - stages                  # previous occupant of slot t % stages
        assert u % stages == t % stages
        m = releasing_k(u)
        assert m < n                    # every reused occupant is released
        slot, phase = kernel_wait(t, stages)
        # (1) the kernel's barrier and phase are those of K_m's commit
        assert slot == k_item(m) % stages and phase == ph[m]
        # (2) the next completion on that barrier is K_{m + period}'s commit,
        # which needs that item loaded, i.e. not before the producer passes t
        nxt = m + period
        assert nxt >= n or ph[nxt] == phase + 1
        assert nxt >= n or k_item(nxt) >= t
        # (3) the release comes at the end of step m - 1, whose MMAs need
        # V_{m-1} and K_m (and, with the joint landing, nothing later): all
        # loaded before the producer blocks at item t
        assert k_item(m) < t


@pytest.mark.parametrize("stages", range(2, 13))
@pytest.mark.parametrize("n", [1, 2, 7, 40])
def test_joint_landing_keeps_one_phase_per_item(stages, n):
    """Joint landing: V_j's FULL barrier is armed for both V_j's and
    K_{j+1}'s bytes; K_{j+1}'s own FULL barrier receives a plain arrival.
    Each slot's FULL barrier therefore completes exactly one phase per item
    placed in it, and the MMA warp's wait on V_j (item t) with parity
    (t // stages) & 1 is the completion that follows both loads."""
    completions = {}
    expected = {}   # (slot, phase) -> bytes the phase was armed for (tiles)
    delivered = {}  # (slot, phase) -> bytes that land on it
    waited = []
    items = [("K", 0)] + [x for j in range(n) for x in
                          ([("V", j)] + ([("K", j + 1)] if j + 1 < n else []))]
    for t, (kind, idx) in enumerate(items):
        s = t % stages
        phase = completions.get(s, 0)
        completions[s] = phase + 1
        assert phase == t // stages     # one phase per item in its slot
        if kind == "V":
            joint = idx + 1 < n
            expected[(s, phase)] = 2 if joint else 1
            delivered[(s, phase)] = delivered.get((s, phase), 0) + 1
            waited.append((t, phase & 1))
            last_v = (s, phase)
        elif idx == 0:
            expected[(s, phase)] = 1    # K_0: armed and filled on its own
            delivered[(s, phase)] = 1
        else:
            expected[(s, phase)] = 0    # plain arrival: completes at once
            delivered[last_v] += 1      # the bytes land on V_{idx-1}'s phase
    assert expected == {k: delivered.get(k, 0) for k in expected}
    for t, parity in waited:
        assert parity == (t // stages) & 1


def pair_relay_events(n, stages, k_first):
    """Happens-before graph of the CTA pair's ring under the joint landing.

    The odd CTA loads its halves onto its own FULL barriers; its relay thread
    waits for each and forwards it (a remote arrival) to the even CTA's
    barrier, which also takes the even producer's own arrival.  The even CTA's
    MMA thread waits only for V_j's barrier (joint landing) and issues S(j+1)
    after it; the commit that follows frees the slots of V_j and K_{j+1} in
    both CTAs.  Nodes: ("OA", t) odd producer arms item t, ("OC", t) the odd
    barrier completes t's phase, ("RW", t) relay has seen it, ("RF", t) relay
    forwards it, ("EA", t) even producer arms t, ("MV", j) MMA has seen V_j
    complete (("MK0",) for K_0), ("S", m) MMA issues S(m), ("EC", m) the
    commit after S(m) lands.  k_first: the relay forwards K_{j+1} before V_j
    (the kernel's order) instead of after."""
    items = [("K", 0)] + [x for j in range(n) for x in
                          ([("V", j)] + ([("K", j + 1)] if j + 1 < n else []))]
    edges = {}

    def edge(a, b):
        edges.setdefault(a, set()).add(b)
        edges.setdefault(b, set())

    def release_wait(t):
        return (t - stages + 1) // 2  # the K whose commit frees slot t mod stages

    for t, (kind, idx) in enumerate(items):
        if t > 0:
            edge(("OA", t - 1), ("OA", t))      # producers arm in item order
            edge(("EA", t - 1), ("EA", t))
        if t >= stages:
            edge(("EC", release_wait(t)), ("OA", t))
            edge(("EC", release_wait(t)), ("EA", t))
        joint_v = kind == "V" and idx + 1 < n
        if kind == "K" and idx > 0:
            edge(("OA", t), ("OC", t))          # plain arrival: completes at once
        elif joint_v:
            edge(("OA", t + 1), ("OC", t))      # needs K_{idx+1}'s bytes, loaded after its arrival
        else:
            edge(("OA", t), ("OC", t))
        edge(("OC", t), ("RW", t))
    # relay program order
    order = [("RW", 0), ("RF", 0)]
    for j in range(n):
        tv = 2 * j + 1
        if j + 1 < n:
            if k_first:
                order += [("RW", tv), ("RW", tv + 1), ("RF", tv + 1), ("RF", tv)]
            else:
                order += [("RW", tv), ("RF", tv), ("RW", tv + 1), ("RF", tv + 1)]
        else:
            order += [("RW", tv), ("RF", tv)]
    for a, b in zip(order, order[1:]):
        edge(a, b)
    for t in range(len(items)):
        edge(("RW", t), ("RF", t))
    # MMA: K_0, then per step V_j, S(j+1); commits after each S
    edge(("RF", 0), ("MK0",))
    edge(("EA", 0), ("MK0",))
    edge(("MK0",), ("S", 0))
    edge(("S", 0), ("EC", 0))
    prev = ("S", 0)
    for j in range(n):
        tv = 2 * j + 1
        edge(("RF", tv), ("MV", j))
        edge(("EA", tv + (1 if j + 1 < n else 0)), ("MV", j))
        edge(prev, ("MV", j))
        if j + 1 < n:
            edge(("MV", j), ("S", j + 1))
            edge(("S", j + 1), ("EC", j + 1))
            prev = ("S", j + 1)
        else:
            prev = ("MV", j)
    return items, edges


def reach(edges):
    """Transitive closure (the graph is small) and an acyclicity check."""
    indeg = {v: 0 for v in edges}
    for a in edges:
        for b in edges[a]:
            indeg[b] += 1
    topo, stack = [], [v for v, d in indeg.items() if d == 0]
    while stack:
        v = stack.pop()
        topo.append(v)
        for b in edges[v]:
            indeg[b] -= 1
            if indeg[b] == 0:
                stack.append(b)
    assert len(topo) == len(edges), "cycle: the protocol deadlocks"
    after = {v: set() for v in edges}
    for v in reversed(topo):
        for b in edges[v]:
            after[v] |= {b} | after[b]
    return after


def pair_relay_violations(n, stages, k_first):
    items, edges = pair_relay_events(n, stages, k_first)
    after = reach(edges)
    bad = []
    for t in range(len(items)):
        nxt = t + stages
        if nxt >= len(items):
            continue
        # the relay's parity wait on t cannot be overtaken by the slot's next phase
        if ("OC", nxt) not in after[("RW", t)]:
            bad.append(("relay wait may alias", t))
        # the even barrier's phase for t (its forward) precedes the next arm
        if ("EA", nxt) not in after[("RF", t)]:
            bad.append(("forward may land in the next phase", t))
    return bad


@pytest.mark.parametrize("stages", [4, 6, 10, 12])
@pytest.mark.parametrize("n", [1, 2, 5, 32])
def test_pair_relay_under_joint_landing(stages, n):
    """CTA pair with the joint landing: with K_{j+1} forwarded before V_j the
    protocol is deadlock-free, no relay wait can alias, and every forwarded
    phase completes before the even producer arms the slot again."""
    assert pair_relay_violations(n, stages, k_first=True) == []


@pytest.mark.parametrize("stages", [4, 10])
def test_pair_relay_model_catches_the_other_order(stages):
    """Planted mistake: forwarding V_j before K_{j+1} leaves both orderings
    to timing, and the model says so."""
    bad = pair_relay_violations(8, stages, k_first=False)
    kinds = {b[0] for b in bad}
    assert "relay wait may alias" in kinds and "forward may land in the next phase" in kinds
