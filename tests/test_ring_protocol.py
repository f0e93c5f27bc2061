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
