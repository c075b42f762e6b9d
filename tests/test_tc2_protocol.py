"""Model check of attn_tc2_kernel's barrier protocol (futon_b200/csrc/
attention_tc2.cuh), on the CPU, for both of its forms: head_dim 32 (a unit
is a head pair and serves both softmax groups) and head_dim 64 (a unit is
one head; units alternate between the groups).

The kernel's four roles — TMA producer, MMA thread, and the two softmax
groups (four warps each) — are restated as coroutines that wait on and
arrive at mbarriers with the hardware's phase-parity semantics, in the same
order and with the same parities as the kernel. TMA copies land and MMAs
complete asynchronously (copies in any order, MMAs in issue order; a commit
arrives once every earlier MMA is done). Random schedules then check that
the protocol never deadlocks and never lets a buffer be used out of turn:
a q·k or v slot is not reloaded before the MMAs that read it are issued and
done, an MMA reads only the unit it expects, S is not overwritten before its
group has read it, P is not rewritten while a P·V reads it, and O is not read
while a P·V writes it. The model must change whenever the kernel's protocol
does.
"""
from __future__ import annotations

import random

import pytest

QK_STAGES, V_STAGES = 3, 2


class Bar:
    def __init__(self, name: str, count: int):
        self.name, self.count, self.arrived, self.phase = name, count, 0, 0

    def arrive(self):
        self.arrived += 1
        assert self.arrived <= self.count, self.name
        if self.arrived == self.count:
            self.arrived, self.phase = 0, self.phase + 1

    def passed(self, parity: int) -> bool:  # mbarrier.try_wait.parity
        return (self.phase & 1) != parity


def simulate(units: int, seed: int, pair: bool) -> None:
    rng = random.Random(seed)
    qkfull = [Bar(f"qkfull{i}", 1) for i in range(QK_STAGES)]
    qkempty = [Bar(f"qkempty{i}", 1) for i in range(QK_STAGES)]
    vfull = [Bar(f"vfull{i}", 1) for i in range(V_STAGES)]
    vempty = [Bar(f"vempty{i}", 1) for i in range(V_STAGES)]
    sfull = [Bar(f"sfull{e}", 1) for e in range(2)]
    sfree = [Bar(f"sfree{e}", 4) for e in range(2)]
    pfull = [Bar(f"pfull{e}", 4) for e in range(2)]
    ofull = [Bar(f"ofull{e}", 1) for e in range(2)]

    copies = []       # (barrier, buffer, unit) in flight
    mma_queue = []    # ("mma", reads, writes) | ("commit", barrier), completed in order
    reads_pending, writes_pending = {}, {}
    content = {}      # buffer -> unit whose data it holds (None while a copy writes it)
    s_state = [None, None]   # None | ("pending", u) | "read"
    p_unit = [None, None]
    s_reads, p_writes = [0, 0], [0, 0]

    def mma(reads, writes):
        for r in reads:
            reads_pending[r] = reads_pending.get(r, 0) + 1
        for w in writes:
            writes_pending[w] = writes_pending.get(w, 0) + 1
        mma_queue.append(("mma", reads, writes))

    def copy(bar, buf, unit):
        assert reads_pending.get(buf, 0) == 0, f"copy into {buf} while an MMA reads it"
        content[buf] = None
        copies.append((bar, buf, unit))

    def producer():
        def issue_qk(u):
            slot = u % QK_STAGES
            if u >= QK_STAGES:
                yield ("wait", qkempty[slot], (u // QK_STAGES - 1) & 1)
            copy(qkfull[slot], f"QK{slot}", u)

        def issue_v(u):
            slot = u & 1
            if u >= 2:
                yield ("wait", vempty[slot], ((u >> 1) - 1) & 1)
            copy(vfull[slot], f"V{slot}", u)

        for u in range(min(2, units)):
            yield from issue_qk(u)
        for u in range(units):
            if u + 2 < units:
                yield from issue_qk(u + 2)
            yield from issue_v(u)

    def mma_thread():
        def issue_s(u, e):
            assert content.get(f"QK{u % QK_STAGES}") == u, ("S reads a stale q·k slot", u)
            assert s_state[e] in (None, "read"), ("S overwritten before its group read it", e, u)
            s_state[e] = ("pending", u)
            mma([f"QK{u % QK_STAGES}"], [f"S{e}"])
            mma_queue.append(("commit", sfull[e]))

        def issue_pv(u, e):
            vs = u & 1
            assert content.get(f"V{vs}") == u, ("P·V reads a stale v slot", u)
            assert p_unit[e] == u, ("P·V reads a stale P", e, u)
            mma([f"P{e}", f"V{vs}"], [f"O{e}"])
            mma_queue.append(("commit", ofull[e]))

        if units == 0:
            return
        if not pair:
            for u in range(min(2, units)):
                yield ("wait", qkfull[u], 0)
                issue_s(u, u & 1)
                mma_queue.append(("commit", qkempty[u]))
            for u in range(units):
                e, i = u & 1, u >> 1
                if u + 2 < units:
                    w = u + 2
                    yield ("wait", qkfull[w % QK_STAGES], (w // QK_STAGES) & 1)
                    yield ("wait", sfree[e], i & 1)
                    issue_s(w, e)
                    mma_queue.append(("commit", qkempty[w % QK_STAGES]))
                yield ("wait", vfull[u & 1], (u >> 1) & 1)
                yield ("wait", pfull[e], i & 1)
                issue_pv(u, e)
                mma_queue.append(("commit", vempty[u & 1]))
            return
        yield ("wait", qkfull[0], 0)
        issue_s(0, 0)
        issue_s(0, 1)
        mma_queue.append(("commit", qkempty[0]))
        for u in range(units):
            if u + 1 < units:
                nu, qs = u + 1, (u + 1) % QK_STAGES
                yield ("wait", qkfull[qs], (nu // QK_STAGES) & 1)
                for e in range(2):
                    yield ("wait", sfree[e], u & 1)
                    issue_s(nu, e)
                mma_queue.append(("commit", qkempty[qs]))
            vs = u & 1
            yield ("wait", vfull[vs], (u >> 1) & 1)
            for e in range(2):
                yield ("wait", pfull[e], u & 1)
                issue_pv(u, e)
            mma_queue.append(("commit", vempty[vs]))

    def group_warp(e):
        mine = list(range(units)) if pair else list(range(e, units, 2))
        for i, u in enumerate(mine):
            yield ("wait", sfull[e], i & 1)
            assert writes_pending.get(f"S{e}", 0) == 0 and s_state[e] == ("pending", u), \
                ("group reads the wrong S", e, u)
            s_reads[e] += 1
            if s_reads[e] == 4:
                s_state[e], s_reads[e] = "read", 0
            yield ("act", sfree[e].arrive)
            if i > 0:
                yield ("wait", ofull[e], (i - 1) & 1)
                assert writes_pending.get(f"O{e}", 0) == 0, "O read while a P·V writes it"
                assert reads_pending.get(f"P{e}", 0) == 0, "P written while a P·V reads it"
            p_writes[e] += 1
            if p_writes[e] == 4:
                p_unit[e], p_writes[e] = u, 0
            yield ("act", pfull[e].arrive)
        if mine:
            yield ("wait", ofull[e], (len(mine) - 1) & 1)
            assert writes_pending.get(f"O{e}", 0) == 0

    roles = [producer(), mma_thread()] + [group_warp(e) for e in range(2) for _ in range(4)]
    blocked = [None] * len(roles)
    alive = [True] * len(roles)
    for _ in range(500000):
        choices = [("role", i) for i in range(len(roles))
                   if alive[i] and (blocked[i] is None or blocked[i][1].passed(blocked[i][2]))]
        if copies:
            choices.append(("copy", None))
        if mma_queue:
            choices.append(("mma", None))
        if not choices:
            stuck = [(i, blocked[i][1].name) for i in range(len(roles)) if alive[i]]
            assert not stuck, f"deadlock: {stuck}"
            return
        kind, i = rng.choice(choices)
        if kind == "copy":
            bar, buf, unit = copies.pop(rng.randrange(len(copies)))
            content[buf] = unit
            bar.arrive()
        elif kind == "mma":
            op = mma_queue.pop(0)
            if op[0] == "mma":
                for r in op[1]:
                    reads_pending[r] -= 1
                for w in op[2]:
                    writes_pending[w] -= 1
            else:
                op[1].arrive()
        else:
            blocked[i] = None
            try:
                while True:
                    step = next(roles[i])
                    if step[0] == "act":
                        step[1]()
                    elif not step[1].passed(step[2]):
                        blocked[i] = step
                        break
            except StopIteration:
                alive[i] = False
    raise AssertionError("schedule did not finish")


@pytest.mark.parametrize("units", [1, 2, 3, 4, 5, 6, 7, 12, 24])
def test_tc2_pair_protocol_random_schedules(units):
    for seed in range(200):
        simulate(units, seed, pair=True)


@pytest.mark.parametrize("units", [2, 4, 6, 8, 12, 24, 48])
def test_tc2_single_head_protocol_random_schedules(units):
    for seed in range(200):
        simulate(units, seed, pair=False)
