"""A randomised model of the barrier protocol of ``attend_persistent_kernel`` (csrc/attend.cu).

The kernel's three roles are restated as Python generators that yield their waits, in the same
order and with the same completion indices as the CUDA code:

* the producer (TMA warp): a ring of two stages (slot pairs); stage G holds V of the CTA's block
  G-1 and K of its block G, blocks counted over all of its items, so an item's first stage (its
  K_0 with the previous item's last V) goes out before the wait for the Q buffers; fill f of a
  buffer waits for completion #(f-1) of its empty barrier (q_empty, kv_empty[stage]);
* the issuer (UMMA warp): S_t(0), then per KV block one wait for stage b0 + j + 1 (V_j, K_{j+1}),
  P.V_t(j) in two chunks and S_t(j+1), with commits on s_full[t] and, after an item's last
  block, on o_full[t];
* 16 softmax warps: exp of S into P (two hand-over chunks), the row-sum exchange over a named
  barrier (double-buffered by item parity) and the epilogue read of O; one warp of the item's
  last query tile releases stage b0 + j (and, at the last block, Q) once it has seen S(j)
  complete, right after its own chunk-0 hand-over.

The 'hardware' runs at random times: TMA copies land, UMMAs execute in issue order, commits
arrive. mbarrier waits use the hardware's parity semantics (a wait for parity p returns once the
current phase's parity differs from p), and every wait checks that this answer is the intended
one, i.e. that the awaited completion has happened and the barrier is not a further phase on.
Every operand read (Q, K and V slots by UMMAs, S and O by the softmax warps, P by P.V, the
partner's row sum) checks the version it must see. Warps react within nanoseconds while copies
and UMMAs take microseconds, so a ready warp mostly runs first.
"""
from __future__ import annotations

import random

import pytest


class ProtocolError(AssertionError):
    pass


class Bar:
    def __init__(self, name: str, count: int = 1):
        self.name, self.count, self.arrived, self.completed = name, count, 0, 0

    def arrive(self):
        self.arrived += 1
        if self.arrived == self.count:
            self.arrived = 0
            self.completed += 1


def schedule(n_tiles, n_splits, bh):
    """(n_full, n_a, s_a, s_b) of AttendSchedule (attend_schedule.cuh) from a KV split count (every
    item split that many ways) or such a tuple (whole items first, then two tiers of pieces)."""
    n_items = bh * ((n_tiles + 1) // 2)
    if isinstance(n_splits, tuple):
        return n_splits
    return (n_items, 0, 1, 1) if n_splits == 1 else (0, n_items, n_splits, n_splits)


def decode(w, n_tiles, sched):
    """decode_item (attend.cu): work unit -> (query tiles, KV range)."""
    n_full, n_a, s_a, s_b = sched
    n_pairs = (n_tiles + 1) // 2
    if w < n_full:
        item, split, splits = w, 0, 1
    elif w - n_full < n_a * s_a:
        item, split, splits = n_full + (w - n_full) // s_a, (w - n_full) % s_a, s_a
    else:
        u = w - n_full - n_a * s_a
        item, split, splits = n_full + n_a + u // s_b, u % s_b, s_b
    t0 = (item % n_pairs) * 2
    kv0 = n_tiles * split // splits
    return dict(w=w, nt=min(2, n_tiles - t0), n_kv=n_tiles * (split + 1) // splits - kv0)


def run_cta(n_tiles, n_splits, bh, grid, cta, rng, p_hw=0.05, release_from_tile0=False):
    sched = schedule(n_tiles, n_splits, bh)
    n_full, n_a, s_a, s_b = sched
    n_units = n_full + n_a * s_a + (bh * ((n_tiles + 1) // 2) - n_full - n_a) * s_b
    items = [decode(w, n_tiles, sched) for w in range(cta, n_units, grid)]
    q_full = Bar("q_full")
    kv_full = [Bar(f"kv_full{s}") for s in range(2)]
    s_full = [Bar(f"s_full{t}") for t in range(2)]
    p_part = [[Bar(f"p_part{t}{c}", 8) for c in range(2)] for t in range(2)]
    o_full = [Bar(f"o_full{t}") for t in range(2)]
    kv_empty = [Bar(f"kv_empty{s}") for s in range(2)]
    q_empty = Bar("q_empty")
    qbuf, q_inflight = [None, None], [False, False]
    kv, kv_inflight = [None] * 4, [False] * 4
    s_reg = [[[None] * 2 for _ in range(4)] for _ in range(2)]  # [tile][quad][half]
    p_reg = [[[[None, None] for _ in range(2)] for _ in range(4)] for _ in range(2)]  # [tile][quad][half][chunk]
    o_reg = [None, None]
    l_part = [[[[None] * 4 for _ in range(2)] for _ in range(2)] for _ in range(2)]  # [parity][tile][half][quad]
    tma, mma = [], []
    named = [[0, 0], [0, 0]]  # per tile: arrivals, generation

    def answer(b, k):
        done = (b.completed & 1) != (k & 1)
        if done and b.completed != k + 1:
            raise ProtocolError(f"wait for {b.name} #{k} returned with {b.completed} completions")
        if not done and b.completed >= k + 2:
            raise ProtocolError(f"wait for {b.name} #{k} missed: {b.completed} completions")
        return done

    def producer():
        stage = [0]
        q_fills = 0

        def issue(v, k):  # stage G: v into slot 2 (G % 2), k into slot 2 (G % 2) + 1
            sp, use = stage[0] % 2, stage[0] // 2
            if use > 0:
                yield ("wait", kv_empty[sp], use - 1)
            for slot, tile in ((2 * sp, v), (2 * sp + 1, k)):
                if tile is not None:
                    if kv_inflight[slot]:
                        raise ProtocolError("slot refilled while a copy into it is in flight")
                    kv_inflight[slot] = True
            tma.append(("kv", sp, v, k))
            stage[0] += 1

        pending_v = None  # the previous item's last V, loaded with this item's first K
        for it in items:
            yield from issue(pending_v, ("K", it["w"], 0))
            if q_fills > 0:
                yield ("wait", q_empty, q_fills - 1)
            if any(q_inflight):
                raise ProtocolError("Q refilled while a copy into it is in flight")
            for t in range(it["nt"]):
                q_inflight[t] = True
            tma.append(("q", it["w"], it["nt"]))
            q_fills += 1
            for j in range(it["n_kv"] - 1):
                yield from issue(("V", it["w"], j), ("K", it["w"], j + 1))
            pending_v = ("V", it["w"], it["n_kv"] - 1)
        if pending_v is not None:
            yield from issue(pending_v, None)

    def issuer():
        b0, done, blocks = 0, 0, [0, 0]
        for it in items:
            yield ("wait", q_full, done)
            if b0 == 0:  # later items' first stage was waited for with the previous item's last V
                yield ("wait", kv_full[0], 0)
            for t in range(it["nt"]):
                mma.append(("S", it["w"], t, 0, 2 * (b0 % 2) + 1))
                mma.append(("commit", s_full[t]))
            n_kv = it["n_kv"]
            for j in range(n_kv):
                st = b0 + j + 1
                last = j == n_kv - 1
                yield ("wait", kv_full[st % 2], st // 2)
                for t in range(it["nt"]):
                    for c in range(2):
                        yield ("wait", p_part[t][c], blocks[t] + j)
                        mma.append(("PV", it["w"], t, j, c, 2 * (st % 2)))
                    if last:
                        mma.append(("commit", o_full[t]))
                    else:
                        mma.append(("S", it["w"], t, j + 1, 2 * (st % 2) + 1))
                        mma.append(("commit", s_full[t]))
            for t in range(it["nt"]):
                blocks[t] += n_kv
            b0 += n_kv
            done += 1

    def softmax(t, quad, half):
        s_seen = o_seen = n_done = b0 = 0
        for it in items:
            item_b0 = b0
            b0 += it["n_kv"]
            if t >= it["nt"]:
                continue
            n_kv = it["n_kv"]
            # planted mistake: releases made by tile 0's warp, whose commit does not cover tile 1
            releaser = t == (0 if release_from_tile0 else it["nt"] - 1) and quad == 2 and half == 0
            for j in range(n_kv):
                yield ("wait", s_full[t], s_seen)
                s_seen += 1
                if s_reg[t][quad][half] != ("S", it["w"], t, j):
                    raise ProtocolError(f"softmax read S {s_reg[t][quad][half]}, wanted {('S', it['w'], t, j)}")
                for c in range(2):
                    yield ("step",)
                    p_reg[t][quad][half][c] = ("P", it["w"], t, j)
                    p_part[t][c].arrive()
                    if c == 0 and releaser:  # after its own chunk-0 hand-over, as the kernel does
                        kv_empty[(item_b0 + j) % 2].arrive()  # stage b0 + j: V_{j-1} (or the last V before) and K_j
                        if j == n_kv - 1:
                            q_empty.arrive()
            lb = n_done & 1
            l_part[lb][t][half][quad] = it["w"]
            gen = named[t][1]
            named[t][0] += 1
            if named[t][0] == 8:
                named[t] = [0, gen + 1]
            yield ("named", t, gen)
            if l_part[lb][t][1 - half][quad] != it["w"]:
                raise ProtocolError("partner's row sum overwritten before it was read")
            yield ("wait", o_full[t], o_seen)
            o_seen += 1
            n_done += 1
            yield ("step",)
            if o_reg[t] != (it["w"], 2 * n_kv - 1):
                raise ProtocolError(f"epilogue read O {o_reg[t]}, wanted {(it['w'], 2 * n_kv - 1)}")

    def execute_mma():
        e = mma.pop(0)
        if e[0] == "commit":
            e[1].arrive()
        elif e[0] == "S":
            _, w, t, j, slot = e
            if qbuf[t] != w or q_inflight[t]:
                raise ProtocolError(f"S read Q {qbuf[t]} (copy in flight: {q_inflight[t]}), wanted {w}")
            if kv[slot] != ("K", w, j) or kv_inflight[slot]:
                raise ProtocolError(f"S read K {kv[slot]} (copy in flight: {kv_inflight[slot]}), wanted {('K', w, j)}")
            for quad in range(4):
                for half in range(2):
                    s_reg[t][quad][half] = ("S", w, t, j)
                    p_reg[t][quad][half] = [None, None]
        else:
            _, w, t, j, c, slot = e
            if kv[slot] != ("V", w, j) or kv_inflight[slot]:
                raise ProtocolError(f"P.V read V {kv[slot]} (copy in flight: {kv_inflight[slot]}), wanted {('V', w, j)}")
            for quad in range(4):
                for half in range(2):
                    if p_reg[t][quad][half][c] != ("P", w, t, j):
                        raise ProtocolError(f"P.V read P {p_reg[t][quad][half][c]}, wanted {('P', w, t, j)}")
            step = 2 * j + c
            if step > 0 and o_reg[t] != (w, step - 1):
                raise ProtocolError(f"P.V accumulated onto O {o_reg[t]}, wanted {(w, step - 1)}")
            o_reg[t] = (w, step)

    def land_copy(k):
        e = tma.pop(k)
        if e[0] == "q":
            for t in range(e[2]):
                qbuf[t], q_inflight[t] = e[1], False
            q_full.arrive()
        else:
            _, sp, v, k = e
            for slot, tile in ((2 * sp, v), (2 * sp + 1, k)):
                if tile is not None:
                    kv[slot], kv_inflight[slot] = tile, False
            kv_full[sp].arrive()

    agents = [producer(), issuer()] + [softmax(t, q, h) for t in range(2) for q in range(4) for h in range(2)]
    req = [None] * len(agents)

    def advance(i):
        req[i] = next(agents[i], None)

    for i in range(len(agents)):
        advance(i)

    def ready(i):
        r = req[i]
        if r is None:
            return False
        if r[0] == "step":
            return True
        if r[0] == "wait":
            return answer(r[1], r[2])
        return named[r[1]][1] > r[2]

    for _ in range(1_000_000):
        warps = [i for i in range(len(agents)) if ready(i)]
        if warps and rng.random() > p_hw:
            advance(rng.choice(warps))
            continue
        hw = [("copy", k) for k in range(len(tma))] + ([("mma", 0)] if mma else [])
        acts = [("warp", i) for i in warps] + hw
        if not acts:
            if all(r is None for r in req):
                assert not tma and not mma
                return len(items)
            raise ProtocolError("deadlock: " + ", ".join(f"{i}: {r}" for i, r in enumerate(req) if r is not None))
        kind, i = rng.choice(acts)
        if kind == "warp":
            advance(i)
        elif kind == "copy":
            land_copy(i)
        else:
            execute_mma()
    raise ProtocolError("no progress")


# (tile count, KV splits, batch x heads, grid): even and odd tile counts (items of one and two
# query tiles mixed), with and without KV splits, one or several items per CTA, single-block items,
# and tiered schedules (n_full, n_a, s_a, s_b): whole items, then pieces of two sizes, so one CTA
# walks items of different lengths.
CASES = [(2, 1, 2, 1), (3, 1, 2, 1), (4, 1, 3, 2), (5, 1, 3, 2), (6, 4, 1, 1), (7, 2, 3, 2), (8, 3, 3, 2),
         (2, 2, 3, 1), (3, 3, 2, 1), (1, 1, 5, 2), (4, 4, 3, 2), (6, 6, 2, 3), (9, 1, 2, 1), (10, 1, 2, 1),
         (6, (3, 2, 2, 3), 2, 3), (7, (2, 1, 3, 5), 2, 2), (8, (4, 1, 2, 2), 3, 4), (5, (3, 2, 2, 5), 2, 3)]


@pytest.mark.parametrize("case", CASES)
def test_protocol_holds(case):
    n_tiles, n_splits, bh, grid = case
    rng = random.Random(hash(case) & 0xFFFF)
    for cta in range(grid):
        for _ in range(6):
            for p_hw in (0.02, 0.3):
                assert run_cta(n_tiles, n_splits, bh, grid, cta, rng, p_hw) > 0


def test_model_catches_an_early_release():
    """Planted in the model: buffers released by a warp of tile 0, whose s_full commit does not
    cover tile 1's UMMAs, so a refill can land before tile 1 has read the old tile."""
    rng = random.Random(7)
    with pytest.raises(ProtocolError, match="read"):
        for _ in range(200):
            run_cta(4, 1, 3, 1, 0, rng, 0.5, release_from_tile0=True)


@pytest.mark.parametrize("case", [(4, 1, 3, 1), (5, 2, 2, 1)])
def test_waits_never_fall_behind_under_any_schedule(case):
    """Fully random scheduling (a copy or UMMA as likely as a ready warp): the empty barriers
    make every parity wait unambiguous however late a warp runs."""
    n_tiles, n_splits, bh, grid = case
    rng = random.Random(11)
    for _ in range(40):
        run_cta(n_tiles, n_splits, bh, grid, 0, rng, 1.0)
