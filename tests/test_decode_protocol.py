"""CPU model of the decode kernel's barrier protocol (csrc/decode_sm100.cu, decode_split_kernel).

One producer thread fills a ring of kStages shared-memory stages (query row, K
and V rows of one 256-key chunk) with bulk copies; 16 consumer warps each score
16 keys of the stage, release the stage (empty) and write their partial row into
the stage's merge slot (merged); a merge warp folds the 16 partials and releases
the merge slot (merge_free).  The last use of a stage is an end marker (n = -1)
published without data.

This model runs the producer, every consumer warp as its own actor and the merge
warp through U stage uses under random interleavings (copies land at random
times) and checks that each parity wait, whenever polled, finds its barrier at
the awaited phase or one past it; that no stage, merge slot or item record is
overwritten while still read, or read before written; and that all roles finish.
"""

from __future__ import annotations

import random

import pytest

K_STAGES = 3
CONSUMERS = 16


class ProtocolError(AssertionError):
    pass


def simulate(uses: int, seed: int, omit: frozenset = frozenset()) -> None:
    rnd = random.Random(seed)
    arrivals: dict[str, int] = {}
    need = {"empty": CONSUMERS, "merged": CONSUMERS, "merge_free": 1}
    full_done: dict[int, int] = {}  # stage -> completed phases of full[]
    read_done = {u: 0 for u in range(uses + 1)}      # consumers done reading stage data
    part_written = {u: 0 for u in range(uses + 1)}   # consumers' merge partials written
    merged_read: set[int] = set()                    # uses whose partials were folded
    item_read = {u: 0 for u in range(uses + 1)}      # consumers that read item[] of use u
    landed: set[int] = set()

    def phases(bar: str) -> int:
        kind, st = bar.rsplit("_", 1)
        if kind == "full":
            return full_done.get(int(st), 0)
        return arrivals.get(bar, 0) // need[kind]

    def producer():
        for u in range(uses + 1):  # the last use is the end marker
            st = u % K_STAGES
            if u >= K_STAGES and "empty" not in omit:
                yield ("wait", f"empty_{st}", u // K_STAGES - 1)
            if u >= K_STAGES:
                yield ("check", ("stage_free", u - K_STAGES))
            yield ("do", ("item_written", u))
            if u < uses:
                yield ("copy", st, u)
            else:
                yield ("full_arrive", st)

    def consumer(w: int):
        for u in range(uses + 1):
            st = u % K_STAGES
            yield ("wait", f"full_{st}", u // K_STAGES)
            if u >= K_STAGES and "merge_free" not in omit:
                yield ("wait", f"merge_free_{st}", u // K_STAGES - 1)
            yield ("do", ("item_read", u))
            if u == uses:
                yield ("arrive", f"merged_{st}")
                return
            yield ("check", ("landed", u))
            yield ("do", ("read_done", u))
            yield ("arrive", f"empty_{st}")
            yield ("check", ("merge_slot_free", u - K_STAGES))
            yield ("do", ("part_written", u))
            yield ("arrive", f"merged_{st}")

    def merge():
        for u in range(uses + 1):
            st = u % K_STAGES
            yield ("wait", f"merged_{st}", u // K_STAGES)
            if u == uses:
                return
            yield ("check", ("parts_complete", u))
            yield ("do", ("merged_read", u))
            yield ("arrive", f"merge_free_{st}")

    roles = {"prod": producer(), "merge": merge()}
    roles.update({f"c{w}": consumer(w) for w in range(CONSUMERS)})
    cur = {r: next(g, None) for r, g in roles.items()}
    copies: list[tuple[int, int]] = []
    written_item = [-1] * K_STAGES  # use whose record item[st] holds

    def check(what) -> None:
        kind, u = what
        if kind == "stage_free" and read_done[u] < CONSUMERS:
            raise ProtocolError(f"stage of use {u} refilled while consumers still read it")
        if kind == "stage_free" and item_read[u] < CONSUMERS:
            raise ProtocolError(f"item record of use {u} overwritten before all consumers read it")
        if kind == "landed" and u not in landed:
            raise ProtocolError(f"use {u} read before its copies landed")
        if kind == "merge_slot_free" and u >= 0 and u not in merged_read:
            raise ProtocolError(f"merge slot of use {u} overwritten before it was merged")
        if kind == "parts_complete" and part_written[u] < CONSUMERS:
            raise ProtocolError(f"use {u} merged before every consumer wrote its partial")

    for _ in range(10 ** 6):
        runnable = []
        for r, op in cur.items():
            if op is None:
                continue
            if op[0] == "wait":
                have, want = phases(op[1]), op[2]
                if have not in (want, want + 1):
                    raise ProtocolError(f"{r}: parity wait on {op[1]} for phase {want} "
                                        f"while {have} phases have completed")
                if have == want + 1:
                    runnable.append(r)
            else:
                runnable.append(r)
        if copies:
            runnable.append("dma")
        if not runnable:
            if all(op is None for op in cur.values()):
                return
            raise ProtocolError(f"deadlock: {cur}")
        r = rnd.choice(runnable)
        if r == "dma":
            st, u = copies.pop(rnd.randrange(len(copies)))
            landed.add(u)
            full_done[st] = full_done.get(st, 0) + 1
            continue
        op = cur[r]
        if op[0] == "copy":
            copies.append((op[1], op[2]))
        elif op[0] == "full_arrive":
            full_done[op[1]] = full_done.get(op[1], 0) + 1
        elif op[0] == "arrive":
            arrivals[op[1]] = arrivals.get(op[1], 0) + 1
        elif op[0] == "check":
            check(op[1])
        elif op[0] == "do":
            key, u = op[1]
            if key == "item_written":
                written_item[u % K_STAGES] = u
            elif key == "item_read":
                if written_item[u % K_STAGES] != u:
                    raise ProtocolError(f"{r} read the item record of use "
                                        f"{written_item[u % K_STAGES]} for use {u}")
                item_read[u] += 1
            elif key == "read_done":
                read_done[u] += 1
            elif key == "part_written":
                part_written[u] += 1
            elif key == "merged_read":
                merged_read.add(u)
        cur[r] = next(roles[r], None)
    raise ProtocolError("no progress")


@pytest.mark.parametrize("uses", [0, 1, 2, 3, 4, 7, 12])
def test_decode_split_kernel_protocol(uses):
    for seed in range(25):
        simulate(uses, seed)


@pytest.mark.parametrize("wait", ["empty", "merge_free"])
def test_model_catches_each_missing_wait(wait):
    caught = 0
    for seed in range(30):
        try:
            simulate(9, seed, omit=frozenset({wait}))
        except ProtocolError:
            caught += 1
    assert caught > 0, wait
