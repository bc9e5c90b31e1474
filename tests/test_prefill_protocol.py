"""CPU model of the two-tile prefill kernel's barrier protocol (csrc/attn_bf16_2q_sm100.cu).

The kernel's roles (K and V TMA producers, the QK^T and P.V MMA issuers, the
softmax of tiles A and B) synchronise through mbarriers waited on by phase
parity.  A parity wait is only meaningful while the barrier is at the awaited
phase or one past it; two phases off in either direction it returns at the
wrong time.  This model runs every role's sequence of waits and signals for
the items one CTA walks (the kernel's own item order, grouped order included)
under random interleavings, with TMA loads landing in random order and MMA
commits completing in issue order per issuing thread, and checks:

* every parity wait, each time it is polled, finds its barrier at the awaited
  phase or one past it;
* no buffer is overwritten while it is still read (K/V ring stages, Q slots,
  S, P and O of each tile, the output staging slab that a TMA store reads
  asynchronously) and none is read before it is written;
* every role finishes (no deadlock).

Each softmax tile is one actor here (its 128 threads arrive together); the
kernel's barriers count all 128 arrivals, so a fast warp can only wait on a
phase its slower warps have already made possible.
"""

from __future__ import annotations

import random

import pytest

K_STAGES = 3
BM = 128  # rows per query tile; keys per K/V tile


def item_indices(n_items: int, blocks: int, cta: int, interleave: bool = False) -> list[int]:
    """Indices (in the heaviest-first order) of the items CTA `cta` takes, in its order: round
    k's item of this CTA, snake-wise; with `interleave` (the kernel's gather modes) the full
    rounds alternate between the heavy and the light end, a partial last round last."""
    full = n_items // blocks
    out = []
    k = 0
    while True:
        r = k
        if interleave and r < full:
            r = full - 1 - (r >> 1) if (r & 1) else (r >> 1)
        idx = r * blocks + ((blocks - 1 - cta) if (k & 1) else cta)
        if idx >= n_items:
            return out
        out.append(idx)
        k += 1


def item_order(sq: int, sk: int, bh: int, grid: int, cta: int, causal: bool,
               interleave: bool = False) -> list[list[int]]:
    """nkv = [key tiles of tile A, of tile B] for each item of CTA `cta`, in its order."""
    n_pairs = (sq + 2 * BM - 1) // (2 * BM)
    n_items = n_pairs * bh
    blocks = min(n_items, grid)
    group = 8 if (n_pairs >= 16 and n_items >= 32 * blocks) else 1
    off = sk - sq
    out = []
    for idx in item_indices(n_items, blocks, cta, interleave):
        n_full = n_pairs // group
        if idx < n_full * group * bh:
            g, r = divmod(idx, group * bh)
            blk = g * group + r % group
        else:
            gl = n_pairs - n_full * group
            r = idx - n_full * group * bh
            blk = n_full * group + r % gl
        q0 = (n_pairs - 1 - blk) * 2 * BM
        nkv = []
        for t in range(2):
            r0 = q0 + t * BM
            rows = min(BM, sq - r0) if r0 < sq else 0
            kend = min(sk, r0 + rows + off) if (causal and rows > 0) else sk
            nkv.append((kend + BM - 1) // BM if rows > 0 else 0)
        out.append(nkv)
    return out


@pytest.mark.parametrize("n_items,blocks", [(384, 148), (3072, 148), (148, 148), (100, 148),
                                            (1000, 148), (296, 148), (3, 1)])
@pytest.mark.parametrize("interleave", [False, True])
def test_item_order_covers_every_item_once(n_items, blocks, interleave):
    seen = sorted(i for c in range(blocks) for i in item_indices(n_items, blocks, c, interleave))
    assert seen == list(range(n_items))


def test_interleaved_rounds_alternate_heavy_and_light():
    # 5 full rounds of 148 and a partial one of 20: 0, 4, 1, 3, 2, then the partial round 5,
    # whose items go (snake order, reversed in odd rounds) to the last 20 CTAs
    rounds = [[i // 148 for i in item_indices(5 * 148 + 20, 148, c, interleave=True)]
              for c in (0, 147)]
    assert rounds == [[0, 4, 1, 3, 2], [0, 4, 1, 3, 2, 5]]


class ProtocolError(AssertionError):
    pass


WAITS = ("q_empty", "k_empty", "v_empty", "s_free", "o_free", "o_done_before_p", "slab_read")


def simulate(items: list[list[int]], seed: int, omit: frozenset = frozenset()) -> None:
    """Runs one interleaving; `omit` drops named waits (to show the checks catch it)."""
    rnd = random.Random(seed)
    count: dict[str, int] = {}
    state = {"s_read": [0, 0], "p_written": [0, 0], "o_read_items": [0, 0]}
    done = {"qk": set(), "pv": set(), "load": set()}

    def c(name: str) -> int:
        return count.get(name, 0)

    def k_producer():
        issued = 0
        for k, nkv in enumerate(items):
            slot = k & 1
            if k >= 2:
                if "q_empty" not in omit:
                    yield ("wait", f"q_empty{slot}", (k >> 1) - 1)
                # every QK^T of item k-2 (the slot's readers) has completed
                yield ("check", ("q_slot_free", k - 2))
            yield ("load", f"q_full{slot}", ("q", k))
            for _ in range(max(nkv)):
                st = issued % K_STAGES
                if issued >= K_STAGES:
                    if "k_empty" not in omit:
                        yield ("wait", f"k_empty{st}", issued // K_STAGES - 1)
                    yield ("check", ("k_stage_free", issued - K_STAGES))
                yield ("load", f"k_full{st}", ("k", issued))
                issued += 1

    def v_producer():
        issued = 0
        for nkv in items:
            for _ in range(max(nkv)):
                st = issued % K_STAGES
                if issued >= K_STAGES:
                    if "v_empty" not in omit:
                        yield ("wait", f"v_empty{st}", issued // K_STAGES - 1)
                    yield ("check", ("v_stage_free", issued - K_STAGES))
                yield ("load", f"v_full{st}", ("v", issued))
                issued += 1

    def qk_issuer():
        ring, n = 0, [0, 0]
        for k, nkv in enumerate(items):
            slot = k & 1
            yield ("wait", f"q_full{slot}", k >> 1)
            yield ("check", ("loaded", ("q", k)))
            for j in range(max(nkv)):
                st = ring % K_STAGES
                yield ("wait", f"k_full{st}", ring // K_STAGES)
                yield ("check", ("loaded", ("k", ring)))
                for t in range(2):
                    if j >= nkv[t]:
                        continue
                    if n[t] > 0 and "s_free" not in omit:
                        yield ("wait", f"s_free{t}", n[t] - 1)
                    yield ("check", ("s_free_read", t, n[t]))
                    yield ("mma", "qk", ("qk", t, n[t], k, ring))
                    yield ("commit", "qk", f"s_full{t}")
                    n[t] += 1
                yield ("commit", "qk", f"k_empty{st}")
                ring += 1
            yield ("commit", "qk", f"q_empty{slot}")

    def pv_issuer():
        ring, n, nit = 0, [0, 0], [0, 0]
        for nkv in items:
            for j in range(max(nkv)):
                st = ring % K_STAGES
                yield ("wait", f"v_full{st}", ring // K_STAGES)
                yield ("check", ("loaded", ("v", ring)))
                for t in range(2):
                    if j >= nkv[t]:
                        continue
                    if j == 0 and nit[t] > 0:
                        if "o_free" not in omit:
                            yield ("wait", f"o_free{t}", nit[t] - 1)
                        yield ("check", ("o_read", t, nit[t]))
                    yield ("wait", f"p_full{t}", n[t])
                    yield ("check", ("p_written", t, n[t]))
                    yield ("mma", "pv", ("pv", t, n[t], ring))
                    yield ("commit", "pv", f"o_done{t}")
                    n[t] += 1
                yield ("commit", "pv", f"v_empty{st}")
                ring += 1
            for t in range(2):
                nit[t] += nkv[t] > 0

    def softmax(t: int):
        ns = 0
        for nkv in items:
            n = nkv[t]
            if n == 0:
                continue
            for j in range(n):
                yield ("wait", f"s_full{t}", ns)
                yield ("check", ("s_written", t, ns))
                yield ("do", ("s_read", t))
                yield ("arrive", f"s_free{t}")
                if ns > 0 and "o_done_before_p" not in omit:
                    yield ("wait", f"o_done{t}", ns - 1)
                yield ("check", ("pv_done", t, ns))  # P may be overwritten, O rescaled
                yield ("do", ("p_written", t))
                yield ("arrive", f"p_full{t}")
                ns += 1
            yield ("wait", f"o_done{t}", ns - 1)
            yield ("check", ("pv_done", t, ns))
            yield ("do", ("o_read", t))
            # the output staging slab: the previous item's TMA store must have
            # read it (bulk wait_group.read) before it is written again
            if "slab_read" not in omit:
                yield ("slab_wait", t)
            yield ("check", ("slab_free", t))
            yield ("store", t)
            yield ("arrive", f"o_free{t}")

    roles = {"kp": k_producer(), "vp": v_producer(), "qk": qk_issuer(), "pv": pv_issuer(),
             "sA": softmax(0), "sB": softmax(1)}
    cur = {r: next(g, None) for r, g in roles.items()}
    pipes: dict[str, list] = {"qk": [], "pv": []}
    loads: list = []
    stores: list = []  # tiles whose slab an output TMA store is still reading

    def check(what) -> None:
        kind = what[0]
        if kind == "loaded":
            if what[1] not in done["load"]:
                raise ProtocolError(f"{what[1]} read before its TMA load landed")
        elif kind == "q_slot_free":
            _, k = what
            pend = [x for x in pipes["qk"] if x[0] == "mma" and x[1][3] == k]
            if pend:
                raise ProtocolError(f"Q slot of item {k} reloaded while its QK^T is pending")
        elif kind in ("k_stage_free", "v_stage_free"):
            _, r = what
            pipe = pipes["qk" if kind == "k_stage_free" else "pv"]
            if any(x[0] == "mma" and x[1][-1] == r for x in pipe):
                raise ProtocolError(f"{kind}: ring tile {r} reloaded while an MMA reads it")
        elif kind == "s_free_read":
            _, t, n = what
            if state["s_read"][t] < n:
                raise ProtocolError(f"S of tile {t} overwritten before softmax read S({n - 1})")
        elif kind == "s_written":
            _, t, n = what
            if ("qk", t, n) not in done["qk"]:
                raise ProtocolError(f"S({n}) of tile {t} read before its QK^T completed")
        elif kind == "p_written":
            _, t, n = what
            if state["p_written"][t] < n + 1:
                raise ProtocolError(f"P.V({n}) of tile {t} issued before P({n}) was written")
        elif kind == "pv_done":
            _, t, n = what
            if any(("pv", t, i) not in done["pv"] for i in range(max(0, n - 2), n)):
                raise ProtocolError(f"tile {t}: P/O touched at step {n} with a P.V pending")
        elif kind == "slab_free":
            if what[1] in stores:
                raise ProtocolError(f"tile {what[1]}'s staging slab rewritten while a store reads it")
        elif kind == "o_read":
            _, t, items_done = what
            if state["o_read_items"][t] < items_done:
                raise ProtocolError(f"O of tile {t} overwritten before its previous item was read")

    for _ in range(10 ** 6):
        runnable = []
        for r, op in cur.items():
            if op is None:
                continue
            if op[0] == "slab_wait":
                if op[1] not in stores:
                    runnable.append(r)
                continue
            if op[0] == "wait":
                have, want = c(op[1]), op[2]
                if have not in (want, want + 1):
                    raise ProtocolError(f"{r}: parity wait on {op[1]} for phase {want} "
                                        f"while {have} phases have completed")
                if have == want + 1:
                    runnable.append(r)
            else:
                runnable.append(r)
        runnable += [f"pipe_{p}" for p, q in pipes.items() if q]
        if loads:
            runnable.append("tma")
        # odd seeds: a store finishes reading its slab only when nothing else can move
        if stores and (not (seed & 1) or not runnable):
            runnable.append("store_read")
        if not runnable:
            if all(op is None for op in cur.values()):
                return
            raise ProtocolError(f"deadlock: {cur}")
        r = rnd.choice(runnable)
        if r == "store_read":
            stores.pop(rnd.randrange(len(stores)))
            continue
        if r == "tma":
            bar, tag = loads.pop(rnd.randrange(len(loads)))
            count[bar] = c(bar) + 1
            done["load"].add(tag)
            continue
        if r.startswith("pipe_"):
            kind, x = pipes[r[5:]].pop(0)
            if kind == "mma":
                done[x[0]].add(x[:3])
            else:
                count[x] = c(x) + 1
            continue
        op = cur[r]
        if op[0] == "load":
            loads.append((op[1], op[2]))
        elif op[0] == "mma":
            pipes[op[1]].append(("mma", op[2]))
        elif op[0] == "commit":
            pipes[op[1]].append(("commit", op[2]))
        elif op[0] == "arrive":  # the arrival of the last of the role's threads
            count[op[1]] = c(op[1]) + 1
        elif op[0] == "store":
            stores.append(op[1])
        elif op[0] == "check":
            check(op[1])
        elif op[0] == "do":
            key, t = op[1]
            if key == "o_read":
                state["o_read_items"][t] += 1
            else:
                state[key][t] += 1
        cur[r] = next(roles[r], None)
    raise ProtocolError("no progress")


# (Sq, Sk, batch*heads, causal): the GPU tests' shapes and the bench workloads
CASES = [
    (1, 1, 160, True), (100, 100, 160, True), (129, 129, 160, True), (300, 300, 160, True),
    (1000, 1000, 160, True), (777, 777, 15, True), (1024, 1024, 96, True),
    (4500, 4500, 272, True), (8192, 8192, 768, True), (300, 700, 160, False),
    (129, 1000, 6, False), (4096, 4096, 128, True),
]


@pytest.mark.parametrize("interleave", [False, True])
@pytest.mark.parametrize("sq,sk,bh,causal", CASES)
def test_two_tile_kernel_protocol(sq, sk, bh, causal, interleave):
    grid = min(148, ((sq + 255) // 256) * bh)
    for cta in sorted({0, 1, grid // 2, grid - 1}):
        items = item_order(sq, sk, bh, grid, cta, causal, interleave)[:10]
        for seed in range(12):
            simulate(items, seed)


@pytest.mark.parametrize("wait", WAITS)
def test_model_catches_each_missing_wait(wait):
    """Dropping any one of the protocol's waits is caught (a hazard, an off-phase wait or a
    deadlock) in some interleaving: the checks above are not vacuous."""
    items = item_order(300, 300, 160, 148, 0, True) + item_order(1000, 1000, 160, 148, 3, True)
    caught = 0
    for seed in range(40):
        try:
            simulate(items, seed, omit=frozenset({wait}))
        except ProtocolError:
            caught += 1
    assert caught > 0, wait
