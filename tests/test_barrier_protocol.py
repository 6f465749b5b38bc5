"""The producer / compute-warp protocol of the persistent kernels, as a model.

`k_fused_step` (csrc/fh_fused.cuh) and `k_stage2_inv` (csrc/fh_batched.cuh)
run 16 compute warps (512 threads) and one producer/reducer warp (32) that
meet on hardware named barriers, which cannot time out. This test replays the
exact sequence of `bar.arrive` / `bar.sync` / mbarrier operations each side
issues, under the hardware rules (an instance of barrier id X completes when
544 thread arrivals have been counted; `bar.sync` blocks until the instance
it joined completes; `bar.arrive` never blocks; an mbarrier chunk is waited
on only after the producer issued its copy), for every chunk count and ring
depth the kernels can meet, and checks that both sides always finish and
leave no barrier instance half-counted.

Stage 1 of `k_fused_step`: compute warps arrive on barrier 1 after each full
round of slots (except the last); the producer waits there before refilling.
Stage 2 (both kernels): per chunk, compute warps arrive on barrier 1 + slot
after consuming it, and at a tile's last chunk, for tiles >= 2, first wait on
barrier 5 + (tile & 1) until the producer has reduced tile - 2 from that
partial buffer; the producer waits on the slot barrier, refills the slot,
reduces the tile and arrives on its partial barrier; an end-of-work chunk
makes both sides leave without touching a barrier; compute warps finally wait
on the partial barriers of the last two tiles.
"""

from __future__ import annotations

import itertools

import pytest

BLOCK = 544
COMPUTE, PRODUCER = 512, 32


class _Bar:
    def __init__(self):
        self.count = 0
        self.gen = 0


def _run(programs):
    """Interleave the agents until all finish; raise on deadlock or miscount."""
    bars: dict[int, _Bar] = {}
    ready = set()
    pcs = [0] * len(programs)
    waiting = [None] * len(programs)
    while True:
        progressed = False
        for i, prog in enumerate(programs):
            while pcs[i] < len(prog):
                op = prog[pcs[i]]
                if op[0] == "wait":
                    if op[1] not in ready:
                        break
                elif op[0] == "issue":
                    ready.add(op[1])
                else:  # arrive / sync
                    b = bars.setdefault(op[1], _Bar())
                    if waiting[i] is None:
                        b.count += op[2]
                        gen = b.gen
                        if b.count > BLOCK:
                            raise AssertionError(f"barrier {op[1]} over-counted")
                        if b.count == BLOCK:
                            b.count, b.gen = 0, b.gen + 1
                        if op[0] == "sync" and b.gen == gen:
                            waiting[i] = (op[1], gen)
                            break
                    else:
                        bid, gen = waiting[i]
                        if bars[bid].gen == gen:
                            break
                        waiting[i] = None
                pcs[i] += 1
                progressed = True
        if all(pc == len(p) for pc, p in zip(pcs, programs)):
            left = {k: b.count for k, b in bars.items() if b.count}
            assert not left, f"barrier instances left half-counted: {left}"
            return
        if not progressed:
            raise AssertionError(f"deadlock at {pcs}")


def _stage1_rounds(n1, ns):
    c, p = [], []
    for k in range(min(ns, n1)):
        p.append(("issue", ("s1", k)))
    for k in range(n1):
        c.append(("wait", ("s1", k)))
        if k % ns == ns - 1 and k + 1 < n1:
            c.append(("arrive", 1, COMPUTE))
    for r0 in range(ns, n1, ns):
        p.append(("sync", 1, PRODUCER))
        for k in range(r0, min(r0 + ns, n1)):
            p.append(("issue", ("s1", k)))
    return c, p


def _stage2(n_items, ndc, ns):
    n_real = n_items * ndc
    c, p = [], []
    for k in range(ns):
        p.append(("issue", ("s2", k)))
    tile = 0
    for k in itertools.count():
        c.append(("wait", ("s2", k)))
        if k >= n_real:  # end-of-work chunk
            break
        if k % ndc == ndc - 1:
            if tile >= 2:
                c.append(("sync", 5 + tile % 2, COMPUTE))
            tile += 1
        c.append(("arrive", 1 + k % ns, COMPUTE))
    for t in range(max(tile - 2, 0), tile):
        c.append(("sync", 5 + t % 2, COMPUTE))
    tile = 0
    for k in range(n_real):
        p.append(("sync", 1 + k % ns, PRODUCER))
        p.append(("issue", ("s2", k + ns)))  # refill before reducing
        if k % ndc == ndc - 1:
            p.append(("arrive", 5 + tile % 2, PRODUCER))
            tile += 1
    return c, p


@pytest.mark.parametrize("ns", [2, 4])
def test_stage1_round_barrier(ns):
    for n1 in range(0, 9):
        _run(list(_stage1_rounds(n1, ns)))


@pytest.mark.parametrize("ns", [2, 4])
@pytest.mark.parametrize("ndc", [1, 2, 3])
def test_stage2_slot_and_partial_barriers(ns, ndc):
    for n_items in range(0, 14):
        _run(list(_stage2(n_items, ndc, ns)))


def test_the_model_catches_a_missing_arrival():
    c, p = _stage2(5, 1, 2)
    p_bad = [op for op in p if not (op[0] == "arrive" and op[1] >= 5)]
    with pytest.raises(AssertionError, match="deadlock"):
        _run([c, p_bad])
    c_bad = c[:-1]  # drop the last leftover wait on a partial barrier
    with pytest.raises(AssertionError, match="half-counted"):
        _run([c_bad, p])
