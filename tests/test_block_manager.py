"""C++ paged block manager: allocation, COW, prefix index, eviction, invariants."""
import random

import numpy as np
import pytest

from lightbulb_b200.kv.block_manager import BlockManager


def test_append_and_free():
    bm = BlockManager(8, 4)
    bm.add_sequence(1)
    slots, cow = bm.append_slots(1, 6, list(range(6)))
    assert len(slots) == 6 and cow == []
    t = bm.block_table(1)
    assert len(t) == 2 and slots[:4] == [t[0] * 4 + i for i in range(4)]
    assert bm.num_free_blocks() == 6
    bm.free_sequence(1)
    assert bm.check_invariants()


def test_prefix_match_and_cow():
    bm = BlockManager(16, 4)
    bm.add_sequence(1)
    toks = list(range(100, 110))
    bm.append_slots(1, 10, toks)
    bm.add_sequence(2)
    n = bm.match_prefix(2, toks + [5, 6])
    assert n == 8  # two full blocks shared
    assert bm.block_table(2)[:2] == bm.block_table(1)[:2]
    assert bm.refcount(bm.block_table(1)[0]) == 2
    # fork shares the partial tail block -> COW on first write
    bm.fork(1, 3)
    slots, cow = bm.append_slots(3, 1, [7])
    assert len(cow) == 2 and cow[0] == bm.block_table(1)[2]
    assert bm.check_invariants()
    for s in (1, 2, 3):
        bm.free_sequence(s)
    assert bm.check_invariants()
    assert bm.num_free_blocks() == 16


def test_cached_blocks_evicted_lru():
    bm = BlockManager(4, 2)
    bm.add_sequence(1)
    bm.append_slots(1, 4, [1, 2, 3, 4])
    bm.free_sequence(1)
    assert bm.num_cached_blocks() == 2 and bm.num_free_blocks() == 4
    bm.add_sequence(2)
    bm.append_slots(2, 8, list(range(50, 58)))  # needs every block: evicts the cached ones
    assert bm.num_free_blocks() == 0
    assert bm.check_invariants()


def test_collision_safe_prefix():
    bm = BlockManager(8, 2)
    bm.add_sequence(1)
    bm.append_slots(1, 4, [1, 2, 3, 4])
    bm.add_sequence(2)
    assert bm.match_prefix(2, [1, 2, 9, 9, 9]) == 2
    bm.add_sequence(3)
    assert bm.match_prefix(3, [2, 1, 3, 4, 5]) == 0


def test_out_of_blocks_raises():
    bm = BlockManager(2, 4)
    bm.add_sequence(1)
    with pytest.raises(RuntimeError):
        bm.append_slots(1, 9)


def test_randomized_invariants():
    rng = random.Random(0)
    bm = BlockManager(64, 4)
    live = {}
    for step in range(2000):
        op = rng.random()
        if op < 0.3 and len(live) < 12:
            sid = step
            bm.add_sequence(sid)
            toks = [rng.randrange(5) for _ in range(rng.randrange(1, 20))]
            bm.match_prefix(sid, toks)
            live[sid] = toks
        elif op < 0.7 and live:
            sid = rng.choice(list(live))
            n = rng.randrange(1, 6)
            if bm.can_allocate(sid, n):
                bm.append_slots(sid, n, [rng.randrange(5) for _ in range(n)])
        elif op < 0.8 and live:
            sid = rng.choice(list(live))
            if bm.num_free_blocks() > 4:
                bm.fork(sid, 10_000 + step)
                live[10_000 + step] = []
        elif live:
            sid = rng.choice(list(live))
            bm.free_sequence(sid)
            del live[sid]
        assert bm.check_invariants()


def test_fill_block_tables():
    bm = BlockManager(8, 4)
    for s in (1, 2):
        bm.add_sequence(s)
        bm.append_slots(s, 5 * s)
    out = np.zeros((2, 4), dtype=np.int32)
    bm.fill_block_tables([1, 2], out, 4)
    assert list(out[0, :2]) == bm.block_table(1) and list(out[1, :3]) == bm.block_table(2)
