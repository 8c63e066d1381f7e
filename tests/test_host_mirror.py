"""The native host mirror (BlockAllocator / BlockTable / Scheduler in
libpagedkv_b200.so) against the oracle restatement (oracle/host_ref.py) and
the reference's known answers. CPU only."""

import numpy as np
import pytest

from oracle import host_ref as H
from pagedkv import CacheError, OutOfBlocks, UnknownSequence
from pagedkv.host import BlockAllocator, BlockTable, Scheduler
from pagedkv.workloads import Stream


def test_allocator_known_answers():  # allocator.rs:274-387
    a = BlockAllocator(4)
    ids = a.allocate_many(4)
    assert ids == [0, 1, 2, 3]
    with pytest.raises(OutOfBlocks) as e:
        a.allocate()
    assert e.value == OutOfBlocks(1, 0)
    a.decref(ids[1])
    a.decref(ids[3])
    assert a.allocate() == ids[3] and a.allocate() == ids[1]
    a.check_invariants()
    b = BlockAllocator(4)
    with pytest.raises(OutOfBlocks) as e:
        b.allocate_many(5)
    assert e.value == OutOfBlocks(5, 4) and b.total_allocated() == 0


def test_allocator_churn_matches_oracle():  # the LCG of allocator.rs:389-435, with a larger pool
    mine, ref = BlockAllocator(64), H.Allocator(64)
    live = []
    seed = 0x243F_6A88_85A3_08D3
    m = (1 << 64) - 1
    for _ in range(5000):
        seed = (seed * 6364136223846793005 + 1) & m
        roll = (seed >> 33) % 3
        if roll == 0:
            try:
                x = ref.allocate()
            except H.RefError:
                with pytest.raises(OutOfBlocks):
                    mine.allocate()
                continue
            assert mine.allocate() == x
            live.append(x)
        elif roll == 1 and live:
            i = live[(seed >> 13) % len(live)]
            assert mine.incref(i) == ref.incref(i)
            live.append(i)
        elif live:
            j = (seed >> 17) % len(live)
            live[j], live[-1] = live[-1], live[j]
            x = live.pop()
            assert mine.decref(x) == ref.decref(x)
    mine.check_invariants()
    assert mine.num_free() == ref.num_free()
    assert [mine.allocate() for _ in range(mine.num_free())] == \
        [ref.allocate() for _ in range(ref.num_free())]


def test_block_table_known_answers():  # block_table.rs:313-347, 392-403
    a = BlockAllocator(8)
    t = BlockTable(4)
    for _ in range(3):
        t.append(a)
    parent = t.physical_blocks()[0]
    child = t.fork(a)
    slot, cow = child.append(a)
    assert cow is not None and cow[0] == parent and slot.block == cow[1] and slot.slot == 3
    pslot, pcow = t.append(a)
    assert pcow is None and pslot.block == parent
    a2, t2 = BlockAllocator(2), BlockTable(4)
    with pytest.raises(OutOfBlocks):
        t2.append_many(a2, 20)
    assert t2.num_tokens() == 0 and a2.num_free() == 2


@pytest.mark.parametrize("seed", range(6))
def test_block_table_random_ops_match_oracle(seed):
    st = Stream(seed)
    bs = int(st.integers(1, 1, 8)[0])
    nb = 48
    ma, ra = BlockAllocator(nb), H.Allocator(nb)
    mt, rt = [BlockTable(bs)], [H.BlockTable(bs)]
    for _ in range(400):
        op = int(st.integers(1, 0, 5)[0])
        i = int(st.integers(1, 0, len(mt) - 1)[0])
        try:
            if op <= 1:
                exp = rt[i].append(ra)
            elif op == 2:
                n = int(st.integers(1, 0, 3 * bs)[0])
                exp = rt[i].append_many(ra, n)
            elif op == 3 and len(mt) < 12:
                rt.append(rt[i].fork(ra))
                mt.append(mt[i].fork(ma))
                continue
            elif op == 4 and len(mt) > 1:
                rt.pop(i).free(ra)
                mt.pop(i).free(ma)
                continue
            else:
                continue
        except H.RefError as e:
            with pytest.raises(CacheError) as me:
                (mt[i].append(ma) if op <= 1 else mt[i].append_many(ma, n))
            assert me.value.code == e.code
            continue
        got = mt[i].append(ma) if op <= 1 else mt[i].append_many(ma, n)
        if op <= 1:
            assert (got[0].block, got[0].slot) == exp[0] and got[1] == exp[1]
        else:
            assert [(s.block, s.slot) for s in got[0]] == exp[0]
            assert [tuple(c) for c in got[1]] == [tuple(c) for c in exp[1]]
        assert mt[i].physical_blocks() == rt[i].blocks and mt[i].num_tokens() == rt[i].num_tokens
    ma.check_invariants()
    assert ma.num_free() == ra.num_free()


def test_scheduler_known_answers():  # scheduler.rs:434-517
    s = Scheduler(3, 2, 2)
    s.add_request(1, 2, 2)
    s.add_request(2, 2, 2)
    o1 = s.step()
    assert len(o1.admitted) == 2 and o1.preempted == [2] and [d.id for d in o1.decoded] == [1]
    o2 = s.step()
    assert o2.admitted == [2] and o2.preempted == [2] and o2.finished == [1]
    f = Scheduler(16, 8, 4)
    f.add_request(1, 3, 5)
    shared = f.step().decoded[0].slot.block
    f.fork_sequence(1, 2, 5)
    o = f.step()
    par = next(d for d in o.decoded if d.id == 1)
    chi = next(d for d in o.decoded if d.id == 2)
    assert par.cow is not None and par.cow[0] == shared and par.slot.block == par.cow[1]
    assert chi.cow is None and chi.slot.block == shared
    with pytest.raises(UnknownSequence):
        f.fork_sequence(99, 100, 1)
    with pytest.raises(OutOfBlocks):
        Scheduler(4, 2, 4).add_request(1, 5, 5)


@pytest.mark.parametrize("seed", range(4))
def test_scheduler_traces_match_oracle(seed):
    """Poisson arrivals, log-uniform prompts, geometric outputs, occasional
    forks, a tight pool: every step's outcome must agree exactly."""
    st = Stream(100 + seed)
    nb, bs, mb = 32, 4, 8
    mine, ref = Scheduler(nb, bs, mb), H.Scheduler(nb, bs, mb)
    sid = 0
    preempted = 0
    for _ in range(300):
        for _ in range(int(st.poisson(1, 1.0)[0])):
            p = int(st.log_uniform_int(1, 1, 40)[0])
            g = int(st.geometric(1, 6.0)[0])
            try:
                ref.add_request(sid, p, g)
            except H.RefError:
                with pytest.raises(OutOfBlocks):
                    mine.add_request(sid, p, g)
                sid += 1
                continue
            mine.add_request(sid, p, g)
            sid += 1
        if ref.running and st.uniform(1)[0] < 0.2:
            parent = ref.running[int(st.integers(1, 0, len(ref.running) - 1)[0])].id
            ref.fork_sequence(parent, sid, 3)
            mine.fork_sequence(parent, sid, 3)
            sid += 1
        e = ref.step()
        g = mine.step()
        assert g.admitted == e.admitted
        assert [(d.id, (d.slot.block, d.slot.slot), d.cow) for d in g.decoded] == \
            [(d[0], d[1], d[2]) for d in e.decoded]
        assert g.preempted == e.preempted and g.finished == e.finished
        preempted += len(g.preempted)
        assert set(g.freed) == {b for b in range(nb) if ref.allocator.ref_counts[b] == 0} & set(g.freed)
        assert mine.num_running() == len(ref.running) and mine.num_waiting() == len(ref.waiting)
    assert preempted > 0  # the trace exercises recompute preemption
    ids, tok, gen, tab = mine.running(table_stride=nb)
    assert [int(x) for x in ids] == [r.id for r in ref.running]
    for row, r in zip(tab, ref.running):
        assert [int(x) for x in row[: len(r.table.blocks)]] == r.table.blocks
        assert (row[len(r.table.blocks):] == -1).all()


def test_freed_blocks_are_free_at_the_end_of_the_step():
    s = Scheduler(8, 2, 4)
    for i in range(4):
        s.add_request(i, 3, 1)
    o = s.step()
    assert sorted(o.finished) == [0, 1, 2, 3]
    assert sorted(o.freed) == list(range(8))
    assert s.pool_utilization() == 0.0
