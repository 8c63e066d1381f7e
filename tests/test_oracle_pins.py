"""Pins the CPU oracle to the reference's own known-answer tests.

Every #[test] in crates/paged-kv-core/src/{cpu,config,allocator,block_table,
scheduler}.rs is restated here against the oracle (oracle/pkv_oracle.c for
CpuBackend, oracle/host_ref.py for the host bookkeeping), with the same
inputs and the same expected values. The reference cannot be built here (no
Rust toolchain), so these known answers are what make the oracle trustworthy.
"""

import numpy as np
import pytest

from oracle import host_ref as H
from oracle.cpu import OracleBackend, digest_plane, digest_rows, resolve_slots
from pagedkv.config import CacheConfig


def entry(seed, n):  # cpu.rs:171-173
    return np.array([seed + i * 0.25 for i in range(n)], dtype=np.float32)


def backend():  # cpu.rs:175-177
    return OracleBackend(CacheConfig.tiny(8))


def err(fn, *a):
    with pytest.raises(H.RefError) as e:
        fn(*a)
    return (e.value.code,) + tuple(e.value.fields)


# ---- cpu.rs tests ------------------------------------------------------------


def test_write_then_read_round_trips():  # cpu.rs:179-192
    b = backend()
    n = b.cfg.entry_elems()
    k, v = entry(1.0, n), entry(100.0, n)
    b.write_kv(1, (3, 2), k, v)
    ko, vo = b.read_entry(1, (3, 2))
    assert (ko == k).all() and (vo == v).all()


def test_writes_do_not_bleed_across_slots_blocks_or_layers():  # cpu.rs:194-216
    b = backend()
    n = b.cfg.entry_elems()
    b.write_kv(1, (3, 2), entry(7.0, n), entry(70.0, n))
    for layer, slot in [(1, (3, 1)), (1, (3, 3)), (1, (2, 2)), (1, (4, 2)), (0, (3, 2))]:
        ko, vo = b.read_entry(layer, slot)
        assert (ko == 0).all() and (vo == 0).all()


def test_copy_block_duplicates_every_slot_and_layer():  # cpu.rs:218-250
    b = backend()
    cfg = b.cfg
    n = cfg.entry_elems()
    for layer in range(cfg.num_layers):
        for slot in range(cfg.block_size):
            seed = layer * 100 + slot
            b.write_kv(layer, (0, slot), entry(seed, n), entry(seed + 0.5, n))
    b.copy_block(0, 5)
    for layer in range(cfg.num_layers):
        for slot in range(cfg.block_size):
            seed = layer * 100 + slot
            ko, vo = b.read_entry(layer, (5, slot))
            assert (ko == entry(seed, n)).all() and (vo == entry(seed + 0.5, n)).all()


def test_copy_is_a_snapshot_not_an_alias():  # cpu.rs:252-271
    b = backend()
    n = b.cfg.entry_elems()
    b.write_kv(0, (0, 0), entry(1.0, n), entry(2.0, n))
    b.copy_block(0, 1)
    b.write_kv(0, (0, 0), entry(9.0, n), entry(9.0, n))
    ko, vo = b.read_entry(0, (1, 0))
    assert (ko == entry(1.0, n)).all() and (vo == entry(2.0, n)).all()


def test_zero_block_clears_all_layers():  # cpu.rs:273-295
    b = backend()
    n = b.cfg.entry_elems()
    for layer in range(b.cfg.num_layers):
        b.write_kv(layer, (2, 1), entry(5.0, n), entry(5.0, n))
    b.zero_block(2)
    for layer in range(b.cfg.num_layers):
        ko, vo = b.read_entry(layer, (2, 1))
        assert (ko == 0).all() and (vo == 0).all()


def test_self_copy_is_a_no_op_not_a_corruption():  # cpu.rs:297-310
    b = backend()
    n = b.cfg.entry_elems()
    b.write_kv(0, (1, 0), entry(3.0, n), entry(4.0, n))
    b.copy_block(1, 1)
    ko, vo = b.read_entry(0, (1, 0))
    assert (ko == entry(3.0, n)).all() and (vo == entry(4.0, n)).all()


def test_bad_addresses_and_shapes_are_rejected():  # cpu.rs:312-351
    b = backend()
    cfg = b.cfg
    n = cfg.entry_elems()
    k, v = entry(0.0, n), entry(0.0, n)
    assert err(b.write_kv, 99, (0, 0), k, v) == (H.INVALID_LAYER, 99, cfg.num_layers)
    assert err(b.write_kv, 0, (99, 0), k, v) == (H.INVALID_BLOCK, 99, cfg.num_blocks)
    assert err(b.write_kv, 0, (0, 99), k, v) == (H.SLOT_OUT_OF_RANGE, 99, cfg.block_size)
    assert err(b.write_kv, 0, (0, 0), k[: n - 1], v) == (H.SHAPE_MISMATCH, n, n - 1)


def test_allocated_bytes_tracks_config():  # cpu.rs:353-358
    b = OracleBackend(CacheConfig.llama_3_2_1b(512))
    assert b.allocated_bytes() == 512 * 16 * 32 * 1024


def test_write_kv_batch_matches_repeated_write_kv():  # cpu.rs:360-383
    b = backend()
    n = b.cfg.entry_elems()
    dsts = [(0, 0), (0, 1), (3, 2)]
    k = np.arange(len(dsts) * n, dtype=np.float32) * 0.5
    v = np.arange(len(dsts) * n, dtype=np.float32) * 0.25 + 1.0
    b.write_kv_batch(1, dsts, k, v)
    for i, d in enumerate(dsts):
        ko, vo = b.read_entry(1, d)
        assert (ko == k[i * n:(i + 1) * n]).all() and (vo == v[i * n:(i + 1) * n]).all()


def test_write_kv_batch_rejects_mismatched_lengths_without_panicking():  # cpu.rs:385-400
    b = backend()
    n = b.cfg.entry_elems()
    assert err(b.write_kv_batch, 0, [(0, 0), (0, 1)], np.zeros(n), np.zeros(2 * n)) == (
        H.SHAPE_MISMATCH, 2 * n, n)


# ---- default trait semantics the oracle must reproduce (backend.rs:55-74, 104-109) ----


def test_batch_stops_at_first_bad_token_and_keeps_earlier_writes():
    b = backend()
    n = b.cfg.entry_elems()
    k = np.arange(3 * n, dtype=np.float32) + 1
    assert err(b.write_kv_batch, 0, [(1, 0), (99, 0), (2, 0)], k, k) == (H.INVALID_BLOCK, 99, 8)
    assert (b.read_entry(0, (1, 0))[0] == k[:n]).all()
    assert (b.read_entry(0, (2, 0))[0] == 0).all()


def test_copy_blocks_apply_in_order_including_chains():
    b = backend()
    n = b.cfg.entry_elems()
    for blk in range(4):
        b.write_kv(0, (blk, 0), entry(blk, n), entry(blk, n))
    b.copy_blocks([(0, 1), (1, 2), (3, 0)])  # 2 <- 1 <- 0 (chain), then 0 <- 3
    assert (b.read_entry(0, (2, 0))[0] == entry(0, n)).all()
    assert (b.read_entry(0, (1, 0))[0] == entry(0, n)).all()
    assert (b.read_entry(0, (0, 0))[0] == entry(3, n)).all()


# ---- config.rs tests -----------------------------------------------------------


def test_llama_bytes_per_token_is_sane():  # config.rs:104-109
    assert CacheConfig.llama_3_2_1b(1024).bytes_per_token() == 32 * 1024


def test_blocks_for_tokens_rounds_up():  # config.rs:111-118
    c = CacheConfig.tiny(64)
    assert [c.blocks_for_tokens(x) for x in (0, 1, 4, 5)] == [0, 1, 1, 2]


def test_split_position_matches_block_size():  # config.rs:120-127
    c = CacheConfig.tiny(64)
    assert [c.split_position(p) for p in (0, 3, 4, 9)] == [(0, 0), (0, 3), (1, 0), (2, 1)]


def test_total_bytes_is_consistent_with_per_block_math():  # config.rs:129-137
    c = CacheConfig.llama_3_2_1b(1000)
    per_block = 2 * c.num_layers * c.block_elems() * c.dtype_bytes
    assert c.total_bytes() == per_block * c.num_blocks
    assert per_block == 16 * c.bytes_per_token()


# ---- allocator.rs tests -------------------------------------------------------------


def test_fresh_pool_is_entirely_free():  # allocator.rs:247-254
    a = H.Allocator(8)
    assert (a.num_free(), a.num_used(), a.utilization()) == (8, 0, 0.0)
    a.check_invariants()


def test_allocate_hands_out_distinct_blocks_with_refcount_one():  # allocator.rs:256-272
    a = H.Allocator(4)
    ids = [a.allocate() for _ in range(4)]
    assert len(set(ids)) == 4 and all(a.ref_count(i) == 1 for i in ids)
    assert a.num_free() == 0 and a.utilization() == 1.0


def test_exhausted_pool_reports_out_of_blocks():  # allocator.rs:274-286
    a = H.Allocator(2)
    a.allocate()
    a.allocate()
    assert err(a.allocate) == (H.OUT_OF_BLOCKS, 1, 0)


def test_allocate_many_is_all_or_nothing():  # allocator.rs:288-303
    a = H.Allocator(4)
    assert err(a.allocate_many, 5) == (H.OUT_OF_BLOCKS, 5, 4)
    assert a.num_free() == 4 and a.total_allocated == 0


def test_decref_to_zero_returns_block_to_the_pool():  # allocator.rs:305-315
    a = H.Allocator(2)
    i = a.allocate()
    assert a.decref(i) == 0 and a.num_free() == 2


def test_shared_block_survives_one_owner_leaving():  # allocator.rs:317-338
    a = H.Allocator(2)
    i = a.allocate()
    assert a.incref(i) == 2 and a.incref(i) == 3 and a.is_shared(i)
    assert a.decref(i) == 2 and a.num_free() == 1
    assert a.decref(i) == 1 and not a.is_shared(i)
    assert a.decref(i) == 0 and a.num_free() == 2


def test_double_free_is_an_error_not_a_silent_corruption():  # allocator.rs:340-353
    a = H.Allocator(2)
    i = a.allocate()
    a.decref(i)
    assert err(a.decref, i) == (H.BLOCK_NOT_ALLOCATED, i)
    assert a.num_free() == 2


def test_incref_on_a_free_block_is_rejected():  # allocator.rs:355-363
    assert err(H.Allocator(2).incref, 0) == (H.BLOCK_NOT_ALLOCATED, 0)


def test_out_of_range_block_is_rejected():  # allocator.rs:365-373
    assert err(H.Allocator(2).ref_count, 7) == (H.INVALID_BLOCK, 7, 2)


def test_free_list_is_lifo():  # allocator.rs:375-387
    a = H.Allocator(4)
    ids = a.allocate_many(4)
    a.decref(ids[1])
    a.decref(ids[3])
    assert a.allocate() == ids[3] and a.allocate() == ids[1]


def test_churn_preserves_invariants():  # allocator.rs:389-435
    a = H.Allocator(16)
    live = []
    seed = 0x243F_6A88_85A3_08D3
    m = (1 << 64) - 1
    for _ in range(2000):
        seed = (seed * 6364136223846793005 + 1) & m
        roll = (seed >> 33) % 3
        if roll == 0:
            try:
                live.append(a.allocate())
            except H.RefError:
                pass
        elif roll == 1:
            if live:
                i = live[(seed >> 13) % len(live)]
                a.incref(i)
                live.append(i)
        elif live:
            i = (seed >> 17) % len(live)
            live[i], live[-1] = live[-1], live[i]
            a.decref(live.pop())
        a.check_invariants()
    for i in live:
        a.decref(i)
    assert a.num_free() == 16


# ---- block_table.rs tests -------------------------------------------------------------


def setup(nb, bs):
    return H.Allocator(nb), H.BlockTable(bs)


def test_append_allocates_lazily_and_fills_one_block_before_growing():  # block_table.rs:250-269
    a, t = setup(8, 4)
    for i in range(4):
        slot, cow = t.append(a)
        assert cow is None and slot[1] == i and len(t.blocks) == 1
    slot, cow = t.append(a)
    assert cow is None and slot[1] == 0 and len(t.blocks) == 2 and t.num_tokens == 5
    assert a.num_used() == 2


def test_resolve_matches_the_slots_append_handed_out():  # block_table.rs:271-281
    a, t = setup(8, 4)
    slots = [t.append(a)[0] for _ in range(10)]
    assert [t.resolve(p) for p in range(10)] == slots


def test_resolve_rejects_unwritten_positions():  # block_table.rs:283-289
    a, t = setup(8, 4)
    t.append(a)
    t.resolve(0)
    with pytest.raises(H.RefError):
        t.resolve(1)


def test_fork_shares_blocks_without_copying():  # block_table.rs:291-311
    a, t = setup(8, 4)
    for _ in range(6):
        t.append(a)
    child = t.fork(a)
    assert child.blocks == t.blocks and a.num_used() == 2
    assert all(a.ref_count(b) == 2 for b in t.blocks)
    t.free(a)
    child.free(a)
    assert a.num_free() == 8


def test_writing_to_a_forked_sequence_triggers_cow_on_the_shared_tail_only():  # :313-347
    a, t = setup(8, 4)
    for _ in range(3):
        t.append(a)
    parent_block = t.blocks[0]
    child = t.fork(a)
    slot, cow = child.append(a)
    assert cow is not None and cow[0] == parent_block and cow[1] != parent_block
    assert slot == (cow[1], 3)
    assert a.ref_count(parent_block) == 1 and a.ref_count(cow[1]) == 1
    pslot, pcow = t.append(a)
    assert pcow is None and pslot == (parent_block, 3)
    t.free(a)
    child.free(a)
    assert a.num_free() == 8


def test_cow_only_touches_the_tail_block_earlier_blocks_stay_shared():  # :349-373
    a, t = setup(16, 2)
    for _ in range(6):
        t.append(a)
    orig = list(t.blocks)
    child = t.fork(a)
    _, cow = child.append(a)
    assert cow is None
    assert all(a.ref_count(b) == 2 for b in orig) and child.blocks[:3] == orig


def test_append_many_matches_repeated_append():  # :375-390
    a1, t1 = setup(16, 4)
    a2, t2 = setup(16, 4)
    s1 = [t1.append(a1)[0] for _ in range(11)]
    s2, _ = t2.append_many(a2, 11)
    assert s1 == s2 and len(t1.blocks) == len(t2.blocks) and a1.num_used() == a2.num_used()


def test_append_many_rolls_back_cleanly_on_exhaustion():  # :392-403
    a, t = setup(2, 4)
    assert err(t.append_many, a, 20)[0] == H.OUT_OF_BLOCKS
    assert t.num_tokens == 0 and not t.blocks and a.num_free() == 2
    a.check_invariants()


def test_free_releases_every_block_and_is_safe_on_an_empty_table():  # :405-418
    a, t = setup(4, 4)
    for _ in range(9):
        t.append(a)
    assert a.num_used() == 3
    t.free(a)
    assert a.num_free() == 4
    H.BlockTable(4).free(a)
    a.check_invariants()


def test_three_way_fork_shares_correctly_and_last_writer_pays_the_copy():  # :420-447
    a, t = setup(16, 4)
    for _ in range(4):
        t.append(a)
    orig = t.blocks[0]
    ba, bb = t.fork(a), t.fork(a)
    assert a.ref_count(orig) == 3
    assert ba.append(a)[1] is None and bb.append(a)[1] is None
    assert a.ref_count(orig) == 3
    for x in (t, ba, bb):
        x.free(a)
    assert a.num_free() == 16


# ---- scheduler.rs tests ----------------------------------------------------------------


def sched(nb, bs, mb):
    return H.Scheduler(nb, bs, mb)


def test_admits_and_decodes_a_single_sequence_to_completion():  # scheduler.rs:375-398
    s = sched(8, 4, 2)
    s.add_request(1, 3, 2)
    o1 = s.step()
    assert o1.admitted == [1] and len(o1.decoded) == 1
    assert o1.decoded[0][1][1] == 3 and o1.decoded[0][2] is None and not o1.finished
    o2 = s.step()
    assert not o2.admitted and len(o2.decoded) == 1 and o2.finished == [1]
    assert s.is_idle() and s.allocator.utilization() == 0.0


def test_batch_size_caps_concurrent_admission():  # scheduler.rs:400-424
    s = sched(16, 4, 1)
    s.add_request(1, 2, 3)
    s.add_request(2, 2, 1)
    assert s.step().admitted == [1] and len(s.waiting) == 1
    assert not s.step().admitted
    assert s.step().finished == [1] and len(s.waiting) == 1
    o4 = s.step()
    assert o4.admitted == [2] and o4.finished == [2] and s.is_idle()


def test_oversized_request_is_rejected_up_front():  # scheduler.rs:426-432
    s = sched(4, 2, 4)
    assert err(s.add_request, 1, 5, 5)[0] == H.OUT_OF_BLOCKS
    assert not s.waiting


def test_pool_pressure_forces_preemption_then_both_sequences_complete():  # :434-484
    s = sched(3, 2, 2)
    s.add_request(1, 2, 2)
    s.add_request(2, 2, 2)
    o1 = s.step()
    assert len(o1.admitted) == 2 and o1.preempted == [2] and [d[0] for d in o1.decoded] == [1]
    o2 = s.step()
    assert o2.admitted == [2] and o2.preempted == [2] and o2.finished == [1]
    assert s.allocator.utilization() == 0.0
    seen = []
    for _ in range(20):
        if s.is_idle():
            break
        seen += s.step().finished
    assert s.is_idle() and seen == [2]


def test_fork_shares_the_tail_block_and_the_second_writer_pays_the_cow():  # :486-517
    s = sched(16, 8, 4)
    s.add_request(1, 3, 5)
    shared = s.step().decoded[0][1][0]
    s.fork_sequence(1, 2, 5)
    o2 = s.step()
    parent = next(d for d in o2.decoded if d[0] == 1)
    child = next(d for d in o2.decoded if d[0] == 2)
    assert parent[2] is not None and parent[2][0] == shared and parent[2][1] != shared
    assert parent[1][0] == parent[2][1]
    assert child[2] is None and child[1][0] == shared


def test_fork_of_unknown_sequence_is_rejected():  # :519-524
    assert err(sched(8, 4, 2).fork_sequence, 99, 100, 1) == (H.UNKNOWN_SEQUENCE, 99)


def test_many_small_sequences_drain_cleanly_with_no_leaks():  # :566-590
    s = sched(6, 2, 3)
    for i in range(10):
        s.add_request(i, 2, 2)
    fin = []
    for _ in range(200):
        if s.is_idle():
            break
        fin += s.step().finished
    assert s.is_idle() and sorted(set(fin)) == list(range(10))


# ---- slot resolution and digest oracles ------------------------------------------------------


def test_resolve_slots_oracle_matches_block_table_append():
    """Device slot resolution's oracle equals the slots BlockTable::append hands out."""
    a = H.Allocator(64)
    tables = [H.BlockTable(4) for _ in range(5)]
    ctx = [3, 0, 7, 4, 9]
    for t, c in zip(tables, ctx):
        t.append_many(a, c)
    new = [2, 5, 1, 0, 6]
    expect = []
    for t, n in zip(tables, new):
        for _ in range(n):
            blk, off = t.append(a)[0]
            expect.append(blk * 4 + off)
    stride = max(len(t.blocks) for t in tables)
    tab = np.full((5, stride), -1, np.int32)
    for q, t in enumerate(tables):
        tab[q, : len(t.blocks)] = t.blocks
    rc, cu, slots = resolve_slots(tab, np.array(ctx), np.array(new), sum(new), 4, 64)
    assert rc == 0
    assert list(cu) == [0, 2, 7, 8, 8, 14]
    assert list(slots) == expect


def test_resolve_slots_oracle_flags_bad_tables():
    tab = np.array([[0, 70]], np.int32)  # 70 is outside a 64-block pool
    rc, _, slots = resolve_slots(tab, np.array([3]), np.array([3]), 3, 4, 64)
    assert rc == 2 and list(slots) == [3, -1, -1]  # position 5 also lies past the table
    rc, _, _ = resolve_slots(tab, np.array([0]), np.array([2]), 5, 4, 64)
    assert rc == -2


def test_digest_is_additive_over_shards_and_zero_for_an_empty_pool():
    cfg = CacheConfig(4, 2, 4, 2, 2, 4)
    b = OracleBackend(cfg)
    assert b.digest() == (0, 0)
    rng = np.random.default_rng(0)
    e = cfg.entry_elems()
    for layer in range(2):
        for blk in range(4):
            for s in range(2):
                b.write_kv(layer, (blk, s), rng.standard_normal(e), rng.standard_normal(e))
    kd, vd = b.digest()
    kp, vp = b.planes()
    # Two shards along the entry axis; each shard's elements keep their full-plane indices.
    acc = 0
    for g in range(2):
        part = np.zeros_like(kp)
        part[..., g * e // 2:(g + 1) * e // 2] = kp[..., g * e // 2:(g + 1) * e // 2]
        acc = (acc + digest_plane(part, 0)) % (1 << 64)
    assert acc == kd
    # Rows scattered into an empty plane digest like the plane itself.
    rows = rng.standard_normal((3, e)).astype(np.float32)
    slots = np.array([5, 0, 7])
    b2 = OracleBackend(cfg)
    b2.write_kv_batch(1, [(s // 2, s % 2) for s in slots], rows.ravel(), rows.ravel())
    assert digest_rows(rows, slots, 1, 8, 0) == b2.digest()[0]
    assert vd != kd
