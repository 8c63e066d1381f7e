"""The seeded workload generators against the oracle's allocator: block
tables built from a "shuffled free list" must be exactly what the reference
allocator and block tables hand out (allocator.rs:40-170,
block_table.rs:135-209, scheduler.rs:228-297). CPU only."""

import numpy as np

from oracle import host_ref as H
from pagedkv import CacheConfig
from pagedkv.workloads import Stream, decode_batch, prefill_chunk, shuffled_pop_order


def shuffled_allocator(nb, perm):
    a = H.Allocator(nb)
    ids = a.allocate_many(nb)
    assert ids == list(range(nb))
    for b in perm:
        a.decref(int(b))
    return a


def test_shuffled_pop_order_is_what_the_allocator_hands_out():
    st = Stream(3)
    order = shuffled_pop_order(64, st)
    perm = Stream(3).permutation(64)
    a = shuffled_allocator(64, perm)
    assert [a.allocate() for _ in range(64)] == order.tolist()


def test_decode_batch_tables_match_admission_then_decode():
    cfg = CacheConfig(num_blocks=512, block_size=4, num_kv_heads=1, head_dim=4, num_layers=1,
                      dtype_bytes=2)
    b = decode_batch(seed=None, num_seqs=20, max_ctx=70, cfg=cfg)
    # Replay: same draws, then the allocator and tables of the reference.
    st = Stream(b.seed)
    ctx = st.integers(20, 1, 70)
    a = shuffled_allocator(512, st.permutation(512))
    tabs = []
    for c in ctx:  # Scheduler::admit, in order
        t = H.BlockTable(4)
        t.append_many(a, int(c))
        tabs.append(t)
    slots = [t.append(a)[0] for t in tabs]  # Scheduler::decode, in order
    for q, t in enumerate(tabs):
        assert b.tables[q, : len(t.blocks)].tolist() == t.blocks
        assert (b.tables[q, len(t.blocks):] == -1).all()
    assert b.slot_mapping().tolist() == [blk * 4 + s for blk, s in slots]


def test_prefill_chunk_fills_the_budget_and_matches_admission():
    cfg = CacheConfig(num_blocks=2048, block_size=16, num_kv_heads=1, head_dim=4, num_layers=1,
                      dtype_bytes=2)
    b = prefill_chunk(seed=4, num_prompts=20, lo=16, hi=500, budget=2500, cfg=cfg)
    assert b.num_tokens == 2500 and (b.ctx == 0).all()
    st = Stream(4)
    lens = st.log_uniform_int(20, 16, 500)
    a = shuffled_allocator(2048, st.permutation(2048))
    for q, n in enumerate(lens):
        t = H.BlockTable(16)
        t.append_many(a, int(n))
        if q < len(b.new):
            assert b.tables[q, : len(t.blocks)].tolist() == t.blocks
            assert b.new[q] == n or q == len(b.new) - 1


def test_generators_are_deterministic_and_shaped():
    a, b = Stream(9), Stream(9)
    assert (a.u64(100) == b.u64(100)).all()
    u = Stream(1).uniform(100000)
    assert 0.0 <= u.min() and u.max() < 1.0 and abs(u.mean() - 0.5) < 0.01
    z = Stream(2).normal(100000)
    assert abs(z.mean()) < 0.02 and abs(z.std() - 1) < 0.02
    g = Stream(3).geometric(100000, 256.0)
    assert g.min() >= 1 and abs(g.mean() / 256 - 1) < 0.03
    p = Stream(4).poisson(100000, 8.0)
    assert abs(p.mean() - 8) < 0.05 and abs(p.var() - 8) < 0.2
    x = Stream(5).log_uniform_int(100000, 64, 8192)
    assert x.min() >= 64 and x.max() <= 8192 and 1500 < x.mean() < 1900
    assert sorted(Stream(6).permutation(1000).tolist()) == list(range(1000))
    np.testing.assert_array_equal(Stream(7).integers(1000, 1, 3) >= 1, True)
