"""Copy waves: pairs of one step ordered into waves that run in parallel
must give the result of applying them one after another (backend.rs:104-109).
The parallel semantics of one wave (every source read before any write) is
modelled on the CPU; the beam-search trace, which chains copies within a step
when old beams are freed group by group, is checked too."""

import numpy as np
import pytest

from pagedkv import CacheConfig
from pagedkv.driver import copy_waves
from pagedkv.traces import beam_cow_trace
from pagedkv.workloads import Stream


def sequential(pool, pairs):
    for s, d in pairs:
        pool[d] = pool[s]
    return pool


def by_waves(pool, pairs):
    ordered, waves = copy_waves(np.asarray(pairs, np.int64).reshape(-1, 2))
    for start, count in waves:
        w = ordered[start:start + count]
        assert len(set(w[:, 1].tolist())) == count  # no two writes to one block in a wave
        assert not set(w[:, 0].tolist()) & set(w[:, 1].tolist())  # nothing read and written
        snapshot = pool[w[:, 0]].copy()  # all sources read, then all writes land
        pool[w[:, 1]] = snapshot
    return pool


@pytest.mark.parametrize("seed", range(20))
def test_waves_equal_sequential_application(seed):
    st = Stream(seed)
    nb = int(st.integers(1, 2, 12)[0])
    p = int(st.integers(1, 0, 30)[0])
    pairs = st.integers(2 * p, 0, nb - 1).reshape(p, 2)
    pool = np.arange(nb * 3, dtype=np.int64).reshape(nb, 3)
    np.testing.assert_array_equal(by_waves(pool.copy(), pairs), sequential(pool.copy(), pairs))


def test_copy_on_write_pairs_without_chains_form_one_wave():
    pairs = np.array([[1, 10], [1, 11], [2, 12], [3, 13]])
    ordered, waves = copy_waves(pairs)
    assert waves == [(0, 4)] and (ordered == pairs).all()
    assert copy_waves(np.array([[5, 5]]))[1] == []


def test_beam_trace_chains_within_a_step_and_waves_keep_its_meaning():
    cfg = CacheConfig(num_blocks=512, block_size=8, num_kv_heads=1, head_dim=1, num_layers=1,
                      dtype_bytes=2)
    chained = 0
    for plan in beam_cow_trace(cfg, groups=6, width=4, prefix=37, steps=30, zero_per_step=5, seed=2,
                               interleave=True):
        if not len(plan.copies):
            continue
        waves = copy_waves(plan.copies)[1]
        chained += len(waves) > 1
        pool = np.arange(512 * 2, dtype=np.int64).reshape(512, 2)
        np.testing.assert_array_equal(by_waves(pool.copy(), plan.copies),
                                      sequential(pool.copy(), plan.copies))
    assert chained > 0  # freeing old beams group by group does chain copies within a step


def test_batched_beam_steps_do_not_chain():
    cfg = CacheConfig(num_blocks=4096, block_size=16, num_kv_heads=1, head_dim=1, num_layers=1,
                      dtype_bytes=2)
    for plan in beam_cow_trace(cfg, groups=16, width=4, prefix=100, steps=20, seed=1):
        if len(plan.copies):
            assert len(copy_waves(plan.copies)[1]) == 1
