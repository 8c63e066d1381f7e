"""group_copy_zero: the host side of the fused copy + zero launch. Applied
as the kernel applies it (each source read once, written to its
destinations, then zeroed if freed; then the other freed blocks zeroed), the
grouped arrays must give the pool that copy_blocks of the pairs in order
followed by zero_blocks gives (crates/paged-kv-core/src/backend.rs:104-109,
cpu.rs:131-160). A toy pool of block ids stands in for the planes."""

import numpy as np
import pytest

from pagedkv.driver import copy_waves, group_copy_zero


def sequential(pool, copies, zero):
    p = pool.copy()
    for s, d in copies:
        p[d] = p[s]
    p[list(zero)] = -1
    return p


def grouped(pool, g):
    srcs, offs, dsts, zsrc, zonly = g
    p = pool.copy()
    vals = {int(s): pool[s] for s in srcs}  # each source read once, before any store
    for i, s in enumerate(srcs):
        for d in dsts[offs[i]:offs[i + 1]]:
            p[d] = vals[int(s)]
        if zsrc[i]:
            p[s] = -1
    p[zonly] = -1
    return p


@pytest.mark.parametrize("seed", range(40))
def test_grouped_arrays_apply_like_copy_then_zero(seed):
    rng = np.random.default_rng(seed)
    nb = 200
    pool = rng.integers(0, 10**6, nb)
    ids = rng.permutation(nb)
    nsrc = int(rng.integers(1, 12))
    srcs = ids[:nsrc]
    ndst = int(rng.integers(nsrc, 40))
    dsts = ids[nsrc:nsrc + ndst]
    copies = np.stack([rng.choice(srcs, ndst), dsts], 1)  # sources shared, as beams share tails
    zero = rng.choice(np.concatenate([srcs, ids[100:150]]), int(rng.integers(1, 20)), replace=False)
    assert len(copy_waves(copies)[1]) == 1
    g = group_copy_zero(copies, zero, np.zeros(0, np.int64))
    assert g is not None
    srcs_g, offs, dsts_g, zsrc, zonly = g
    assert offs[-1] == len(copies) and sorted(dsts_g.tolist()) == sorted(dsts.tolist())
    assert set(zonly.tolist()) | set(srcs_g[zsrc == 1].tolist()) == set(zero.tolist())
    np.testing.assert_array_equal(grouped(pool, g), sequential(pool, copies, zero))


def test_not_eligible_when_a_destination_is_zeroed_or_a_zeroed_block_is_written():
    copies = np.array([[1, 2], [1, 3]])
    assert group_copy_zero(copies, np.array([3]), np.zeros(0, np.int64)) is None
    assert group_copy_zero(copies, np.array([7]), np.array([7])) is None
    assert group_copy_zero(copies, np.zeros(0, np.int64), np.zeros(0, np.int64)) is None
    g = group_copy_zero(copies, np.array([1, 9]), np.array([2, 3]))
    assert g[0].tolist() == [1] and g[1].tolist() == [0, 2] and g[2].tolist() == [2, 3]
    assert g[3].tolist() == [1] and g[4].tolist() == [9]
