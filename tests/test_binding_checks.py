"""Argument checks of the Python binding (pagedkv.B200Backend) that run on the
host before any library call, so they need no GPU: the destination array of
write_kv_batch_pairs and the tensor shapes of paged_attention. The backend
object is made without a device pool (its methods raise before using one)."""

import numpy as np
import pytest
import torch

from pagedkv import B200Backend


def hollow():
    """A B200Backend with no device handle: only the host-side checks run."""
    return object.__new__(B200Backend)


def test_slot_pairs_layout():
    p = B200Backend.slot_pairs(np.array([3, 0, 7]), np.array([1, 15, 0]))
    assert p.dtype == np.uint64 and p.shape == (3, 2) and p.flags.c_contiguous
    assert p.tolist() == [[3, 1], [0, 15], [7, 0]]


@pytest.mark.parametrize("bad", [
    np.zeros((4, 2), np.int64),            # wrong dtype
    np.zeros((4, 3), np.uint64),           # wrong width
    np.zeros((4, 2), np.uint64, order="F")[::2],  # not contiguous
    np.zeros(8, np.uint64),                # flat
])
def test_write_kv_batch_pairs_rejects_other_layouts(bad):
    k = np.zeros((len(bad) if bad.ndim == 2 else 1, 8), np.float32)
    with pytest.raises(ValueError):
        hollow().write_kv_batch_pairs(0, bad, k, k)


def test_paged_attention_shape_checks():
    b = hollow()
    t = torch.zeros((2, 4), dtype=torch.int32)
    c = torch.full((2,), 8, dtype=torch.int32)
    q = torch.zeros((6, 4, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # 6 rows are not whole sequences of 4 tokens
        b.paged_attention(q, t, c, 16, q.clone(), 0, q_len=4)
    with pytest.raises(ValueError):  # q_len below 1
        b.paged_attention(q, t, c, 16, q.clone(), 0, q_len=0)
    with pytest.raises(ValueError):  # head rows not contiguous
        b.paged_attention(q.transpose(1, 2).contiguous().transpose(1, 2), t, c, 16, q.clone(), 0)
    with pytest.raises(ValueError):  # output of another shape
        b.paged_attention(q, t, c, 16, torch.zeros((6, 4, 32), dtype=torch.bfloat16), 0)
    with pytest.raises(ValueError):  # output of another dtype
        b.paged_attention(q, t, c, 16, q.float(), 0)
