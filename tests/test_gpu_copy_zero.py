"""pkv_copy_zero_blocks_dev, one launch for a step's copy-on-write pairs and
freed blocks, against copy_blocks followed by zero_blocks on an identical
pool (and, through them, the oracle semantics of cpu.rs:131-160): shared
sources, freed sources zeroed after their copies, small and large block
planes, and bad ids recorded with their documented index and skipped."""

import numpy as np
import pytest

from pagedkv import B200Backend, CacheConfig, InvalidBlock
from pagedkv.driver import group_copy_zero
from pagedkv.workloads import Stream

pytestmark = pytest.mark.gpu


def filled(cfg, seed, shards=(0, 1), dtype="bf16"):
    import torch

    b = B200Backend(cfg, dtype=dtype, shard_rank=shards[0], num_shards=shards[1])
    g = torch.Generator(device="cuda").manual_seed(seed)
    for p in b.planes():
        x = torch.randn(p.shape, generator=g, device="cuda")
        p.copy_(x.to(p.dtype))
    return b


def bits(p):
    import torch

    return p.view(torch.uint8) if p.element_size() == 1 else p.view(torch.int16)


def dev(x):
    import torch

    return torch.from_numpy(np.ascontiguousarray(x, np.int64)).cuda()


@pytest.mark.parametrize("heads,shards,dtype", [(4, 1, "bf16"), (4, 8, "bf16"), (3, 1, "bf16"),
                                                (4, 1, "f32"), (4, 2, "fp8_e4m3"), (1, 1, "f16")])
def test_fused_launch_equals_copy_then_zero(cuda, heads, shards, dtype):
    import torch

    nbytes = {"bf16": 2, "f16": 2, "f32": 4, "fp8_e4m3": 1}[dtype]
    cfg = CacheConfig(num_blocks=600, block_size=16, num_kv_heads=heads, head_dim=128,
                      num_layers=5, dtype_bytes=nbytes)
    st = Stream(heads * 10 + shards)
    ids = st.permutation(cfg.num_blocks)
    srcs = ids[:40]
    dsts = ids[40:200]
    pick = st.integers(len(dsts), 0, len(srcs) - 1)
    copies = np.stack([srcs[pick], dsts], 1).astype(np.int64)
    zero = np.concatenate([srcs[:25], ids[300:340]]).astype(np.int64)
    g = group_copy_zero(copies, zero, np.zeros(0, np.int64))
    assert g is not None and g[3].sum() > 0
    a = filled(cfg, 7, (0, shards), dtype)
    b = filled(cfg, 7, (0, shards), dtype)
    a.copy_blocks_dev(dev(copies))
    a.zero_blocks_dev(dev(zero))
    b.copy_zero_blocks_dev(*(dev(x) for x in g))
    torch.cuda.synchronize()
    assert a.device_error() is None and b.device_error() is None
    for x, y in zip(a.planes(), b.planes()):
        assert torch.equal(bits(x), bits(y))
    assert int(torch.count_nonzero(bits(b.planes()[0])[:, dev(zero)])) == 0
    # Every destination holds its source's plane as it was before the step.
    ref = filled(cfg, 7, (0, shards), dtype)
    for p_new, p_old in zip(b.planes(), ref.planes()):
        assert torch.equal(bits(p_new)[:, dev(copies[:, 1])], bits(p_old)[:, dev(copies[:, 0])])


def test_bad_ids_are_recorded_and_skipped(cuda):
    import torch

    cfg = CacheConfig(num_blocks=64, block_size=16, num_kv_heads=2, head_dim=64, num_layers=2,
                      dtype_bytes=2)
    b = filled(cfg, 3)
    ref = [p.clone() for p in b.planes()]
    # source 70 is outside the pool (its pairs are skipped); dst 99 likewise.
    srcs, offs = np.array([5, 70, 9]), np.array([0, 2, 3, 5])
    dsts, zsrc = np.array([20, 21, 22, 99, 23]), np.array([1, 1, 0])
    b.copy_zero_blocks_dev(dev(srcs), dev(offs), dev(dsts), dev(zsrc), dev(np.array([30])))
    err = b.device_error()
    assert isinstance(err[0], InvalidBlock) and err[1] in (2, 3)
    for p, r in zip(b.planes(), ref):
        for d in (20, 21):
            assert torch.equal(p[:, d].view(torch.int16), r[:, 5].view(torch.int16))
        assert torch.equal(p[:, 23].view(torch.int16), r[:, 9].view(torch.int16))
        assert torch.equal(p[:, 22].view(torch.int16), r[:, 22].view(torch.int16))
        assert int(torch.count_nonzero(p[:, 5])) == 0 and int(torch.count_nonzero(p[:, 30])) == 0
        assert torch.equal(p[:, 9].view(torch.int16), r[:, 9].view(torch.int16))
    b.copy_zero_blocks_dev(dev(np.array([1])), dev(np.array([0, 0])), dev(np.array([0])),
                           dev(np.array([0])), dev(np.array([-4])))
    err = b.device_error()
    assert isinstance(err[0], InvalidBlock) and err[1] == 0  # dst_offsets[1] + 0
