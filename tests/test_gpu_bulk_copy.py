"""copy_blocks on the bulk-copy (TMA) engine: bit-exact against the oracle.

The bulk engine (pkv_set_copy_engine(PKV_COPY_BULK)) moves each block plane
global -> shared -> global with cp.async.bulk; these tests give it the same
inputs as the register engine's tests and compare whole pools with
oracle/pkv_oracle.c, the restated CpuBackend (cpu.rs:131-149 and the
trait's sequential copy_blocks loop, backend.rs:104-109).
"""

import numpy as np
import pytest

from oracle import host_ref as H
from oracle.cpu import OracleBackend
from pagedkv import B200Backend, CacheConfig
from pagedkv.errors import CacheError
from pagedkv.workloads import Stream, bf16_bits_to_f32, config1, f32_to_bf16_bits

from test_gpu_parity import apply, assert_pools_equal, random_ops

pytestmark = pytest.mark.gpu


def test_config1_through_the_bulk_engine(cuda):
    """The CpuBackend-runnable case (f32, 32 KiB block planes)."""
    w = config1(seed=0)
    cpu, gpu = OracleBackend(w.cfg), B200Backend(w.cfg)
    gpu.set_copy_engine("bulk")
    bs = w.cfg.block_size
    for layer in range(w.cfg.num_layers):
        dsts = [(int(s) // bs, int(s) % bs) for s in w.slots]
        cpu.write_kv_batch(layer, dsts, w.k[layer].ravel(), w.v[layer].ravel())
        gpu.write_kv_batch(layer, dsts, w.k[layer].ravel(), w.v[layer].ravel())
    cpu.copy_blocks(w.pairs)
    gpu.copy_blocks(w.pairs)
    cpu.zero_blocks(w.zero)
    gpu.zero_blocks(w.zero)
    assert_pools_equal(gpu, cpu)
    assert gpu.digest() == cpu.digest()


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("seed", [4, 5])
def test_bulk_engine_random_sequences(cuda, dtype, seed):
    """Chained pairs (wave-ordered by the host), self-copies, out-of-pool ids."""
    bytes_ = 4 if dtype == "f32" else 2
    cfg = CacheConfig(24, 4, 2, 8, 3, bytes_)  # 128- or 256-byte block planes
    cpu, gpu = OracleBackend(cfg), B200Backend(cfg, dtype=dtype)
    gpu.set_copy_engine("bulk")
    for op in random_ops(seed, cfg):
        if dtype == "f16" and op[0] == "write":
            op = op[:3] + tuple(np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
                                for x in op[3:])
        errs = []
        for b in (gpu, cpu):
            try:
                apply(b, op)
                errs.append(None)
            except (CacheError, H.RefError) as ex:
                errs.append((ex.code, tuple(getattr(ex, "values", getattr(ex, "fields", ())))))
        assert errs[0] == errs[1], op[0]
    assert_pools_equal(gpu, cpu)


@pytest.mark.parametrize("heads,head_dim", [(4, 128), (12, 128), (8, 256)])
def test_bulk_engine_split_planes_and_long_rings(cuda, heads, head_dim):
    """Many items per CTA (the shared-memory ring wraps many times). Block
    planes of 16, 48 and 64 KiB: the last two move as 24 and 32 KiB runs."""
    import torch

    cfg = CacheConfig(1200, 16, heads, head_dim, 2, 2)
    st = Stream(heads * head_dim)
    gpu = B200Backend(cfg, dtype="bf16")
    gpu.set_copy_engine("bulk")
    pk, pv = gpu.planes()
    g = torch.Generator(device=cuda).manual_seed(heads * head_dim)
    pk.copy_(torch.randn(pk.shape, device=cuda, generator=g).to(torch.bfloat16))
    pv.copy_(torch.randn(pv.shape, device=cuda, generator=g).to(torch.bfloat16))
    ids = st.permutation(cfg.num_blocks)
    pairs = np.stack([ids[:560], ids[560:1120]], 1)
    pairs[7, 1] = pairs[7, 0]  # one self-copy
    want_k, want_v = pk.clone(), pv.clone()
    src = torch.from_numpy(pairs[:, 0].astype(np.int64)).to(cuda)
    dst = torch.from_numpy(pairs[:, 1].astype(np.int64)).to(cuda)
    want_k[:, dst] = want_k[:, src]
    want_v[:, dst] = want_v[:, src]
    gpu.copy_blocks_dev(torch.from_numpy(pairs.astype(np.int64)).to(cuda))
    torch.cuda.synchronize()
    assert gpu.device_error() is None
    assert torch.equal(pk.view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(pv.view(torch.int16), want_v.view(torch.int16))


def test_bulk_engine_flags_out_of_pool_pairs(cuda):
    import torch

    cfg = CacheConfig(40, 16, 2, 64, 3, 2)
    st = Stream(9)
    cpu, gpu = OracleBackend(cfg), B200Backend(cfg, dtype="bf16")
    gpu.set_copy_engine("bulk")
    e = cfg.entry_elems()
    for layer in range(cfg.num_layers):
        dsts = [(blk, s) for blk in range(cfg.num_blocks) for s in range(cfg.block_size)]
        k = bf16_bits_to_f32(f32_to_bf16_bits(st.normal(len(dsts) * e)))
        cpu.write_kv_batch(layer, dsts, k, -k)
        gpu.write_kv_batch(layer, dsts, k, -k)
    gpu.copy_blocks_dev(torch.tensor([[1, 2], [3, 99], [4, 5]], dtype=torch.int64, device=cuda))
    cpu.copy_blocks([(1, 2), (4, 5)])  # the device path skips the bad pair and carries on
    err = gpu.device_error()
    assert err is not None and err[1] == 1
    assert_pools_equal(gpu, cpu)


def test_bulk_engine_rejects_unaligned_planes(cuda):
    # block_size 3 x entry 3 x 2 bytes = 18-byte planes: not a multiple of 16.
    b = B200Backend(CacheConfig(8, 3, 1, 3, 1, 2), dtype="bf16")
    with pytest.raises(CacheError):
        b.set_copy_engine("bulk")
    b.copy_blocks([(0, 1)])  # still on the register engine
    with pytest.raises(KeyError):
        b.set_copy_engine("dma")


@pytest.mark.parametrize("heads,head_dim", [(4, 128), (12, 128), (1, 64)])
def test_bulk_engine_zero_blocks(cuda, heads, head_dim):
    """zero_blocks through bulk stores of a zeroed shared-memory run: 16, 48
    (two 24 KiB runs) and 2 KiB block planes, many items per issuing lane,
    repeated ids, and an id outside the pool that is recorded and skipped."""
    import torch

    cfg = CacheConfig(1200, 16, heads, head_dim, 3, 2)
    st = Stream(heads * head_dim + 1)
    gpu = B200Backend(cfg, dtype="bf16")
    gpu.set_copy_engine("bulk")
    pk, pv = gpu.planes()
    g = torch.Generator(device=cuda).manual_seed(heads + head_dim)
    pk.copy_(torch.randn(pk.shape, device=cuda, generator=g).to(torch.bfloat16))
    pv.copy_(torch.randn(pv.shape, device=cuda, generator=g).to(torch.bfloat16))
    ids = st.permutation(cfg.num_blocks)[:700].astype(np.int64)
    ids[10] = ids[11]  # a repeated id
    want_k, want_v = pk.clone(), pv.clone()
    good = torch.from_numpy(ids).to(cuda)
    want_k[:, good] = 0
    want_v[:, good] = 0
    with_bad = np.concatenate([ids[:300], [cfg.num_blocks + 5], ids[300:]])
    gpu.zero_blocks_dev(torch.from_numpy(with_bad).to(cuda))
    torch.cuda.synchronize()
    err = gpu.device_error()
    assert err is not None and err[1] == 300
    assert torch.equal(pk.view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(pv.view(torch.int16), want_v.view(torch.int16))
    # The host-buffer path on the same engine.
    more = [int(b) for b in st.permutation(cfg.num_blocks)[:5]]
    gpu.zero_blocks(more)
    torch.cuda.synchronize()
    assert gpu.device_error() is None
    want_k[:, more] = 0
    want_v[:, more] = 0
    assert torch.equal(pk.view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(pv.view(torch.int16), want_v.view(torch.int16))
