"""The config-2, -3 and -4 operations at their full sizes on the device, checked
through properties that hold at any size (the whole-pool oracle comparison of
the smaller cases does not fit a CPU at these sizes):

- slot resolution equals the C oracle's (oracle/pkv_oracle.c, the rule of
  BlockTable::slot_for_position, block_table.rs:97-101) token for token;
- every token lands exactly once: the plane digest of the pool (order
  independent, summed over elements) equals the digest the written rows
  predict, which holds because the pool starts at zero and the slots are
  distinct; a strided sample of rows is also compared bit for bit;
- copy_blocks and zero_blocks change exactly the destination blocks, in every
  layer and both planes: the whole pool is compared with a device copy
  updated by plain tensor indexing (cpu.rs:131-160 semantics).

Geometry: Qwen2-7B KV heads (28 layers, 4 KV heads x 128, bf16, block size
16) over a 32,768-block pool (30 GiB), as the benchmark configurations; and
config 5's 70B-like geometry over its 150 GB single-GPU pool.
"""

import numpy as np
import pytest

from oracle.cpu import resolve_slots as ref_resolve_slots
from pagedkv import B200Backend, CacheConfig
from pagedkv.workloads import Stream, decode_batch, prefill_chunk

pytestmark = pytest.mark.gpu

GEOM = dict(num_blocks=32768, block_size=16, num_kv_heads=4, head_dim=128, num_layers=28)


def _fused_step_holds_its_properties(cuda, batch, pool_dtype, cfg=None):
    import torch

    cfg = cfg or CacheConfig(dtype_bytes=1 if pool_dtype == "fp8_e4m3" else 2, **GEOM)
    b = B200Backend(cfg, dtype=pool_dtype)
    if pool_dtype == "fp8_e4m3":
        st = Stream(7)
        n = cfg.num_layers * cfg.num_kv_heads
        b.set_kv_scales(st.uniform(n, 0.5, 2.0).astype(np.float32),
                        st.uniform(n, 0.5, 2.0).astype(np.float32))
    L, E, T, S = cfg.num_layers, cfg.entry_elems(), batch.num_tokens, len(batch.new)
    g = torch.Generator(device=cuda).manual_seed(T)
    k = torch.randn((L, T, E), generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn((L, T, E), generator=g, device=cuda).to(torch.bfloat16)
    d_tab = torch.from_numpy(batch.tables).to(cuda)
    d_ctx = torch.from_numpy(batch.ctx).to(cuda)
    d_new = torch.from_numpy(batch.new).to(cuda)
    cu = torch.empty(S + 1, dtype=torch.int32, device=cuda)
    slots = torch.empty(T, dtype=torch.int64, device=cuda)
    b.resolve_and_cache(d_tab, d_ctx, d_new, T, cu, k, v, slots_out=slots)
    torch.cuda.synchronize()
    assert b.device_error() is None

    rc, want_cu, want_slots = ref_resolve_slots(batch.tables, batch.ctx, batch.new, T,
                                                cfg.block_size, cfg.num_blocks)
    assert rc == 0
    np.testing.assert_array_equal(cu.cpu().numpy(), want_cu)
    np.testing.assert_array_equal(slots.cpu().numpy(), want_slots)
    assert len(np.unique(want_slots)) == T

    assert b.digest() == b.digest_rows(k, v, slots)

    kp, vp = b.planes()
    sample = torch.arange(0, T, 997, device=cuda)
    s = slots[sample]
    for plane, rows in ((kp, k), (vp, v)):
        got = plane.view(L, -1, E)[:, s]
        if pool_dtype == "fp8_e4m3":
            assert torch.isfinite(got.float()).all()  # values checked through the digests
        else:
            assert torch.equal(got.view(torch.int16), rows[:, sample].view(torch.int16))
    del kp, vp, k, v
    b.close()
    torch.cuda.empty_cache()


@pytest.mark.parametrize("pool_dtype", ["bf16", "fp8_e4m3"])
def test_config3_prefill_chunk_full_size(cuda, pool_dtype):
    """65,536 tokens of 96 log-uniform prompts, shuffled free list, one launch."""
    batch = prefill_chunk(seed=0, num_prompts=96, budget=65536,
                          cfg=CacheConfig(dtype_bytes=2, **GEOM))
    assert batch.num_tokens == 65536
    _fused_step_holds_its_properties(cuda, batch, pool_dtype)


def test_config2_decode_step_full_size(cuda):
    """256 sequences with contexts U[1,4096] append one token each."""
    batch = decode_batch(seed=None, cfg=CacheConfig(dtype_bytes=2, **GEOM))
    _fused_step_holds_its_properties(cuda, batch, "bf16")


@pytest.mark.parametrize("engine", ["vector", "bulk"])
def test_config4_copy_and_zero_full_size(cuda, engine):
    """256 copy-on-write pairs (distinct blocks, no chains) across all 28
    layers, then zero_blocks on 64 other blocks, over a pool of random
    contents; the device result is compared with a device copy of the pool
    updated by tensor indexing."""
    import torch

    cfg = CacheConfig(dtype_bytes=2, **GEOM)
    b = B200Backend(cfg, dtype="bf16")
    b.set_copy_engine(engine)
    g = torch.Generator(device=cuda).manual_seed(4)
    planes = b.planes()
    for p in planes:
        for layer in range(cfg.num_layers):
            p[layer].copy_(torch.randn(p[layer].shape, generator=g, device=cuda).to(torch.bfloat16))
    st = Stream(44)
    ids = st.permutation(cfg.num_blocks)
    pairs = np.stack([ids[:256], ids[256:512]], 1).astype(np.int64)
    zero = ids[512:576].astype(np.int64)
    want = [p.clone() for p in planes]
    src = torch.from_numpy(pairs[:, 0]).to(cuda)
    dst = torch.from_numpy(pairs[:, 1]).to(cuda)
    z = torch.from_numpy(zero).to(cuda)
    for w in want:
        w[:, dst] = w[:, src]
        w[:, z] = 0
    b.copy_blocks_dev(torch.from_numpy(pairs).to(cuda))
    b.zero_blocks_dev(z)
    torch.cuda.synchronize()
    assert b.device_error() is None
    for p, w in zip(planes, want):
        assert torch.equal(p.view(torch.int16), w.view(torch.int16))
    del want, planes
    b.close()
    torch.cuda.empty_cache()


def test_config5_geometry_full_pool(cuda):
    """Config 5 on one GPU: 80 layers, 8 KV heads x 128, bf16, the 150 GB pool
    (28,610 blocks: 3.75e10 elements per plane, far past 2^31). One step of a
    16,384-token chunk of prompts (log-uniform 64..8192) written through the
    fused kernel into blocks drawn from the whole pool."""
    import torch

    cfg = CacheConfig(num_blocks=28610, block_size=16, num_kv_heads=8, head_dim=128,
                      num_layers=80, dtype_bytes=2)
    torch.cuda.empty_cache()  # the pool and its rows need 155 GB of the 183
    batch = prefill_chunk(seed=5, num_prompts=40, lo=64, hi=8192, budget=16384, cfg=cfg)
    assert batch.tables.max() > cfg.num_blocks * 3 // 4  # reaches the top of the pool
    _fused_step_holds_its_properties(cuda, batch, "bf16", cfg=cfg)
