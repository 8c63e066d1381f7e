"""The host stager behind the host-buffer writes (pkv_write_kv_batch): large
batches from pageable memory, and f32 rows for a bf16 pool, are copied or
narrowed to bf16 by worker threads into pinned chunks before they cross the
host link.

The trait's own call is write_kv_batch(&[f32]) (crates/paged-kv-core/src/
backend.rs:55-74) from ordinary memory. These tests hold that path, at sizes
that take many chunks of the ring per call, to:
- the CPU oracle (CpuBackend semantics) on bf16-representable rows, bit for bit;
- the device's own f32 -> bf16 conversion on every class of f32 value (ties,
  subnormals, infinities, values past the largest bf16, NaNs), bit for bit;
- the unstaged path (PKV_HOST_STAGING=off) and pinned rows;
- CpuBackend's error order and partial effects when a destination is bad.
"""

import numpy as np
import pytest

from oracle import host_ref as H
from oracle.cpu import OracleBackend
from pagedkv import B200Backend, CacheConfig, InvalidBlock
from pagedkv.workloads import Stream, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def planes_bits(b):
    import torch

    k, v = b.planes()
    return k.view(torch.int16).cpu().numpy(), v.view(torch.int16).cpu().numpy()


def special_f32(n, seed):
    """n f32 values: random bit patterns (NaNs and infinities among them) and
    every special class the narrowing must get right."""
    rng = np.random.default_rng(seed)
    bits = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32).copy()
    fmax = np.finfo(np.float32).max
    sp = np.array([0.0, -0.0, np.inf, -np.inf, fmax, -fmax, 1.00390625, 1.01171875,
                   -2.00390625, 3.0e-39, -3.0e-39, 1e-45, -1e-45, 3.3895e38, 3.39617e38,
                   3.3961e38, 1.0 + 2**-8, 1.0 + 3 * 2**-8], np.float32)
    nan = np.array([0x7fc00000, 0xffc00000, 0x7f800001, 0x7fbfffff, 0xff800001, 0x7fffffff,
                    0x7fc0ffff], np.uint32).view(np.float32)
    idx = rng.permutation(n)[: len(sp) + len(nan)]
    x[idx] = np.concatenate([sp, nan])
    return x


def test_host_narrowing_matches_device_conversion_on_every_class_of_value(cuda):
    import torch

    cfg = CacheConfig(num_blocks=1024, block_size=16, num_kv_heads=3, head_dim=40, num_layers=2,
                      dtype_bytes=2)
    e = cfg.entry_elems()
    t = 9000  # 4.3 MiB of f32 per plane: staged, in chunks that split rows
    st = Stream(8)
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:t].astype(np.int64)
    k = special_f32(t * e, 1).reshape(t, e)
    v = special_f32(t * e, 2).reshape(t, e)
    host = B200Backend(cfg, dtype="bf16")
    host.write_kv_batch_slots(1, slots // 16, slots % 16, k, v)  # pageable f32 rows
    dev = B200Backend(cfg, dtype="bf16")
    dev.reshape_and_cache(torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda),
                          torch.from_numpy(slots).to(cuda), layer=1)
    torch.cuda.synchronize()
    assert host.device_error() is None and dev.device_error() is None
    for a, b in zip(planes_bits(host), planes_bits(dev)):
        np.testing.assert_array_equal(a, b)
    # Non-NaN values also equal the oracle's round to nearest even.
    hk, _ = planes_bits(host)
    got = hk[1].reshape(-1, e)[slots].view(np.uint16)
    keep = ~np.isnan(k)
    np.testing.assert_array_equal(got[keep], f32_to_bf16_bits(k)[keep])
    assert np.all((got[~keep] & 0x7f80) == 0x7f80) and np.all(got[~keep] & 0x7f)


@pytest.mark.parametrize("host_dtype", ["f32", "bf16"])
def test_large_pageable_batches_match_the_oracle(cuda, host_dtype):
    """Three calls of 16,384 tokens x 512 elements (32 MiB of f32 rows per
    plane, 16 chunks each): every layer, bit for bit against CpuBackend."""
    cfg = CacheConfig(num_blocks=2048, block_size=16, num_kv_heads=4, head_dim=128, num_layers=3,
                      dtype_bytes=2)
    e = cfg.entry_elems()
    t = 16384
    st = Stream(31)
    b = B200Backend(cfg, dtype="bf16")
    cpu = OracleBackend(cfg)
    for layer in range(cfg.num_layers):
        slots = st.permutation(cfg.num_blocks * cfg.block_size)[:t].astype(np.int64)
        kb = f32_to_bf16_bits(st.normal(t * e)).reshape(t, e)
        vb = f32_to_bf16_bits(st.normal(t * e)).reshape(t, e)
        kf, vf = bf16_bits_to_f32(kb), bf16_bits_to_f32(vb)
        blocks, offs = slots // 16, slots % 16
        if host_dtype == "f32":
            b.write_kv_batch_slots(layer, blocks, offs, kf, vf)
        else:
            b.write_kv_batch_slots(layer, blocks, offs, kb, vb, host_dtype="bf16")
        cpu.write_kv_batch_pairs(layer, np.stack([blocks, offs], 1).astype(np.uint64), kf, vf)
    assert b.device_error() is None
    dk, dv = b.planes()
    ok, ov = cpu.planes()
    np.testing.assert_array_equal(dk.float().cpu().numpy().view(np.uint32), ok.view(np.uint32))
    np.testing.assert_array_equal(dv.float().cpu().numpy().view(np.uint32), ov.view(np.uint32))
    assert b.digest() == cpu.digest()


def test_staged_and_unstaged_paths_write_the_same_pool(cuda, monkeypatch):
    import torch

    cfg = CacheConfig(num_blocks=1024, block_size=16, num_kv_heads=2, head_dim=128, num_layers=2,
                      dtype_bytes=2)
    e = cfg.entry_elems()
    t = 6000
    st = Stream(77)
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:t].astype(np.int64)
    k = (st.normal(t * e) * 7).astype(np.float32).reshape(t, e)  # not bf16-representable
    v = (st.normal(t * e) * 7).astype(np.float32).reshape(t, e)
    pools = []
    for mode in ("auto", "off"):
        monkeypatch.setenv("PKV_HOST_STAGING", mode)
        b = B200Backend(cfg, dtype="bf16")
        b.write_kv_batch_slots(0, slots // 16, slots % 16, k, v)
        # Pinned bf16 rows of the same values: straight from the caller's buffer.
        kb = torch.from_numpy(f32_to_bf16_bits(v).view(np.int16)).pin_memory().numpy()
        b.write_kv_batch_slots(1, slots // 16, slots % 16, kb.view(np.uint16),
                               kb.view(np.uint16), host_dtype="bf16")
        assert b.device_error() is None
        pools.append(planes_bits(b))
        b.close()
    for a, c in zip(pools[0], pools[1]):
        np.testing.assert_array_equal(a, c)
    np.testing.assert_array_equal(pools[0][1][0], pools[0][1][1])  # V of layers 0 and 1 alike


def test_bad_destination_mid_batch_applies_the_prefix_like_cpubackend(cuda):
    cfg = CacheConfig(num_blocks=512, block_size=16, num_kv_heads=2, head_dim=64, num_layers=1,
                      dtype_bytes=2)
    e = cfg.entry_elems()
    t = 5000
    st = Stream(5)
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:t].astype(np.int64)
    blocks, offs = slots // 16, slots % 16
    blocks[3210] = cfg.num_blocks + 9
    k = bf16_bits_to_f32(f32_to_bf16_bits(st.normal(t * e))).reshape(t, e)
    v = bf16_bits_to_f32(f32_to_bf16_bits(st.normal(t * e))).reshape(t, e)
    b = B200Backend(cfg, dtype="bf16")
    cpu = OracleBackend(cfg)
    pairs = np.stack([blocks, offs], 1).astype(np.uint64)
    with pytest.raises(InvalidBlock) as ed:
        b.write_kv_batch_pairs(0, pairs, k, v)
    with pytest.raises(H.RefError) as eo:
        cpu.write_kv_batch_pairs(0, pairs, k, v)
    assert ed.value.code == eo.value.code
    assert tuple(ed.value.values) == tuple(eo.value.fields)[: len(ed.value.values)]
    dk, _ = b.planes()
    ok, _ = cpu.planes()
    np.testing.assert_array_equal(dk.float().cpu().numpy().view(np.uint32), ok.view(np.uint32))
    # The next call reuses the ring and the staging buffers.
    b.write_kv_batch_pairs(0, np.ascontiguousarray(pairs[:3210]), k[:3210] * 0, v[:3210] * 0)
    assert b.device_error() is None
    assert int(np.count_nonzero(b.planes()[0].float().cpu().numpy())) == 0


@pytest.mark.parametrize("pool,host", [("f16", "f32"), ("fp8_e4m3", "bf16"), ("f32", "f32")])
def test_staged_copies_for_other_pool_types_equal_the_unstaged_path(cuda, monkeypatch, pool, host):
    """Pageable rows the stager copies unchanged (no host narrowing) and the
    device then converts or quantises: the same pool as the direct path."""
    import torch

    nbytes = {"f16": 2, "fp8_e4m3": 1, "f32": 4}[pool]
    cfg = CacheConfig(num_blocks=512, block_size=16, num_kv_heads=2, head_dim=128, num_layers=2,
                      dtype_bytes=nbytes)
    e = cfg.entry_elems()
    t = 4000
    st = Stream(91)
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:t].astype(np.int64)
    k = (st.normal(t * e) * 2).astype(np.float32).reshape(t, e)
    v = (st.normal(t * e) * 2).astype(np.float32).reshape(t, e)
    if host == "bf16":
        k, v = f32_to_bf16_bits(k), f32_to_bf16_bits(v)
    pools = []
    for mode in ("auto", "off"):
        monkeypatch.setenv("PKV_HOST_STAGING", mode)
        b = B200Backend(cfg, dtype=pool)
        if pool == "fp8_e4m3":
            b.set_kv_scales(np.full((2, 2), 0.5, np.float32), np.full((2, 2), 0.25, np.float32))
        b.write_kv_batch_slots(1, slots // 16, slots % 16, k, v, host_dtype=host)
        assert b.device_error() is None
        pools.append([p.view(torch.uint8).cpu().numpy() for p in b.planes()])
        b.close()
    for a, c in zip(pools[0], pools[1]):
        np.testing.assert_array_equal(a, c)
    assert np.count_nonzero(pools[0][0]) > 0


def test_stager_settings_from_the_environment(cuda, monkeypatch):
    cfg = CacheConfig(num_blocks=16, block_size=16, num_kv_heads=1, head_dim=64, num_layers=1,
                      dtype_bytes=2)
    monkeypatch.setenv("PKV_HOST_THREADS", "3")
    assert B200Backend(cfg, dtype="bf16").host_threads() == 3
    monkeypatch.setenv("PKV_STAGE_SLOTS", "4")  # at most half the ring's chunks
    assert B200Backend(cfg, dtype="bf16").host_threads() == 2
