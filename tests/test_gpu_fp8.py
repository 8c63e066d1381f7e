"""fp8 (E4M3) pools on the device, bit-exact against the oracle.

Every write path into an fp8 pool -- the trait's host-buffer writes, the
per-layer and all-layer device scatter, and the fused slot resolution +
scatter -- is compared code for code with oracle/pkv_oracle.c in fp8 mode
(E4M3(x * (1/scale)) per layer and kv head), including saturation,
subnormals, per-head scales, shards that split a head, and the scalar
fallback for heads that are not a multiple of 16 elements.
"""

import numpy as np
import pytest

from oracle import host_ref as H
from oracle.cpu import OracleBackend, e4m3_from_f32, resolve_slots
from pagedkv import B200Backend, CacheConfig
from pagedkv.errors import CacheError, ShapeMismatch
from pagedkv.workloads import Stream, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def dev_codes(b):
    k, v = b.planes()
    import torch
    return k.view(torch.uint8).cpu().numpy(), v.view(torch.uint8).cpu().numpy()


def orc_codes(orc):
    """The oracle's planes hold widened E4M3 values; re-encoding them is exact."""
    k, v = orc.planes()
    return e4m3_from_f32(k), e4m3_from_f32(v)


def assert_codes_equal(dev, orc):
    dk, dv = dev_codes(dev)
    ok, ov = orc_codes(orc)
    np.testing.assert_array_equal(dk, ok)
    np.testing.assert_array_equal(dv, ov)


def scales(cfg, seed):
    st = Stream(seed)
    n = cfg.num_layers * cfg.num_kv_heads
    k = st.uniform(n, 0.02, 3.0).astype(np.float32).reshape(cfg.num_layers, cfg.num_kv_heads)
    v = st.uniform(n, 0.02, 3.0).astype(np.float32).reshape(cfg.num_layers, cfg.num_kv_heads)
    return k, v


def rows(st, n, spread=6.0):
    """f32 rows with a wide magnitude range: saturating, normal and subnormal codes."""
    return (st.normal(n) * np.exp(st.uniform(n, -9.0, spread))).astype(np.float32)


def pair(cfg, dtype="fp8_e4m3", seed=1, **kw):
    cpu, gpu = OracleBackend(cfg), B200Backend(cfg, dtype=dtype, **kw)
    ks, vs = scales(cfg, seed)
    cpu.set_fp8(ks, vs)
    gpu.set_kv_scales(ks, vs)
    return cpu, gpu, ks, vs


def test_every_bf16_value_quantises_as_the_oracle(cuda):
    """All 65,536 bf16 bit patterns through write_kv_batch (bf16 host rows)."""
    cfg = CacheConfig(64, 16, 4, 64, 2, 1)  # entry 256: 256 tokens x 256 = 65,536 values
    cpu, gpu, ks, vs = pair(cfg)
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    x = bf16_bits_to_f32(bits)
    nan = np.isnan(x)
    bits = np.where(nan, np.uint16(0), bits)  # NaN codes are checked separately
    e = cfg.entry_elems()
    dsts = [(t // 16, t % 16) for t in range(256)]
    for layer in range(2):
        kb = bits.reshape(256, e)
        vb = np.ascontiguousarray(kb[::-1])
        gpu.write_kv_batch(layer, dsts, kb.ravel(), vb.ravel(), host_dtype="bf16")
        cpu.write_kv_batch(layer, dsts, bf16_bits_to_f32(kb).ravel(), bf16_bits_to_f32(vb).ravel())
    assert_codes_equal(gpu, cpu)
    assert gpu.digest() == cpu.digest()


def test_nan_and_infinity(cuda):
    cfg = CacheConfig(4, 4, 1, 16, 1, 1)
    gpu = B200Backend(cfg, dtype="fp8_e4m3")
    x = np.array([np.nan, -np.nan, np.inf, -np.inf, 1e30, -1e30, 448, 464] + [0.5] * 8, np.float32)
    gpu.write_kv(0, (1, 2), x, -x)
    dk, dv = dev_codes(gpu)
    k, v = dk[0, 1, 2], dv[0, 1, 2]
    assert ((k[:2] & 0x7F) == 0x7F).all() and ((v[:2] & 0x7F) == 0x7F).all()
    np.testing.assert_array_equal(k[2:8], [0x7E, 0xFE, 0x7E, 0xFE, 0x7E, 0x7E])
    np.testing.assert_array_equal(v[2:8], [0xFE, 0x7E, 0xFE, 0x7E, 0xFE, 0xFE])


@pytest.mark.parametrize("head_dim", [32, 8])  # 8: the one-element-per-thread fallback
@pytest.mark.parametrize("seed", [1, 2])
def test_host_writes_copies_zeros_reads_match_oracle(cuda, head_dim, seed):
    cfg = CacheConfig(48, 16, 4, head_dim, 3, 1)
    cpu, gpu, ks, vs = pair(cfg, seed=seed)
    st = Stream(100 + seed)
    e = cfg.entry_elems()
    for step in range(12):
        layer = int(st.integers(1, 0, cfg.num_layers - 1)[0])
        t = int(st.integers(1, 1, 60)[0])
        dsts = list(zip(st.integers(t, 0, cfg.num_blocks - 1).tolist(),
                        st.integers(t, 0, cfg.block_size - 1).tolist()))
        k, v = rows(st, t * e), rows(st, t * e)
        if step == 5:
            dsts[t // 2] = (cfg.num_blocks + 1, 0)  # invalid mid-batch: prefix applied
        errs = []
        for b, kk, vv in ((gpu, k, v), (cpu, k, v)):
            try:
                b.write_kv_batch(layer, dsts, kk, vv)
                errs.append(None)
            except (CacheError, H.RefError) as ex:
                errs.append(ex.code)
        assert errs[0] == errs[1]
        if step % 4 == 3:
            ids = st.permutation(cfg.num_blocks)
            pairs = np.stack([ids[:6], ids[6:12]], 1)
            cpu.copy_blocks(pairs)
            gpu.copy_blocks(pairs)
            cpu.zero_blocks(ids[12:14])
            gpu.zero_blocks(ids[12:14])
    assert_codes_equal(gpu, cpu)
    assert gpu.digest() == cpu.digest()
    for d in [(0, 0), (7, 3), (47, 15)]:
        for layer in range(cfg.num_layers):
            a, b = cpu.read_entry(layer, d), gpu.read_entry(layer, d)
            np.testing.assert_array_equal(a[0].view(np.uint32), b[0].view(np.uint32))
            np.testing.assert_array_equal(a[1].view(np.uint32), b[1].view(np.uint32))


@pytest.mark.parametrize("src", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("all_layers", [True, False])
def test_device_scatter_quantises_as_the_oracle(cuda, src, all_layers):
    import torch

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[src]
    cfg = CacheConfig(96, 16, 2, 64, 5, 1)
    cpu, gpu, ks, vs = pair(cfg, seed=7)
    st = Stream(8)
    e, T = cfg.entry_elems(), 300
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:T].astype(np.int64)
    slots[17] = -1  # padding
    kx = torch.from_numpy(rows(st, cfg.num_layers * T * e).reshape(cfg.num_layers, T, e)).to(tdt)
    vx = torch.from_numpy(rows(st, cfg.num_layers * T * e).reshape(cfg.num_layers, T, e)).to(tdt)
    d_slots = torch.from_numpy(slots).to(cuda)
    kd, vd = kx.to(cuda), vx.to(cuda)
    if all_layers:
        gpu.reshape_and_cache(kd, vd, d_slots)
    else:
        for layer in range(cfg.num_layers):
            gpu.reshape_and_cache(kd[layer], vd[layer], d_slots, layer=layer)
    torch.cuda.synchronize()
    assert gpu.device_error() is None
    keep = slots >= 0
    dsts = [(int(s) // 16, int(s) % 16) for s in slots[keep]]
    for layer in range(cfg.num_layers):
        cpu.write_kv_batch(layer, dsts, kx[layer][keep].float().numpy().ravel(),
                           vx[layer][keep].float().numpy().ravel())
    assert_codes_equal(gpu, cpu)
    kdg, vdg = gpu.digest_rows(kd, vd, d_slots)
    assert (kdg, vdg) == gpu.digest() == cpu.digest()


@pytest.mark.parametrize("head_dim,shape", [(128, "ragged"), (8, "ragged"), (128, "decode"),
                                            (128, "decode_mixed"), (8, "decode")])
def test_fused_resolve_and_quantise_matches_oracle(cuda, head_dim, shape):
    """Ragged batches, and one-token-per-sequence batches: the decode form
    (every new_lens 1) and its fallback to the general form (lengths that
    also sum to the sequence count), over 5 layers so that the layers past
    the prefetched ones are quantised too."""
    import torch

    cfg = CacheConfig(2048, 16, 4, head_dim, 5, 1)
    cpu, gpu, ks, vs = pair(cfg, seed=11)
    st = Stream(12)
    s = 40
    ctx = st.integers(s, 0, 200).astype(np.int32)
    if shape == "ragged":
        new = st.integers(s, 1, 180).astype(np.int32)
        new[::7] = 0
    else:
        new = np.ones(s, np.int32)
        if shape == "decode_mixed":
            new[0], new[1] = 2, 0
    need = -(-(ctx + new) // 16)
    stride = int(need.max())
    perm = st.permutation(cfg.num_blocks)
    tables = np.full((s, stride), -1, np.int32)
    pos = 0
    for q in range(s):
        tables[q, : need[q]] = perm[pos:pos + need[q]]
        pos += need[q]
    t = int(new.sum())
    rc, cu, slots = resolve_slots(tables, ctx, new, t, 16, cfg.num_blocks)
    assert rc == 0
    e = cfg.entry_elems()
    kx = torch.from_numpy(rows(st, cfg.num_layers * t * e).reshape(cfg.num_layers, t, e)).to(torch.bfloat16)
    vx = torch.from_numpy(rows(st, cfg.num_layers * t * e).reshape(cfg.num_layers, t, e)).to(torch.bfloat16)
    d_cu = torch.zeros(s + 1, dtype=torch.int32, device=cuda)
    d_sl = torch.zeros(t, dtype=torch.int64, device=cuda)
    gpu.resolve_and_cache(torch.from_numpy(tables).to(cuda), torch.from_numpy(ctx).to(cuda),
                          torch.from_numpy(new).to(cuda), t, d_cu, kx.to(cuda), vx.to(cuda),
                          slots_out=d_sl)
    torch.cuda.synchronize()
    assert gpu.device_error() is None
    np.testing.assert_array_equal(d_cu.cpu().numpy(), cu)
    np.testing.assert_array_equal(d_sl.cpu().numpy(), slots)
    dsts = [(int(x) // 16, int(x) % 16) for x in slots]
    for layer in range(cfg.num_layers):
        cpu.write_kv_batch(layer, dsts, kx[layer].float().numpy().ravel(), vx[layer].float().numpy().ravel())
    assert_codes_equal(gpu, cpu)


@pytest.mark.parametrize("shards", [2, 8])
def test_fp8_shards_reassemble_to_the_oracle_pool(cuda, shards):
    """With 8 shards of 4 heads x 64, each shard holds half a head: the scale
    index comes from the shard's offset in the full entry."""
    import torch

    cfg = CacheConfig(32, 16, 4, 64, 2, 1)
    e, w = cfg.entry_elems(), cfg.entry_elems() // shards
    cpu = OracleBackend(cfg)
    ks, vs = scales(cfg, 21)
    cpu.set_fp8(ks, vs)
    backs = [B200Backend(cfg, dtype="fp8_e4m3", shard_rank=r, num_shards=shards) for r in range(shards)]
    for b in backs:
        b.set_kv_scales(ks, vs)
    st = Stream(22)
    for layer in range(cfg.num_layers):
        slots = st.permutation(cfg.num_blocks * cfg.block_size)[:100]
        dsts = [(int(x) // 16, int(x) % 16) for x in slots]
        k = f32_to_bf16_bits(rows(st, 100 * e)).reshape(100, e)
        v = f32_to_bf16_bits(rows(st, 100 * e)).reshape(100, e)
        cpu.write_kv_batch(layer, dsts, bf16_bits_to_f32(k).ravel(), bf16_bits_to_f32(v).ravel())
        for r, b in enumerate(backs):
            b.write_kv_batch(layer, dsts, k[:, r * w:(r + 1) * w].copy(), v[:, r * w:(r + 1) * w].copy(),
                             host_dtype="bf16")
    ok, ov = orc_codes(cpu)
    parts = [dev_codes(b) for b in backs]
    np.testing.assert_array_equal(np.concatenate([p[0] for p in parts], -1), ok)
    np.testing.assert_array_equal(np.concatenate([p[1] for p in parts], -1), ov)
    kd = sum(b.digest()[0] for b in backs) % (1 << 64)
    vd = sum(b.digest()[1] for b in backs) % (1 << 64)
    assert (kd, vd) == cpu.digest()
    for r, b in enumerate(backs):  # reads dequantise with the right head's scale
        got_k, got_v = b.read_entry(1, dsts[3])
        want_k, want_v = cpu.read_entry(1, dsts[3])
        np.testing.assert_array_equal(got_k, want_k[r * w:(r + 1) * w])
        np.testing.assert_array_equal(got_v, want_v[r * w:(r + 1) * w])


def test_e4m3_rows_move_unchanged_and_only_into_fp8_pools(cuda):
    import torch

    cfg = CacheConfig(8, 4, 2, 16, 2, 1)
    gpu = B200Backend(cfg, dtype="fp8_e4m3")
    codes = np.arange(64, dtype=np.uint8).reshape(2, 32)
    gpu.write_kv_batch(1, [(3, 1), (5, 2)], codes.ravel(), codes[::-1].ravel())
    dk, dv = dev_codes(gpu)
    np.testing.assert_array_equal(dk[1, 3, 1], codes[0])
    np.testing.assert_array_equal(dv[1, 5, 2], codes[0])
    raw_k, raw_v = np.zeros(32, np.uint8), np.zeros(32, np.uint8)
    gpu.read_kv(1, (5, 2), raw_k, raw_v)
    np.testing.assert_array_equal(raw_k, codes[1])
    bf = B200Backend(CacheConfig(8, 4, 2, 16, 2, 2), dtype="bf16")
    with pytest.raises(CacheError):
        bf.write_kv(0, (0, 0), codes[0], codes[1])
    with pytest.raises(CacheError):
        bf.set_kv_scales(np.ones((2, 2)), np.ones((2, 2)))
    d = torch.from_numpy(codes).to(cuda).view(torch.float8_e4m3fn)
    gpu.reshape_and_cache(d, d, torch.tensor([0, 31], dtype=torch.int64, device=cuda), layer=0)
    torch.cuda.synchronize()
    dk, _ = dev_codes(gpu)
    np.testing.assert_array_equal(dk[0, 7, 3], codes[1])


def test_scale_validation(cuda):
    cfg = CacheConfig(8, 4, 2, 16, 2, 1)
    gpu = B200Backend(cfg, dtype="fp8_e4m3")
    with pytest.raises(ShapeMismatch):
        gpu.set_kv_scales(np.ones(3), np.ones(3))
    for bad in (0.0, -1.0, np.inf, np.nan, 1e-39):
        k = np.ones(4, np.float32)
        k[2] = bad
        with pytest.raises(CacheError):
            gpu.set_kv_scales(k, np.ones(4))
    gpu.set_kv_scales(np.full(4, 2.0), np.full(4, 0.5))
    gpu.write_kv(1, (2, 3), np.full(32, 3.0, np.float32), np.full(32, 3.0, np.float32))
    k, v = gpu.read_entry(1, (2, 3))
    np.testing.assert_array_equal(k, np.full(32, 3.0, np.float32))  # 1.5 * 2
    np.testing.assert_array_equal(v, np.full(32, 3.0, np.float32))  # 6 * 0.5


def test_device_name_of_an_fp8_pool(cuda):
    """KvBackend::device_name (backend.rs:123) names the pool dtype."""
    b = B200Backend(CacheConfig(8, 16, 2, 64, 1, 1), dtype="fp8_e4m3")
    name = b.device_name()
    assert "fp8_e4m3" in name and name.startswith("cuda:")
