"""Parity of the B200 data path with the CPU oracle, bit for bit.

Every test drives libpagedkv_b200.so through its C ABI (pagedkv.B200Backend)
and compares the whole pool, or the entries it touched, with
oracle/pkv_oracle.c (the restated CpuBackend) on the same seeded inputs.
The first three tests restate the reference's own GPU-vs-CPU tests
(crates/paged-kv-cuda/src/backend.rs:345-416), which never ran upstream.
"""

import numpy as np
import pytest

from oracle import host_ref as H
from oracle.cpu import OracleBackend, resolve_slots
from pagedkv import (B200Backend, CacheConfig, InvalidBlock, InvalidLayer, ShapeMismatch,
                     SlotOutOfRange)
from pagedkv.errors import CacheError
from pagedkv.workloads import Stream, bf16_bits_to_f32, config1, decode_batch, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def entry(seed, n):
    return np.array([seed + i * 0.25 for i in range(n)], dtype=np.float32)


def dev_planes_f32(b):
    k, v = b.planes()
    return k.float().cpu().numpy(), v.float().cpu().numpy()


def assert_pools_equal(dev, orc):
    dk, dv = dev_planes_f32(dev)
    ok, ov = orc.planes()
    assert dk.shape == ok.shape
    np.testing.assert_array_equal(dk.view(np.uint32), ok.view(np.uint32))
    np.testing.assert_array_equal(dv.view(np.uint32), ov.view(np.uint32))


def same_error(f_dev, f_orc):
    """Both raise; same variant and fields."""
    with pytest.raises(CacheError) as ed:
        f_dev()
    with pytest.raises(H.RefError) as eo:
        f_orc()
    assert ed.value.code == eo.value.code
    assert tuple(ed.value.values) == tuple(eo.value.fields)[: len(ed.value.values)]


# ---- the reference's CUDA oracle tests (cuda/src/backend.rs:345-416) -------------------


def test_constructs_and_reports_sane_metadata(cuda):
    cfg = CacheConfig.tiny(8)
    b = B200Backend(cfg)
    assert b.allocated_bytes() == cfg.total_bytes()
    assert b.device_name().startswith("cuda:")


def test_matches_cpu_oracle_on_scatter_write_then_read(cuda):
    cfg = CacheConfig.tiny(8)
    cpu, gpu = OracleBackend(cfg), B200Backend(cfg)
    n = cfg.entry_elems()
    dsts = [(0, 0), (0, 1), (3, 2)]
    k = np.arange(len(dsts) * n, dtype=np.float32) * 0.5
    v = np.arange(len(dsts) * n, dtype=np.float32) * 0.25 + 1.0
    for i, d in enumerate(dsts):
        cpu.write_kv(1, d, k[i * n:(i + 1) * n], v[i * n:(i + 1) * n])
    gpu.write_kv_batch(1, dsts, k, v)
    for d in dsts:
        for a, b in zip(cpu.read_entry(1, d), gpu.read_entry(1, d)):
            np.testing.assert_array_equal(a, b)
    assert_pools_equal(gpu, cpu)


def test_matches_cpu_oracle_on_copy_block(cuda):
    cfg = CacheConfig.tiny(8)
    cpu, gpu = OracleBackend(cfg), B200Backend(cfg)
    n = cfg.entry_elems()
    for layer in range(cfg.num_layers):
        for slot in range(cfg.block_size):
            seed = layer * 100 + slot
            k = np.arange(n, dtype=np.float32) + seed
            v = np.arange(n, dtype=np.float32) + seed + 0.5
            cpu.write_kv(layer, (2, slot), k, v)
            gpu.write_kv(layer, (2, slot), k, v)
    cpu.copy_block(2, 5)
    gpu.copy_block(2, 5)
    for layer in range(cfg.num_layers):
        for slot in range(cfg.block_size):
            for a, b in zip(cpu.read_entry(layer, (5, slot)), gpu.read_entry(layer, (5, slot))):
                np.testing.assert_array_equal(a, b)
    assert_pools_equal(gpu, cpu)


# ---- cpu.rs known answers on the device -------------------------------------------------


def test_cpu_rs_known_answers_hold_on_the_device(cuda):
    b = B200Backend(CacheConfig.tiny(8))
    n = 8
    b.write_kv(1, (3, 2), entry(1.0, n), entry(100.0, n))  # cpu.rs:179-192
    k, v = b.read_entry(1, (3, 2))
    assert (k == entry(1.0, n)).all() and (v == entry(100.0, n)).all()
    for layer, slot in [(1, (3, 1)), (1, (3, 3)), (1, (2, 2)), (1, (4, 2)), (0, (3, 2))]:
        assert not b.read_entry(layer, slot)[0].any()  # cpu.rs:194-216
    b.write_kv(0, (0, 0), entry(1.0, n), entry(2.0, n))  # cpu.rs:252-271
    b.copy_block(0, 1)
    b.write_kv(0, (0, 0), entry(9.0, n), entry(9.0, n))
    assert (b.read_entry(0, (1, 0))[0] == entry(1.0, n)).all()
    b.copy_block(1, 1)  # cpu.rs:297-310
    assert (b.read_entry(0, (1, 0))[1] == entry(2.0, n)).all()
    for layer in range(2):  # cpu.rs:273-295
        b.write_kv(layer, (2, 1), entry(5.0, n), entry(5.0, n))
    b.zero_block(2)
    for layer in range(2):
        assert not np.concatenate(b.read_entry(layer, (2, 1))).any()


def test_bad_addresses_and_shapes_are_rejected(cuda):  # cpu.rs:312-351
    cfg = CacheConfig.tiny(8)
    b = B200Backend(cfg)
    n = cfg.entry_elems()
    k = v = entry(0.0, n)
    with pytest.raises(InvalidLayer) as e:
        b.write_kv(99, (0, 0), k, v)
    assert e.value == InvalidLayer(99, cfg.num_layers)
    with pytest.raises(InvalidBlock) as e:
        b.write_kv(0, (99, 0), k, v)
    assert e.value == InvalidBlock(99, cfg.num_blocks)
    with pytest.raises(SlotOutOfRange) as e:
        b.write_kv(0, (0, 99), k, v)
    assert e.value == SlotOutOfRange(99, cfg.block_size)
    with pytest.raises(ShapeMismatch) as e:
        b.write_kv(0, (0, 0), k[: n - 1], v)
    assert e.value == ShapeMismatch(n, n - 1)
    with pytest.raises(ShapeMismatch) as e:  # cpu.rs:385-400
        b.write_kv_batch(0, [(0, 0), (0, 1)], np.zeros(n), np.zeros(2 * n))
    assert e.value == ShapeMismatch(2 * n, n)


def test_allocated_bytes_tracks_config(cuda):  # cpu.rs:353-358
    b = B200Backend(CacheConfig.llama_3_2_1b(512), dtype="bf16")
    assert b.allocated_bytes() == 512 * 16 * 32 * 1024


# ---- config 1 (the CpuBackend-runnable case), whole pool bit for bit ----------------------


@pytest.mark.parametrize("zero_batched", [False, True])
def test_config1_oracle_case_bit_exact(cuda, zero_batched):
    w = config1(seed=0)
    cpu, gpu = OracleBackend(w.cfg), B200Backend(w.cfg)
    bs = w.cfg.block_size
    for layer in range(w.cfg.num_layers):
        dsts = [(int(s) // bs, int(s) % bs) for s in w.slots]
        cpu.write_kv_batch(layer, dsts, w.k[layer].ravel(), w.v[layer].ravel())
        gpu.write_kv_batch(layer, dsts, w.k[layer].ravel(), w.v[layer].ravel())
    cpu.copy_blocks(w.pairs)
    gpu.copy_blocks(w.pairs)
    if zero_batched:
        cpu.zero_blocks(w.zero)
        gpu.zero_blocks(w.zero)
    else:
        for z in w.zero:
            cpu.zero_block(int(z))
            gpu.zero_block(int(z))
    assert_pools_equal(gpu, cpu)
    assert gpu.digest() == cpu.digest()


# ---- seeded random operation sequences, every dtype ----------------------------------------


def random_ops(seed, cfg, steps=40):
    """A seeded mix of batched writes (duplicates included), chained copy
    lists, zeros and invalid calls."""
    st = Stream(seed)
    e = cfg.entry_elems()
    ops = []
    for _ in range(steps):
        kind = int(st.integers(1, 0, 9)[0])
        if kind <= 4:
            t = int(st.integers(1, 0, 40)[0])
            layer = int(st.integers(1, 0, cfg.num_layers - 1)[0])
            blocks = st.integers(t, 0, cfg.num_blocks - 1)
            slots = st.integers(t, 0, cfg.block_size - 1)
            k = bf16_bits_to_f32(f32_to_bf16_bits(st.normal(t * e)))
            v = bf16_bits_to_f32(f32_to_bf16_bits(st.normal(t * e)))
            if kind == 4 and t > 0:  # an invalid token in the middle of the batch
                bad = int(st.integers(1, 0, t - 1)[0])
                blocks[bad] = cfg.num_blocks + 3
            ops.append(("write", layer, list(zip(blocks.tolist(), slots.tolist())), k, v))
        elif kind <= 6:
            p = int(st.integers(1, 0, 12)[0])
            ids = st.integers(2 * p, 0, cfg.num_blocks - 1).reshape(p, 2)  # chains, dups, self
            ops.append(("copy", ids))
        elif kind == 7:
            ops.append(("zero", st.integers(int(st.integers(1, 0, 5)[0]), 0, cfg.num_blocks - 1)))
        elif kind == 8:
            ops.append(("copy", np.array([[0, 1], [cfg.num_blocks, 2], [3, 4]])))
        else:
            ops.append(("zero", np.array([1, cfg.num_blocks + 1, 2])))
    return ops


def apply(b, op):
    kind = op[0]
    if kind == "write":
        _, layer, dsts, k, v = op
        b.write_kv_batch(layer, dsts, k, v)
    elif kind == "copy":
        b.copy_blocks(op[1])
    else:
        b.zero_blocks(op[1])


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("seed", [1, 2, 3])
def test_random_operation_sequences_match_oracle(cuda, dtype, seed):
    bytes_ = 4 if dtype == "f32" else 2
    cfg = CacheConfig(24, 4, 2, 8, 3, bytes_)
    cpu, gpu = OracleBackend(cfg), B200Backend(cfg, dtype=dtype)
    for op in random_ops(seed, cfg):
        if dtype == "f16" and op[0] == "write":
            # f16 holds every value these tests write exactly only after rounding to f16 first.
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
    assert gpu.digest() == cpu.digest()


def test_f32_writes_into_a_bf16_pool_round_to_nearest_even(cuda):
    cfg = CacheConfig(8, 4, 1, 64, 1, 2)
    b = B200Backend(cfg, dtype="bf16")
    x = Stream(11).normal(64).astype(np.float32)
    x[:4] = [1.00390625, 1.01171875, -2.00390625, 3.0e-39]  # exact ties and a subnormal
    b.write_kv(0, (1, 2), x, -x)
    k, v = b.read_entry(0, (1, 2))
    np.testing.assert_array_equal(k, bf16_bits_to_f32(f32_to_bf16_bits(x)))
    np.testing.assert_array_equal(v, bf16_bits_to_f32(f32_to_bf16_bits(-x)))


def test_bf16_host_data_is_copied_bit_for_bit(cuda):
    cfg = CacheConfig(8, 4, 2, 32, 2, 2)
    b = B200Backend(cfg, dtype="bf16")
    bits = f32_to_bf16_bits(Stream(5).normal(3 * 64))
    b.write_kv_batch(1, [(0, 1), (7, 3), (2, 0)], bits, bits[::-1].copy(), host_dtype="bf16")
    k = np.zeros(64, np.uint16)
    v = np.zeros(64, np.uint16)
    b.read_kv(1, (7, 3), k, v)
    np.testing.assert_array_equal(k, bits[64:128])


# ---- device entry points --------------------------------------------------------------------


def test_device_reshape_per_layer_and_all_layers_match_oracle(cuda):
    import torch

    cfg = CacheConfig(64, 16, 4, 32, 5, 2)
    e = cfg.entry_elems()
    st = Stream(21)
    t = 300
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:t].astype(np.int64)
    slots[7] = -1  # padding tokens are skipped
    slots[100] = -5
    kv = f32_to_bf16_bits(st.normal(2 * cfg.num_layers * t * e)).reshape(2, cfg.num_layers, t, e)
    cpu = OracleBackend(cfg)
    for layer in range(cfg.num_layers):
        keep = slots >= 0
        dsts = [(int(s) // 16, int(s) % 16) for s in slots[keep]]
        cpu.write_kv_batch(layer, dsts, bf16_bits_to_f32(kv[0, layer][keep]).ravel(),
                           bf16_bits_to_f32(kv[1, layer][keep]).ravel())
    d_kv = torch.from_numpy(kv.view(np.int16)).view(torch.bfloat16).to(cuda)
    d_slots = torch.from_numpy(slots).to(cuda)
    a = B200Backend(cfg, dtype="bf16")
    a.reshape_and_cache(d_kv[0], d_kv[1], d_slots)  # one launch, every layer
    b = B200Backend(cfg, dtype="bf16")
    for layer in range(cfg.num_layers):
        b.reshape_and_cache(d_kv[0, layer], d_kv[1, layer], d_slots, layer=layer)
    torch.cuda.synchronize()
    assert a.device_error() is None and b.device_error() is None
    assert_pools_equal(a, cpu)
    assert_pools_equal(b, cpu)


@pytest.mark.parametrize("tokens", [2000, 1150, 700])
def test_all_layer_scatter_at_70b_geometry_equals_per_layer_calls(cuda, tokens):
    """80 layers of 2 KiB entries (the churn trace's geometry), token counts
    of its decode steps: the all-layer launch (several waves at 2 CTAs per
    SM, every thread walking all 80 layers) must write the pool that 80
    per-layer launches write, and every row must land at its slot."""
    import torch

    cfg = CacheConfig(200, 16, 8, 128, 80, 2)
    e, L = cfg.entry_elems(), cfg.num_layers
    st = Stream(tokens)
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:tokens].astype(np.int64)
    slots[3] = -1  # a padding token
    g = torch.Generator(device=cuda).manual_seed(tokens)
    k = torch.randn((L, tokens, e), generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn((L, tokens, e), generator=g, device=cuda).to(torch.bfloat16)
    d_slots = torch.from_numpy(slots).to(cuda)
    a = B200Backend(cfg, dtype="bf16")
    a.reshape_and_cache(k, v, d_slots)
    b = B200Backend(cfg, dtype="bf16")
    for layer in range(L):
        b.reshape_and_cache(k[layer], v[layer], d_slots, layer=layer)
    torch.cuda.synchronize()
    assert a.device_error() is None and b.device_error() is None
    keep = torch.from_numpy(slots >= 0).to(cuda)
    for pa, pb, src in zip(a.planes(), b.planes(), (k, v)):
        assert torch.equal(pa.view(torch.int16), pb.view(torch.int16))
        flat = pa.view(L, -1, e)
        assert torch.equal(flat[:, d_slots[keep]], src[:, keep])
        assert int(torch.count_nonzero(flat.view(torch.int16))) == int(keep.sum()) * L * e - int(
            (src[:, keep].view(torch.int16) == 0).sum())
    a.close()
    b.close()


def test_device_reshape_reads_strided_rows_and_converts(cuda):
    import torch

    cfg = CacheConfig(16, 8, 2, 16, 2, 2)
    e = cfg.entry_elems()
    qkv = torch.randn(50, 3 * e, generator=torch.Generator().manual_seed(3)).to(cuda)
    k, v = qkv[:, e:2 * e], qkv[:, 2 * e:]  # views into a fused projection output
    slots = torch.arange(50, dtype=torch.int64, device=cuda) * 2 + 1
    b = B200Backend(cfg, dtype="bf16")
    b.reshape_and_cache(k, v, slots, layer=1)
    pk, pv = b.planes()
    flat_k = pk[1].reshape(-1, e)[slots]
    flat_v = pv[1].reshape(-1, e)[slots]
    assert torch.equal(flat_k, k.to(torch.bfloat16))
    assert torch.equal(flat_v, v.to(torch.bfloat16))
    assert torch.count_nonzero(pk[0]) == 0


def test_device_reshape_flags_out_of_pool_slots_without_writing(cuda):
    import torch

    cfg = CacheConfig(4, 4, 1, 16, 1, 4)
    b = B200Backend(cfg)
    k = torch.ones(3, 16, device=cuda)
    slots = torch.tensor([2, 16, 5], dtype=torch.int64, device=cuda)  # 16 slots in the pool
    b.reshape_and_cache(k, k, slots, layer=0)
    err = b.device_error()
    assert err is not None and err[1] == 1 and isinstance(err[0], InvalidBlock)
    pk, _ = b.planes()
    assert int(torch.count_nonzero(pk)) == 2 * 16
    assert b.device_error() is None  # reading clears the word


def test_device_copy_and_zero_match_oracle(cuda):
    import torch

    cfg = CacheConfig(40, 16, 2, 64, 3, 2)
    st = Stream(8)
    cpu, gpu = OracleBackend(cfg), B200Backend(cfg, dtype="bf16")
    e = cfg.entry_elems()
    for layer in range(cfg.num_layers):
        dsts = [(blk, s) for blk in range(cfg.num_blocks) for s in range(cfg.block_size)]
        k = bf16_bits_to_f32(f32_to_bf16_bits(st.normal(len(dsts) * e)))
        cpu.write_kv_batch(layer, dsts, k, -k)
        gpu.write_kv_batch(layer, dsts, k, -k)
    ids = st.permutation(cfg.num_blocks)
    pairs = np.stack([ids[:12], ids[12:24]], 1)  # distinct: no chains
    cpu.copy_blocks(pairs)
    gpu.copy_blocks_dev(torch.from_numpy(pairs.astype(np.int64)).to(cuda))
    zero = ids[24:30]
    cpu.zero_blocks(zero)
    gpu.zero_blocks_dev(torch.from_numpy(zero.astype(np.int64)).to(cuda))
    torch.cuda.synchronize()
    assert gpu.device_error() is None
    assert_pools_equal(gpu, cpu)
    gpu.copy_blocks_dev(torch.tensor([[1, 2], [3, 99]], dtype=torch.int64, device=cuda))
    err = gpu.device_error()
    assert err is not None and err[1] == 1


@pytest.mark.parametrize("case", ["decode", "ragged", "empty_seqs", "single", "no_seqs"])
def test_device_slot_resolution_matches_oracle(cuda, case):
    import torch

    cfg = CacheConfig(16384, 16, 1, 8, 1, 2)
    st = Stream({"decode": 1, "ragged": 2, "empty_seqs": 3, "single": 4, "no_seqs": 5}[case])
    if case == "decode":
        batch = decode_batch(seed=None, num_seqs=300, max_ctx=200, cfg=cfg)
        tables, ctx, new = batch.tables, batch.ctx, batch.new
    else:
        s = {"ragged": 150, "empty_seqs": 40, "single": 1, "no_seqs": 0}[case]
        ctx = st.integers(s, 0, 300).astype(np.int32)
        new = st.integers(s, 1, 500).astype(np.int32)
        if case == "empty_seqs":
            new[::3] = 0
        need = -(-(ctx + new) // 16)
        stride = int(need.max()) if s else 1
        perm = st.permutation(cfg.num_blocks)
        tables = np.full((s, stride), -1, np.int32)
        pos = 0
        for q in range(s):
            tables[q, : need[q]] = perm[pos:pos + need[q]]
            pos += need[q]
    t = int(new.sum())
    rc, cu, slots = resolve_slots(tables, ctx, new, t, 16, cfg.num_blocks)
    assert rc == 0
    b = B200Backend(cfg, dtype="bf16")
    d_cu = torch.full((len(ctx) + 1,), -9, dtype=torch.int32, device=cuda)
    d_slots = torch.full((max(t, 1),), -9, dtype=torch.int64, device=cuda)
    b.resolve_slots(torch.from_numpy(np.ascontiguousarray(tables)).to(cuda),
                    torch.from_numpy(ctx).to(cuda), torch.from_numpy(new).to(cuda), t, d_cu, d_slots)
    torch.cuda.synchronize()
    assert b.device_error() is None
    np.testing.assert_array_equal(d_cu.cpu().numpy(), cu)
    np.testing.assert_array_equal(d_slots[:t].cpu().numpy(), slots)
    if case == "decode":
        np.testing.assert_array_equal(slots, batch.slot_mapping())


def test_device_slot_resolution_flags_bad_inputs(cuda):
    import torch

    b = B200Backend(CacheConfig(64, 4, 1, 8, 1, 2), dtype="bf16")
    tables = torch.tensor([[0, 70]], dtype=torch.int32, device=cuda)
    cu = torch.zeros(2, dtype=torch.int32, device=cuda)
    slots = torch.zeros(3, dtype=torch.int64, device=cuda)
    ctx = torch.tensor([3], dtype=torch.int32, device=cuda)
    new = torch.tensor([3], dtype=torch.int32, device=cuda)
    b.resolve_slots(tables, ctx, new, 3, cu, slots)
    err = b.device_error()
    assert err is not None and err[1] in (1, 2)
    assert slots.tolist() == [3, -1, -1]
    b.resolve_slots(tables, ctx, new, 5, cu, slots)  # wrong total: nothing written
    err = b.device_error()
    assert isinstance(err[0], ShapeMismatch)


# ---- head-sharded pools (the multi-GPU layout, here on one GPU) ------------------------------


@pytest.mark.parametrize("shards", [2, 4, 8])
def test_head_shards_reassemble_to_the_oracle_pool(cuda, shards):
    cfg = CacheConfig(32, 16, 4, 32, 2, 2)
    e = cfg.entry_elems()
    w = e // shards
    st = Stream(shards)
    cpu = OracleBackend(cfg)
    backs = [B200Backend(cfg, dtype="bf16", shard_rank=r, num_shards=shards) for r in range(shards)]
    for layer in range(cfg.num_layers):
        slots = st.permutation(cfg.num_blocks * cfg.block_size)[:100]
        dsts = [(int(s) // 16, int(s) % 16) for s in slots]
        k = f32_to_bf16_bits(st.normal(100 * e)).reshape(100, e)
        v = f32_to_bf16_bits(st.normal(100 * e)).reshape(100, e)
        cpu.write_kv_batch(layer, dsts, bf16_bits_to_f32(k).ravel(), bf16_bits_to_f32(v).ravel())
        for r, b in enumerate(backs):
            b.write_kv_batch(layer, dsts, k[:, r * w:(r + 1) * w].copy(), v[:, r * w:(r + 1) * w].copy(),
                             host_dtype="bf16")
    pairs = np.array([[1, 30], [2, 31]])
    cpu.copy_blocks(pairs)
    cpu.zero_blocks([5, 6])
    for b in backs:
        b.copy_blocks(pairs)
        b.zero_blocks([5, 6])
    ok, ov = cpu.planes()
    parts = [dev_planes_f32(b) for b in backs]
    np.testing.assert_array_equal(np.concatenate([p[0] for p in parts], -1), ok)
    np.testing.assert_array_equal(np.concatenate([p[1] for p in parts], -1), ov)
    kd = sum(b.digest()[0] for b in backs) % (1 << 64)
    vd = sum(b.digest()[1] for b in backs) % (1 << 64)
    assert (kd, vd) == cpu.digest()


@pytest.mark.parametrize("src", ["bf16", "f32"])
def test_rows_digest_predicts_the_pool_digest(cuda, src):
    """pkv_digest_rows_dev (used to verify shards without reading pools back)
    equals pkv_digest of the pool the rows were written into."""
    import torch

    cfg = CacheConfig(64, 16, 4, 32, 3, 2)
    e = cfg.entry_elems()
    st = Stream(31)
    slots = torch.from_numpy(st.permutation(cfg.num_blocks * cfg.block_size)[:500].astype(np.int64)).to(cuda)
    slots[9] = -1
    dt = torch.bfloat16 if src == "bf16" else torch.float32
    k = torch.randn((cfg.num_layers, 500, e), device=cuda).to(dt)
    v = torch.randn((cfg.num_layers, 500, e), device=cuda).to(dt)
    for shards in (1, 2):
        digs, rows = [], []
        for r in range(shards):
            w = e // shards
            b = B200Backend(cfg, dtype="bf16", shard_rank=r, num_shards=shards)
            ks, vs = k[..., r * w:(r + 1) * w], v[..., r * w:(r + 1) * w]
            b.reshape_and_cache(ks, vs, slots)
            digs.append(b.digest())
            rows.append(b.digest_rows(ks, vs, slots))
            assert digs[-1] == rows[-1]
        if shards == 1:
            whole = digs[0]
        else:
            assert tuple(sum(d[i] for d in digs) % 2**64 for i in range(2)) == whole


def test_offsets_beyond_2_31_elements_per_plane(cuda):
    """A plane of 80 layers x 2,048 blocks x 16 slots x 1,024 elements holds
    2.7e9 elements (> 2^31): the last layer's last block must be addressed
    exactly, through every entry point."""
    import torch

    cfg = CacheConfig(num_blocks=2048, block_size=16, num_kv_heads=8, head_dim=128, num_layers=80,
                      dtype_bytes=2)
    assert cfg.num_layers * cfg.layer_elems() > 2**31
    b = B200Backend(cfg, dtype="bf16")
    e = cfg.entry_elems()
    st = Stream(55)
    bits = f32_to_bf16_bits(st.normal(2 * 3 * e)).reshape(2, 3, e)
    dsts = [(2047, 15), (2047, 0), (1500, 7)]
    b.write_kv_batch(79, dsts, bits[0].ravel(), bits[1].ravel(), host_dtype="bf16")
    for i, d in enumerate(dsts):
        k = np.zeros(e, np.uint16)
        v = np.zeros(e, np.uint16)
        b.read_kv(79, d, k, v)
        assert (k == bits[0, i]).all() and (v == bits[1, i]).all()
    b.copy_blocks([(2047, 2046)])
    k = np.zeros(e, np.uint16)
    b.read_kv(79, (2046, 15), k, np.zeros(e, np.uint16))
    assert (k == bits[0, 0]).all()
    # Device path, all layers, into the last block.
    rows = torch.randn((80, 2, e), device=cuda).to(torch.bfloat16)
    slots = torch.tensor([2047 * 16 + 3, 2047 * 16 + 4], dtype=torch.int64, device=cuda)
    b.reshape_and_cache(rows, rows, slots)
    pk, _ = b.planes()
    assert torch.equal(pk[79, 2047, 3:5], rows[79])
    assert torch.equal(pk[0, 2047, 3:5], rows[0])
    b.zero_blocks([2047])
    assert int(torch.count_nonzero(pk[:, 2047])) == 0
    assert b.device_error() is None


def test_empty_device_calls_launch_nothing_and_succeed(cuda):
    import torch

    b = B200Backend(CacheConfig(8, 4, 1, 8, 2, 2), dtype="bf16")
    z64 = torch.zeros(0, dtype=torch.int64, device=cuda)
    e = torch.zeros((0, 8), dtype=torch.bfloat16, device=cuda)
    b.reshape_and_cache(e, e, z64, layer=0)
    b.copy_blocks_dev(z64.view(0, 2) if z64.numel() else torch.zeros((0, 2), dtype=torch.int64, device=cuda))
    b.zero_blocks_dev(z64)
    b.write_kv_batch(1, [], np.zeros(0, np.float32), np.zeros(0, np.float32))
    b.copy_blocks([])
    b.zero_blocks([])
    cu = torch.full((1,), 7, dtype=torch.int32, device=cuda)
    z32 = torch.zeros(0, dtype=torch.int32, device=cuda)
    b.resolve_slots(torch.zeros((0, 1), dtype=torch.int32, device=cuda), z32, z32, 0, cu,
                    torch.zeros(1, dtype=torch.int64, device=cuda))
    torch.cuda.synchronize()
    assert cu.item() == 0 and b.device_error() is None
    pk, pv = b.planes()
    assert int(torch.count_nonzero(pk)) == 0 and int(torch.count_nonzero(pv)) == 0


@pytest.mark.parametrize("case", ["prefill", "decode", "per_layer", "no_slot_output", "sharded"])
def test_fused_resolve_and_cache_equals_resolve_then_reshape(cuda, case):
    """pkv_resolve_and_cache_dev (slots resolved inside the scatter) gives the
    pool, cu_seqlens and slot mapping of pkv_resolve_slots_dev followed by
    pkv_reshape_and_cache_dev, and the oracle's pool."""
    import torch

    cfg = CacheConfig(4096, 16, 4, 32, 4, 2)
    e = cfg.entry_elems()
    st = Stream({"prefill": 1, "decode": 2, "per_layer": 3, "no_slot_output": 4, "sharded": 5}[case])
    if case == "decode":
        batch = decode_batch(seed=None, num_seqs=200, max_ctx=500, cfg=cfg)
    else:
        from pagedkv.workloads import prefill_chunk
        batch = prefill_chunk(seed=int(st.integers(1, 0, 100)[0]), num_prompts=30, lo=16, hi=600,
                              budget=5000, cfg=cfg)
    t = batch.num_tokens
    shards = 2 if case == "sharded" else 1
    w = e // shards
    kv = f32_to_bf16_bits(st.normal(2 * cfg.num_layers * t * e)).reshape(2, cfg.num_layers, t, e)
    d_kv = torch.from_numpy(kv.view(np.int16)).view(torch.bfloat16).to(cuda)
    tab = torch.from_numpy(batch.tables).to(cuda)
    ctx = torch.from_numpy(batch.ctx).to(cuda)
    new = torch.from_numpy(batch.new).to(cuda)
    layer = 2 if case == "per_layer" else None
    for r in range(shards):
        ks, vs = d_kv[0, ..., r * w:(r + 1) * w], d_kv[1, ..., r * w:(r + 1) * w]
        if layer is not None:
            ks, vs = ks[layer], vs[layer]
        ref = B200Backend(cfg, dtype="bf16", shard_rank=r, num_shards=shards)
        cu_ref = torch.empty(len(batch.new) + 1, dtype=torch.int32, device=cuda)
        sl_ref = torch.empty(t, dtype=torch.int64, device=cuda)
        ref.resolve_slots(tab, ctx, new, t, cu_ref, sl_ref)
        ref.reshape_and_cache(ks, vs, sl_ref, layer=layer)
        fus = B200Backend(cfg, dtype="bf16", shard_rank=r, num_shards=shards)
        cu = torch.full_like(cu_ref, -1)
        sl = None if case == "no_slot_output" else torch.full_like(sl_ref, -9)
        fus.resolve_and_cache(tab, ctx, new, t, cu, ks, vs, layer=layer, slots_out=sl)
        torch.cuda.synchronize()
        assert ref.device_error() is None and fus.device_error() is None
        assert torch.equal(cu, cu_ref)
        if sl is not None:
            assert torch.equal(sl, sl_ref)
        for a, b in zip(fus.planes(), ref.planes()):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    if shards == 1 and layer is None:
        cpu = OracleBackend(cfg)
        slots = batch.slot_mapping()
        dsts = [(int(x) // 16, int(x) % 16) for x in slots]
        for l in range(cfg.num_layers):
            cpu.write_kv_batch(l, dsts, bf16_bits_to_f32(kv[0, l]).ravel(), bf16_bits_to_f32(kv[1, l]).ravel())
        assert_pools_equal(fus, cpu)


@pytest.mark.parametrize("case", ["ones", "mixed_lengths", "bad_block", "past_table",
                                  "negative_ctx"])
def test_decode_form_of_the_fused_step_matches_the_general_form(cuda, case):
    """With one token per sequence (num_tokens == num_seqs) the fused step
    takes its decode form: no length scan when every new_lens is 1, the
    general scan otherwise (lengths such as [2, 0, 1, ...] that also sum to
    the sequence count, or a negative context). Pools, cu_seqlens, slots and
    the recorded error must equal resolve_slots + reshape_and_cache."""
    import torch

    cfg = CacheConfig(2048, 16, 2, 64, 5, 2)
    e = cfg.entry_elems()
    st = Stream(70)
    batch = decode_batch(seed=None, num_seqs=96, max_ctx=300, cfg=cfg)
    tables, ctx, new = batch.tables.copy(), batch.ctx.copy(), batch.new.copy()
    if case == "mixed_lengths":
        new[0], new[1] = 2, 0  # still 96 tokens for 96 sequences
        need = -(-(ctx[0] + 2) // 16)
        if tables[0, need - 1] < 0:
            tables[0, need - 1] = int(np.setdiff1d(np.arange(cfg.num_blocks), tables)[0])
    elif case == "bad_block":
        q = 7
        tables[q, int(ctx[q]) // 16] = cfg.num_blocks + 3
    elif case == "past_table":
        q = 11
        ctx[q] = tables.shape[1] * 16  # its new token's block is past the table
    elif case == "negative_ctx":
        ctx[5] = -1
    t = int(new.sum())
    assert t == len(new)
    kv = f32_to_bf16_bits(st.normal(2 * cfg.num_layers * t * e)).reshape(2, cfg.num_layers, t, e)
    d_kv = torch.from_numpy(kv.view(np.int16)).view(torch.bfloat16).to(cuda)
    tab, dctx, dnew = (torch.from_numpy(x).to(cuda) for x in (tables, ctx, new))
    ref = B200Backend(cfg, dtype="bf16")
    cu_ref = torch.full((len(new) + 1,), -5, dtype=torch.int32, device=cuda)
    sl_ref = torch.full((t,), -9, dtype=torch.int64, device=cuda)
    ref.resolve_slots(tab, dctx, dnew, t, cu_ref, sl_ref)
    torch.cuda.synchronize()
    err_ref = ref.device_error()
    if case != "negative_ctx":
        ref.reshape_and_cache(d_kv[0], d_kv[1], sl_ref)
    fus = B200Backend(cfg, dtype="bf16")
    cu = torch.full_like(cu_ref, -5)
    sl = torch.full_like(sl_ref, -9)
    fus.resolve_and_cache(tab, dctx, dnew, t, cu, d_kv[0], d_kv[1], slots_out=sl)
    torch.cuda.synchronize()
    err = fus.device_error()
    if case in ("ones", "mixed_lengths"):
        assert err is None and err_ref is None
    else:
        assert err is not None and err_ref is not None
        assert type(err[0]) is type(err_ref[0]) and err[1] == err_ref[1]
    if case == "negative_ctx":  # nothing is written; cu_seqlens is still published
        assert torch.equal(cu, cu_ref)
        for p_ in fus.planes():
            assert int(torch.count_nonzero(p_)) == 0
        return
    assert torch.equal(cu, cu_ref)
    assert torch.equal(sl, sl_ref)
    assert ref.device_error() is None
    for a, b in zip(fus.planes(), ref.planes()):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("form", ["decode", "general"])
def test_consecutive_fused_steps_keep_stream_order(cuda, form):
    """The fused step kernels are launched as programmatic dependents of the
    previous grid in their stream and wait for it before touching memory.
    Eight steps on one stream write the same slots: with a torch kernel
    rewriting the source rows before each step (and a torch gather of the
    written rows after it), every step must write the rows copied just before
    it; back to back, eagerly and replayed from a CUDA graph, the pool must
    end with the last step's rows."""
    import torch

    cfg = CacheConfig(1024, 16, 2, 64, 4, 2)
    e, L = cfg.entry_elems(), cfg.num_layers
    batch = decode_batch(seed=None, num_seqs=64, max_ctx=300, cfg=cfg)
    tables, ctx, new = batch.tables.copy(), batch.ctx.copy(), batch.new.copy()
    if form == "general":  # still one token per sequence on average: the scan runs
        new[0], new[1] = 2, 0
        need = -(-(ctx[0] + 2) // 16)
        if tables[0, need - 1] < 0:
            tables[0, need - 1] = int(np.setdiff1d(np.arange(cfg.num_blocks), tables)[0])
    t, steps = int(new.sum()), 8
    tab, dctx, dnew = (torch.from_numpy(x).to(cuda) for x in (tables, ctx, new))
    g = torch.Generator(device=cuda).manual_seed(31)
    src = torch.randn((steps, 2, L, t, e), generator=g, device=cuda).to(torch.bfloat16)
    b = B200Backend(cfg, dtype="bf16")
    cu = torch.empty(len(new) + 1, dtype=torch.int32, device=cuda)
    sl = torch.empty(t, dtype=torch.int64, device=cuda)
    b.resolve_and_cache(tab, dctx, dnew, t, cu, src[0, 0], src[0, 1], slots_out=sl)
    torch.cuda.synchronize()
    assert b.device_error() is None
    kp, vp = (x.view(L, -1, e) for x in b.planes())

    def rows():
        return torch.stack([kp[:, sl], vp[:, sl]])

    stream = torch.cuda.Stream()
    k = torch.empty_like(src[0, 0])
    v = torch.empty_like(src[0, 1])
    snaps = []
    with torch.cuda.stream(stream):
        for i in range(steps):
            k.copy_(src[i, 0])
            v.copy_(src[i, 1])
            b.resolve_and_cache(tab, dctx, dnew, t, cu, k, v, slots_out=sl, stream=stream)
            snaps.append(rows())
    stream.synchronize()
    for i in range(steps):
        assert torch.equal(snaps[i], src[i]), f"step {i}"
    for order in (list(range(steps)), list(reversed(range(steps)))):
        last = order[-1]
        with torch.cuda.stream(stream):
            for i in order:
                b.resolve_and_cache(tab, dctx, dnew, t, cu, src[i, 0], src[i, 1], slots_out=sl,
                                    stream=stream)
        stream.synchronize()
        assert torch.equal(rows(), src[last])
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            b.resolve_and_cache(tab, dctx, dnew, t, cu, src[i, 0], src[i, 1], slots_out=sl,
                                stream=stream)
    b.resolve_and_cache(tab, dctx, dnew, t, cu, src[0, 0], src[0, 1], slots_out=sl)
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(rows(), src[steps - 1])
    assert b.device_error() is None
    del graph


def test_fused_resolve_and_cache_flags_bad_tables_and_writes_nothing_for_them(cuda):
    import torch

    cfg = CacheConfig(64, 4, 1, 8, 2, 2)
    b = B200Backend(cfg, dtype="bf16")
    tables = torch.tensor([[0, 70]], dtype=torch.int32, device=cuda)  # 70 is outside the pool
    ctx = torch.tensor([3], dtype=torch.int32, device=cuda)
    new = torch.tensor([3], dtype=torch.int32, device=cuda)
    k = torch.ones((2, 3, 8), dtype=torch.bfloat16, device=cuda)
    cu = torch.zeros(2, dtype=torch.int32, device=cuda)
    sl = torch.zeros(3, dtype=torch.int64, device=cuda)
    b.resolve_and_cache(tables, ctx, new, 3, cu, k, k, slots_out=sl)
    err = b.device_error()
    assert err is not None and isinstance(err[0], InvalidBlock)
    assert sl.tolist() == [3, -1, -1]
    pk, _ = b.planes()
    assert int(torch.count_nonzero(pk)) == 2 * 8  # token 0 in both layers only
    with pytest.raises(Exception, match="dtype"):
        b.resolve_and_cache(tables, ctx, new, 3, cu, k.float(), k.float())


def test_a_pool_larger_than_hbm_fails_cleanly_and_leaves_the_device_usable(cuda):
    """Failure at init (CudaBackend::new's alloc_zeros): a 2.7 TB pool is a
    Device error, not a crash, and the next backend works normally."""
    from pagedkv import Device

    huge = CacheConfig(num_blocks=2**20, block_size=16, num_kv_heads=8, head_dim=128,
                       num_layers=80, dtype_bytes=2)
    with pytest.raises(Device, match="allocating"):
        B200Backend(huge, dtype="bf16")
    b = B200Backend(CacheConfig.tiny(8))
    b.write_kv(1, (3, 2), entry(1.0, 8), entry(2.0, 8))
    assert (b.read_entry(1, (3, 2))[0] == entry(1.0, 8)).all()
