"""pkv_resolve_and_cache_noalloc, the entry point for callers that cannot
allocate device memory (for example a plugin inside an engine that has
already reserved nearly all HBM for its own pool). It keeps its scratch in a
fixed static device array and takes every buffer from the caller.

Its results must equal those of the regular entry points,
pkv_resolve_slots_dev followed by pkv_reshape_and_cache_dev, bit for bit,
and the CPU oracle's, on calls in a row: each call after the first sees the
scratch the one before left behind. One call carries a block id outside the
pool after a call that resolved every token, so a stale slot in the shared
array would show up as a write the regular path does not make.

This file is collected last on purpose; it also passes on its own.
"""

import ctypes as C

import numpy as np
import pytest

from oracle.cpu import OracleBackend, resolve_slots
from pagedkv import B200Backend, CacheConfig
from pagedkv import _lib
from pagedkv.workloads import Stream, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu

MAX_TOKENS = 131072  # PKV_NOALLOC_MAX_TOKENS in include/pkv_b200.h


def make_batch(st, cfg, num_seqs, max_ctx, max_new, perm_off, min_new=0):
    """Sequences with ctx cached tokens and new tokens, tables from a permutation."""
    ctx = st.integers(num_seqs, 0, max_ctx).astype(np.int32)
    new = st.integers(num_seqs, min_new, max_new).astype(np.int32)
    need = -(-(ctx + new) // cfg.block_size)
    stride = max(int(need.max()), 1)
    perm = (st.permutation(cfg.num_blocks) + perm_off) % cfg.num_blocks
    tables = np.full((num_seqs, stride), -1, np.int32)
    pos = 0
    for q in range(num_seqs):
        tables[q, : need[q]] = perm[pos:pos + need[q]]
        pos += need[q]
    return tables, ctx, new


def noalloc(cfg, k_plane, v_plane, tables, ctx, new, t, cu, layer, k, v, src_tag, status,
            stream, shard=(0, 1)):
    c = _lib.Config(cfg.num_blocks, cfg.block_size, cfg.num_kv_heads, cfg.head_dim,
                    cfg.num_layers, cfg.dtype_bytes)
    lay = -1 if layer is None else layer
    tok_stride = k.stride(1) if layer is None else k.stride(0)
    lay_stride = k.stride(0) if layer is None else 0
    return _lib.lib.pkv_resolve_and_cache_noalloc(
        C.byref(c), _lib.BF16, shard[0], shard[1], k_plane.data_ptr(), v_plane.data_ptr(),
        tables.data_ptr(), tables.shape[1], ctx.data_ptr(), new.data_ptr(), ctx.shape[0], t,
        cu.data_ptr(), lay, k.data_ptr(), v.data_ptr(), tok_stride, lay_stride, src_tag,
        status.data_ptr(), stream.cuda_stream)


def bf16_rows(st, shape):
    """bf16-representable values as f32 (so an f32 source narrows exactly)."""
    n = int(np.prod(shape))
    return bf16_bits_to_f32(f32_to_bf16_bits(st.normal(n))).reshape(shape)


@pytest.mark.parametrize("shard", [(0, 1), (1, 2)])
def test_noalloc_matches_regular_entry_points_and_oracle_over_calls_in_a_row(cuda, shard):
    import torch

    cfg = CacheConfig(num_blocks=2048, block_size=16, num_kv_heads=4, head_dim=64, num_layers=3,
                      dtype_bytes=2)
    full = cfg.entry_elems()
    rank, ways = shard
    es = full // ways
    lo = rank * es
    reg = B200Backend(cfg, dtype="bf16", shard_rank=rank, num_shards=ways)
    rk, rv = reg.planes()
    # Caller-owned pool for the no-alloc path, laid out like the backend's.
    k_plane = torch.zeros_like(rk)
    v_plane = torch.zeros_like(rv)
    cpu = OracleBackend(cfg)
    stream = torch.cuda.current_stream()
    st = Stream(4242 + rank)
    dec_tables, dec_ctx, dec_new = make_batch(st, cfg, 100, 300, 1, 911, min_new=1)
    bad_q = 37
    bad_tables = dec_tables.copy()
    bad_tables[bad_q, int(dec_ctx[bad_q]) // cfg.block_size] = cfg.num_blocks + 3
    calls = [
        # (layer, batch, source dtype, token with a bad table entry)
        (None, make_batch(st, cfg, 40, 300, 400, 0), "bf16", None),   # prefill-like, every layer
        (1, make_batch(st, cfg, 100, 300, 2, 17), "f32", None),      # decode-like, one layer, f32 rows
        (None, (bad_tables, dec_ctx, dec_new), "bf16", bad_q),       # one token rejected
        (2, make_batch(st, cfg, 64, 200, 9, 401), "bf16", None),     # clean again after the bad call
    ]
    for layer, (tables, ctx, new), src, bad in calls:
        t = int(new.sum())
        d_tab = torch.from_numpy(tables).to(cuda)
        d_ctx = torch.from_numpy(ctx).to(cuda)
        d_new = torch.from_numpy(new).to(cuda)
        layers = cfg.num_layers if layer is None else 1
        kf = bf16_rows(st, (layers, t, full))
        vf = bf16_rows(st, (layers, t, full))
        tdt = torch.float32 if src == "f32" else torch.bfloat16
        # This shard's head slice of the rows, as a tensor-parallel rank holds them.
        k = torch.from_numpy(np.ascontiguousarray(kf[:, :, lo:lo + es])).to(cuda).to(tdt)
        v = torch.from_numpy(np.ascontiguousarray(vf[:, :, lo:lo + es])).to(cuda).to(tdt)
        if layer is not None:
            k, v = k[0], v[0]
        tag = _lib.F32 if src == "f32" else _lib.BF16
        # Regular path: resolve into a slot buffer, then scatter.
        cu_ref = torch.empty(len(ctx) + 1, dtype=torch.int32, device=cuda)
        slots = torch.empty(max(t, 1), dtype=torch.int64, device=cuda)
        reg.resolve_slots(d_tab, d_ctx, d_new, t, cu_ref, slots, stream=stream)
        reg.reshape_and_cache(k, v, slots[:t], layer=layer, stream=stream)
        # No-alloc path.
        cu = torch.full((len(ctx) + 1,), -3, dtype=torch.int32, device=cuda)
        status = torch.full((2,), -9, dtype=torch.int64, device=cuda)
        rc = noalloc(cfg, k_plane, v_plane, d_tab, d_ctx, d_new, t, cu, layer, k, v, tag, status,
                     stream, shard)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        err_ref = reg.device_error()
        # Oracle: the same tokens through CpuBackend semantics, full entries.
        orc_rc, orc_cu, orc_slots = resolve_slots(tables, ctx, new, t, cfg.block_size,
                                                  cfg.num_blocks)
        for li in range(layers):
            keep = orc_slots >= 0
            dsts = [(int(s) // cfg.block_size, int(s) % cfg.block_size) for s in orc_slots[keep]]
            lay_id = li if layer is None else layer
            cpu.write_kv_batch(lay_id, dsts, kf[li][keep].ravel(), vf[li][keep].ravel())
        if bad is None:
            assert err_ref is None and orc_rc == 0
            assert status.tolist() == [0, 0]
        else:
            # The bad token's index and variant, as the regular path records them.
            assert orc_rc == 1 and err_ref is not None and err_ref[1] == bad
            assert status.tolist() == [err_ref[0].code, bad]
        assert torch.equal(cu, cu_ref)
        np.testing.assert_array_equal(cu.cpu().numpy(), orc_cu)
        assert torch.equal(k_plane.view(torch.int16), rk.view(torch.int16))
        assert torch.equal(v_plane.view(torch.int16), rv.view(torch.int16))
        ok, ov = cpu.planes()
        np.testing.assert_array_equal(k_plane.float().cpu().numpy().view(np.uint32),
                                      ok[..., lo:lo + es].view(np.uint32))
        np.testing.assert_array_equal(v_plane.float().cpu().numpy().view(np.uint32),
                                      ov[..., lo:lo + es].view(np.uint32))
    assert int(torch.count_nonzero(k_plane)) > 0


def test_noalloc_rejects_sizes_beyond_its_scratch_without_device_work(cuda):
    import torch

    z = torch.zeros(1, dtype=torch.int32, device=cuda)
    c = _lib.Config(16, 16, 1, 8, 1, 2)
    rc = _lib.lib.pkv_resolve_and_cache_noalloc(
        C.byref(c), _lib.BF16, 0, 1, z.data_ptr(), z.data_ptr(), z.data_ptr(), 1, z.data_ptr(),
        z.data_ptr(), 1, MAX_TOKENS + 1, z.data_ptr(), 0, z.data_ptr(), z.data_ptr(), 8, 0,
        _lib.BF16, None, None)
    code, a, b, msg = _lib.last_error()
    assert rc == code == 6 and (a, b) == (MAX_TOKENS, MAX_TOKENS + 1) and "at most" in msg
    assert int(z.item()) == 0
