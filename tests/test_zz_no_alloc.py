"""pkv_resolve_and_cache_noalloc, the entry point for callers that cannot
allocate device memory (for example a plugin inside an engine that has
already reserved nearly all HBM for its own pool). It keeps its scratch in a
fixed static device array and takes every buffer from the caller.

Its results must equal those of the regular entry points,
pkv_resolve_slots_dev followed by pkv_reshape_and_cache_dev, bit for bit, on
two calls in a row (the second call sees the scratch the first one left
behind). This file is collected last on purpose; it also passes on its own.
"""

import ctypes as C

import numpy as np
import pytest

from pagedkv import B200Backend, CacheConfig
from pagedkv import _lib
from pagedkv.workloads import Stream

pytestmark = pytest.mark.gpu

MAX_TOKENS = 131072  # PKV_NOALLOC_MAX_TOKENS in include/pkv_b200.h


def make_batch(st, cfg, num_seqs, max_ctx, max_new, perm_off):
    """Sequences with ctx cached tokens and new tokens, tables from a permutation."""
    ctx = st.integers(num_seqs, 0, max_ctx).astype(np.int32)
    new = st.integers(num_seqs, 0, max_new).astype(np.int32)
    need = -(-(ctx + new) // cfg.block_size)
    stride = max(int(need.max()), 1)
    perm = (st.permutation(cfg.num_blocks) + perm_off) % cfg.num_blocks
    tables = np.full((num_seqs, stride), -1, np.int32)
    pos = 0
    for q in range(num_seqs):
        tables[q, : need[q]] = perm[pos:pos + need[q]]
        pos += need[q]
    return tables, ctx, new


def noalloc(cfg, dtype_tag, k_plane, v_plane, tables, ctx, new, t, cu, layer, k, v, status,
            stream):
    c = _lib.Config(cfg.num_blocks, cfg.block_size, cfg.num_kv_heads, cfg.head_dim,
                    cfg.num_layers, cfg.dtype_bytes)
    lay = -1 if layer is None else layer
    tok_stride = k.stride(1) if layer is None else k.stride(0)
    lay_stride = k.stride(0) if layer is None else 0
    return _lib.lib.pkv_resolve_and_cache_noalloc(
        C.byref(c), dtype_tag, 0, 1, k_plane.data_ptr(), v_plane.data_ptr(), tables.data_ptr(),
        tables.shape[1], ctx.data_ptr(), new.data_ptr(), ctx.shape[0], t, cu.data_ptr(), lay,
        k.data_ptr(), v.data_ptr(), tok_stride, lay_stride, _lib.BF16, status.data_ptr(),
        stream.cuda_stream)


def test_noalloc_matches_regular_entry_points_twice_in_a_row(cuda):
    import torch

    cfg = CacheConfig(num_blocks=2048, block_size=16, num_kv_heads=4, head_dim=64, num_layers=3,
                      dtype_bytes=2)
    e = cfg.entry_elems()
    reg = B200Backend(cfg, dtype="bf16")
    rk, rv = reg.planes()
    # Caller-owned pool for the no-alloc path, laid out like the backend's.
    k_plane = torch.zeros_like(rk)
    v_plane = torch.zeros_like(rv)
    stream = torch.cuda.current_stream()
    st = Stream(4242)
    calls = [
        (None, make_batch(st, cfg, 40, 300, 400, 0)),     # prefill-like chunk, every layer
        (1, make_batch(st, cfg, 100, 300, 2, 17)),        # decode-like step, one layer
    ]
    for layer, (tables, ctx, new) in calls:
        t = int(new.sum())
        d_tab = torch.from_numpy(tables).to(cuda)
        d_ctx = torch.from_numpy(ctx).to(cuda)
        d_new = torch.from_numpy(new).to(cuda)
        shape = (cfg.num_layers, t, e) if layer is None else (t, e)
        k = torch.randn(shape, device=cuda).to(torch.bfloat16)
        v = torch.randn(shape, device=cuda).to(torch.bfloat16)
        # Regular path: resolve into a slot buffer, then scatter.
        cu_ref = torch.empty(len(ctx) + 1, dtype=torch.int32, device=cuda)
        slots = torch.empty(max(t, 1), dtype=torch.int64, device=cuda)
        reg.resolve_slots(d_tab, d_ctx, d_new, t, cu_ref, slots, stream=stream)
        reg.reshape_and_cache(k, v, slots[:t], layer=layer, stream=stream)
        # No-alloc path.
        cu = torch.full((len(ctx) + 1,), -3, dtype=torch.int32, device=cuda)
        status = torch.full((2,), -9, dtype=torch.int64, device=cuda)
        rc = noalloc(cfg, _lib.BF16, k_plane, v_plane, d_tab, d_ctx, d_new, t, cu, layer, k, v,
                     status, stream)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert reg.device_error() is None
        assert status.tolist() == [0, 0]
        assert torch.equal(cu, cu_ref)
        assert torch.equal(k_plane.view(torch.int16), rk.view(torch.int16))
        assert torch.equal(v_plane.view(torch.int16), rv.view(torch.int16))
    assert int(torch.count_nonzero(k_plane)) > 0


def test_noalloc_rejects_sizes_beyond_its_scratch_without_device_work(cuda):
    import torch

    cfg = CacheConfig(num_blocks=16, block_size=16, num_kv_heads=1, head_dim=8, num_layers=1,
                      dtype_bytes=2)
    z = torch.zeros(1, dtype=torch.int32, device=cuda)
    c = _lib.Config(16, 16, 1, 8, 1, 2)
    rc = _lib.lib.pkv_resolve_and_cache_noalloc(
        C.byref(c), _lib.BF16, 0, 1, z.data_ptr(), z.data_ptr(), z.data_ptr(), 1, z.data_ptr(),
        z.data_ptr(), 1, MAX_TOKENS + 1, z.data_ptr(), 0, z.data_ptr(), z.data_ptr(), 8, 0,
        _lib.BF16, None, None)
    code, a, b, msg = _lib.last_error()
    assert rc == code == 6 and (a, b) == (MAX_TOKENS, MAX_TOKENS + 1) and "at most" in msg
    assert int(z.item()) == 0
