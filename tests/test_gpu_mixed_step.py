"""pkv_resolve_and_cache_mixed_dev: a scheduler step's admitted prompts
(slots resolved from block tables) and decoded tokens (slots from the host)
in one launch, against pkv_resolve_and_cache_dev followed by
pkv_reshape_and_cache_dev of the decoded tokens, and against the oracle;
padding and out-of-pool host slots, and the refusal of fp8 pools."""

import numpy as np
import pytest

from oracle.cpu import OracleBackend, resolve_slots
from pagedkv import B200Backend, CacheConfig, Device, InvalidBlock
from pagedkv.workloads import Stream, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def step(cfg, st, seqs, max_ctx, max_new, direct):
    ctx = st.integers(seqs, 0, max_ctx).astype(np.int32)
    new = st.integers(seqs, 1, max_new).astype(np.int32)
    need = -(-(ctx + new) // cfg.block_size)
    perm = st.permutation(cfg.num_blocks)
    tables = np.full((seqs, int(need.max())), -1, np.int32)
    off = 0
    for q in range(seqs):
        tables[q, : need[q]] = perm[off:off + need[q]]
        off += need[q]
    # Host slots in blocks no table uses.
    free = perm[off:]
    dslots = (free[st.integers(direct, 0, len(free) - 1)] * cfg.block_size +
              st.integers(direct, 0, cfg.block_size - 1)).astype(np.int64)
    dslots = np.unique(dslots)  # distinct, as a step's decoded tokens are
    return tables, ctx, new, dslots


@pytest.mark.parametrize("layers,heads", [(6, 4), (28, 1)])
def test_one_launch_equals_the_two_launches_and_the_oracle(cuda, layers, heads):
    import torch

    cfg = CacheConfig(num_blocks=4096, block_size=16, num_kv_heads=heads, head_dim=128,
                      num_layers=layers, dtype_bytes=2)
    e = cfg.entry_elems()
    st = Stream(layers)
    tables, ctx, new, dslots = step(cfg, st, 40, 500, 300, 700)
    tr, d = int(new.sum()), len(dslots)
    dslots[5] = -1                     # padding: skipped
    kv = f32_to_bf16_bits(st.normal(2 * layers * (tr + d) * e)).reshape(2, layers, tr + d, e)
    dk = torch.from_numpy(kv.view(np.int16)).view(torch.bfloat16).cuda()
    tab, dctx, dnew = (torch.from_numpy(x).cuda() for x in (tables, ctx, new))
    ddir = torch.from_numpy(dslots).cuda()
    one = B200Backend(cfg, dtype="bf16")
    cu1 = torch.full((len(new) + 1,), -1, dtype=torch.int32, device=cuda)
    sl1 = torch.full((tr,), -9, dtype=torch.int64, device=cuda)
    one.resolve_and_cache_mixed(tab, dctx, dnew, tr, cu1, ddir, d, dk[0], dk[1], slots_out=sl1)
    two = B200Backend(cfg, dtype="bf16")
    cu2 = torch.full_like(cu1, -1)
    sl2 = torch.full_like(sl1, -9)
    two.resolve_and_cache(tab, dctx, dnew, tr, cu2, dk[0][:, :tr], dk[1][:, :tr], slots_out=sl2)
    two.reshape_and_cache(dk[0][:, tr:], dk[1][:, tr:], ddir)
    torch.cuda.synchronize()
    assert one.device_error() is None and two.device_error() is None
    assert torch.equal(cu1, cu2) and torch.equal(sl1, sl2)
    for a, b in zip(one.planes(), two.planes()):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    if layers == 6:
        rc, _, res = resolve_slots(tables, ctx, new, tr, cfg.block_size, cfg.num_blocks)
        assert rc == 0
        slots = np.concatenate([res, dslots])
        keep = slots >= 0
        dsts = [(int(x) // 16, int(x) % 16) for x in slots[keep]]
        cpu = OracleBackend(cfg)
        for l in range(layers):
            cpu.write_kv_batch(l, dsts, bf16_bits_to_f32(kv[0, l][keep]).ravel(),
                               bf16_bits_to_f32(kv[1, l][keep]).ravel())
        ok, ov = cpu.planes()
        pk, pv = one.planes()
        np.testing.assert_array_equal(pk.float().cpu().numpy().view(np.uint32), ok.view(np.uint32))
        np.testing.assert_array_equal(pv.float().cpu().numpy().view(np.uint32), ov.view(np.uint32))


def test_out_of_pool_host_slot_is_recorded_and_fp8_is_refused(cuda):
    import torch

    cfg = CacheConfig(num_blocks=64, block_size=16, num_kv_heads=2, head_dim=64, num_layers=2,
                      dtype_bytes=2)
    e = cfg.entry_elems()
    tab = torch.tensor([[3, 4]], dtype=torch.int32, device=cuda)
    ctx = torch.tensor([10], dtype=torch.int32, device=cuda)
    new = torch.tensor([2], dtype=torch.int32, device=cuda)
    ddir = torch.tensor([7 * 16 + 1, 64 * 16 + 3, 9 * 16], dtype=torch.int64, device=cuda)
    k = torch.randn((2, 5, e), device=cuda).to(torch.bfloat16)
    b = B200Backend(cfg, dtype="bf16")
    cu = torch.empty(2, dtype=torch.int32, device=cuda)
    b.resolve_and_cache_mixed(tab, ctx, new, 2, cu, ddir, 3, k, k)
    err = b.device_error()
    assert isinstance(err[0], InvalidBlock) and err[1] == 3  # token 2 + 1: the second host slot
    pk, _ = b.planes()
    assert torch.equal(pk[1, 7, 1], k[1, 2]) and torch.equal(pk[1, 9, 0], k[1, 4])
    assert torch.equal(pk[0, 3, 10], k[0, 0]) and torch.equal(pk[0, 3, 11], k[0, 1])
    f = B200Backend(CacheConfig(64, 16, 2, 64, 2, 1), dtype="fp8_e4m3")
    with pytest.raises(Device):
        f.resolve_and_cache_mixed(tab, ctx, new, 2, cu, ddir, 3, k, k)
