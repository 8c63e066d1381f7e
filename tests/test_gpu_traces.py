"""Whole scheduler traces through the device data path, bit for bit against
the CPU oracle: a decode step and a prefill chunk at reduced geometry
(configs 2 and 3), beam search with copy-on-write every step (config 4) and
continuous batching with preemption and forks (config 5). Each step runs
copy_blocks -> slot resolution -> all-layer reshape_and_cache -> zero_blocks
on the GPU through the C ABI, and the same step on the oracle."""

import numpy as np
import pytest

from oracle.cpu import OracleBackend, resolve_slots
from pagedkv import B200Backend, CacheConfig
from pagedkv.driver import DeviceStepper
from pagedkv.traces import StepPlan, beam_cow_trace, churn_trace, plan_from_batch
from pagedkv.workloads import Stream, bf16_bits_to_f32, decode_batch, f32_to_bf16_bits, prefill_chunk

pytestmark = pytest.mark.gpu


def apply_to_oracle(orc, plan: StepPlan, k: np.ndarray, v: np.ndarray, resolve) -> None:
    """The same step on the CPU oracle (CpuBackend semantics): copies, writes
    of every token (slots resolved by the oracle's slot rule), zeroes.
    k, v: f32 [L][R][entry]; token i uses row i % R."""
    cfg = orc.cfg
    bs = cfg.block_size
    if len(plan.copies):
        orc.copy_blocks(plan.copies)
    tr = plan.resolved_tokens
    if len(plan.new):
        rc, _, res = resolve(plan.tables, plan.ctx, plan.new, tr, bs, cfg.num_blocks)
        assert rc == 0
    else:
        res = np.zeros(0, np.int64)
    slots = np.concatenate([res, plan.direct_slots.astype(np.int64)])
    rows = np.arange(len(slots)) % k.shape[1]
    keep = slots >= 0
    dsts = [(int(x) // bs, int(x) % bs) for x in slots[keep]]
    for layer in range(cfg.num_layers):
        orc.write_kv_batch(layer, dsts, k[layer][rows[keep]].ravel(), v[layer][rows[keep]].ravel())
    if len(plan.zero):
        orc.zero_blocks(plan.zero)


def rows(cfg, r, seed):
    """bf16 K/V rows [L][r][entry] on the device and their exact f32 copies."""
    import torch

    st = Stream(seed)
    bits = f32_to_bf16_bits(st.normal(2 * cfg.num_layers * r * cfg.entry_elems()))
    bits = bits.reshape(2, cfg.num_layers, r, cfg.entry_elems())
    d = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    return d[0], d[1], bf16_bits_to_f32(bits[0]), bf16_bits_to_f32(bits[1])


def assert_same_pool(gpu, cpu):
    gk, gv = (p.float().cpu().numpy() for p in gpu.planes())
    ok, ov = cpu.planes()
    np.testing.assert_array_equal(gk.view(np.uint32), ok.view(np.uint32))
    np.testing.assert_array_equal(gv.view(np.uint32), ov.view(np.uint32))


def run(cfg, plans, r=2048, check_every=0, fuse=True, fused_steps=None, mixed_steps=None):
    import torch

    gpu, cpu = B200Backend(cfg, dtype="bf16"), OracleBackend(cfg)
    k, v, kf, vf = rows(cfg, r, 9)
    stepper = DeviceStepper(gpu, fuse_copy_zero=fuse, fuse_mixed=fuse)
    stats = []
    for i, plan in enumerate(plans):
        stepper.apply(plan, k, v)
        apply_to_oracle(cpu, plan, kf, vf, resolve_slots)
        stats.append(plan.stats)
        if check_every and i % check_every == 0:
            torch.cuda.synchronize()
            assert_same_pool(gpu, cpu)
    torch.cuda.synchronize()
    assert gpu.device_error() is None
    assert_same_pool(gpu, cpu)
    assert gpu.digest() == cpu.digest()
    if fused_steps is not None:
        fused_steps.append(stepper.fused_steps)
    if mixed_steps is not None:
        mixed_steps.append(stepper.mixed_steps)
    return stats


def test_decode_step_from_a_shuffled_allocator(cuda):  # config 2 at reduced geometry
    cfg = CacheConfig(num_blocks=2048, block_size=16, num_kv_heads=2, head_dim=32, num_layers=4,
                      dtype_bytes=2)
    batch = decode_batch(seed=None, num_seqs=96, max_ctx=300, cfg=cfg)
    run(cfg, [plan_from_batch(batch)])


def test_ragged_prefill_chunk(cuda):  # config 3 at reduced geometry
    cfg = CacheConfig(num_blocks=1024, block_size=16, num_kv_heads=2, head_dim=32, num_layers=3,
                      dtype_bytes=2)
    batch = prefill_chunk(seed=3, num_prompts=24, lo=16, hi=900, budget=3000, cfg=cfg)
    assert batch.num_tokens == 3000
    run(cfg, [plan_from_batch(batch)], r=4096)


@pytest.mark.parametrize("fuse", [True, False])
@pytest.mark.parametrize("interleave", [False, True])
def test_beam_search_copy_on_write_trace(cuda, interleave, fuse):  # config 4 at reduced geometry
    """interleave=True frees old beams group by group, which chains copy
    pairs within a step; the driver must keep their sequential meaning.
    fuse=True runs each eligible step's copies and zeroes as one launch
    (sources grouped, freed sources zeroed after their copies); with one
    wave of copies per step every step with zeroes is eligible."""
    cfg = CacheConfig(num_blocks=512, block_size=8, num_kv_heads=2, head_dim=16, num_layers=3,
                      dtype_bytes=2)
    plans = list(beam_cow_trace(cfg, groups=6, width=4, prefix=37, steps=30, zero_per_step=5, seed=2,
                                interleave=interleave))
    fused = []
    stats = run(cfg, plans, r=512, check_every=7, fuse=fuse, fused_steps=fused)
    if fuse and not interleave:
        assert fused[0] > 20
    if not fuse:
        assert fused[0] == 0
    copies = sum(s["copies"] for s in stats)
    # Every child pays a copy except on steps whose append opens a new block.
    assert copies == sum(24 for s in range(1, 31) if (37 + s - 1) % 8 != 0)


@pytest.mark.parametrize("fuse", [True, False])
@pytest.mark.parametrize("fork_rate", [0.0, 0.5])
def test_continuous_batching_churn_trace(cuda, fork_rate, fuse):  # config 5 at reduced geometry
    """fuse=True writes a step's admitted prompts and decoded tokens in one
    launch (pkv_resolve_and_cache_mixed_dev) and its copies and zeroes in
    another, where the step allows; fuse=False issues every part apart."""
    cfg = CacheConfig(num_blocks=96, block_size=4, num_kv_heads=2, head_dim=16, num_layers=2,
                      dtype_bytes=2)
    plans = list(churn_trace(cfg, steps=250, arrival_rate=1.2, prompt_lo=2, prompt_hi=60,
                             out_mean=12.0, max_batch=24, fork_rate=fork_rate, seed=5))
    mixed = []
    stats = run(cfg, plans, r=1024, check_every=50, fuse=fuse, mixed_steps=mixed)
    assert (mixed[0] > 50) if fuse else (mixed[0] == 0)
    assert sum(s["preempted"] for s in stats) > 0
    assert sum(s["finished"] for s in stats) > 100
    if fork_rate:
        assert sum(len(p.copies) for p in plans) > 0
