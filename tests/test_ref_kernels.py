"""The reference's own CUDA kernels (crates/paged-kv-cuda/kernels/kernels.cu,
built from the reference checkout into oracle/_ref by oracle/ref.mk; they
never ran upstream) on a B200:

* on config 1 they produce exactly the C oracle's pool -- a second pin of the
  oracle, this time against the reference's device code; and
* on a prefill chunk at Qwen2-7B KV geometry (f32, the only type they
  support) they are the device-side "before": the B200 kernels must beat them
  and write the same pool.
"""

import numpy as np
import pytest

from oracle import ref_kernels as ref
from oracle.cpu import OracleBackend
from pagedkv import B200Backend, CacheConfig
from pagedkv.workloads import config1, prefill_chunk

pytestmark = pytest.mark.gpu

if not ref.available():
    pytest.skip("oracle/_ref/libref_kernels.so was not built (needs the reference checkout)",
                allow_module_level=True)


def test_reference_kernels_agree_with_the_c_oracle_on_config1(cuda):
    import torch

    w = config1(seed=0)
    cfg = w.cfg
    e, bs, nb, L = cfg.entry_elems(), cfg.block_size, cfg.num_blocks, cfg.num_layers
    kc = torch.zeros(L * nb * bs * e, dtype=torch.float32, device=cuda)
    vc = torch.zeros_like(kc)
    slots = torch.from_numpy(w.slots.astype(np.int64)).to(cuda)
    cpu = OracleBackend(cfg)
    for layer in range(L):
        k = torch.from_numpy(w.k[layer]).to(cuda)
        v = torch.from_numpy(w.v[layer]).to(cuda)
        ref.reshape_and_cache(k, v, kc, vc, slots, layer, nb, bs, e)
        cpu.write_kv_batch(layer, [(int(s) // bs, int(s) % bs) for s in w.slots],
                           w.k[layer].ravel(), w.v[layer].ravel())
    ref.copy_blocks(kc, vc, torch.from_numpy(w.pairs.astype(np.int64)).to(cuda), L, nb, bs * e)
    cpu.copy_blocks(w.pairs)
    for z in w.zero:
        ref.zero_block(kc, vc, int(z), L, nb, bs * e)
        cpu.zero_block(int(z))
    torch.cuda.synchronize()
    ok, ov = cpu.planes()
    np.testing.assert_array_equal(kc.cpu().numpy().view(np.uint32), ok.ravel().view(np.uint32))
    np.testing.assert_array_equal(vc.cpu().numpy().view(np.uint32), ov.ravel().view(np.uint32))


def _timed(fn, reps=10):
    import torch

    times = []
    for i in range(reps + 2):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        if i >= 2:
            times.append(a.elapsed_time(b))
    return sum(times) / len(times)


def test_b200_kernels_beat_the_reference_kernels_on_a_prefill_chunk(cuda):
    import torch

    cfg = CacheConfig(num_blocks=8192, block_size=16, num_kv_heads=4, head_dim=128, num_layers=28,
                      dtype_bytes=4)
    batch = prefill_chunk(seed=0, num_prompts=24, budget=16384, cfg=cfg)
    t, e, L, nb, bs = batch.num_tokens, cfg.entry_elems(), cfg.num_layers, cfg.num_blocks, 16
    slots = torch.from_numpy(batch.slot_mapping()).to(cuda)
    k = torch.randn((L, t, e), device=cuda)
    v = torch.randn((L, t, e), device=cuda)
    kc = torch.zeros(L * nb * bs * e, dtype=torch.float32, device=cuda)
    vc = torch.zeros_like(kc)

    def reference():  # CudaBackend::write_kv_batch once per layer
        for layer in range(L):
            ref.reshape_and_cache(k[layer], v[layer], kc, vc, slots, layer, nb, bs, e)

    ours = B200Backend(cfg, dtype="f32")
    t_ref = _timed(reference)
    t_ours = _timed(lambda: ours.reshape_and_cache(k, v, slots))
    t_ours_per_layer = _timed(lambda: [ours.reshape_and_cache(k[l], v[l], slots, layer=l)
                                       for l in range(L)])
    torch.cuda.synchronize()
    pk, pv = ours.planes()
    assert torch.equal(pk.reshape(-1).view(torch.int32), kc.view(torch.int32))
    assert torch.equal(pv.reshape(-1).view(torch.int32), vc.view(torch.int32))
    gb = t * L * 2 * e * 4 * 2 / 1e9
    print(f"\nprefill chunk {t} tokens x {L} layers, f32 ({gb:.2f} GB moved): reference kernels "
          f"{t_ref:.3f} ms ({gb / t_ref * 1e3:.0f} GB/s); B200 all-layer {t_ours:.3f} ms "
          f"({gb / t_ours * 1e3:.0f} GB/s); B200 per-layer {t_ours_per_layer:.3f} ms "
          f"({gb / t_ours_per_layer * 1e3:.0f} GB/s)")
    assert t_ours < t_ref
