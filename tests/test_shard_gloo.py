"""The N>1 path on CPU: two gloo ranks, each holding one KV-head shard of a
pool (written through the oracle), verify the shards with the same
all-gather of digests that the benchmark runs over NCCL; a planted mistake
in one rank's shard is caught."""

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _rank_main(rank: int, world: int, port: int, plant: bool, out_dir: str) -> None:
    sys.path[:0] = [str(ROOT / "paged-kv-cache_b200"), str(ROOT)]
    import torch.distributed as dist

    from oracle.cpu import OracleBackend, digest_rows
    from pagedkv.config import CacheConfig
    from pagedkv.shard import entry_slice, verify_over_group
    from pagedkv.workloads import Stream

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = CacheConfig(num_blocks=16, block_size=4, num_kv_heads=4, head_dim=8, num_layers=2,
                      dtype_bytes=4)
    e = cfg.entry_elems()
    off, w = entry_slice(e, rank, world)
    st = Stream(77)  # same inputs on every rank; each keeps its own columns
    t = 20
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:t]
    dsts = [(int(s) // 4, int(s) % 4) for s in slots]
    orc = OracleBackend(cfg)  # this rank's shard, held as a full-width pool zero outside the slice
    pool, expect = [0, 0], [0, 0]
    full_expect = [0, 0]
    for layer in range(cfg.num_layers):
        k = st.normal(t * e).astype(np.float32).reshape(t, e)
        v = st.normal(t * e).astype(np.float32).reshape(t, e)
        km, vm = np.zeros_like(k), np.zeros_like(v)
        km[:, off:off + w], vm[:, off:off + w] = k[:, off:off + w], v[:, off:off + w]
        if plant and rank == 1 and layer == 1:
            km[3, off] += 1.0  # a wrong value lands in this shard only
        orc.write_kv_batch(layer, dsts, km.ravel(), vm.ravel())
        for p, rows in ((0, k), (1, v)):
            masked = np.zeros_like(rows)
            masked[:, off:off + w] = rows[:, off:off + w]
            expect[p] += digest_rows(masked, slots, layer, cfg.num_blocks * cfg.block_size, p)
            full_expect[p] += digest_rows(rows, slots, layer, cfg.num_blocks * cfg.block_size, p)
    pool = orc.digest()
    res = verify_over_group(tuple(pool), tuple(x % 2**64 for x in expect))
    ok_total = int(res["pool_digest_k"], 16) == full_expect[0] % 2**64
    Path(out_dir, f"rank{rank}.txt").write_text(f"{res['ok']} {res['shards_ok']} {ok_total}\n")
    dist.destroy_process_group()


def _run(plant: bool, tmp_path, port: int):
    import torch.multiprocessing as mp

    mp.start_processes(_rank_main, args=(2, port, plant, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    return [Path(tmp_path, f"rank{r}.txt").read_text().split(" ", 1) for r in range(2)]


def test_two_gloo_ranks_verify_their_shards(tmp_path):
    out = _run(False, tmp_path, 29531)
    for ok, rest in out:
        assert ok == "True" and rest.strip() == "[True, True] True"


def test_a_wrong_value_in_one_shard_is_caught(tmp_path):
    out = _run(True, tmp_path, 29532)
    for ok, rest in out:
        assert ok == "False" and rest.strip().startswith("[True, False]")


def test_entry_slices_tile_the_entry():
    sys.path[:0] = [str(ROOT / "paged-kv-cache_b200")]
    from pagedkv.shard import entry_slice

    for world in (1, 2, 4, 8):
        cols = [c for r in range(world) for c in range(*(lambda o, w: (o, o + w))(*entry_slice(512, r, world)))]
        assert cols == list(range(512))
    with pytest.raises(ValueError):
        entry_slice(512, 0, 3)


def _dying_rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    """Rank 1 exits between steps, before the verification collective; rank 0
    must learn it from the collective (an error within the process-group
    timeout), not hang."""
    sys.path[:0] = [str(ROOT / "paged-kv-cache_b200"), str(ROOT)]
    from datetime import timedelta

    import torch.distributed as dist

    from pagedkv.shard import verify_over_group

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    dist.barrier()
    if rank == 1:
        os._exit(3)  # a rank that dies between steps
    try:
        verify_over_group((1, 2), (1, 2))
        outcome = "no error"
    except Exception as e:  # noqa: BLE001 -- any collective failure is the detection
        outcome = "error: " + type(e).__name__
    Path(out_dir, "rank0.txt").write_text(outcome)
    os._exit(0)


def test_a_rank_that_dies_is_detected_by_the_survivor(tmp_path):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_dying_rank_main, args=(r, 2, 29533, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a surviving rank hung instead of failing"
    assert procs[1].exitcode == 3
    assert Path(tmp_path, "rank0.txt").read_text().startswith("error")


def _breakdown_rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    """bench.py's per-rank view of a multi-GPU trace, over gloo on CPU: each
    rank contributes its per-step device times and token-write time."""
    sys.path[:0] = [str(ROOT / "paged-kv-cache_b200"), str(ROOT)]
    import json
    import types

    import torch
    import torch.distributed as dist

    import bench

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    run = types.SimpleNamespace(torch=torch, dist=dist, world=world, rank=rank,
                                dev=torch.device("cpu"))
    # Rank 1 is slower on steps 1 and 3; rank 0 on steps 0, 2 and 4.
    steps = [2.0, 1.0, 2.0, 1.0, 2.0] if rank == 0 else [1.0, 3.0, 1.0, 3.0, 1.0]
    out = bench.rank_breakdown(run, steps, write_bytes=6.55e9, write_ms=1000.0 * (1 + rank))
    Path(out_dir, f"rank{rank}.json").write_text(json.dumps(out))
    dist.destroy_process_group()


def test_rank_breakdown_over_two_gloo_ranks(tmp_path):
    import json

    import torch.multiprocessing as mp

    mp.start_processes(_breakdown_rank_main, args=(2, 29534, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    outs = [json.loads(Path(tmp_path, f"rank{r}.json").read_text()) for r in range(2)]
    assert outs[0] == outs[1]  # every rank computes the same view
    o = outs[0]
    assert o["device_ms_per_rank"] == [8.0, 9.0]
    assert o["steps_bounded_by_rank"] == [3, 2]
    fr = o["token_write_frac_of_peak_per_rank"]
    assert abs(fr[0] / fr[1] - 2.0) < 1e-9  # rank 1 took twice as long for the same bytes


def _gather_rank_main(rank: int, world: int, port: int, out_dir: str) -> None:
    """Each rank holds its head shard of a pool written through the oracle;
    rank 0 reassembles the full pool from the shards and compares it, element
    for element, with the pool the oracle writes unsharded."""
    sys.path[:0] = [str(ROOT / "paged-kv-cache_b200"), str(ROOT)]
    import torch
    import torch.distributed as dist

    from oracle.cpu import OracleBackend
    from pagedkv.config import CacheConfig
    from pagedkv.shard import entry_slice, gather_shards
    from pagedkv.workloads import Stream

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = CacheConfig(num_blocks=12, block_size=4, num_kv_heads=4, head_dim=8, num_layers=2,
                      dtype_bytes=4)
    e = cfg.entry_elems()
    off, w = entry_slice(e, rank, world)
    st = Stream(3)
    t = 30
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:t]
    dsts = [(int(s) // 4, int(s) % 4) for s in slots]
    full = OracleBackend(cfg)
    for layer in range(cfg.num_layers):
        k = st.normal(t * e).astype(np.float32).reshape(t, e)
        v = st.normal(t * e).astype(np.float32).reshape(t, e)
        full.write_kv_batch(layer, dsts, k.ravel(), v.ravel())
    fk, fv = full.planes()
    # This rank's shard: its slice of the entry axis.
    mine = (torch.from_numpy(np.ascontiguousarray(fk[..., off:off + w])),
            torch.from_numpy(np.ascontiguousarray(fv[..., off:off + w])))
    got = gather_shards(*mine)
    if rank == 0:
        ok = np.array_equal(got[0].numpy(), fk) and np.array_equal(got[1].numpy(), fv)
        Path(out_dir, "gather.txt").write_text(str(ok))
    else:
        assert got is None
    dist.destroy_process_group()


def test_shards_gathered_to_rank_zero_reassemble_the_pool(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_gather_rank_main, args=(2, 29535, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    assert Path(tmp_path, "gather.txt").read_text() == "True"
