"""Benchmark of the paged KV cache data path on B200.

Headline workload: a ragged prefill chunk at Qwen2-7B-like geometry
(28 layers, 4 KV heads x 128, bf16, block_size 16). One step is the hot path
over one chunk: device slot resolution from block tables, then
reshape_and_cache of every token into all 28 layers (one launch).

Scaling: the pool is sharded by KV head (each GPU owns entry slice
[r*E/N, (r+1)*E/N) of every block). At N GPUs a step processes N chunks of
65,536 tokens (N x 96 prompts) over a pool of N x 32,768 blocks, so every GPU
moves the same bytes per step at every N (weak scaling); no collective runs on
the data path. `value` is tokens/s over all GPUs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference algorithm (CpuBackend semantics, the C
restatement in oracle/) on the host cores, on a bounded sample of the same
workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "paged-kv-cache_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "KV tokens/s & HBM GB/s (reshape_and_cache, copy_blocks) at 1/2/4/8 B200"
CHUNK_TOKENS = 65536
CHUNK_PROMPTS = 96
BLOCKS_PER_CHUNK = 32768
GEOM = dict(block_size=16, num_kv_heads=4, head_dim=128, num_layers=28, dtype_bytes=2)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-ops", action="store_true")
    p.add_argument("--profile-small", action="store_true",
                   help="an 8,192-token chunk over a 2,048-block pool and nothing else, "
                        "for ncu captures")
    a = p.parse_args()
    a.chunk_tokens, a.chunk_prompts, a.chunk_blocks = CHUNK_TOKENS, CHUNK_PROMPTS, BLOCKS_PER_CHUNK
    if a.profile_small:
        a.chunk_tokens, a.chunk_prompts, a.chunk_blocks = 8192, 16, 2048
        a.no_e2e = a.no_cpu = a.no_ops = True
    return a


# ---- clocks ---------------------------------------------------------------------------------


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak_gbs() -> tuple[float, str]:
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def profile_traffic(name: str):
    """Per-launch DRAM bytes (read + write) from the committed ncu summary, if any."""
    p = ROOT / "profiles" / f"{name}.txt"
    try:
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1]))
    except OSError:
        pass
    return None


# ---- workload ---------------------------------------------------------------------------------


def build_batch(world: int, tokens: int = CHUNK_TOKENS, prompts: int = CHUNK_PROMPTS,
                blocks: int = BLOCKS_PER_CHUNK):
    """N prefill chunks, chunk c drawing its blocks from its own shuffled
    `blocks`-block range of the pool."""
    import numpy as np

    from pagedkv import CacheConfig
    from pagedkv.workloads import prefill_chunk

    cfg = CacheConfig(num_blocks=blocks * world, **GEOM)
    one = CacheConfig(num_blocks=blocks, **GEOM)
    ctx, new, tabs = [], [], []
    for c in range(world):
        b = prefill_chunk(seed=c, num_prompts=prompts, budget=tokens, cfg=one)
        t = b.tables.astype(np.int64)
        t[t >= 0] += c * blocks
        ctx.append(b.ctx)
        new.append(b.new)
        tabs.append(t.astype(np.int32))
    stride = max(t.shape[1] for t in tabs)
    tables = np.full((sum(len(x) for x in ctx), stride), -1, np.int32)
    r = 0
    for t in tabs:
        tables[r:r + len(t), : t.shape[1]] = t
        r += len(t)
    ctx = np.concatenate(ctx).astype(np.int32)
    new = np.concatenate(new).astype(np.int32)
    return cfg, tables, ctx, new


def host_slots(tables, ctx, new, block_size):
    import numpy as np

    q = np.repeat(np.arange(len(new)), new)
    starts = np.concatenate([[0], np.cumsum(new)[:-1]])
    j = np.arange(int(new.sum())) - np.repeat(starts, new)
    pos = ctx[q] + j
    return tables[q, pos // block_size].astype(np.int64), pos % block_size


# ---- our arm ----------------------------------------------------------------------------------


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from pagedkv import B200Backend, CacheConfig

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    cfg, tables, ctx, new = build_batch(world, args.chunk_tokens, args.chunk_prompts,
                                        args.chunk_blocks)
    T = int(new.sum())
    S = len(new)
    backend = B200Backend(cfg, dtype="bf16", device=local, shard_rank=rank, num_shards=world)
    es = backend.shard_entry_elems
    L = cfg.num_layers

    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    k = torch.randn((L, T, es), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn((L, T, es), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    d_tab = torch.from_numpy(tables).to(dev)
    d_ctx = torch.from_numpy(ctx).to(dev)
    d_new = torch.from_numpy(new).to(dev)
    d_cu = torch.empty(S + 1, dtype=torch.int32, device=dev)
    d_slots = torch.empty(T, dtype=torch.int64, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step():
        backend.resolve_slots(d_tab, d_ctx, d_new, T, d_cu, d_slots, stream=stream)
        backend.reshape_and_cache(k, v, d_slots, stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    barrier()
    if backend.device_error() is not None:
        raise SystemExit(f"device error in warm-up: {backend.device_error()}")

    # Correctness of the timed configuration: every token's entry landed in its slot.
    pk, pv = backend.planes()
    slot_host = d_slots.cpu().numpy()
    chk = torch.from_numpy(slot_host[:: max(1, T // 4096)]).to(dev)
    idx = torch.arange(0, T, max(1, T // 4096), device=dev)
    ok = all(torch.equal(pk[l].reshape(-1, es)[chk], k[l, idx]) and
             torch.equal(pv[l].reshape(-1, es)[chk], v[l, idx]) for l in (0, L // 2, L - 1))
    if not ok:
        raise SystemExit("bench: pool contents differ from the inputs")

    K = args.steps
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]

    def load(seconds: float) -> None:
        """Untimed steps that keep the GPU busy while the clocks are sampled."""
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            with torch.cuda.stream(stream):
                for _ in range(20):
                    step()
            stream.synchronize()

    barrier()
    with ClockSampler(local) as clocks:
        load(1.0)
        barrier()
        with torch.cuda.stream(stream):
            for i in range(K):
                ev[i][0].record(stream)
                backend.resolve_slots(d_tab, d_ctx, d_new, T, d_cu, d_slots, stream=stream)
                ev[i][1].record(stream)
                backend.reshape_and_cache(k, v, d_slots, stream=stream)
                ev[i][2].record(stream)
        barrier()
        load(0.3)
    barrier()
    total_ms = ev[0][0].elapsed_time(ev[K - 1][2])
    resolve_ms = [ev[i][0].elapsed_time(ev[i][1]) for i in range(K)]
    reshape_ms = [ev[i][1].elapsed_time(ev[i][2]) for i in range(K)]
    total_ms = max_over_ranks(total_ms)
    reshape_avg = max_over_ranks(sum(reshape_ms) / K)
    resolve_avg = max_over_ranks(sum(resolve_ms) / K)

    # Shard verification: each rank digests its shard and the rows it wrote;
    # the ranks all-gather the digests (NCCL) and check them.
    from pagedkv.shard import verify_over_group

    verify = verify_over_group(backend.digest(stream=stream),
                               backend.digest_rows(k, v, d_slots, stream=stream), device=dev)
    if not verify["ok"]:
        raise SystemExit(f"bench: shard verification failed: {verify}")

    # Every rank writes its head slice of all T tokens, so a step stores T
    # whole tokens across the N GPUs.
    tokens_all = T
    value = tokens_all * K / (total_ms / 1e3)
    eb = es * 2
    alg_bytes = T * L * 2 * eb * 2 + T * 8  # read + write K and V, one slot read per token
    peak, peak_kind = measured_peak_gbs()
    achieved = alg_bytes / (reshape_avg / 1e3) / 1e9

    out = {
        "metric": METRIC,
        "value": value,
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": total_ms / K,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded: log-uniform prompt lengths, shuffled free list, normal K/V)",
        "config": {
            "workload": f"ragged prefill chunk x{world}: {world}x{args.chunk_tokens} tokens "
                        f"({S} prompts, log-uniform 128..4096), Qwen2-7B KV geometry "
                        f"(28 layers, 4 KV heads x 128, bs 16), pool {cfg.num_blocks} blocks "
                        f"head-sharded {world} ways; step = device slot resolution + "
                        "all-layer reshape_and_cache",
            "tokens_per_step": tokens_all,
            "layers": L,
            "entry_elems_per_gpu": es,
            "pool_gib_per_gpu": round(backend.allocated_bytes() / 2**30, 2),
            "parallelism": f"kv-head shards x{world}",
            "l2": "inputs (K/V %.2f GiB per GPU) exceed the 126 MB L2; no flush needed" %
                  (2 * L * T * eb / 2**30),
        },
        "gb_per_s": alg_bytes * world / (total_ms / K / 1e3) / 1e9,
        "roofline": {
            "kernel": "reshape_copy_kernel (all layers)",
            "bound": "hbm",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / peak,
            "traffic": profile_traffic("reshape_prefill_ncu"),
            "algorithmic_bytes_per_launch": alg_bytes,
            "kernel_ms": reshape_avg,
        },
        "resolve_slots_ms": resolve_avg,
        "gpu_launches": 2 * K,
        "verify": verify,
        "clocks": {**clocks.summary(),
                   "window": "sampled every 200 ms over 1.3 s of continuous load around the timed steps"},
    }

    if not args.no_ops and rank == 0:
        out["ops"] = bench_ops(backend, cfg, dev, stream)

    if not args.no_e2e:
        out["e2e"] = e2e_host_path(args, backend, tables, ctx, new, k, v, barrier, max_over_ranks,
                                   world)

    if rank == 0 and world == 1 and not args.no_cpu:
        n = 4096
        out["cpu_baseline"] = cpu_sample(tables, ctx, new, k[:, :n].float().cpu().numpy(),
                                         v[:, :n].float().cpu().numpy(), seconds=8.0, threads=1)

    backend.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def e2e_host_path(args, backend, tables, ctx, new, k, v, barrier, max_over_ranks, world):
    """Same step through the C ABI's KvBackend entry points with host buffers:
    per layer pkv_write_kv_batch from pinned bf16 rows (host->device copies in
    the timed region), then the device error word read back."""
    import numpy as np
    import torch

    L, T, es = k.shape
    blocks, offs = host_slots(tables, ctx, new, backend.config().block_size)
    hk = k.view(torch.int16).cpu().pin_memory().numpy().view(np.uint16)
    hv = v.view(torch.int16).cpu().pin_memory().numpy().view(np.uint16)
    steps = max(1, min(args.steps, 5))

    def one():
        for layer in range(L):
            backend.write_kv_batch_slots(layer, blocks, offs, hk[layer], hv[layer], host_dtype="bf16")
        if backend.device_error() is not None:
            raise SystemExit("device error in e2e step")

    one()
    barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    barrier()
    dt = max_over_ranks(time.perf_counter() - t0)
    return {"value": T * steps / dt, "unit": "tokens/s",
            "h2d_bytes_per_step": int(L * (2 * T * es * 2 + T * 8)),
            "d2h_bytes_per_step": 16, "steps": steps,
            "path": "pkv_write_kv_batch per layer, pinned bf16 host rows, + pkv_device_error"}


def bench_ops(backend, cfg, dev, stream, reps: int = 10) -> dict:
    """Per-kernel timings on this GPU's shard: copy_blocks (256 copy-on-write
    pairs, every layer), zero_blocks (64 blocks) and a 256-token decode step."""
    import numpy as np
    import torch

    from pagedkv.workloads import Stream

    peak, _ = measured_peak_gbs()
    es = backend.shard_entry_elems
    L, bs = cfg.num_layers, cfg.block_size
    block_bytes = bs * es * 2
    flush = torch.ones(256 * 2**20, dtype=torch.uint8, device=dev)
    st = Stream(77)
    ids = st.permutation(cfg.num_blocks)
    res = {}

    def timed(fn, nbytes, name, extra=None):
        """Mean over `reps` launches; before each, a 256 MB read on the same
        stream evicts the previous launch's lines from the 126 MB L2."""
        times = []
        for i in range(reps + 2):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                flush.sum(dtype=torch.int64)
                a.record(stream)
                fn()
                b.record(stream)
            stream.synchronize()
            if i >= 2:
                times.append(a.elapsed_time(b))
        ms = sum(times) / len(times)
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"ms": ms, "gb_per_s": gbs, "frac_of_peak": gbs / peak,
                     "algorithmic_bytes": nbytes, **(extra or {})}

    pairs = torch.from_numpy(np.stack([ids[:256], ids[256:512]], 1).astype(np.int64)).to(dev)
    timed(lambda: backend.copy_blocks_dev(pairs, stream=stream),
          256 * L * 2 * block_bytes * 2 + 256 * 16, "copy_blocks", {"pairs": 256, "layers": L})
    zero = torch.from_numpy(ids[512:576].astype(np.int64)).to(dev)
    timed(lambda: backend.zero_blocks_dev(zero, stream=stream),
          64 * L * 2 * block_bytes + 64 * 8, "zero_blocks", {"blocks": 64})
    td = 256
    kd = torch.randn((L, td, es), device=dev).to(torch.bfloat16)
    sl = torch.from_numpy((ids[600:856] * bs + st.integers(256, 0, bs - 1)).astype(np.int64)).to(dev)
    timed(lambda: backend.reshape_and_cache(kd, kd, sl, stream=stream),
          td * L * 2 * es * 2 * 2 + td * 8, "decode_reshape_all_layers", {"tokens": td})
    assert backend.device_error() is None
    return res


class CpuArm:
    """CpuBackend semantics (the C restatement in oracle/, f32 planes like the
    reference) on a bounded sample of the workload: the first `sample` tokens
    of the chunk, all layers, slots folded into a 1,024-block pool. Rows are
    split over `threads` host threads (disjoint tokens)."""

    NB = 1024

    def __init__(self, tables, ctx, new, kf, vf, threads: int):
        import numpy as np

        from oracle.cpu import OracleBackend
        from pagedkv import CacheConfig

        L, sample, es = kf.shape
        self.L, self.sample, self.es = L, sample, es
        cfg = CacheConfig(num_blocks=self.NB, block_size=16, num_kv_heads=1, head_dim=es,
                          num_layers=L, dtype_bytes=4)
        blocks, offs = host_slots(tables, ctx, new, 16)
        pairs = np.stack([blocks[:sample] % self.NB, offs[:sample]], 1).astype(np.uint64)
        self.orc = OracleBackend(cfg)
        parts = [p for p in np.array_split(np.arange(sample), threads) if len(p)]
        self.rows = [(np.ascontiguousarray(pairs[p]),
                      [np.ascontiguousarray(kf[l, p]) for l in range(L)],
                      [np.ascontiguousarray(vf[l, p]) for l in range(L)]) for p in parts]
        self.threads = len(self.rows)
        for kp, vp in zip(*self.orc.planes()):  # fault the planes in before timing
            kp.fill(0)
            vp.fill(0)

    def _work(self, pairs, ks, vs):
        for layer in range(self.L):
            self.orc.write_kv_batch_pairs(layer, pairs, ks[layer], vs[layer])

    def one_pass(self) -> None:
        if self.threads == 1:
            self._work(*self.rows[0])
            return
        ts = [threading.Thread(target=self._work, args=r) for r in self.rows]
        for t in ts:
            t.start()
        for t in ts:
            t.join()

    def describe(self, passes: int) -> str:
        return (f"{self.sample} tokens x {self.L} layers per pass, {passes} pass(es), f32 planes "
                f"of {self.NB} blocks x 16 slots x {self.es} (CpuBackend semantics, "
                "oracle/pkv_oracle.c)")


def cpu_sample(tables, ctx, new, kf, vf, seconds: float, threads: int) -> dict:
    arm = CpuArm(tables, ctx, new, kf, vf, threads)
    arm.one_pass()
    n = 0
    t0 = time.perf_counter()
    while True:
        arm.one_pass()
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    return {"value": arm.sample * n / dt, "unit": "tokens/s", "cores": arm.threads,
            "kind": "port", "sample": arm.describe(n)}


# ---- reference arm ----------------------------------------------------------------------------


def run_reference(args):
    """The reference algorithm on the host cores: CpuBackend semantics
    (oracle/pkv_oracle.c; the Rust crate cannot be built here), one thread
    per core over disjoint tokens, on a bounded sample of the same workload."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from pagedkv.workloads import Stream, bf16_bits_to_f32, f32_to_bf16_bits

    cfg, tables, ctx, new = build_batch(1)
    L = cfg.num_layers
    threads = os.cpu_count() or 1
    sample = 4096
    st = Stream(5)
    kf = bf16_bits_to_f32(f32_to_bf16_bits(st.normal(L * sample * 512))).reshape(L, sample, 512)
    vf = bf16_bits_to_f32(f32_to_bf16_bits(st.normal(L * sample * 512))).reshape(L, sample, 512)
    arm = CpuArm(tables, ctx, new, kf, vf, threads)
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        arm.one_pass()
        if i >= args.warmup:
            times.append(time.perf_counter() - t0)
    per = sum(times) / len(times)
    value = sample / per
    out = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
           "config": {"workload": "ragged prefill chunk, Qwen2-7B KV geometry (28 layers, "
                                  "entry 512); bounded sample per step: 4096 tokens x 28 layers"},
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": arm.threads,
                            "kind": "port", "sample": arm.describe(len(times))},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
