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
    p.add_argument("--workload", choices=["prefill", "decode", "cow", "churn", "attention"],
                   default="prefill",
                   help="prefill: ragged 65,536-token chunk (headline); decode: 256-sequence "
                        "decode step; cow: beam-search copy-on-write trace; churn: "
                        "continuous-batching trace at 70B-like geometry")
    p.add_argument("--fork-rate", type=float, default=0.05,
                   help="churn: probability per step of forking a running sequence")
    p.add_argument("--no-graph", action="store_true", help="decode: launch instead of graph replay")
    p.add_argument("--graph-steps", type=int, default=0,
                   help="decode: steps captured per CUDA graph (0: the largest divisor of "
                        "--steps up to 8)")
    p.add_argument("--strong", action="store_true",
                   help="prefill/decode: strong scaling -- one chunk (or decode batch) over one "
                        "32,768-block pool, head-sharded over the N GPUs, instead of N of them")
    p.add_argument("--unfused", action="store_true",
                   help="resolve slots and scatter in two launches instead of the fused kernel")
    p.add_argument("--pool-dtype", choices=["bf16", "fp8"], default="bf16",
                   help="prefill/decode: pool element type; fp8 quantises the bf16 rows to E4M3 "
                        "with per-(layer, kv head) scales in the same launch")
    p.add_argument("--compare-library", action="store_true",
                   help="attention: also time flashinfer's paged decode (tensor-core path) on "
                        "the same pool, for comparison")
    p.add_argument("--no-fuse", action="store_true",
                   help="cow/churn: copy_blocks and zero_blocks as two launches per step, and "
                        "a step's resolved and host-slot tokens as two launches")
    p.add_argument("--copy-engine", choices=["auto", "vector", "bulk"], default="auto",
                   help="cow/churn: copy_blocks engine (pkv_set_copy_engine)")
    p.add_argument("--q-len", type=int, default=1,
                   help="attention: query tokens per sequence (the last q_len positions, causal; "
                        "q_len * 7 <= 16)")
    p.add_argument("--no-plan", action="store_true",
                   help="attention: sequences in batch order (no pkv_paged_attention_plan_dev)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-ops", action="store_true")
    p.add_argument("--profile-small", action="store_true",
                   help="an 8,192-token chunk over a 2,048-block pool and nothing else, "
                        "for ncu captures")
    p.add_argument("--with-ops", action="store_true",
                   help="with --profile-small: also the per-kernel timings (copy_blocks, "
                        "zero_blocks, decode step) over the small pool")
    a = p.parse_args()
    a.chunk_tokens, a.chunk_prompts, a.chunk_blocks = CHUNK_TOKENS, CHUNK_PROMPTS, BLOCKS_PER_CHUNK
    if a.profile_small:
        a.chunk_tokens, a.chunk_prompts, a.chunk_blocks = 8192, 16, 2048
        a.no_e2e = a.no_cpu = True
        a.no_ops = not a.with_ops
    return a


# ---- clocks ---------------------------------------------------------------------------------


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons of the GPUs in `indices`
    while the timed region runs. One process (rank 0) samples every GPU of
    the job; it waits for the first sample before the load starts."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, indices, active: bool = True):
        self.indices = list(indices)
        self.active = active
        self.proc = None
        self.lines: list[str] = []
        self.first = threading.Event()

    def __enter__(self):
        if not self.active:
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", ",".join(str(i) for i in self.indices),
                 f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
            self.first.wait(timeout=20.0)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())
            self.first.set()

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
                "reasons": sorted(reasons), "samples": len(sm), "gpus": self.indices}


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


class Run:
    """One rank of the benchmark: device, stream, process group and timing helpers."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.args = args
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if args.gpus != self.world and self.world > 1:
            raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {self.world}")
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        # The ranks of one box share its host cores: give each rank's host
        # stager (the e2e paths) its share instead of one thread per core each.
        local_world = int(os.environ.get("LOCAL_WORLD_SIZE", "1"))
        if local_world > 1:
            os.environ.setdefault("PKV_HOST_THREADS",
                                  str(max(1, (os.cpu_count() or 1) // local_world)))
        if self.world > 1:
            from datetime import timedelta

            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=self.dev)
        self.stream = torch.cuda.Stream(device=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def load(self, step, seconds: float) -> None:
        """Untimed steps that keep the GPU busy while the clocks are sampled."""
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < seconds:
            with self.torch.cuda.stream(self.stream):
                for _ in range(20):
                    step()
            self.stream.synchronize()

    def timed_steps(self, step, K: int, marks_per_step: int = 1):
        """K steps between CUDA events on the benchmark stream, with the
        clocks sampled over 1.3 s of continuous load around them. `step(i, ev)`
        records its own inner events into ev (a list) if it wants."""
        torch = self.torch
        evs = []
        self.barrier()
        with ClockSampler(range(self.world), active=self.rank == 0) as clocks:
            self.barrier()
            self.load(lambda: step(-1, None), 1.0)
            self.barrier()
            start = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(self.stream):
                start.record(self.stream)
                for i in range(K):
                    ev = []
                    step(i, ev)
                    evs.append(ev)
                end = torch.cuda.Event(enable_timing=True)
                end.record(self.stream)
            self.barrier()
            self.load(lambda: step(-1, None), 0.3)
        self.barrier()
        total = self.max_over_ranks(start.elapsed_time(end))
        return total, evs, {**clocks.summary(),
                            "window": "sampled every 200 ms over 1.3 s of continuous load "
                                      "around the timed steps"}

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def _event_ms(evs, i, j):
    return sum(e[i].elapsed_time(e[j]) for e in evs) / max(len(evs), 1)


def base_line(run, value, K, ms_per_step, scaling, workload, extra_config, data) -> dict:
    return {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": run.world, "steps": K,
        "warmup": run.args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "bf16", "data": data,
        "config": {"workload": workload, **extra_config},
    }


def roofline(kernel, alg_bytes, kernel_ms, traffic=None) -> dict:
    peak, peak_kind = measured_peak_gbs()
    achieved = alg_bytes / (kernel_ms / 1e3) / 1e9
    return {"kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": peak,
            "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
            "algorithmic_bytes_per_launch": alg_bytes, "kernel_ms": kernel_ms}


def check_rows_landed(backend, k, v, d_slots, T, L, inv=None):
    """Every token's entry is in its slot (strided sample of tokens, 3 layers).
    For an fp8 pool, `inv` = ([L][heads_here] K, V reciprocal scales): the
    slot holds E4M3(row * inv), which torch's round-to-nearest-even
    float8_e4m3fn conversion reproduces for these unsaturated rows."""
    torch = __import__("torch")
    es = k.shape[2]
    pk, pv = backend.planes()
    stride = max(1, T // 4096)
    idx = torch.arange(0, T, stride, device=k.device)
    chk = d_slots[idx]

    def want(x, l, plane):
        if inv is None:
            return x[l, idx]
        r = inv[plane][l].repeat_interleave(es // inv[plane].shape[1])
        return (x[l, idx].float() * r).to(torch.float8_e4m3fn).view(torch.uint8)

    def got(p, l):
        rows = p[l].reshape(-1, es)[chk]
        return rows.view(torch.uint8) if inv is not None else rows

    ok = all(torch.equal(got(pk, l), want(k, l, 0)) and torch.equal(got(pv, l), want(v, l, 1))
             for l in (0, L // 2, L - 1))
    if not ok:
        raise SystemExit("bench: pool contents differ from the inputs")


def wl_table_batch(run, kind: str) -> dict:
    """Prefill chunk (config 3, the headline) or decode step (config 2): one
    step = device slot resolution + one all-layer reshape_and_cache."""
    import numpy as np

    torch = run.torch
    from pagedkv import B200Backend
    from pagedkv.shard import verify_over_group

    args, world, dev, stream = run.args, run.world, run.dev, run.stream
    copies = 1 if args.strong else world  # chunks (decode batches) per step over all GPUs
    if kind == "prefill":
        cfg, tables, ctx, new = build_batch(copies, args.chunk_tokens, args.chunk_prompts,
                                            args.chunk_blocks)
    else:
        cfg, tables, ctx, new = build_decode(copies)
    T, S = int(new.sum()), len(new)
    fp8 = args.pool_dtype == "fp8"
    if fp8:
        from pagedkv import CacheConfig
        cfg = CacheConfig(num_blocks=cfg.num_blocks, block_size=cfg.block_size,
                          num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                          num_layers=cfg.num_layers, dtype_bytes=1)
    backend = B200Backend(cfg, dtype="fp8_e4m3" if fp8 else "bf16", device=run.local,
                          shard_rank=run.rank, num_shards=world)
    es, L = backend.shard_entry_elems, cfg.num_layers
    inv = None
    if fp8:
        # Seeded per-(layer, kv head) scales in [0.5, 2]; rows here hold this GPU's heads.
        from pagedkv.workloads import Stream
        st = Stream(55)
        n = L * cfg.num_kv_heads
        sk = st.uniform(n, 0.5, 2.0).astype(np.float32).reshape(L, cfg.num_kv_heads)
        sv = st.uniform(n, 0.5, 2.0).astype(np.float32).reshape(L, cfg.num_kv_heads)
        backend.set_kv_scales(sk, sv)
        h0 = backend.elem_offset // cfg.head_dim
        h1 = -(-(backend.elem_offset + es) // cfg.head_dim)
        inv = tuple(torch.from_numpy(np.float32(1.0) / s_[:, h0:h1]).to(dev) for s_ in (sk, sv))
    gen = torch.Generator(device=dev).manual_seed(1000 + run.rank)
    k = torch.randn((L, T, es), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn((L, T, es), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    d_tab = torch.from_numpy(tables).to(dev)
    d_ctx = torch.from_numpy(ctx).to(dev)
    d_new = torch.from_numpy(new).to(dev)
    d_cu = torch.empty(S + 1, dtype=torch.int32, device=dev)
    d_slots = torch.empty(T, dtype=torch.int64, device=dev)

    def launch():
        if args.unfused:
            backend.resolve_slots(d_tab, d_ctx, d_new, T, d_cu, d_slots, stream=stream)
            backend.reshape_and_cache(k, v, d_slots, stream=stream)
        else:  # one launch: slots resolved inline, also published to d_slots
            backend.resolve_and_cache(d_tab, d_ctx, d_new, T, d_cu, k, v, slots_out=d_slots,
                                      stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            launch()
    run.barrier()
    if backend.device_error() is not None:
        raise SystemExit(f"device error in warm-up: {backend.device_error()}")
    check_rows_landed(backend, k, v, d_slots, T, L, inv)

    graph, per_graph = None, 1
    if kind == "decode" and not args.no_graph:
        # The decode step is launch-bound. An engine replays its whole decode
        # iteration as one CUDA graph, so the cache write runs back to back
        # with other kernels; here G consecutive steps are captured in one
        # graph (each a full launch over all 256 tokens and 28 layers), so
        # one replay from Python does not cost more than G steps of device work.
        per_graph = args.graph_steps or max(d for d in range(1, 9) if args.steps % d == 0)
        if args.steps % per_graph:
            raise SystemExit(f"--steps {args.steps} is not a multiple of --graph-steps {per_graph}")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(per_graph):
                launch()
        torch.cuda.synchronize()

    def step(i, ev):
        if graph is not None:
            if i < 0 or i % per_graph == 0:  # steps i .. i + G - 1 (i = -1: untimed load)
                graph.replay()
            return
        if ev is not None and args.unfused:
            for _ in range(3):
                ev.append(torch.cuda.Event(enable_timing=True))
            ev[0].record(stream)
            backend.resolve_slots(d_tab, d_ctx, d_new, T, d_cu, d_slots, stream=stream)
            ev[1].record(stream)
            backend.reshape_and_cache(k, v, d_slots, stream=stream)
            ev[2].record(stream)
        elif ev is not None:
            for _ in range(2):
                ev.append(torch.cuda.Event(enable_timing=True))
            ev[0].record(stream)
            launch()
            ev[1].record(stream)
        else:
            launch()

    K = args.steps
    total_ms, evs, clocks = run.timed_steps(step, K)
    eb = es * 2
    pool_eb = es * (1 if fp8 else 2)
    # Read K and V rows (bf16) + write them into the pool, one slot per token.
    alg_bytes = T * L * 2 * (eb + pool_eb) + T * 8
    if graph is None and args.unfused:
        kernel_ms = run.max_over_ranks(_event_ms(evs, 1, 2))
        resolve_ms = run.max_over_ranks(_event_ms(evs, 0, 1))
    elif graph is None:
        kernel_ms = run.max_over_ranks(_event_ms(evs, 0, 1))
        resolve_ms = 0.0
    else:
        # Kernel time inside the graph: the steps run back to back, so the
        # device time per step is the kernel plus the gap between launches.
        # A launch bracketed by events on its own is reported beside it.
        kernel_ms = total_ms / K
        evs2 = []
        with torch.cuda.stream(stream):
            for _ in range(max(K, 10)):
                e = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
                e[0].record(stream)
                launch()
                e[1].record(stream)
                evs2.append(e)
        stream.synchronize()
        single_launch_ms = run.max_over_ranks(_event_ms(evs2, 0, 1))
        resolve_ms = 0.0 if not args.unfused else None

    verify = verify_over_group(backend.digest(stream=stream),
                               backend.digest_rows(k, v, d_slots, stream=stream), device=dev)
    if not verify["ok"]:
        raise SystemExit(f"bench: shard verification failed: {verify}")

    workload, extra = table_batch_config(args, kind, world, cfg, T, S,
                                         per_graph if graph is not None else 0)
    out = base_line(run, T * K / (total_ms / 1e3), K, total_ms / K,
                    "strong" if args.strong else "weak", workload, extra,
                    "synthetic (seeded: shuffled free list, " + ("log-uniform prompt lengths" if kind == "prefill"
                                                       else "uniform context lengths") + ", normal K/V)")
    out["gb_per_s"] = alg_bytes * world / (total_ms / K / 1e3) / 1e9
    if fp8:
        kname = ("reshape_fp8_kernel (all layers)" if args.unfused else
                 "resolve_cache_fp8_kernel (slot resolution fused with the all-layer quantising "
                 "reshape_and_cache)")
        prof = "reshape_fp8_prefill_ncu" if args.unfused else "resolve_cache_fp8_prefill_ncu"
    else:
        kname = ("reshape_copy_kernel (all layers)" if args.unfused else
                 "resolve_cache_kernel (slot resolution fused with the all-layer reshape_and_cache)")
        prof = "reshape_prefill_ncu" if args.unfused else "resolve_cache_prefill_ncu"
    out["roofline"] = roofline(kname, alg_bytes, kernel_ms,
                               profile_traffic(prof) if kind == "prefill" else None)
    if args.unfused:
        out["resolve_slots_ms"] = resolve_ms
    out["gpu_launches"] = (2 if args.unfused else 1) * K
    if graph is not None:
        out["config"]["steps_per_graph"] = per_graph
        out["single_launch_ms"] = single_launch_ms
    out["verify"] = verify
    out["clocks"] = clocks
    if kind == "prefill" and not args.no_ops and run.rank == 0:
        ops = bench_ops(backend, cfg, dev, stream)
        cb = ops["copy_blocks"]
        # The second kernel the metric names, as its own roofline object:
        # the copy-on-write microbenchmark (distinct pairs, L2 flushed).
        out["copy_blocks"] = {
            **roofline("copy_blocks_kernel (256 distinct pairs x 28 layers x K,V planes of "
                       f"{cfg.block_size * es * 2 // 1024} KiB, L2 flushed before each launch)",
                       cb["algorithmic_bytes"], cb["ms"],
                       profile_traffic("copy_blocks_pairs_ncu") if world == 1 else None),
            "pairs": cb["pairs"], "layers": L, "launches_timed": cb["launches"]}
        out["ops"] = {name: {"ms": round(r["ms"], 4), "frac": round(r["frac_of_peak"], 3)}
                      for name, r in ops.items()}
    if not args.no_e2e:
        out["e2e"] = e2e_host_path(args, backend, tables, ctx, new, k, v, run.barrier,
                                   run.max_over_ranks, mode="bf16_pinned")
        out["e2e_f32"] = e2e_host_path(args, backend, tables, ctx, new, k, v, run.barrier,
                                       run.max_over_ranks, mode="f32_pageable",
                                       link=out["e2e"]["link_h2d_gb_per_s"])
    if run.rank == 0 and world == 1 and not args.no_cpu:
        n = min(4096, T)
        out["cpu_baseline"] = cpu_sample(tables, ctx, new, k[:, :n].float().cpu().numpy(),
                                         v[:, :n].float().cpu().numpy(), seconds=8.0, threads=1,
                                         head_dim=cfg.head_dim,
                                         fp8_scales=(sk, sv) if fp8 else None)
    graph = None  # release the captured graph before its pool is freed
    backend.close()
    if "copy_blocks" in out:  # last, so that a truncated tail of the line still holds it
        out["copy_blocks"] = out.pop("copy_blocks")
    return out


def table_batch_config(args, kind: str, world: int, cfg, T: int, S: int,
                       per_graph: int = 0) -> tuple[str, dict]:
    """`config.workload` and the other config keys of a prefill-chunk or
    decode-step line. Both arms print the same ones: the reference arm
    describes its bounded sample under `cpu_baseline.sample`."""
    copies = 1 if args.strong else world
    fp8 = args.pool_dtype == "fp8"
    L = cfg.num_layers
    es = cfg.num_kv_heads * cfg.head_dim // world
    eb = es * 2
    # Every rank writes its head slice of all T tokens, so a step stores T
    # whole tokens across the N GPUs.
    if kind == "prefill":
        workload = (f"ragged prefill chunk x{copies}: {copies}x{args.chunk_tokens} tokens ({S} prompts, "
                    "log-uniform 128..4096)")
    else:
        workload = f"decode step x{copies}: {copies}x256 sequences, context U[1,4096], +1 token each"
    workload += (f", Qwen2-7B KV geometry (28 layers, 4 KV heads x 128, bs 16), pool "
                 f"{cfg.num_blocks} blocks (shuffled free list) head-sharded {world} ways, "
                 + ("fp8 E4M3 pool (bf16 rows quantised with per-layer, per-head scales)"
                    if fp8 else "bf16 pool") + "; step = "
                 + ("device slot resolution + all-layer reshape_and_cache" if args.unfused else
                  "slot resolution fused with the all-layer reshape_and_cache (one launch)")
                 + (f" ({per_graph} steps captured per CUDA graph)" if per_graph else ""))
    pool_bytes = 2 * L * cfg.num_blocks * cfg.block_size * es * (1 if fp8 else 2)
    return workload, {
        "tokens_per_step": T, "sequences_per_step": S, "layers": L, "entry_elems_per_gpu": es,
        "pool_gib_per_gpu": round(pool_bytes / 2**30, 2),
        "parallelism": f"kv-head shards x{world}",
        "l2": ("inputs (K/V %.2f GiB per GPU) exceed the 126 MB L2; no flush needed"
               % (2 * L * T * eb / 2**30)) if 2 * L * T * eb > 2**28 else
              "inputs (%.1f MiB) fit in L2; every step rewrites the same rows, as a decode "
              "step re-reads a projection's fresh output" % (2 * L * T * eb / 2**20),
        "pool_dtype": "fp8_e4m3" if fp8 else "bf16",
    }


def build_decode(world: int):
    """N decode batches of 256 sequences (config 2), batch c on its own
    32,768-block range of the pool, each from a shuffled free list; batch c
    uses the c-th seed (from 0 up) whose demand fits the range."""
    import numpy as np

    from pagedkv import CacheConfig
    from pagedkv.workloads import decode_batch

    cfg = CacheConfig(num_blocks=BLOCKS_PER_CHUNK * world, **GEOM)
    one = CacheConfig(num_blocks=BLOCKS_PER_CHUNK, **GEOM)
    parts, seed = [], 0
    for c in range(world):
        b = decode_batch(seed=None, first_seed=seed, cfg=one)
        seed = b.seed + 1
        t = b.tables.astype(np.int64)
        t[t >= 0] += c * BLOCKS_PER_CHUNK
        parts.append((b.ctx, b.new, t.astype(np.int32)))
    return (cfg, np.concatenate([p[2] for p in parts]),
            np.concatenate([p[0] for p in parts]).astype(np.int32),
            np.concatenate([p[1] for p in parts]).astype(np.int32))


def wl_attention(run) -> dict:
    """Decode attention over the config-2 batch (256 sequences, context
    U[1,4096] + the appended token, Qwen2-7B: 28 query heads over 4 kv heads
    x 128, bf16): one step = paged attention for all 28 layers."""
    import numpy as np

    torch = run.torch
    from pagedkv import B200Backend

    args, world, dev, stream = run.args, run.world, run.dev, run.stream
    cfg, tables, ctx, new = build_decode(world)
    if args.profile_small:  # the same per-layer launches over a 2-layer pool (2.1 GB), for ncu
        from pagedkv import CacheConfig
        cfg = CacheConfig(num_blocks=cfg.num_blocks, block_size=cfg.block_size,
                          num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, num_layers=2,
                          dtype_bytes=cfg.dtype_bytes)
    if cfg.num_kv_heads % world:
        raise SystemExit("attention workload: kv heads must split evenly over the GPUs")
    fp8 = args.pool_dtype == "fp8"
    if fp8:
        from pagedkv import CacheConfig
        cfg = CacheConfig(num_blocks=cfg.num_blocks, block_size=cfg.block_size,
                          num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                          num_layers=cfg.num_layers, dtype_bytes=1)
    backend = B200Backend(cfg, dtype="fp8_e4m3" if fp8 else "bf16", device=run.local,
                          shard_rank=run.rank, num_shards=world)
    L, D = cfg.num_layers, cfg.head_dim
    kvh = backend.shard_entry_elems // D
    hq = kvh * 7  # Qwen2-7B: 28 query heads over 4 kv heads
    ql = args.q_len
    if ql < 1 or ql * 7 > 16:
        raise SystemExit("attention workload: q_len * 7 query heads per kv head must be <= 16")
    lens = (ctx + new).astype(np.int32)  # the appended token is in the cache too
    if int(lens.min()) < ql:  # the query tokens are the last q_len of each context
        raise SystemExit("attention workload: a context is shorter than q_len")
    S = len(lens)
    max_ctx = int(lens.max())
    gen = torch.Generator(device=dev).manual_seed(3000 + run.rank)
    h0 = backend.elem_offset // D
    scales = None
    if fp8:
        # Codes of N(0, 3) values with seeded per-(layer, kv head) scales in
        # [0.2, 0.5]: the cache holds values of about N(0, 1).
        from pagedkv.workloads import Stream
        st = Stream(55)
        n = L * cfg.num_kv_heads
        sk = st.uniform(n, 0.2, 0.5).astype(np.float32).reshape(L, cfg.num_kv_heads)
        sv = st.uniform(n, 0.2, 0.5).astype(np.float32).reshape(L, cfg.num_kv_heads)
        backend.set_kv_scales(sk, sv)
        scales = tuple(torch.from_numpy(x[:, h0:h0 + kvh]).to(dev) for x in (sk, sv))
    with torch.cuda.stream(stream):
        for p_ in backend.planes():
            for l in range(L):
                x = torch.randn(p_[l].shape, generator=gen, device=dev)
                p_[l].copy_((x * 3).to(torch.float8_e4m3fn) if fp8 else x.to(torch.bfloat16))
        q = torch.randn((S * ql, hq, D), generator=gen, device=dev).to(torch.bfloat16)
    stream.synchronize()
    d_tab = torch.from_numpy(tables).to(dev)
    d_len = torch.from_numpy(lens).to(dev)
    out = torch.empty((L, S * ql, hq, D), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((L, S * ql, hq), dtype=torch.float32, device=dev)

    plan = not args.no_plan  # one longest-first order per step, for all its layers

    def step(i, ev):
        if ev is not None:
            ev.extend(torch.cuda.Event(enable_timing=True) for _ in range(2))
            ev[0].record(stream)
        if plan:
            backend.paged_attention_plan(d_len, max_ctx, stream=stream)
        for l in range(L):
            backend.paged_attention(q, d_tab, d_len, max_ctx, out[l], l, lse=lse[l], stream=stream,
                                    q_len=ql)
        if ev is not None:
            ev[1].record(stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step(0, None)
    stream.synchronize()
    if backend.device_error() is not None:
        raise SystemExit(f"device error in attention warm-up: {backend.device_error()}")
    # Spot check against a float32 torch attention of 8 sequences on 2 layers.
    kp, vp = backend.planes()
    worst = 0.0
    for l in (0, L - 1):
        for s_ in range(0, S, S // 8):
            n = int(lens[s_])
            t = torch.arange(n, device=dev)
            blk = d_tab[s_, t // 16].long()
            kk = kp[l, blk, t % 16].float().view(n, kvh, D)
            vv = vp[l, blk, t % 16].float().view(n, kvh, D)
            if fp8:  # code * scale per kv head
                kk = kk * scales[0][l].view(1, kvh, 1)
                vv = vv * scales[1][l].view(1, kvh, 1)
            kk, vv = kk.repeat_interleave(7, 1), vv.repeat_interleave(7, 1)
            for i in range(ql):  # query token i sees keys 0 .. n - ql + i
                m, r = n - ql + i + 1, s_ * ql + i
                sc = torch.einsum("hd,thd->ht", q[r].float(), kk[:m]) * D ** -0.5
                ref = torch.einsum("ht,thd->hd", torch.softmax(sc, -1), vv[:m])
                worst = max(worst, float((out[l, r].float() - ref).abs().max()))
    if worst > 2e-2:
        raise SystemExit(f"attention spot check failed: max abs error {worst}")

    graph = None
    if not args.no_graph:
        # The step's 2 x L launches replayed as one CUDA graph (the workspace
        # and tensor maps exist already after the warm-up).
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            if plan:
                backend.paged_attention_plan(d_len, max_ctx, stream=stream)
            for l in range(L):
                backend.paged_attention(q, d_tab, d_len, max_ctx, out[l], l, lse=lse[l], stream=stream,
                                        q_len=ql)
        torch.cuda.synchronize()

        def step(i, ev):  # noqa: F811
            if ev is not None:
                ev.extend(torch.cuda.Event(enable_timing=True) for _ in range(2))
                ev[0].record(stream)
            graph.replay()
            if ev is not None:
                ev[1].record(stream)

    K = args.steps
    total_ms, evs, clocks = run.timed_steps(step, K)
    kernel_ms = run.max_over_ranks(_event_ms(evs, 0, 1))
    kv_bytes = int(lens.sum()) * backend.shard_entry_elems * 2 * backend.elem_bytes  # K and V, per layer
    io_bytes = S * ql * (hq * D * 2 * 2 + hq * 4) + tables.nbytes + lens.nbytes
    alg = L * (kv_bytes + io_bytes)
    workload = (f"decode attention x{world}: {world}x256 sequences, context U[1,4096]+1 "
                f"(mean {lens.mean():.0f}), Qwen2-7B (28 query heads over 4 kv heads x 128, "
                f"{L} layers, bs 16, bf16 queries), pool {cfg.num_blocks} blocks "
                + ("of E4M3 codes with per-(layer, kv head) scales" if fp8 else "bf16")
                + f" head-sharded {world} ways; step = "
                + ("a longest-first order of the sequences (one plan kernel), then " if plan else "")
                + "paged attention over every layer"
                + (f" with its last {ql} tokens as causal query tokens" if ql > 1 else "")
                + (" replayed as one CUDA graph" if graph is not None else ""))
    out_line = base_line(run, int(lens.sum()) * world * K / (total_ms / 1e3), K, total_ms / K,
                         "weak", workload, {
                             "sequences": S, "query_heads_per_gpu": hq, "kv_heads_per_gpu": kvh,
                             "layers": L, "max_context": max_ctx,
                             "kv_gib_read_per_step_per_gpu": round(L * kv_bytes / 2**30, 2),
                             "parallelism": f"kv-head shards x{world}",
                             "l2": "each step reads %.1f GiB of cache, far more than the 126 MB L2"
                                   % (L * kv_bytes / 2**30)},
                         "synthetic (seeded: shuffled free list, uniform context lengths, "
                         "normal K/V/Q)")
    out_line["metric"] = "KV tokens attended/s & HBM GB/s (paged decode attention)"
    out_line["unit"] = "tokens/s"
    out_line["gb_per_s"] = alg * world / (total_ms / K / 1e3) / 1e9
    out_line["roofline"] = roofline(f"paged_attention_kernel + combine ({L} layers)", alg, kernel_ms)
    out_line["gpu_launches"] = K * (L * 2 + (1 if plan else 0))
    out_line["spot_check_max_abs_err"] = worst
    out_line["config"]["pool_dtype"] = "fp8_e4m3" if fp8 else "bf16"
    out_line["config"]["q_len"] = ql
    if args.compare_library and world == 1 and not fp8 and ql == 1:
        out_line["library_comparison"] = flashinfer_decode(backend, q, tables, lens, out, L, stream,
                                                           kernel_ms / L, kv_bytes)
    graph = None  # release the captured graph before the backend's buffers go
    out_line["clocks"] = clocks
    backend.close()
    return out_line


def flashinfer_decode(backend, q, tables, lens, ours_out, L, stream, ours_layer_ms, kv_bytes):
    """flashinfer's batched paged decode (tensor-core path, NHD pages) over the
    same pool layer by layer: the per-layer pool view [num_blocks][16][entry]
    is its [pages][page_size][kv_heads][head_dim]. Comparison only; nothing of
    ours runs through it."""
    import numpy as np
    import torch

    try:
        import flashinfer
    except Exception as ex:  # noqa: BLE001
        return {"unavailable": repr(ex)[:200]}
    cfg = backend.config()
    dev = q.device
    npages = (lens + 15) // 16
    indptr = torch.from_numpy(np.concatenate([[0], np.cumsum(npages)]).astype(np.int32)).to(dev)
    indices = torch.from_numpy(np.concatenate([tables[s_, :npages[s_]] for s_ in range(len(lens))])
                               .astype(np.int32)).to(dev)
    last = torch.from_numpy((lens - (npages - 1) * 16).astype(np.int32)).to(dev)
    kvh = backend.shard_entry_elems // cfg.head_dim
    ws = torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)
    w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, "NHD", use_tensor_cores=True)
    w.plan(indptr, indices, last, q.shape[1], kvh, cfg.head_dim, 16, q_data_type=torch.bfloat16,
           kv_data_type=torch.bfloat16)
    kp, vp = backend.planes()
    views = [(kp[l].view(cfg.num_blocks, 16, kvh, cfg.head_dim),
              vp[l].view(cfg.num_blocks, 16, kvh, cfg.head_dim)) for l in range(L)]
    with torch.cuda.stream(stream):
        diff = float((w.run(q, views[0]).float() - ours_out[0].float()).abs().max())
        for _ in range(3):
            for l in range(L):
                w.run(q, views[l])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            for l in range(L):
                w.run(q, views[l])
        e1.record(stream)
    stream.synchronize()
    ms = e0.elapsed_time(e1) / (5 * L)
    peak, _ = measured_peak_gbs()
    return {"library": f"flashinfer {flashinfer.__version__} BatchDecodeWithPagedKVCacheWrapper "
                       "(tensor cores, NHD)",
            "layer_ms": ms, "kv_gb_per_s": kv_bytes / ms / 1e6,
            "kv_frac_of_peak": kv_bytes / ms / 1e6 / peak,
            "ours_layer_ms": ours_layer_ms, "ours_kv_frac_of_peak": kv_bytes / ours_layer_ms / 1e6 / peak,
            "max_abs_diff_vs_ours_layer0": diff}


def wl_trace(run, kind: str) -> dict:
    """Config 4 (beam-search copy-on-write, Qwen2-7B geometry) or config 5
    (continuous-batching churn, 70B-like geometry): a host trace of StepPlans
    applied to the device by the StepOutcome driver, copy_blocks ->
    resolve_slots -> reshape_and_cache -> zero_blocks per step."""
    import numpy as np

    torch = run.torch
    from pagedkv import B200Backend, CacheConfig
    from pagedkv.driver import DeviceStepper
    from pagedkv.traces import beam_cow_trace, churn_trace

    args, world, dev, stream = run.args, run.world, run.dev, run.stream
    W, K = args.warmup, args.steps
    if kind == "cow":
        small = args.profile_small  # 512-token prefixes over a 4,096-block pool, for ncu
        prefix = 512 if small else 2048
        cfg = CacheConfig(num_blocks=4096 if small else BLOCKS_PER_CHUNK, **GEOM)
        plans = list(beam_cow_trace(cfg, groups=64, width=4, prefix=prefix, steps=W + K,
                                    zero_per_step=64, seed=0))
        rows = 64 * prefix
        workload = (f"beam search: 64 prefixes of {prefix} tokens forked to 4 beams; every step "
                    "re-forks 4 children per group from seeded parents and appends one token to "
                    "each (copy-on-write of the shared tail), frees the old beams, zeroes 64 freed "
                    f"blocks; Qwen2-7B KV geometry, {cfg.num_blocks}-block pool")
    else:
        heads, hd, layers = 8, 128, 80
        per_gpu = 150e9
        nb = int(per_gpu // (layers * 2 * 16 * (heads * hd // world) * 2))
        cfg = CacheConfig(num_blocks=nb, block_size=16, num_kv_heads=heads, head_dim=hd,
                          num_layers=layers, dtype_bytes=2)
        plans = list(churn_trace(cfg, steps=W + K, arrival_rate=8.0, prompt_lo=64,
                                 prompt_hi=8192, out_mean=256.0, max_batch=4096,
                                 fork_rate=args.fork_rate, zero_freed=False, seed=0))
        rows = 16384
        workload = (f"continuous batching: Poisson(8) arrivals per step, prompts log-uniform "
                    f"[64, 8192], outputs geometric mean 256, max batch 4096, recompute "
                    f"preemption, forks of a running sequence with probability {args.fork_rate} "
                    f"per step; 80 layers, 8 KV heads x 128, bs 16, pool {nb} blocks "
                    f"(150 GB per GPU); per step: copy_blocks, slot resolution of admitted "
                    f"prompts, all-layer reshape_and_cache (freed blocks are not zeroed: the "
                    f"reference marks zero_block a debugging aid)")
    backend = B200Backend(cfg, dtype="bf16", device=run.local, shard_rank=run.rank, num_shards=world)
    backend.set_copy_engine(args.copy_engine)
    es, L = backend.shard_entry_elems, cfg.num_layers
    gen = torch.Generator(device=dev).manual_seed(2000 + run.rank)
    k = torch.randn((L, rows, es), generator=gen, device=dev, dtype=torch.bfloat16)
    v = torch.randn((L, rows, es), generator=gen, device=dev, dtype=torch.bfloat16)
    stepper = DeviceStepper(backend, stream=stream, timing=False, fuse_copy_zero=not args.no_fuse,
                            fuse_mixed=not args.no_fuse)
    with torch.cuda.stream(stream):
        for p in plans[: 1 + W if kind == "cow" else W]:
            stepper.apply(p, k, v)
    run.barrier()
    timed = plans[1 + W:] if kind == "cow" else plans[W:]
    # Host-side preparation (copy waves, packing) and the upload of every
    # step's metadata happen before the timed region, as the inputs of the
    # other workloads lie in HBM before theirs; each timed step launches.
    prepared = [stepper.prepare(p) for p in timed]
    resident = stepper.make_resident(prepared)
    stepper.timing = True
    run.barrier()
    busy = torch.ones(2**30, dtype=torch.uint8, device=dev)
    with ClockSampler(range(world), active=run.rank == 0) as clocks:
        run.barrier()
        # A second of streaming reads first, so the clock samples see the GPU under load.
        t_load = time.perf_counter()
        while time.perf_counter() - t_load < 1.0:
            busy.sum(dtype=torch.int64)
            torch.cuda.synchronize()
        t0 = time.perf_counter()
        with torch.cuda.stream(stream):
            for p in prepared:
                stepper.apply(p, k, v)
        run.barrier()
        host_s = time.perf_counter() - t0
    ph = stepper.phase_ms()
    if backend.device_error() is not None:
        raise SystemExit(f"device error in trace: {backend.device_error()}")
    total = run.max_over_ranks(ph["total"])
    tokens = sum(p.num_tokens for p in timed)
    copies = sum(len(p.copies) for p in timed)
    zeros = sum(len(p.zero) for p in timed)
    eb, bb = es * 2, cfg.block_size * es * 2
    copy_bytes = copies * L * 2 * bb * 2 + 16 * copies
    write_bytes = tokens * L * 2 * eb * 2 + 8 * tokens
    zero_bytes = zeros * L * 2 * bb + 8 * zeros
    phase = {p: run.max_over_ranks(ph[p]) for p in stepper.PHASES}
    out = base_line(run, tokens / (total / 1e3), len(timed), total / len(timed), "strong", workload, {
        "steps_timed": len(timed), "warmup_steps": W, "layers": L, "entry_elems_per_gpu": es,
        "pool_gib_per_gpu": round(backend.allocated_bytes() / 2**30, 2),
        "parallelism": f"kv-head shards x{world}", "tokens_written": tokens,
        "copy_pairs": copies, "zeroed_blocks": zeros, "copy_engine": args.copy_engine,
        "l2": "copies and writes stream through far more than the 126 MB L2 over the trace",
    }, "synthetic (seeded host trace through the native BlockAllocator/BlockTable/Scheduler)")
    out["gb_per_s"] = (copy_bytes + write_bytes + zero_bytes) * world / (total / 1e3) / 1e9
    out["phases_ms"] = phase
    out["device_ms_per_step"] = sum(phase[p] for p in stepper.PHASES) / len(timed)
    write_ms = phase["resolve_and_cache"] + phase["reshape_and_cache"]
    out["phase_gb_per_s"] = {
        "copy_blocks": copy_bytes / (phase["copy_blocks"] / 1e3) / 1e9 if phase["copy_blocks"] else None,
        "token_writes": write_bytes / (write_ms / 1e3) / 1e9 if write_ms else None,
        "zero_blocks": zero_bytes / (phase["zero_blocks"] / 1e3) / 1e9 if phase["zero_blocks"] else None,
    }
    fused = stepper.fused_steps
    out["config"]["fused_copy_zero_steps"] = fused
    out["config"]["one_launch_token_write_steps"] = stepper.mixed_steps
    if kind == "cow" and fused:
        # Steps that ran their copies and zeroes as one launch move both in
        # the copy phase; the others zero in their own phase.
        fz = sum(len(p_.zero) for p_, q_ in zip(timed, prepared) if q_.fused is not None)
        cz_bytes = copy_bytes + fz * L * 2 * bb + 8 * fz
        rest_zero = zero_bytes - (fz * L * 2 * bb + 8 * fz)
        out["roofline"] = roofline("copy_zero_kernel (256 copy-on-write pairs grouped by source "
                                   "+ 64 freed blocks zeroed, 28 layers, one launch per step)",
                                   cz_bytes / len(timed), phase["copy_blocks"] / len(timed),
                                   profile_traffic("copy_zero_cow_ncu"))
        out["roofline"]["fused_steps"] = fused
        out["phase_gb_per_s"]["copy_blocks"] = cz_bytes / (phase["copy_blocks"] / 1e3) / 1e9
        out["phase_gb_per_s"]["zero_blocks"] = (rest_zero / (phase["zero_blocks"] / 1e3) / 1e9
                                                if rest_zero and phase["zero_blocks"] else None)
    elif kind == "cow":
        kern = "copy_blocks_bulk_kernel" if args.copy_engine == "bulk" else "copy_blocks_kernel"
        out["roofline"] = roofline(f"{kern} (256 pairs x 28 layers per step)",
                                   copy_bytes / len(timed), phase["copy_blocks"] / len(timed),
                                   None if args.copy_engine == "bulk" else
                                   profile_traffic("copy_blocks_cow_ncu"))
    else:
        out["roofline"] = roofline("resolve_cache_kernel + reshape_copy_kernel (token writes, all "
                                   "layers)", write_bytes / len(timed), write_ms / len(timed))
        st = [p.stats for p in timed]
        out["trace"] = {"admitted": sum(s["admitted"] for s in st),
                        "preempted": sum(s["preempted"] for s in st),
                        "finished": sum(s["finished"] for s in st),
                        "rejected": st[-1]["rejected"],
                        "running_final": st[-1]["running"],
                        "utilization_max": max(s["utilization"] for s in st)}
    out["verify"] = last_step_landed(run, backend, timed[-1], k, v)
    if not out["verify"]["ok"]:
        raise SystemExit(f"bench: trace verification failed: {out['verify']}")
    if world > 1:
        out["ranks"] = rank_breakdown(run, stepper.step_ms(), write_bytes,
                                      ph["resolve_and_cache"] + ph["reshape_and_cache"])
    out["host_driver_s"] = host_s
    out["gpu_launches"] = stepper.launches
    out["clocks"] = {**clocks.summary(),
                     "window": "sampled every 200 ms over 1 s of streaming reads and the timed trace"}
    del resident  # the trace metadata, before the pool goes
    backend.close()
    return out


def link_h2d_gbs(src_np, dev) -> float:
    """The host link's own ceiling: plain pinned host -> device copies of one
    layer's K and V rows."""
    import torch

    src = torch.from_numpy(src_np)
    if not src.is_pinned():
        src = src.pin_memory()
    dst = torch.empty(src.shape, dtype=src.dtype, device=dev)
    best = 0.0
    dst.copy_(src, non_blocking=True)
    for _ in range(5):  # best of 5 runs of 4 back-to-back copies
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        for _ in range(4):
            dst.copy_(src, non_blocking=True)
        ev[1].record()
        torch.cuda.synchronize()
        best = max(best, 4 * src.numel() * src.element_size() / (ev[0].elapsed_time(ev[1]) / 1e3) / 1e9)
    return best


def last_step_landed(run, backend, plan, k, v) -> dict:
    """After a trace: every token the last step wrote from a host-known slot
    (nothing later overwrote them) holds its row, in 3 layers of this rank's
    shard; the per-rank results are all-gathered (NCCL) and must all hold."""
    import numpy as np

    torch = run.torch
    L, R, es = k.shape
    tr = plan.resolved_tokens
    slots = np.asarray(plan.direct_slots, np.int64)
    ok = True
    if len(slots):
        d_slots = torch.from_numpy(slots).to(run.dev)
        rows = torch.from_numpy((tr + np.arange(len(slots))) % R).to(run.dev)
        pk, pv = backend.planes()
        for l in (0, L // 2, L - 1):
            ok &= bool(torch.equal(pk[l].reshape(-1, es)[d_slots], k[l, rows]))
            ok &= bool(torch.equal(pv[l].reshape(-1, es)[d_slots], v[l, rows]))
    flag = torch.tensor([1 if ok else 0, len(slots)], dtype=torch.int64, device=run.dev)
    if run.world > 1:
        got = [torch.empty_like(flag) for _ in range(run.world)]
        run.dist.all_gather(got, flag)
    else:
        got = [flag]
    per = [bool(g[0].item()) for g in got]
    return {"ok": all(per), "ranks_ok": per, "tokens_checked_per_rank": int(len(slots)),
            "check": "last step's host-slot tokens hold their rows in layers 0, L/2, L-1 of "
                     "every shard" + (" (all_gather over NCCL)" if run.world > 1 else "")}


def rank_breakdown(run, step_ms: list[float], write_bytes: float, write_ms: float) -> dict:
    """Per-rank view of a multi-GPU trace: each rank's device time over the
    timed steps, how many steps each rank bounds (is the slowest on), and
    each rank's token-write bandwidth as a fraction of the measured peak.
    All ranks call the same collectives in the same order."""
    torch, dist = run.torch, run.dist
    t = torch.tensor(step_ms, dtype=torch.float64, device=run.dev)
    per = [torch.empty_like(t) for _ in range(run.world)]
    dist.all_gather(per, t)
    m = torch.stack(per)  # [rank][step]
    w = torch.tensor([write_ms], dtype=torch.float64, device=run.dev)
    ws = [torch.empty_like(w) for _ in range(run.world)]
    dist.all_gather(ws, w)
    peak, _ = measured_peak_gbs()
    bounds = torch.bincount(m.argmax(0), minlength=run.world).tolist()
    return {
        "device_ms_per_rank": [round(x, 3) for x in m.sum(1).tolist()],
        "steps_bounded_by_rank": bounds,
        "token_write_frac_of_peak_per_rank": [
            round(write_bytes / (float(x.item()) / 1e3) / 1e9 / peak, 4) if float(x.item()) else None
            for x in ws],
        "note": "a step's device time is its first to last phase mark on that rank; the rank "
                "with the longest time bounds the step",
    }


def e2e_host_path(args, backend, tables, ctx, new, k, v, barrier, max_over_ranks,
                  mode: str = "f32_pageable", link: float | None = None):
    """Same step through the C ABI's KvBackend entry point with host buffers:
    per layer pkv_write_kv_batch (host->device copies in the timed region),
    then the device error word read back.

    mode "f32_pageable": the trait's own call, write_kv_batch(&[f32]) from
    ordinary (pageable) memory, as a Rust caller holding Vec<f32> rows makes
    it; the library's host stager narrows the rows to bf16 (round to nearest
    even) into pinned chunks while earlier chunks upload.
    mode "bf16_pinned": rows already in bf16 in pinned memory, copied by the
    DMA engine straight from the caller's buffer."""
    import numpy as np
    import torch

    L, T, es = k.shape
    blocks, offs = host_slots(tables, ctx, new, backend.config().block_size)
    if mode == "bf16_pinned":
        hk = k.view(torch.int16).cpu().pin_memory().numpy().view(np.uint16)
        hv = v.view(torch.int16).cpu().pin_memory().numpy().view(np.uint16)
        host_dtype, elem = "bf16", 2
    else:
        hk = k.float().cpu().numpy()  # pageable: torch's ordinary CPU allocator
        hv = v.float().cpu().numpy()
        host_dtype, elem = "f32", 4
    steps = max(1, min(args.steps, 5))

    def one():
        # The step's destinations, built once and passed to every layer's call
        # (a caller of the trait holds one slice of PhysicalSlots per step).
        pairs = backend.slot_pairs(blocks, offs)
        for layer in range(L):
            backend.write_kv_batch_pairs(layer, pairs, hk[layer], hv[layer], host_dtype=host_dtype)
        if backend.device_error() is not None:
            raise SystemExit("device error in e2e step")

    one()
    barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    barrier()
    dt = max_over_ranks(time.perf_counter() - t0)
    # Bytes the caller hands over per step (its rows and its destinations).
    h2d = int(L * (2 * T * es * elem + T * 8))
    # Bytes that cross the link per step: rows as the pool stores them.
    moved = int(L * (2 * T * es * 2 + T * 8))
    if link is None:
        link = link_h2d_gbs(k[0].view(torch.int16).cpu().numpy(), k.device)
    moved_gbs = moved * steps / dt / 1e9
    out = {"value": T * steps / dt, "unit": "tokens/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 16, "steps": steps,
           "link_bytes_per_step": moved, "link_gb_per_s": moved_gbs,
           "link_h2d_gb_per_s": link, "frac_of_link": moved_gbs / link}
    if mode == "bf16_pinned":
        out["path"] = "pkv_write_kv_batch per layer, pinned bf16 host rows, + pkv_device_error"
    else:
        out["path"] = ("pkv_write_kv_batch per layer, PKV_F32 rows in pageable host memory (the "
                       "trait's write_kv_batch(&[f32])), narrowed to bf16 by the library's host "
                       "stager, + pkv_device_error")
        out["host_threads"] = backend.host_threads()
    return out


def bench_ops(backend, cfg, dev, stream, reps: int = 10) -> dict:
    """Per-kernel timings on this GPU's shard: copy_blocks (256 copy-on-write
    pairs, every layer), zero_blocks (64 blocks) and a 256-token decode step."""
    import numpy as np
    import torch

    from pagedkv.workloads import Stream

    peak, _ = measured_peak_gbs()
    es = backend.shard_entry_elems
    L, bs = cfg.num_layers, cfg.block_size
    pe = backend.elem_bytes
    block_bytes = bs * es * pe
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
                     "algorithmic_bytes": nbytes, "launches": len(times), **(extra or {})}

    pairs = torch.from_numpy(np.stack([ids[:256], ids[256:512]], 1).astype(np.int64)).to(dev)
    timed(lambda: backend.copy_blocks_dev(pairs, stream=stream),
          256 * L * 2 * block_bytes * 2 + 256 * 16, "copy_blocks", {"pairs": 256, "layers": L})
    backend.set_copy_engine("bulk")
    timed(lambda: backend.copy_blocks_dev(pairs, stream=stream),
          256 * L * 2 * block_bytes * 2 + 256 * 16, "copy_blocks_bulk",
          {"pairs": 256, "layers": L, "engine": "cp.async.bulk global->shared->global"})
    backend.set_copy_engine("auto")
    zero = torch.from_numpy(ids[512:576].astype(np.int64)).to(dev)
    zero_big = torch.from_numpy(ids[1024:2048].astype(np.int64)).to(dev)
    for engine, suffix in (("auto", ""), ("bulk", "_bulk")):
        backend.set_copy_engine(engine)
        extra = {"engine": "cp.async.bulk stores of a zeroed shared-memory run"} if suffix else {}
        timed(lambda: backend.zero_blocks_dev(zero, stream=stream),
              64 * L * 2 * block_bytes + 64 * 8, "zero_blocks" + suffix, {"blocks": 64, **extra})
        timed(lambda: backend.zero_blocks_dev(zero_big, stream=stream),
              1024 * L * 2 * block_bytes + 1024 * 8, "zero_blocks_1024" + suffix,
              {"blocks": 1024, **extra})
    backend.set_copy_engine("auto")
    td = 256
    kd = torch.randn((L, td, es), device=dev).to(torch.bfloat16)
    sl = torch.from_numpy((ids[600:856] * bs + st.integers(256, 0, bs - 1)).astype(np.int64)).to(dev)
    timed(lambda: backend.reshape_and_cache(kd, kd, sl, stream=stream),
          td * L * 2 * es * (2 + pe) + td * 8, "decode_reshape_all_layers", {"tokens": td})
    assert backend.device_error() is None
    return res


class CpuArm:
    """CpuBackend semantics (the C restatement in oracle/, f32 planes like the
    reference) on a bounded sample of the workload: the first `sample` tokens
    of the chunk, all layers, slots folded into a 1,024-block pool. Rows are
    split over `threads` host threads (disjoint tokens)."""

    NB = 1024

    def __init__(self, tables, ctx, new, kf, vf, threads: int, head_dim: int | None = None,
                 fp8_scales=None):
        import numpy as np

        from oracle.cpu import OracleBackend
        from pagedkv import CacheConfig

        L, sample, es = kf.shape
        self.L, self.sample, self.es = L, sample, es
        hd = head_dim or es
        cfg = CacheConfig(num_blocks=self.NB, block_size=16, num_kv_heads=es // hd, head_dim=hd,
                          num_layers=L, dtype_bytes=4)
        blocks, offs = host_slots(tables, ctx, new, 16)
        pairs = np.stack([blocks[:sample] % self.NB, offs[:sample]], 1).astype(np.uint64)
        self.orc = OracleBackend(cfg)
        self.fp8 = fp8_scales is not None
        if self.fp8:  # the oracle quantises each element, as the device's fp8 path does
            self.orc.set_fp8(*fp8_scales)
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
                "oracle/pkv_oracle.c" + (", E4M3 quantisation per element)" if self.fp8 else ")"))


def cpu_sample(tables, ctx, new, kf, vf, seconds: float, threads: int, head_dim=None,
               fp8_scales=None) -> dict:
    arm = CpuArm(tables, ctx, new, kf, vf, threads, head_dim, fp8_scales)
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
    per core over disjoint tokens, on a bounded sample of the same workload.
    The reference's CpuBackend itself is single-threaded (cpu.rs:95-111): the
    line also carries that figure, measured on the same sample. Nothing here
    loads the device library."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from pagedkv.workloads import Stream, bf16_bits_to_f32, f32_to_bf16_bits

    copies = 1 if args.strong else world
    cfg, tables, ctx, new = build_batch(copies, args.chunk_tokens, args.chunk_prompts,
                                        args.chunk_blocks)
    workload, extra = table_batch_config(args, "prefill", world, cfg, int(new.sum()), len(new))
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
    single = cpu_sample(tables, ctx, new, kf, vf, seconds=2.0, threads=1)
    out = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": per * 1e3, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
           "config": {"workload": workload, **extra, "host_threads": arm.threads},
           "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": arm.threads,
                            "kind": "port", "sample": arm.describe(len(times)) +
                            f"; each step is this sample on {arm.threads} host threads"},
           "single_thread": {"value": single["value"], "unit": "tokens/s", "cores": 1,
                             "sample": single["sample"],
                             "note": "CpuBackend is single-threaded; the arm's value uses "
                                     "every host core, a harder baseline"},
           "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    run = Run(args)
    if args.workload in ("prefill", "decode"):
        out = wl_table_batch(run, args.workload)
    elif args.workload == "attention":
        out = wl_attention(run)
    else:
        out = wl_trace(run, args.workload)
    run.close()
    if run.rank == 0:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
