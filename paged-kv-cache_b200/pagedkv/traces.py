"""Step plans for the data path, built from the host bookkeeping.

A ``StepPlan`` is what one scheduler step asks of the device, in the order it
must happen (crates/paged-kv-core/src/scheduler.rs:57-63): copy-on-write
copies first, then the new tokens' K/V, then zeroing of blocks freed this
step. New tokens come in two kinds:

* sequences whose slots the device resolves from block tables (prefill of
  admitted prompts, whose slots Scheduler::admit discards,
  scheduler.rs:235-236; or decode batches given as tables), and
* single tokens whose slot the host already knows (Scheduler::step's
  decoded tokens).

The token order of a step's K/V rows is: resolved sequences' tokens (in
cu_seqlens order), then the direct tokens.

Traces: ``decode_plan`` (a decode step over a seeded batch),
``prefill_plan`` (a ragged prefill chunk), ``beam_cow_trace`` (beam search
that re-forks beams every step, so appends land on shared tails) and
``churn_trace`` (continuous batching with Poisson arrivals, preemption and
optional forks).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .config import CacheConfig
from .errors import OutOfBlocks
from .host import BlockAllocator, BlockTable, Scheduler
from .workloads import Batch, Stream


@dataclass
class StepPlan:
    copies: np.ndarray  # [P][2] int64 (src, dst)
    tables: np.ndarray  # [S][stride] int32, -1 padded
    ctx: np.ndarray  # [S] int32 tokens already cached
    new: np.ndarray  # [S] int32 tokens written this step
    direct_slots: np.ndarray  # [D] int64 combined slots known on the host
    zero: np.ndarray  # [Z] int64 blocks to zero after the writes
    stats: dict = field(default_factory=dict)

    @property
    def resolved_tokens(self) -> int:
        return int(self.new.sum())

    @property
    def num_tokens(self) -> int:
        return self.resolved_tokens + len(self.direct_slots)

    def slot_mapping(self, block_size: int) -> np.ndarray:
        """Host restatement of the step's slots (resolved part + direct part)."""
        if self.resolved_tokens:
            q = np.repeat(np.arange(len(self.new)), self.new)
            starts = np.concatenate([[0], np.cumsum(self.new)[:-1]])
            j = np.arange(self.resolved_tokens) - np.repeat(starts, self.new)
            pos = self.ctx[q] + j
            res = self.tables[q, pos // block_size].astype(np.int64) * block_size + pos % block_size
        else:
            res = np.zeros(0, np.int64)
        return np.concatenate([res, self.direct_slots.astype(np.int64)])


def _empty_tables():
    return np.zeros((0, 1), np.int32), np.zeros(0, np.int32), np.zeros(0, np.int32)


def plan_from_batch(batch: Batch) -> StepPlan:
    """Decode or prefill batch (workloads.decode_batch / prefill_chunk) as one step."""
    return StepPlan(np.zeros((0, 2), np.int64), batch.tables, batch.ctx, batch.new,
                    np.zeros(0, np.int64), np.zeros(0, np.int64))


def _pack_tables(rows: list[np.ndarray]) -> np.ndarray:
    stride = max([len(r) for r in rows] + [1])
    out = np.full((len(rows), stride), -1, np.int32)
    for i, r in enumerate(rows):
        out[i, : len(r)] = r
    return out


def beam_cow_trace(cfg: CacheConfig, groups: int = 64, width: int = 4, prefix: int = 2048,
                   steps: int = 100, zero_per_step: int = 64, seed: int = 0,
                   interleave: bool = False):
    """Beam search over shared prefixes.

    Step 0 prefills `groups` prefixes of `prefix` tokens and forks each to
    `width` beams (BlockTable::fork, block_table.rs:218-227). Every later
    step selects `width` parents per group (seeded, with replacement), forks
    the children from them, appends one token to every child while the old
    beams are still alive -- so each append onto a partly filled tail is a
    copy-on-write (block_table.rs:135-150) -- then frees the old beams and
    zeroes up to `zero_per_step` of the blocks that freeing released.

    By default the step forks and appends for every group before it frees
    any old beam, as a batched engine does; blocks freed in a step are then
    reused only by later steps. With interleave=True each group frees its old
    beams before the next group appends, so the LIFO free list hands a block
    that an earlier pair of the same step copied from to a later pair as its
    destination: the step's copy list chains."""
    a = BlockAllocator(cfg.num_blocks)
    bs = cfg.block_size
    st = Stream(seed)
    beams = []
    roots = []
    for _ in range(groups):
        t = BlockTable(bs)
        t.append_many(a, prefix)
        roots.append(np.array(t.physical_blocks(), np.int64))
        beams.append([t] + [t.fork(a) for _ in range(width - 1)])
    tables = _pack_tables(roots)
    yield StepPlan(np.zeros((0, 2), np.int64), tables, np.zeros(groups, np.int32),
                   np.full(groups, prefix, np.int32), np.zeros(0, np.int64), np.zeros(0, np.int64),
                   {"step": 0, "copies": 0})
    for step in range(1, steps + 1):
        copies, slots, old = [], [], []
        retired = []
        for g in range(groups):
            parents = st.integers(width, 0, width - 1)
            children = [beams[g][int(p)].fork(a) for p in parents]
            for c in children:
                slot, cow = c.append(a)
                if cow is not None:
                    copies.append(cow)
                slots.append(slot.block * bs + slot.slot)
            retired.append(beams[g])
            beams[g] = children
            if interleave:
                for t in retired.pop():
                    old.append(t.physical_blocks())
                    t.free(a)
        for group in retired:
            for t in group:
                old.append(t.physical_blocks())
                t.free(a)
        cand = np.unique(np.concatenate([np.asarray(o, np.int64) for o in old]))
        freed = cand[a.ref_counts(cand) == 0]
        ti, ci, ni = _empty_tables()
        yield StepPlan(np.asarray(copies, np.int64).reshape(-1, 2), ti, ci, ni,
                       np.asarray(slots, np.int64), freed[:zero_per_step].astype(np.int64),
                       {"step": step, "copies": len(copies), "freed": int(len(freed))})


def churn_trace(cfg: CacheConfig, steps: int = 2000, arrival_rate: float = 8.0,
                prompt_lo: int = 64, prompt_hi: int = 8192, out_mean: float = 256.0,
                max_batch: int = 4096, fork_rate: float = 0.0, zero_freed: bool = True,
                seed: int = 0):
    """Continuous batching through Scheduler::step (scheduler.rs:218-226):
    Poisson(arrival_rate) arrivals per step with log-uniform prompt lengths
    in [prompt_lo, prompt_hi] and geometric output lengths of mean
    `out_mean`, recompute preemption, and, with probability `fork_rate` per
    step, a fork of a random running sequence (parallel sampling), whose
    shared tail makes the next append a copy-on-write.

    Each step's plan writes the prompts of sequences admitted (and not
    preempted again) this step, resolved on the device from their tables,
    then every decoded token at the slot the scheduler returned, and (with
    zero_freed) zeroes every block the step released."""
    sched = Scheduler(cfg.num_blocks, cfg.block_size, max_batch)
    bs = cfg.block_size
    st = Stream(seed)
    sid = 0
    running: list[int] = []
    rejected = 0
    for step in range(steps):
        for _ in range(int(st.poisson(1, arrival_rate)[0])):
            p = int(st.log_uniform_int(1, prompt_lo, prompt_hi)[0])
            g = int(st.geometric(1, out_mean)[0])
            try:
                sched.add_request(sid, p, g)
            except OutOfBlocks:
                rejected += 1
            sid += 1
        if fork_rate > 0 and running and st.uniform(1)[0] < fork_rate:
            parent = running[int(st.integers(1, 0, len(running) - 1)[0])]
            sched.fork_sequence(parent, sid, int(st.geometric(1, out_mean)[0]))
            running.append(sid)
            sid += 1
        r = sched.step_raw()
        pre = set(int(x) for x in r["preempted"])
        fin = set(int(x) for x in r["finished"])
        running = [x for x in running if x not in pre and x not in fin]
        running += [int(x) for x in r["admitted"] if int(x) not in pre and int(x) not in fin]
        off = r["admitted_table_offsets"]
        rows, new = [], []
        for i, seq in enumerate(r["admitted"]):
            if int(seq) in pre:
                continue  # its blocks went back to the pool this same step
            rows.append(r["admitted_blocks"][off[i]:off[i + 1]])
            new.append(int(r["admitted_ctx"][i]))
        cow = r["decoded_cow"].astype(bool)
        copies = np.stack([r["cow_src"][cow], r["cow_dst"][cow]], 1).astype(np.int64)
        yield StepPlan(copies, _pack_tables(rows) if rows else np.zeros((0, 1), np.int32),
                       np.zeros(len(new), np.int32), np.asarray(new, np.int32),
                       (r["decoded_block"] * bs + r["decoded_slot"]).astype(np.int64),
                       r["freed"].astype(np.int64) if zero_freed else np.zeros(0, np.int64),
                       {"step": step, "freed": len(r["freed"]), "admitted": len(r["admitted"]), "preempted": len(pre),
                        "finished": len(fin), "running": sched.num_running(),
                        "waiting": sched.num_waiting(), "rejected": rejected,
                        "utilization": sched.pool_utilization()})
