"""Seeded synthetic workloads for the data path.

One portable generator (splitmix64, Steele, Lea & Flood 2014) drives every
draw so that a workload is fully determined by its seed: uniform doubles from
the top 53 bits, normals by Box-Muller, permutations as a stable argsort of
raw draws, log-uniform and geometric lengths by inversion.

Block tables follow the reference allocator's rules
(crates/paged-kv-core/src/allocator.rs): a LIFO free list; a "shuffled"
free list is what allocate_many(num_blocks) followed by decref of every block
in a seeded permutation order leaves behind (allocator.rs:152-170), so blocks
then come off the stack in reverse permutation order. Sequences take their
blocks in admission order, as Scheduler::admit does (scheduler.rs:228-253),
and a decode step's new blocks come after all admissions
(scheduler.rs:255-297).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .config import CacheConfig

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


class Stream:
    """splitmix64 stream; draw i of seed s is mix(s + (i+1)*golden)."""

    def __init__(self, seed: int):
        self.seed = np.uint64(seed)
        self.pos = 0

    def u64(self, n: int) -> np.ndarray:
        i = np.arange(self.pos + 1, self.pos + n + 1, dtype=np.uint64)
        self.pos += n
        with np.errstate(over="ignore"):
            z = self.seed + i * _GOLDEN
            z = (z ^ (z >> np.uint64(30))) * _M1
            z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))

    def uniform(self, n: int, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
        u = (self.u64(n) >> np.uint64(11)).astype(np.float64) * (1.0 / (1 << 53))
        return lo + (hi - lo) * u

    def integers(self, n: int, lo: int, hi: int) -> np.ndarray:
        """Uniform integers in [lo, hi] inclusive."""
        return lo + np.floor(self.uniform(n) * (hi - lo + 1)).astype(np.int64)

    def normal(self, n: int) -> np.ndarray:
        m = (n + 1) // 2
        u1 = 1.0 - self.uniform(m)  # (0, 1]
        u2 = self.uniform(m)
        r = np.sqrt(-2.0 * np.log(u1))
        z = np.concatenate([r * np.cos(2 * np.pi * u2), r * np.sin(2 * np.pi * u2)])
        return z[:n]

    def permutation(self, n: int) -> np.ndarray:
        return np.argsort(self.u64(n), kind="stable").astype(np.int64)

    def log_uniform_int(self, n: int, lo: int, hi: int) -> np.ndarray:
        u = self.uniform(n)
        x = np.floor(np.exp(np.log(lo) + u * (np.log(hi + 1) - np.log(lo)))).astype(np.int64)
        return np.clip(x, lo, hi)

    def geometric(self, n: int, mean: float) -> np.ndarray:
        """Support {1, 2, ...}, success probability 1/mean, by inversion."""
        p = 1.0 / mean
        u = self.uniform(n)
        k = np.ceil(np.log1p(-u) / np.log1p(-p)).astype(np.int64)
        return np.maximum(k, 1)

    def poisson(self, n: int, lam: float) -> np.ndarray:
        """By inversion of the CDF, one uniform per draw."""
        u = self.uniform(n)
        out = np.zeros(n, np.int64)
        pmf = np.exp(-lam)
        cdf = pmf
        k = 0
        left = u > cdf
        while left.any():
            k += 1
            pmf *= lam / k
            cdf += pmf
            out[left] = k
            left &= u > cdf
            if k > 10 * lam + 100:
                break
        return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (finite inputs)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))
    return ((b + bias) >> np.uint32(16)).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << np.uint32(16)).view(np.float32)


def shuffled_pop_order(num_blocks: int, stream: Stream) -> np.ndarray:
    """Order in which a shuffled free list hands out blocks."""
    perm = stream.permutation(num_blocks)  # decref order = push order
    return perm[::-1].copy()


def fresh_pop_order(num_blocks: int) -> np.ndarray:
    """A fresh allocator pops block 0 first (allocator.rs:40-55)."""
    return np.arange(num_blocks, dtype=np.int64)


# ---- configs ------------------------------------------------------------------


@dataclass
class Oracle1:
    """Config 1, the CpuBackend-runnable oracle case."""

    cfg: CacheConfig
    k: list  # per layer [T][E] f32
    v: list
    slots: np.ndarray  # combined slot index, [T]
    pairs: np.ndarray  # [P][2]
    zero: np.ndarray  # [Z]


def config1(seed: int = 0, tokens: int = 64, pairs: int = 16, zeros: int = 4) -> Oracle1:
    """2 layers, 256 blocks of 16, 8 heads x 64, f32; K/V uniform[-1, 1] drawn
    per layer K then V; slots = first `tokens` of a permutation of all 4096
    slots; `pairs` copy pairs with all ids distinct; `zeros` random blocks."""
    cfg = CacheConfig(256, 16, 8, 64, 2, 4)
    e = cfg.entry_elems()
    st = Stream(seed)
    ks, vs = [], []
    for _ in range(cfg.num_layers):
        ks.append(st.uniform(tokens * e, -1.0, 1.0).astype(np.float32).reshape(tokens, e))
        vs.append(st.uniform(tokens * e, -1.0, 1.0).astype(np.float32).reshape(tokens, e))
    slots = st.permutation(cfg.num_blocks * cfg.block_size)[:tokens]
    ids = st.permutation(cfg.num_blocks)[: 2 * pairs].reshape(pairs, 2)
    zero = st.permutation(cfg.num_blocks)[:zeros]
    return Oracle1(cfg, ks, vs, slots, ids, zero)


QWEN2_7B = dict(block_size=16, num_kv_heads=4, head_dim=128, num_layers=28, dtype_bytes=2)


@dataclass
class Batch:
    """A continuous-batching step's metadata: per-sequence cached and new
    token counts and block tables ([S][stride] int32, -1 past the end)."""

    cfg: CacheConfig
    ctx: np.ndarray
    new: np.ndarray
    tables: np.ndarray
    seed: int
    notes: dict = field(default_factory=dict)

    @property
    def num_tokens(self) -> int:
        return int(self.new.sum())

    def slot_mapping(self) -> np.ndarray:
        """Combined slots, BlockTable::slot_for_position (block_table.rs:97-101)."""
        bs = self.cfg.block_size
        q = np.repeat(np.arange(len(self.new)), self.new)
        starts = np.concatenate([[0], np.cumsum(self.new)[:-1]])
        j = np.arange(self.num_tokens) - np.repeat(starts, self.new)
        pos = self.ctx[q] + j
        return self.tables[q, pos // bs].astype(np.int64) * bs + pos % bs


def _tables_from_order(order: np.ndarray, admit_blocks: np.ndarray, extra: np.ndarray,
                       stride: int) -> np.ndarray:
    """Seq q takes admit_blocks[q] blocks at admission (in q order), then one
    more at decode where extra[q] (in q order)."""
    s = len(admit_blocks)
    tables = np.full((s, stride), -1, np.int32)
    starts = np.concatenate([[0], np.cumsum(admit_blocks)[:-1]])
    for q in range(s):
        tables[q, : admit_blocks[q]] = order[starts[q]: starts[q] + admit_blocks[q]]
    pos = int(admit_blocks.sum())
    for q in np.nonzero(extra)[0]:
        tables[q, admit_blocks[q]] = order[pos]
        pos += 1
    return tables


def decode_batch(seed: int | None = None, num_seqs: int = 256, max_ctx: int = 4096,
                 num_blocks: int = 32768, cfg: CacheConfig | None = None,
                 first_seed: int = 0) -> Batch:
    """Config 2: every sequence has ctx ~ U{1..max_ctx} cached tokens and
    appends one. With seed None the first seed >= first_seed whose demand
    fits the pool is used (roughly half of all seeds overflow 32768 blocks)."""
    cfg = cfg or CacheConfig(num_blocks=num_blocks, **QWEN2_7B)
    bs = cfg.block_size
    s0 = first_seed if seed is None else seed
    for sd in range(s0, s0 + 10_000):
        st = Stream(sd)
        ctx = st.integers(num_seqs, 1, max_ctx)
        need = -(-(ctx + 1) // bs)
        if need.sum() <= cfg.num_blocks:
            break
        if seed is not None:
            raise ValueError(f"seed {seed}: {need.sum()} blocks needed, pool holds {cfg.num_blocks}")
    order = shuffled_pop_order(cfg.num_blocks, st)
    admit = -(-ctx // bs)
    extra = (ctx % bs == 0).astype(np.int64)
    stride = -(-(max_ctx + 1) // bs)
    tables = _tables_from_order(order, admit, extra, stride)
    return Batch(cfg, ctx.astype(np.int32), np.ones(num_seqs, np.int32), tables, sd,
                 {"blocks_used": int(need.sum())})


def prefill_chunk(seed: int = 0, num_prompts: int = 96, lo: int = 128, hi: int = 4096,
                  budget: int = 65536, num_blocks: int = 32768,
                  cfg: CacheConfig | None = None) -> Batch:
    """Config 3: prompts with log-uniform lengths, admitted in order (each
    takes its whole prompt's blocks), packed into a `budget`-token chunk; the
    last prompt in the chunk is cut at the budget."""
    cfg = cfg or CacheConfig(num_blocks=num_blocks, **QWEN2_7B)
    bs = cfg.block_size
    st = Stream(seed)
    lens = st.log_uniform_int(num_prompts, lo, hi)
    order = shuffled_pop_order(cfg.num_blocks, st)
    admit = -(-lens // bs)
    if admit.sum() > cfg.num_blocks:
        raise ValueError("prompts do not fit the pool")
    cum = np.cumsum(lens)
    if cum[-1] <= budget:
        n_in, new = num_prompts, lens.copy()
    else:
        k = int(np.searchsorted(cum, budget, side="left"))  # first prompt reaching the budget
        n_in = k + 1
        new = lens[:n_in].copy()
        new[-1] -= cum[k] - budget
    stride = -(-hi // bs)
    tables = _tables_from_order(order, admit, np.zeros(num_prompts, np.int64), stride)[:n_in]
    return Batch(cfg, np.zeros(n_in, np.int32), new.astype(np.int32), tables, seed,
                 {"prompt_lens": lens, "total_prompt_tokens": int(lens.sum())})
