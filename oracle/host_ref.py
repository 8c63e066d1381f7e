"""TEST INFRASTRUCTURE ONLY -- pure-Python restatement of the reference's host
bookkeeping: ``BlockAllocator`` (crates/paged-kv-core/src/allocator.rs),
``BlockTable`` (crates/paged-kv-core/src/block_table.rs) and ``Scheduler``
(crates/paged-kv-core/src/scheduler.rs).

These produce the slots, copy-on-write pairs and freed blocks that feed the
device data path. The product's native host mirror (C++, in the package) is
checked against this restatement on seeded traces, and this restatement is
itself pinned by the reference's own unit tests (tests/test_oracle_pins.py).
Only tests import it. Pure-Python loops: small cases only.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

# Error variants, numbered as in include/pkv_b200.h (error.rs:12-46).
OUT_OF_BLOCKS = 1
INVALID_BLOCK = 2
BLOCK_NOT_ALLOCATED = 3
REFCOUNT_OVERFLOW = 4
SLOT_OUT_OF_RANGE = 5
SHAPE_MISMATCH = 6
INVALID_LAYER = 7
UNKNOWN_SEQUENCE = 8

MAX_REFCOUNT = 0xFFFF  # u16 counter, allocator.rs:6-7


class RefError(Exception):
    """A CacheError variant: ``code`` plus the variant's fields."""

    def __init__(self, code: int, *fields: int):
        super().__init__(code, *fields)
        self.code = code
        self.fields = fields


class Allocator:
    """allocator.rs:24-241."""

    def __init__(self, num_blocks: int):
        # Descending push so the first allocate pops block 0 (allocator.rs:40-55).
        self.num_blocks = num_blocks
        self.free_list = list(range(num_blocks - 1, -1, -1))
        self.ref_counts = [0] * num_blocks
        self.total_allocated = 0

    def num_free(self) -> int:
        return len(self.free_list)

    def num_used(self) -> int:
        return self.num_blocks - len(self.free_list)

    def utilization(self) -> float:  # allocator.rs:74-79
        return 0.0 if self.num_blocks == 0 else self.num_used() / self.num_blocks

    def allocate(self) -> int:  # allocator.rs:90-105
        if not self.free_list:
            raise RefError(OUT_OF_BLOCKS, 1, 0)
        b = self.free_list.pop()
        self.ref_counts[b] = 1
        self.total_allocated += 1
        return b

    def allocate_many(self, n: int) -> list[int]:  # allocator.rs:113-126
        if len(self.free_list) < n:
            raise RefError(OUT_OF_BLOCKS, n, len(self.free_list))
        return [self.allocate() for _ in range(n)]

    def _validate(self, b: int) -> None:  # allocator.rs:200-208
        if b >= self.num_blocks:
            raise RefError(INVALID_BLOCK, b, self.num_blocks)

    def incref(self, b: int) -> int:  # allocator.rs:132-148
        self._validate(b)
        rc = self.ref_counts[b]
        if rc == 0:
            raise RefError(BLOCK_NOT_ALLOCATED, b)
        if rc == MAX_REFCOUNT:
            raise RefError(REFCOUNT_OVERFLOW, b, MAX_REFCOUNT)
        self.ref_counts[b] = rc + 1
        return rc + 1

    def decref(self, b: int) -> int:  # allocator.rs:152-170
        self._validate(b)
        rc = self.ref_counts[b]
        if rc == 0:
            raise RefError(BLOCK_NOT_ALLOCATED, b)
        rc -= 1
        self.ref_counts[b] = rc
        if rc == 0:
            self.free_list.append(b)
        return rc

    def ref_count(self, b: int) -> int:  # allocator.rs:181-184
        self._validate(b)
        return self.ref_counts[b]

    def is_shared(self, b: int) -> bool:  # allocator.rs:190-192
        return self.ref_count(b) > 1

    def check_invariants(self) -> None:  # allocator.rs:213-240
        seen = [False] * self.num_blocks
        for b in self.free_list:
            assert b < self.num_blocks and not seen[b] and self.ref_counts[b] == 0
            seen[b] = True
        for i in range(self.num_blocks):
            assert self.ref_counts[i] != 0 or seen[i]


@dataclass
class BlockTable:
    """block_table.rs:20-240."""

    block_size: int
    blocks: list[int] = field(default_factory=list)
    num_tokens: int = 0

    def _last_block_has_room(self) -> bool:  # block_table.rs:90-92
        return bool(self.blocks) and self.num_tokens % self.block_size != 0

    def slot_for_position(self, pos: int) -> tuple[int, int]:  # block_table.rs:97-101
        return self.blocks[pos // self.block_size], pos % self.block_size

    def resolve(self, pos: int) -> tuple[int, int]:  # block_table.rs:107-115
        if pos >= self.num_tokens:
            raise RefError(SLOT_OUT_OF_RANGE, pos, self.num_tokens)
        return self.slot_for_position(pos)

    def append(self, a: Allocator):  # block_table.rs:135-160
        cow = None
        if self._last_block_has_room():
            tail = self.blocks[-1]
            if a.is_shared(tail):
                fresh = a.allocate()
                a.decref(tail)
                self.blocks[-1] = fresh
                cow = (tail, fresh)
        else:
            self.blocks.append(a.allocate())
        slot = self.slot_for_position(self.num_tokens)
        self.num_tokens += 1
        return slot, cow

    def append_many(self, a: Allocator, n: int):  # block_table.rs:169-209
        saved_blocks, saved_tokens = list(self.blocks), self.num_tokens
        slots, copies = [], []
        for _ in range(n):
            try:
                slot, cow = self.append(a)
            except RefError:
                for b in self.blocks[min(len(self.blocks), len(saved_blocks)):]:
                    try:
                        a.decref(b)
                    except RefError:
                        pass
                self.blocks, self.num_tokens = saved_blocks, saved_tokens
                raise
            slots.append(slot)
            if cow is not None:
                copies.append(cow)
        return slots, copies

    def fork(self, a: Allocator) -> "BlockTable":  # block_table.rs:218-227
        for b in self.blocks:
            a.incref(b)
        return BlockTable(self.block_size, list(self.blocks), self.num_tokens)

    def free(self, a: Allocator) -> None:  # block_table.rs:233-239
        for b in self.blocks:
            a.decref(b)
        self.blocks = []
        self.num_tokens = 0


@dataclass
class _Pending:
    id: int
    context_len: int
    max_new_tokens: int


@dataclass
class _Running:
    id: int
    table: BlockTable
    max_new_tokens: int
    generated: int = 0


@dataclass
class StepOutcome:  # scheduler.rs:72-86
    admitted: list = field(default_factory=list)
    decoded: list = field(default_factory=list)  # (id, (block, slot), cow or None)
    preempted: list = field(default_factory=list)
    finished: list = field(default_factory=list)


class Scheduler:
    """scheduler.rs:117-358."""

    def __init__(self, num_blocks: int, block_size: int, max_batch_size: int):
        self.allocator = Allocator(num_blocks)
        self.block_size = block_size
        self.max_batch_size = max_batch_size
        self.waiting: deque[_Pending] = deque()
        self.running: list[_Running] = []

    def is_idle(self) -> bool:
        return not self.waiting and not self.running

    def add_request(self, sid: int, prompt_len: int, max_new_tokens: int) -> None:  # :196-213
        cap = self.allocator.num_blocks * self.block_size
        final = prompt_len + max_new_tokens
        if final > cap:
            raise RefError(OUT_OF_BLOCKS, -(-final // self.block_size), self.allocator.num_blocks)
        self.waiting.append(_Pending(sid, prompt_len, max_new_tokens))

    def step(self) -> StepOutcome:  # :218-226
        o = StepOutcome()
        self._admit(o)
        self._decode(o)
        self._retire(o)
        return o

    def _admit(self, o: StepOutcome) -> None:  # :228-253
        while len(self.running) < self.max_batch_size and self.waiting:
            p = self.waiting[0]
            t = BlockTable(self.block_size)
            try:
                t.append_many(self.allocator, p.context_len)
            except RefError as e:
                if e.code == OUT_OF_BLOCKS:
                    break
                raise
            self.waiting.popleft()
            o.admitted.append(p.id)
            self.running.append(_Running(p.id, t, p.max_new_tokens))

    def _index(self, sid: int):
        for i, s in enumerate(self.running):
            if s.id == sid:
                return i
        return None

    def _decode(self, o: StepOutcome) -> None:  # :255-297
        for sid in [s.id for s in self.running]:
            idx = self._index(sid)
            if idx is None:
                continue
            while True:
                try:
                    slot, cow = self.running[idx].table.append(self.allocator)
                except RefError as e:
                    if e.code != OUT_OF_BLOCKS:
                        raise
                    self._preempt(len(self.running) - 1, o)
                    idx = self._index(sid)
                    if idx is None:
                        break
                    continue
                o.decoded.append((sid, slot, cow))
                self.running[idx].generated += 1
                break

    def _preempt(self, idx: int, o: StepOutcome) -> None:  # :299-317
        s = self.running.pop(idx)
        o.decoded = [d for d in o.decoded if d[0] != s.id]
        o.preempted.append(s.id)
        ctx = s.table.num_tokens
        rem = s.max_new_tokens - s.generated
        s.table.free(self.allocator)
        self.waiting.appendleft(_Pending(s.id, ctx, rem))

    def _retire(self, o: StepOutcome) -> None:  # :319-331
        i = 0
        while i < len(self.running):
            if self.running[i].generated >= self.running[i].max_new_tokens:
                s = self.running.pop(i)
                o.finished.append(s.id)
                s.table.free(self.allocator)
            else:
                i += 1

    def fork_sequence(self, parent: int, child: int, max_new_tokens: int) -> None:  # :342-357
        idx = self._index(parent)
        if idx is None:
            raise RefError(UNKNOWN_SEQUENCE, parent)
        t = self.running[idx].table.fork(self.allocator)
        self.running.append(_Running(child, t, max_new_tokens))

    def running_snapshot(self):  # :178-189
        return [(s.id, s.table.num_tokens, s.generated, s.max_new_tokens, list(s.table.blocks))
                for s in self.running]
