"""BlockAllocator, BlockTable and Scheduler of paged-kv-core over the native
host mirror in libpagedkv_b200.so (include/pkv_host.h).

These produce the slots, copy-on-write pairs and freed blocks that the
device data path consumes; they run on the host only.
"""

from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from ._lib import lib
from .backend import _check
from .config import PhysicalSlot

_P, _U64, _U32, _I = C.c_void_p, C.c_uint64, C.c_uint32, C.c_int


class _Outcome(C.Structure):
    _fields_ = [
        ("admitted", C.POINTER(_U64)), ("num_admitted", _U64),
        ("decoded_id", C.POINTER(_U64)), ("decoded_block", C.POINTER(_U32)),
        ("decoded_slot", C.POINTER(_U64)), ("decoded_cow", C.POINTER(C.c_int32)),
        ("decoded_cow_src", C.POINTER(_U32)), ("decoded_cow_dst", C.POINTER(_U32)),
        ("num_decoded", _U64),
        ("preempted", C.POINTER(_U64)), ("num_preempted", _U64),
        ("finished", C.POINTER(_U64)), ("num_finished", _U64),
        ("freed_blocks", C.POINTER(_U32)), ("num_freed", _U64),
        ("admitted_ctx", C.POINTER(_U64)), ("admitted_table_offsets", C.POINTER(_U64)),
        ("admitted_blocks", C.POINTER(_U32)),
    ]


for _n, _r, _a in [
    ("pkv_allocator_new", _P, [_U64]), ("pkv_allocator_free", None, [_P]),
    ("pkv_allocator_allocate", _I, [_P, C.POINTER(_U32)]),
    ("pkv_allocator_allocate_many", _I, [_P, _U64, _P]),
    ("pkv_allocator_incref", _I, [_P, _U32, C.POINTER(_U32)]),
    ("pkv_allocator_decref", _I, [_P, _U32, C.POINTER(_U32)]),
    ("pkv_allocator_ref_count", _I, [_P, _U32, C.POINTER(_U32)]),
    ("pkv_allocator_num_free", _U64, [_P]), ("pkv_allocator_total_allocated", _U64, [_P]),
    ("pkv_allocator_check_invariants", _I, [_P]),
    ("pkv_allocator_ref_counts", _I, [_P, _P, _U64, _P]),
    ("pkv_table_new", _P, [_U64]), ("pkv_table_free_handle", None, [_P]),
    ("pkv_table_num_tokens", _U64, [_P]), ("pkv_table_num_blocks", _U64, [_P]),
    ("pkv_table_blocks", _U64, [_P, _P, _U64]),
    ("pkv_table_append", _I, [_P, _P, C.POINTER(_U32), C.POINTER(_U64), C.POINTER(_I),
                              C.POINTER(_U32), C.POINTER(_U32)]),
    ("pkv_table_append_many", _I, [_P, _P, _U64, _P, _P, _P, C.POINTER(_U64)]),
    ("pkv_table_resolve", _I, [_P, _U64, C.POINTER(_U32), C.POINTER(_U64)]),
    ("pkv_table_fork", _I, [_P, _P, C.POINTER(_P)]),
    ("pkv_table_release", _I, [_P, _P]),
    ("pkv_scheduler_new", _P, [_U64, _U64, _U64]), ("pkv_scheduler_free", None, [_P]),
    ("pkv_scheduler_add_request", _I, [_P, _U64, _U64, _U64]),
    ("pkv_scheduler_step", _I, [_P, C.POINTER(_Outcome)]),
    ("pkv_scheduler_fork_sequence", _I, [_P, _U64, _U64, _U64]),
    ("pkv_scheduler_num_running", _U64, [_P]), ("pkv_scheduler_num_waiting", _U64, [_P]),
    ("pkv_scheduler_pool_utilization", C.c_double, [_P]),
    ("pkv_scheduler_running", _I, [_P, _P, _P, _P, _P, _U64]),
]:
    _f = getattr(lib, _n)
    _f.restype = _r
    _f.argtypes = _a


class BlockAllocator:
    """allocator.rs:24-241."""

    def __init__(self, num_blocks: int):
        self._h = lib.pkv_allocator_new(num_blocks)
        self.num_blocks = num_blocks

    def __del__(self):
        if getattr(self, "_h", None):
            lib.pkv_allocator_free(self._h)
            self._h = None

    def allocate(self) -> int:
        out = _U32()
        _check(lib.pkv_allocator_allocate(self._h, C.byref(out)))
        return out.value

    def allocate_many(self, n: int) -> list[int]:
        out = np.zeros(max(n, 1), np.uint32)
        _check(lib.pkv_allocator_allocate_many(self._h, n, out.ctypes.data))
        return out[:n].tolist()

    def incref(self, b: int) -> int:
        out = _U32()
        _check(lib.pkv_allocator_incref(self._h, b, C.byref(out)))
        return out.value

    def decref(self, b: int) -> int:
        out = _U32()
        _check(lib.pkv_allocator_decref(self._h, b, C.byref(out)))
        return out.value

    def ref_count(self, b: int) -> int:
        out = _U32()
        _check(lib.pkv_allocator_ref_count(self._h, b, C.byref(out)))
        return out.value

    def is_shared(self, b: int) -> bool:
        return self.ref_count(b) > 1

    def num_free(self) -> int:
        return int(lib.pkv_allocator_num_free(self._h))

    def num_used(self) -> int:
        return self.num_blocks - self.num_free()

    def utilization(self) -> float:
        return 0.0 if self.num_blocks == 0 else self.num_used() / self.num_blocks

    def total_allocated(self) -> int:
        return int(lib.pkv_allocator_total_allocated(self._h))

    def check_invariants(self) -> None:
        _check(lib.pkv_allocator_check_invariants(self._h))

    def ref_counts(self, ids: np.ndarray) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        out = np.zeros(max(ids.size, 1), np.uint32)
        _check(lib.pkv_allocator_ref_counts(self._h, ids.ctypes.data, ids.size, out.ctypes.data))
        return out[: ids.size]


class BlockTable:
    """block_table.rs:20-240. Slots come back as PhysicalSlot; CoW copies as (src, dst)."""

    def __init__(self, block_size: int, _handle=None):
        self._h = _handle or lib.pkv_table_new(block_size)
        self.block_size = block_size

    def __del__(self):
        if getattr(self, "_h", None):
            lib.pkv_table_free_handle(self._h)
            self._h = None

    def num_tokens(self) -> int:
        return int(lib.pkv_table_num_tokens(self._h))

    def num_blocks(self) -> int:
        return int(lib.pkv_table_num_blocks(self._h))

    def physical_blocks(self) -> list[int]:
        n = self.num_blocks()
        out = np.zeros(max(n, 1), np.uint32)
        lib.pkv_table_blocks(self._h, out.ctypes.data, n)
        return out[:n].tolist()

    def append(self, a: BlockAllocator):
        b, s, cow, cs, cd = _U32(), _U64(), _I(), _U32(), _U32()
        _check(lib.pkv_table_append(self._h, a._h, C.byref(b), C.byref(s), C.byref(cow),
                                    C.byref(cs), C.byref(cd)))
        return PhysicalSlot(b.value, s.value), ((cs.value, cd.value) if cow.value else None)

    def append_many(self, a: BlockAllocator, n: int):
        blocks = np.zeros(max(n, 1), np.uint32)
        slots = np.zeros(max(n, 1), np.uint64)
        copies = np.zeros(2 * max(n, 1), np.uint32)
        nc = _U64()
        _check(lib.pkv_table_append_many(self._h, a._h, n, blocks.ctypes.data, slots.ctypes.data,
                                         copies.ctypes.data, C.byref(nc)))
        out = [PhysicalSlot(int(b), int(s)) for b, s in zip(blocks[:n], slots[:n])]
        return out, [tuple(copies[2 * i:2 * i + 2].tolist()) for i in range(nc.value)]

    def resolve(self, pos: int) -> PhysicalSlot:
        b, s = _U32(), _U64()
        _check(lib.pkv_table_resolve(self._h, pos, C.byref(b), C.byref(s)))
        return PhysicalSlot(b.value, s.value)

    def fork(self, a: BlockAllocator) -> "BlockTable":
        h = C.c_void_p()
        _check(lib.pkv_table_fork(self._h, a._h, C.byref(h)))
        return BlockTable(self.block_size, _handle=h.value)

    def free(self, a: BlockAllocator) -> None:
        _check(lib.pkv_table_release(self._h, a._h))


@dataclass
class DecodedToken:  # scheduler.rs:64-69
    id: int
    slot: PhysicalSlot
    cow: tuple | None


@dataclass
class StepOutcome:  # scheduler.rs:72-86, plus the blocks freed this step
    admitted: list = field(default_factory=list)
    decoded: list = field(default_factory=list)
    preempted: list = field(default_factory=list)
    finished: list = field(default_factory=list)
    freed: list = field(default_factory=list)


def _arr(ptr, n, dtype):
    if n == 0:
        return np.zeros(0, dtype)
    return np.ctypeslib.as_array(ptr, shape=(n,)).astype(dtype, copy=True)


class Scheduler:
    """scheduler.rs:117-358 (continuous batching with recompute preemption)."""

    def __init__(self, num_blocks: int, block_size: int, max_batch_size: int):
        self._h = lib.pkv_scheduler_new(num_blocks, block_size, max_batch_size)
        self.block_size = block_size

    def __del__(self):
        if getattr(self, "_h", None):
            lib.pkv_scheduler_free(self._h)
            self._h = None

    def add_request(self, sid: int, prompt_len: int, max_new_tokens: int) -> None:
        _check(lib.pkv_scheduler_add_request(self._h, sid, prompt_len, max_new_tokens))

    def step_raw(self) -> dict:
        """One step; outcome as numpy arrays (for driving the device)."""
        o = _Outcome()
        _check(lib.pkv_scheduler_step(self._h, C.byref(o)))
        nd = o.num_decoded
        na = o.num_admitted
        off = _arr(o.admitted_table_offsets, na + 1, np.int64)
        return {
            "admitted_ctx": _arr(o.admitted_ctx, na, np.int64),
            "admitted_table_offsets": off,
            "admitted_blocks": _arr(o.admitted_blocks, int(off[-1]) if na else 0, np.int64),
            "admitted": _arr(o.admitted, o.num_admitted, np.uint64),
            "decoded_id": _arr(o.decoded_id, nd, np.uint64),
            "decoded_block": _arr(o.decoded_block, nd, np.int64),
            "decoded_slot": _arr(o.decoded_slot, nd, np.int64),
            "decoded_cow": _arr(o.decoded_cow, nd, np.int32),
            "cow_src": _arr(o.decoded_cow_src, nd, np.int64),
            "cow_dst": _arr(o.decoded_cow_dst, nd, np.int64),
            "preempted": _arr(o.preempted, o.num_preempted, np.uint64),
            "finished": _arr(o.finished, o.num_finished, np.uint64),
            "freed": _arr(o.freed_blocks, o.num_freed, np.int64),
        }

    def step(self) -> StepOutcome:
        r = self.step_raw()
        dec = []
        for i in range(len(r["decoded_id"])):
            cow = (int(r["cow_src"][i]), int(r["cow_dst"][i])) if r["decoded_cow"][i] else None
            dec.append(DecodedToken(int(r["decoded_id"][i]),
                                    PhysicalSlot(int(r["decoded_block"][i]), int(r["decoded_slot"][i])), cow))
        return StepOutcome([int(x) for x in r["admitted"]], dec, [int(x) for x in r["preempted"]],
                           [int(x) for x in r["finished"]], [int(x) for x in r["freed"]])

    def fork_sequence(self, parent: int, child: int, max_new_tokens: int) -> None:
        _check(lib.pkv_scheduler_fork_sequence(self._h, parent, child, max_new_tokens))

    def num_running(self) -> int:
        return int(lib.pkv_scheduler_num_running(self._h))

    def num_waiting(self) -> int:
        return int(lib.pkv_scheduler_num_waiting(self._h))

    def is_idle(self) -> bool:
        return self.num_running() == 0 and self.num_waiting() == 0

    def pool_utilization(self) -> float:
        return float(lib.pkv_scheduler_pool_utilization(self._h))

    def running(self, table_stride: int):
        """(ids, tokens, generated, tables [n][table_stride] int32) of the running sequences."""
        n = self.num_running()
        ids = np.zeros(max(n, 1), np.uint64)
        tok = np.zeros(max(n, 1), np.uint64)
        gen = np.zeros(max(n, 1), np.uint64)
        tab = np.zeros((max(n, 1), table_stride), np.int32)
        _check(lib.pkv_scheduler_running(self._h, ids.ctypes.data, tok.ctypes.data, gen.ctypes.data,
                                         tab.ctypes.data, table_stride))
        return ids[:n], tok[:n], gen[:n], tab[:n]
