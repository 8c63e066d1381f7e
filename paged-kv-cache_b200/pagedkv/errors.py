"""CacheError (crates/paged-kv-core/src/error.rs:12-46) as Python exceptions.

Each variant carries the same named fields as the reference; two errors are
equal when their variant and fields are equal, so tests can assert on exact
variants the way the reference's own tests do.
"""

from __future__ import annotations


class CacheError(Exception):
    code = -1
    fields: tuple[str, ...] = ()

    def __init__(self, *values):
        super().__init__(*values)
        self.values = tuple(values)
        for name, val in zip(self.fields, values):
            setattr(self, name, val)

    def __eq__(self, other):
        return type(self) is type(other) and self.values == other.values

    def __hash__(self):
        return hash((type(self), self.values))

    def __repr__(self):
        body = ", ".join(f"{n}: {v!r}" for n, v in zip(self.fields, self.values))
        return f"{type(self).__name__} {{ {body} }}"


class OutOfBlocks(CacheError):  # error.rs:14
    code, fields = 1, ("requested", "available")


class InvalidBlock(CacheError):  # error.rs:17
    code, fields = 2, ("id", "num_blocks")


class BlockNotAllocated(CacheError):  # error.rs:20
    code, fields = 3, ("id",)


class RefCountOverflow(CacheError):  # error.rs:24
    code, fields = 4, ("id", "max")


class SlotOutOfRange(CacheError):  # error.rs:27
    code, fields = 5, ("slot", "block_size")


class ShapeMismatch(CacheError):  # error.rs:31
    code, fields = 6, ("expected", "actual")


class InvalidLayer(CacheError):  # error.rs:34
    code, fields = 7, ("layer", "num_layers")


class UnknownSequence(CacheError):  # error.rs:38
    code, fields = 8, ("id",)


class Device(CacheError):  # error.rs:45
    code, fields = 9, ("message",)


BY_CODE = {c.code: c for c in (OutOfBlocks, InvalidBlock, BlockNotAllocated, RefCountOverflow,
                               SlotOutOfRange, ShapeMismatch, InvalidLayer, UnknownSequence, Device)}


def from_status(code: int, a: int, b: int, msg: str) -> CacheError:
    cls = BY_CODE.get(code, Device)
    if cls is Device:
        return Device(msg)
    return cls(*(a, b)[: len(cls.fields)])
