"""pagedkv -- host-side mirror of paged-kv-core's ``KvBackend`` over the B200
data path in libpagedkv_b200.so (include/pkv_b200.h).

The configuration, error and workload modules are plain Python. The native
library is loaded the first time ``B200Backend`` (or ``pagedkv._lib``) is
used, not at ``import pagedkv``: a process that only builds workloads or
configurations never maps the device library. Using ``B200Backend`` without
the built library raises ImportError (there is no fallback).
"""

from .config import CacheConfig, PhysicalSlot
from .errors import (BlockNotAllocated, CacheError, Device, InvalidBlock, InvalidLayer,
                     OutOfBlocks, RefCountOverflow, ShapeMismatch, SlotOutOfRange, UnknownSequence)

__all__ = [
    "B200Backend", "CacheConfig", "PhysicalSlot", "CacheError", "OutOfBlocks", "InvalidBlock",
    "BlockNotAllocated", "RefCountOverflow", "SlotOutOfRange", "ShapeMismatch", "InvalidLayer",
    "UnknownSequence", "Device",
]


def __getattr__(name):
    if name == "B200Backend":
        from .backend import B200Backend

        return B200Backend
    raise AttributeError(f"module 'pagedkv' has no attribute {name!r}")
