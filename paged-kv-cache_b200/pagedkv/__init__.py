"""pagedkv -- host-side mirror of paged-kv-core's ``KvBackend`` over the B200
data path in libpagedkv_b200.so (include/pkv_b200.h)."""

from .backend import B200Backend
from .config import CacheConfig, PhysicalSlot
from .errors import (BlockNotAllocated, CacheError, Device, InvalidBlock, InvalidLayer,
                     OutOfBlocks, RefCountOverflow, ShapeMismatch, SlotOutOfRange, UnknownSequence)

__all__ = [
    "B200Backend", "CacheConfig", "PhysicalSlot", "CacheError", "OutOfBlocks", "InvalidBlock",
    "BlockNotAllocated", "RefCountOverflow", "SlotOutOfRange", "ShapeMismatch", "InvalidLayer",
    "UnknownSequence", "Device",
]
