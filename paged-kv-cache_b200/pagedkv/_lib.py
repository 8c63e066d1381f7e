"""ctypes binding of libpagedkv_b200.so (include/pkv_b200.h).

The library is built in-tree (``make -C paged-kv-cache_b200``) and loaded from
``paged-kv-cache_b200/lib/``. There is no fallback: if the library is missing,
importing this module raises.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent.parent
LIB_PATH = PKG_ROOT / "lib" / "libpagedkv_b200.so"

if not LIB_PATH.exists():
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `make -C {PKG_ROOT}` "
        "(nvcc, sm_100a); the data path has no CPU fallback")

lib = C.CDLL(os.fspath(LIB_PATH))

# pkv_dtype
F32, BF16, F16, FP8_E4M3 = 0, 1, 2, 3
DTYPE_TAGS = {"f32": F32, "bf16": BF16, "f16": F16, "fp8_e4m3": FP8_E4M3}
DTYPE_BYTES = {F32: 4, BF16: 2, F16: 2, FP8_E4M3: 1}

# pkv_copy_engine
COPY_AUTO, COPY_VECTOR, COPY_BULK = 0, 1, 2


class Config(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in
                ("num_blocks", "block_size", "num_kv_heads", "head_dim", "num_layers", "dtype_bytes")]


class Slot(C.Structure):
    _fields_ = [("block", C.c_uint64), ("slot", C.c_uint64)]


_P = C.c_void_p
_U64 = C.c_uint64
_I64 = C.c_int64
_I = C.c_int

_PROTOS = {
    "pkv_last_error": (C.c_char_p, []),
    "pkv_last_error_fields": (_I, [C.POINTER(_I64), C.POINTER(_I64)]),
    "pkv_create": (_I, [C.POINTER(Config), _I, _I, _I, _I, C.POINTER(_P)]),
    "pkv_destroy": (_I, [_P]),
    "pkv_get_config": (_I, [_P, C.POINTER(Config)]),
    "pkv_allocated_bytes": (_U64, [_P]),
    "pkv_device_name": (_I, [_P, C.c_char_p, _U64]),
    "pkv_shard_info": (_I, [_P, C.POINTER(_I), C.POINTER(_I), C.POINTER(_U64), C.POINTER(_U64)]),
    "pkv_device_planes": (_I, [_P, C.POINTER(_P), C.POINTER(_P)]),
    "pkv_write_kv": (_I, [_P, _U64, Slot, _P, _U64, _P, _U64, _I]),
    "pkv_write_kv_batch": (_I, [_P, _U64, _P, _U64, _P, _U64, _P, _U64, _I]),
    "pkv_read_kv": (_I, [_P, _U64, Slot, _P, _U64, _P, _U64, _I]),
    "pkv_copy_block": (_I, [_P, _U64, _U64]),
    "pkv_copy_blocks": (_I, [_P, _P, _U64]),
    "pkv_zero_block": (_I, [_P, _U64]),
    "pkv_zero_blocks": (_I, [_P, _P, _U64]),
    "pkv_reshape_and_cache_dev": (_I, [_P, _I64, _P, _P, _I64, _I64, _P, _I64, _I, _P]),
    "pkv_copy_blocks_dev": (_I, [_P, _P, _I64, _P]),
    "pkv_zero_blocks_dev": (_I, [_P, _P, _I64, _P]),
    "pkv_copy_zero_blocks_dev": (_I, [_P, _P, _P, _P, _P, _I64, _P, _I64, _P]),
    "pkv_resolve_and_cache_mixed_dev": (_I, [_P, _P, _I64, _P, _P, _I64, _I64, _P, _P, _P, _I64,
                                             _I64, _P, _P, _I64, _I64, _I, _P]),
    "pkv_set_copy_engine": (_I, [_P, _I]),
    "pkv_set_kv_scales": (_I, [_P, _P, _P, _U64]),
    "pkv_paged_attention_dev": (_I, [_P, _I64, _P, _I64, _I64, _I64, _P, _I64, _P, _I64, C.c_float,
                                     _P, _P, _P]),
    "pkv_paged_attention_typed_dev": (_I, [_P, _I64, _P, _I, _I64, _I64, _I64, _P, _I64, _P, _I64,
                                           C.c_float, _P, _P, _P]),
    "pkv_paged_attention_multi_dev": (_I, [_P, _I64, _P, _I, _I64, _I64, _I64, _I64, _P, _I64, _P,
                                           _I64, C.c_float, _P, _P, _P]),
    "pkv_paged_attention_plan_dev": (_I, [_P, _P, _I64, _I64, _P]),
    "pkv_resolve_slots_dev": (_I, [_P, _P, _I64, _P, _P, _I64, _I64, _P, _P, _P]),
    "pkv_resolve_and_cache_dev": (_I, [_P, _P, _I64, _P, _P, _I64, _I64, _P, _P, _I64, _P, _P,
                                       _I64, _I64, _I, _P]),
    "pkv_digest": (_I, [_P, C.POINTER(_U64), C.POINTER(_U64), _P]),
    "pkv_resolve_and_cache_noalloc": (_I, [C.POINTER(Config), _I, _I, _I, _P, _P, _P, _I64, _P, _P,
                                           _I64, _I64, _P, _I64, _P, _P, _I64, _I64, _I, _P, _P]),
    "pkv_digest_rows_dev": (_I, [_P, _I64, _P, _P, _I64, _I64, _P, _I64, _I, C.POINTER(_U64),
                                 C.POINTER(_U64), _P]),
    "pkv_f32_to_bf16": (_I, [_P, _P, _U64]),
    "pkv_host_threads": (_I, [_P, C.POINTER(_I)]),
    "pkv_sync": (_I, [_P]),
    "pkv_device_error": (_I, [_P, C.POINTER(_I64)]),
}

for _name, (_res, _args) in _PROTOS.items():
    _f = getattr(lib, _name)
    _f.restype = _res
    _f.argtypes = _args


def last_error() -> tuple[int, int, int, str]:
    """(status, field0, field1, message) of the last call on this thread."""
    a, b = _I64(), _I64()
    code = lib.pkv_last_error_fields(C.byref(a), C.byref(b))
    return code, a.value, b.value, lib.pkv_last_error().decode()
