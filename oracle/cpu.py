"""TEST INFRASTRUCTURE ONLY -- ctypes wrapper of liboracle.so (pkv_oracle.c),
the C restatement of the reference's ``CpuBackend``.

Mirrors the trait's method names so that parity tests read like the
reference's own tests. Raises the same ``RefError`` codes as host_ref.py.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

from .host_ref import RefError

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"


def _load():
    if not LIB.exists():
        subprocess.run(["make", "-s", "-C", os.fspath(HERE)], check=True)
    return C.CDLL(os.fspath(LIB))


_lib = _load()


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in
                ("num_blocks", "block_size", "num_kv_heads", "head_dim", "num_layers", "dtype_bytes")]


class _Slot(C.Structure):
    _fields_ = [("block", C.c_uint64), ("slot", C.c_uint64)]


_P, _U64, _I64 = C.c_void_p, C.c_uint64, C.c_int64
for name, res, args in [
    ("orc_new", _P, [C.POINTER(_Cfg)]),
    ("orc_free", None, [_P]),
    ("orc_k_plane", _P, [_P]),
    ("orc_v_plane", _P, [_P]),
    ("orc_plane_elems", _U64, [_P]),
    ("orc_last_fields", None, [_P, C.POINTER(_I64), C.POINTER(_I64)]),
    ("orc_write_kv", C.c_int, [_P, _U64, _Slot, _P, _U64, _P, _U64]),
    ("orc_write_kv_batch", C.c_int, [_P, _U64, _P, _U64, _P, _U64, _P, _U64]),
    ("orc_read_kv", C.c_int, [_P, _U64, _Slot, _P, _U64, _P, _U64]),
    ("orc_copy_block", C.c_int, [_P, _U64, _U64]),
    ("orc_copy_blocks", C.c_int, [_P, _P, _U64]),
    ("orc_zero_block", C.c_int, [_P, _U64]),
    ("orc_zero_blocks", C.c_int, [_P, _P, _U64]),
    ("orc_allocated_bytes", _U64, [_P]),
    ("orc_resolve_slots", _I64, [_P, _I64, _P, _P, _I64, _I64, _I64, _I64, _P, _P]),
    ("orc_digest_plane", _U64, [_P, _U64, C.c_uint32]),
    ("orc_digest_rows", _U64, [_P, _U64, _U64, _P, _U64, _U64, C.c_uint32]),
    ("orc_set_fp8", C.c_int, [_P, _P, _P]),
    ("orc_e4m3_from_f32_array", None, [_P, _U64, _P]),
    ("orc_e4m3_to_f32", C.c_float, [C.c_uint8]),
]:
    f = getattr(_lib, name)
    f.restype = res
    f.argtypes = args


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


def _slot(s) -> _Slot:
    b, o = (s.block, s.slot) if hasattr(s, "block") else s
    return _Slot(int(b), int(o))


class OracleBackend:
    """CpuBackend (cpu.rs:27-165) restated in C; f32 planes."""

    def __init__(self, cfg):
        c = _Cfg(cfg.num_blocks, cfg.block_size, cfg.num_kv_heads, cfg.head_dim, cfg.num_layers,
                 cfg.dtype_bytes)
        self.cfg = cfg
        self._h = _lib.orc_new(C.byref(c))
        if not self._h:
            raise MemoryError("oracle pool")

    def __del__(self):
        if getattr(self, "_h", None):
            _lib.orc_free(self._h)
            self._h = None

    def _rc(self, rc: int) -> None:
        if rc:
            a, b = _I64(), _I64()
            _lib.orc_last_fields(self._h, C.byref(a), C.byref(b))
            raise RefError(rc, a.value, b.value)

    def set_fp8(self, k_scales, v_scales) -> None:
        """Makes this an fp8 (E4M3) pool with [num_layers][num_kv_heads] scales."""
        self._k_scales = np.ascontiguousarray(k_scales, dtype=np.float32).ravel()
        self._v_scales = np.ascontiguousarray(v_scales, dtype=np.float32).ravel()
        n = self.cfg.num_layers * self.cfg.num_kv_heads
        assert self._k_scales.size == n and self._v_scales.size == n
        self._rc(_lib.orc_set_fp8(self._h, self._k_scales.ctypes.data, self._v_scales.ctypes.data))

    def write_kv(self, layer, dst, k, v):
        k, v = _f32(k), _f32(v)
        self._rc(_lib.orc_write_kv(self._h, layer, _slot(dst), k.ctypes.data, k.size, v.ctypes.data, v.size))

    def write_kv_batch(self, layer, dsts, k, v):
        k, v = _f32(k), _f32(v)
        arr = (_Slot * max(len(dsts), 1))(*[_slot(s) for s in dsts])
        self._rc(_lib.orc_write_kv_batch(self._h, layer, C.addressof(arr), len(dsts), k.ctypes.data,
                                         k.size, v.ctypes.data, v.size))

    def write_kv_batch_pairs(self, layer, pairs: np.ndarray, k: np.ndarray, v: np.ndarray):
        """write_kv_batch with dsts as a contiguous uint64 [n][2] (block, slot)
        array and contiguous f32 rows: no per-token Python work."""
        self._rc(_lib.orc_write_kv_batch(self._h, layer, pairs.ctypes.data, pairs.shape[0],
                                         k.ctypes.data, k.size, v.ctypes.data, v.size))

    def read_kv(self, layer, src, k_out, v_out):
        self._rc(_lib.orc_read_kv(self._h, layer, _slot(src), k_out.ctypes.data, k_out.size,
                                  v_out.ctypes.data, v_out.size))

    def read_entry(self, layer, src):
        n = self.cfg.num_kv_heads * self.cfg.head_dim
        k, v = np.zeros(n, np.float32), np.zeros(n, np.float32)
        self.read_kv(layer, src, k, v)
        return k, v

    def copy_block(self, src, dst):
        self._rc(_lib.orc_copy_block(self._h, src, dst))

    def copy_blocks(self, pairs):
        a = np.ascontiguousarray(np.asarray(pairs, dtype=np.uint64).reshape(-1, 2))
        self._rc(_lib.orc_copy_blocks(self._h, a.ctypes.data, a.shape[0]))

    def zero_block(self, block):
        self._rc(_lib.orc_zero_block(self._h, block))

    def zero_blocks(self, blocks):
        a = np.ascontiguousarray(np.asarray(blocks, dtype=np.uint64))
        self._rc(_lib.orc_zero_blocks(self._h, a.ctypes.data, a.size))

    def allocated_bytes(self) -> int:
        return int(_lib.orc_allocated_bytes(self._h))

    def planes(self) -> tuple[np.ndarray, np.ndarray]:
        """(K, V) as [L][num_blocks][block_size][entry] f32 views (no copy)."""
        n = int(_lib.orc_plane_elems(self._h))
        c = self.cfg
        shape = (c.num_layers, c.num_blocks, c.block_size, c.num_kv_heads * c.head_dim)
        out = []
        for f in (_lib.orc_k_plane, _lib.orc_v_plane):
            p = f(self._h)
            buf = (C.c_float * max(n, 1)).from_address(p)
            out.append(np.frombuffer(buf, dtype=np.float32, count=n).reshape(shape))
        return out[0], out[1]

    def digest(self) -> tuple[int, int]:
        n = int(_lib.orc_plane_elems(self._h))
        return (int(_lib.orc_digest_plane(_lib.orc_k_plane(self._h), n, 0)),
                int(_lib.orc_digest_plane(_lib.orc_v_plane(self._h), n, 1)))


def resolve_slots(tables: np.ndarray, ctx: np.ndarray, new: np.ndarray, num_tokens: int,
                  block_size: int, num_blocks: int):
    """Oracle of the device slot-resolution kernel; returns (status, cu, slots)."""
    tables = np.ascontiguousarray(tables, dtype=np.int32)
    ctx = np.ascontiguousarray(ctx, dtype=np.int32)
    new = np.ascontiguousarray(new, dtype=np.int32)
    s = ctx.shape[0]
    stride = tables.shape[1] if tables.ndim == 2 else 0
    cu = np.zeros(s + 1, np.int32)
    slots = np.full(max(num_tokens, 1), -7, np.int64)
    rc = _lib.orc_resolve_slots(tables.ctypes.data, stride, ctx.ctypes.data, new.ctypes.data, s,
                                num_tokens, block_size, num_blocks, cu.ctypes.data, slots.ctypes.data)
    return int(rc), cu, slots[:num_tokens]


def digest_rows(rows_f32: np.ndarray, slots: np.ndarray, layer: int, slots_per_layer: int,
                plane: int) -> int:
    rows = np.ascontiguousarray(rows_f32, dtype=np.float32)
    sl = np.ascontiguousarray(slots, dtype=np.int64)
    return int(_lib.orc_digest_rows(rows.ctypes.data, rows.shape[0], rows.shape[1], sl.ctypes.data,
                                    layer, slots_per_layer, plane))


def digest_plane(plane_f32: np.ndarray, plane_id: int) -> int:
    p = np.ascontiguousarray(plane_f32, dtype=np.float32)
    return int(_lib.orc_digest_plane(p.ctypes.data, p.size, plane_id))


def e4m3_from_f32(x) -> np.ndarray:
    """E4M3 codes (uint8) of f32 values: round to nearest even, saturating to
    +-448 (pkv_oracle.c, orc_e4m3_from_f32)."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(a.shape, np.uint8)
    _lib.orc_e4m3_from_f32_array(a.ctypes.data, a.size, out.ctypes.data)
    return out


_E4M3_TABLE = np.array([_lib.orc_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)


def e4m3_to_f32(q) -> np.ndarray:
    """Exact f32 values of E4M3 codes."""
    return _E4M3_TABLE[np.asarray(q, dtype=np.uint8)]
