"""B200Backend: the ``KvBackend`` trait (crates/paged-kv-core/src/backend.rs:23-124)
over libpagedkv_b200.so.

Method names, argument meaning, validation order and error variants follow
the trait and ``CpuBackend`` (crates/paged-kv-core/src/cpu.rs); every call goes
through the C ABI of include/pkv_b200.h. Host-buffer methods take numpy
arrays; the device entry points take CUDA tensors (torch) or raw addresses.
"""

from __future__ import annotations

import ctypes as C
from typing import Iterable, Sequence

import numpy as np

from . import _lib
from ._lib import BF16, DTYPE_BYTES, DTYPE_TAGS, F16, F32, FP8_E4M3, lib
from .config import CacheConfig, PhysicalSlot
from .errors import from_status

_NP_TAG = {np.dtype(np.float32): F32, np.dtype(np.float16): F16}


def _check(code: int) -> None:
    if code != 0:
        raise from_status(*_lib.last_error())


def _host_array(x, tag: int | None):
    """Contiguous numpy view of a host buffer plus its dtype tag. bf16 data is
    passed as uint16 bit patterns with tag BF16, E4M3 codes as uint8."""
    a = np.ascontiguousarray(x)
    if tag is None:
        if a.dtype in _NP_TAG:
            tag = _NP_TAG[a.dtype]
        elif a.dtype == np.uint16:
            tag = BF16
        elif a.dtype == np.uint8:
            tag = FP8_E4M3
        else:
            a = a.astype(np.float32)
            tag = F32
    expect = {F32: np.float32, F16: np.float16, BF16: np.uint16, FP8_E4M3: np.uint8}[tag]
    if a.dtype != expect:
        a = a.astype(expect) if tag == F32 else a.view(expect)
    return a, tag


def _slot(s) -> _lib.Slot:
    if isinstance(s, PhysicalSlot):
        return _lib.Slot(s.block, s.slot)
    b, o = s
    return _lib.Slot(int(b), int(o))


def _ptr(t) -> int:
    """Device address of a torch tensor (or an int address)."""
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream_ptr(stream) -> int | None:
    """cudaStream_t for a device entry point: torch's current stream by default."""
    if stream is None:
        import torch

        return torch.cuda.current_stream().cuda_stream or None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


class _DeviceArray:
    """Minimal __cuda_array_interface__ so torch can view the pool planes."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {
            "shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3, "strides": None}


class B200Backend:
    """One device pool (or one KV-head shard of it) on one B200."""

    def __init__(self, config: CacheConfig, dtype: str = "f32", device: int = 0,
                 shard_rank: int = 0, num_shards: int = 1):
        self._cfg = config
        self._dtype = DTYPE_TAGS[dtype]
        self.device = device
        h = C.c_void_p()
        c = _lib.Config(config.num_blocks, config.block_size, config.num_kv_heads,
                        config.head_dim, config.num_layers, config.dtype_bytes)
        _check(lib.pkv_create(C.byref(c), self._dtype, device, shard_rank, num_shards, C.byref(h)))
        self._h = h
        r, g, off, n = C.c_int(), C.c_int(), C.c_uint64(), C.c_uint64()
        _check(lib.pkv_shard_info(h, C.byref(r), C.byref(g), C.byref(off), C.byref(n)))
        self.shard_rank, self.num_shards = r.value, g.value
        self.elem_offset, self.shard_entry_elems = off.value, n.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib.pkv_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- KvBackend ----------------------------------------------------------

    def config(self) -> CacheConfig:  # backend.rs:25
        return self._cfg

    def write_kv(self, layer: int, dst, k, v, host_dtype: str | None = None) -> None:
        """backend.rs:34-40."""
        tag = None if host_dtype is None else DTYPE_TAGS[host_dtype]
        ka, tag = _host_array(k, tag)
        va, _ = _host_array(v, tag)
        _check(lib.pkv_write_kv(self._h, layer, _slot(dst), ka.ctypes.data, ka.size,
                                va.ctypes.data, va.size, tag))

    def write_kv_batch(self, layer: int, dsts: Sequence, k, v, host_dtype: str | None = None) -> None:
        """backend.rs:55-74: k, v flattened, dsts.len() * entry_elems each."""
        tag = None if host_dtype is None else DTYPE_TAGS[host_dtype]
        ka, tag = _host_array(k, tag)
        va, _ = _host_array(v, tag)
        arr = (_lib.Slot * max(len(dsts), 1))(*[_slot(s) for s in dsts])
        _check(lib.pkv_write_kv_batch(self._h, layer, C.addressof(arr), len(dsts), ka.ctypes.data,
                                      ka.size, va.ctypes.data, va.size, tag))

    @staticmethod
    def slot_pairs(blocks: np.ndarray, slots: np.ndarray) -> np.ndarray:
        """Destinations as the C ABI's pkv_slot array ([n][2] uint64: block,
        slot), built once and passed to every layer's write_kv_batch_pairs."""
        pairs = np.empty((len(blocks), 2), dtype=np.uint64)
        pairs[:, 0] = blocks
        pairs[:, 1] = slots
        return pairs

    def write_kv_batch_pairs(self, layer: int, pairs: np.ndarray, k, v,
                             host_dtype: str | None = None) -> None:
        """write_kv_batch with the destinations as a slot_pairs array."""
        if pairs.dtype != np.uint64 or pairs.ndim != 2 or pairs.shape[1] != 2 or not pairs.flags.c_contiguous:
            raise ValueError("pairs must be a contiguous [n][2] uint64 array (see slot_pairs)")
        tag = None if host_dtype is None else DTYPE_TAGS[host_dtype]
        ka, tag = _host_array(k, tag)
        va, _ = _host_array(v, tag)
        _check(lib.pkv_write_kv_batch(self._h, layer, pairs.ctypes.data, len(pairs),
                                      ka.ctypes.data, ka.size, va.ctypes.data, va.size, tag))

    def write_kv_batch_slots(self, layer: int, blocks: np.ndarray, slots: np.ndarray, k, v,
                             host_dtype: str | None = None) -> None:
        """write_kv_batch with the destinations given as two integer arrays."""
        self.write_kv_batch_pairs(layer, self.slot_pairs(blocks, slots), k, v, host_dtype)

    def host_threads(self) -> int:
        """Worker threads of the library's host stager (PKV_HOST_THREADS)."""
        n = C.c_int()
        _check(lib.pkv_host_threads(self._h, C.byref(n)))
        return n.value

    def read_kv(self, layer: int, src, k_out: np.ndarray, v_out: np.ndarray) -> None:
        """backend.rs:82-88: fills k_out and v_out (f32, f16, or uint16 = bf16 bits)."""
        tag = _host_array(k_out[:0], None)[1]
        for a in (k_out, v_out):
            if not a.flags.c_contiguous:
                raise ValueError("read_kv needs contiguous output arrays")
        _check(lib.pkv_read_kv(self._h, layer, _slot(src), k_out.ctypes.data, k_out.size,
                               v_out.ctypes.data, v_out.size, tag))

    def read_entry(self, layer: int, src) -> tuple[np.ndarray, np.ndarray]:
        n = self.shard_entry_elems
        k, v = np.zeros(n, np.float32), np.zeros(n, np.float32)
        self.read_kv(layer, src, k, v)
        return k, v

    def copy_block(self, src: int, dst: int) -> None:  # backend.rs:97
        _check(lib.pkv_copy_block(self._h, src, dst))

    def copy_blocks(self, pairs: Iterable) -> None:  # backend.rs:104-109
        a = np.ascontiguousarray(np.asarray(list(pairs) if not isinstance(pairs, np.ndarray) else pairs,
                                            dtype=np.uint64).reshape(-1, 2))
        _check(lib.pkv_copy_blocks(self._h, a.ctypes.data, a.shape[0]))

    def zero_block(self, block: int) -> None:  # backend.rs:115
        _check(lib.pkv_zero_block(self._h, block))

    def zero_blocks(self, blocks: Iterable[int]) -> None:
        a = np.ascontiguousarray(np.asarray(list(blocks) if not isinstance(blocks, np.ndarray) else blocks,
                                            dtype=np.uint64))
        _check(lib.pkv_zero_blocks(self._h, a.ctypes.data, a.size))

    def allocated_bytes(self) -> int:  # backend.rs:118-120
        return int(lib.pkv_allocated_bytes(self._h))

    def device_name(self) -> str:  # backend.rs:123
        buf = C.create_string_buffer(256)
        _check(lib.pkv_device_name(self._h, buf, 256))
        return buf.value.decode()

    # ---- device entry points ----------------------------------------------------

    def reshape_and_cache(self, k, v, slot_mapping, layer: int | None = None, stream=None) -> None:
        """Scatter device rows into the pool. layer=None: k, v are [L][T][entry]."""
        tag = _torch_tag(k)
        if layer is None:
            n_tok = k.shape[1]
            tok_stride, layer_stride, lay = k.stride(1), k.stride(0), -1
            _same_layout(k, v)
        else:
            n_tok = k.shape[0]
            tok_stride, layer_stride, lay = k.stride(0), 0, layer
            _same_layout(k, v)
        _check(lib.pkv_reshape_and_cache_dev(self._h, lay, _ptr(k), _ptr(v), tok_stride,
                                             layer_stride, _ptr(slot_mapping), n_tok, tag,
                                             _stream_ptr(stream)))

    def copy_blocks_dev(self, pairs, count: int | None = None, stream=None) -> None:
        n = pairs.shape[0] if count is None else count
        _check(lib.pkv_copy_blocks_dev(self._h, _ptr(pairs), n, _stream_ptr(stream)))

    def set_kv_scales(self, k_scales, v_scales) -> None:
        """Scales of an fp8 (E4M3) pool, [num_layers][num_kv_heads] each (pkv_set_kv_scales)."""
        ks = np.ascontiguousarray(k_scales, dtype=np.float32).ravel()
        vs = np.ascontiguousarray(v_scales, dtype=np.float32).ravel()
        if ks.size != vs.size:
            raise ValueError("k_scales and v_scales differ in size")
        _check(lib.pkv_set_kv_scales(self._h, ks.ctypes.data, vs.ctypes.data, ks.size))

    def set_copy_engine(self, engine: str) -> None:
        """Engine of later copy_blocks calls: "auto", "vector" or "bulk" (pkv_set_copy_engine)."""
        tag = {"auto": _lib.COPY_AUTO, "vector": _lib.COPY_VECTOR, "bulk": _lib.COPY_BULK}[engine]
        _check(lib.pkv_set_copy_engine(self._h, tag))

    def zero_blocks_dev(self, blocks, count: int | None = None, stream=None) -> None:
        n = blocks.shape[0] if count is None else count
        _check(lib.pkv_zero_blocks_dev(self._h, _ptr(blocks), n, _stream_ptr(stream)))

    def copy_zero_blocks_dev(self, srcs, dst_offsets, dsts, zero_src, zero_ids, num_srcs=None,
                             num_zero=None, stream=None) -> None:
        """One launch for a step's copies (grouped by source, see
        pkv_copy_zero_blocks_dev) and the blocks it zeroes; int64 device tensors."""
        ns = srcs.shape[0] if num_srcs is None else num_srcs
        nz = zero_ids.shape[0] if num_zero is None else num_zero
        _check(lib.pkv_copy_zero_blocks_dev(self._h, _ptr(srcs), _ptr(dst_offsets), _ptr(dsts),
                                            _ptr(zero_src), ns, _ptr(zero_ids), nz,
                                            _stream_ptr(stream)))

    def resolve_slots(self, block_tables, ctx_lens, new_lens, num_tokens: int, cu_out, slots_out,
                      stream=None) -> None:
        """Device slot resolution: block_tables [S][stride] int32, ctx/new int32 [S]."""
        s = ctx_lens.shape[0]
        stride = block_tables.shape[1] if block_tables.dim() == 2 else 0
        _check(lib.pkv_resolve_slots_dev(self._h, _ptr(block_tables), stride, _ptr(ctx_lens),
                                         _ptr(new_lens), s, num_tokens, _ptr(cu_out),
                                         _ptr(slots_out), _stream_ptr(stream)))

    def resolve_and_cache(self, block_tables, ctx_lens, new_lens, num_tokens: int, cu_out, k, v,
                          layer: int | None = None, slots_out=None, stream=None) -> None:
        """Fused slot resolution + reshape_and_cache (one launch); k, v as in
        reshape_and_cache, slots_out optional."""
        s = ctx_lens.shape[0]
        stride = block_tables.shape[1] if block_tables.dim() == 2 else 0
        tag = _torch_tag(k)
        _same_layout(k, v)
        if layer is None:
            tok_stride, layer_stride, lay = k.stride(1), k.stride(0), -1
        else:
            tok_stride, layer_stride, lay = k.stride(0), 0, layer
        _check(lib.pkv_resolve_and_cache_dev(self._h, _ptr(block_tables), stride, _ptr(ctx_lens),
                                             _ptr(new_lens), s, num_tokens, _ptr(cu_out),
                                             _ptr(slots_out), lay, _ptr(k), _ptr(v), tok_stride,
                                             layer_stride, tag, _stream_ptr(stream)))

    def resolve_and_cache_mixed(self, block_tables, ctx_lens, new_lens, num_tokens: int, cu_out,
                                direct_slots, num_direct: int, k, v, layer: int | None = None,
                                slots_out=None, stream=None) -> None:
        """One launch for a step's resolved tokens (rows [0, num_tokens)) and
        its host-slot tokens (rows num_tokens + j to direct_slots[j])."""
        s = ctx_lens.shape[0]
        stride = block_tables.shape[1] if block_tables.dim() == 2 else 0
        tag = _torch_tag(k)
        _same_layout(k, v)
        if layer is None:
            tok_stride, layer_stride, lay = k.stride(1), k.stride(0), -1
        else:
            tok_stride, layer_stride, lay = k.stride(0), 0, layer
        _check(lib.pkv_resolve_and_cache_mixed_dev(
            self._h, _ptr(block_tables), stride, _ptr(ctx_lens), _ptr(new_lens), s, num_tokens,
            _ptr(cu_out), _ptr(slots_out), _ptr(direct_slots), num_direct, lay, _ptr(k), _ptr(v),
            tok_stride, layer_stride, tag, _stream_ptr(stream)))

    def paged_attention_plan(self, context_lens, max_context_len: int, stream=None) -> None:
        """Longest-first order of the sequences for the following
        paged_attention calls with these context_lens
        (pkv_paged_attention_plan_dev); results unchanged."""
        _check(lib.pkv_paged_attention_plan_dev(self._h, _ptr(context_lens), context_lens.shape[0],
                                                max_context_len, _stream_ptr(stream)))

    def paged_attention(self, q, block_tables, context_lens, max_context_len: int, out,
                        layer: int, softmax_scale: float | None = None, lse=None,
                        stream=None, q_len: int = 1) -> None:
        """Paged attention over one layer: q and out [num_seqs * q_len]
        [num_q_heads][head_dim], bf16 or f16 (the pool dtype, or either over
        an fp8 pool), block_tables int32 [num_seqs][stride], context_lens
        int32 [num_seqs], lse optional f32 [num_seqs * q_len][num_q_heads].
        q_len 1 is decode (pkv_paged_attention_typed_dev); q_len > 1 query
        tokens per sequence are the last q_len positions of its context,
        causal among themselves (pkv_paged_attention_multi_dev)."""
        rows, hq, d = q.shape
        if q_len < 1 or rows % q_len:
            raise ValueError("q must hold q_len rows per sequence")
        if q.stride(2) != 1 or q.stride(1) != d:
            raise ValueError("q must hold contiguous [heads][head_dim] rows")
        if not out.is_contiguous() or tuple(out.shape) != (rows, hq, d):
            raise ValueError("out must be a dense [num_seqs * q_len][num_q_heads][head_dim] tensor")
        if out.dtype != q.dtype:
            raise ValueError("out must have the dtype of q")
        if softmax_scale is None:
            softmax_scale = d ** -0.5
        stride = block_tables.shape[1] if block_tables.dim() == 2 else 0
        if q_len == 1:
            _check(lib.pkv_paged_attention_typed_dev(self._h, layer, _ptr(q), _torch_tag(q), q.stride(0),
                                                     rows, hq, _ptr(block_tables), stride,
                                                     _ptr(context_lens), max_context_len,
                                                     float(softmax_scale), _ptr(out), _ptr(lse),
                                                     _stream_ptr(stream)))
        else:
            _check(lib.pkv_paged_attention_multi_dev(self._h, layer, _ptr(q), _torch_tag(q), q_len,
                                                     q.stride(0), rows // q_len, hq,
                                                     _ptr(block_tables), stride, _ptr(context_lens),
                                                     max_context_len, float(softmax_scale), _ptr(out),
                                                     _ptr(lse), _stream_ptr(stream)))

    def digest(self, stream=None) -> tuple[int, int]:
        k, v = C.c_uint64(), C.c_uint64()
        _check(lib.pkv_digest(self._h, C.byref(k), C.byref(v), _stream_ptr(stream)))
        return k.value, v.value

    def digest_rows(self, k, v, slot_mapping, layer: int | None = None, stream=None) -> tuple[int, int]:
        """Digests the pool would have if these rows were its only contents."""
        tag = _torch_tag(k)
        if layer is None:
            n_tok, tok_stride, layer_stride, lay = k.shape[1], k.stride(1), k.stride(0), -1
        else:
            n_tok, tok_stride, layer_stride, lay = k.shape[0], k.stride(0), 0, layer
        _same_layout(k, v)
        kd, vd = C.c_uint64(), C.c_uint64()
        _check(lib.pkv_digest_rows_dev(self._h, lay, _ptr(k), _ptr(v), tok_stride, layer_stride,
                                       _ptr(slot_mapping), n_tok, tag, C.byref(kd), C.byref(vd),
                                       _stream_ptr(stream)))
        return kd.value, vd.value

    def sync(self) -> None:
        _check(lib.pkv_sync(self._h))

    def device_error(self):
        """None, or (CacheError, index) for the first bad index a device entry point met."""
        idx = C.c_int64()
        code = lib.pkv_device_error(self._h, C.byref(idx))
        if code == 0:
            return None
        return from_status(*_lib.last_error()), idx.value

    def planes(self):
        """(K, V) torch views [L][num_blocks][block_size][entry] of the device pool."""
        import torch

        k, v = C.c_void_p(), C.c_void_p()
        _check(lib.pkv_device_planes(self._h, C.byref(k), C.byref(v)))
        c = self._cfg
        shape = (c.num_layers, c.num_blocks, c.block_size, self.shard_entry_elems)
        typestr = {F32: "<f4", BF16: "<i2", F16: "<f2", FP8_E4M3: "|u1"}[self._dtype]
        out = []
        for p in (k.value, v.value):
            t = torch.as_tensor(_DeviceArray(p or 0, shape, typestr), device=f"cuda:{self.device}")
            if self._dtype == BF16:
                t = t.view(torch.bfloat16)
            elif self._dtype == FP8_E4M3:
                t = t.view(torch.float8_e4m3fn)
            out.append(t)
        return tuple(out)

    @property
    def dtype_tag(self) -> int:
        return self._dtype

    @property
    def elem_bytes(self) -> int:
        return DTYPE_BYTES[self._dtype]


def _torch_tag(t) -> int:
    import torch

    return {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16,
            torch.float8_e4m3fn: FP8_E4M3}[t.dtype]


def _same_layout(k, v) -> None:
    if k.shape != v.shape or k.stride() != v.stride() or k.dtype != v.dtype:
        raise ValueError("k and v must share shape, strides and dtype")
    if k.stride(-1) != 1:
        raise ValueError("entries must be contiguous")
