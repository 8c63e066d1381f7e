"""TEST INFRASTRUCTURE ONLY -- ctypes wrapper of oracle/_ref/libref_kernels.so,
the reference's own CUDA kernels (crates/paged-kv-cuda/kernels/kernels.cu)
built for sm_100a by oracle/ref.mk from the reference checkout. Launch shapes
are those of the reference's CudaBackend. Used by tests to pin the C oracle
against the reference's device code and to time the reference kernels.
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB = Path(__file__).resolve().parent / "_ref" / "libref_kernels.so"


def available() -> bool:
    return LIB.exists()


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(os.fspath(LIB))
        P, I = C.c_void_p, C.c_int
        _lib.ref_reshape_and_cache.argtypes = [P, P, P, P, P, I, I, I, I, I, P]
        _lib.ref_copy_blocks.argtypes = [P, P, P, I, I, I, I, P]
        _lib.ref_zero_block.argtypes = [P, P, I, I, I, I, P]
        for f in (_lib.ref_reshape_and_cache, _lib.ref_copy_blocks, _lib.ref_zero_block):
            f.restype = I
    return _lib


def reshape_and_cache(k, v, kc, vc, slots, layer, num_blocks, block_size, entry, stream=0):
    """One launch for one layer (CudaBackend::write_kv_batch's shape)."""
    rc = lib().ref_reshape_and_cache(k.data_ptr(), v.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                     slots.data_ptr(), slots.numel(), layer, num_blocks,
                                     block_size, entry, stream)
    assert rc == 0, rc


def copy_blocks(kc, vc, pairs, num_layers, num_blocks, block_elems, stream=0):
    rc = lib().ref_copy_blocks(kc.data_ptr(), vc.data_ptr(), pairs.data_ptr(), pairs.shape[0],
                               num_layers, num_blocks, block_elems, stream)
    assert rc == 0, rc


def zero_block(kc, vc, block, num_layers, num_blocks, block_elems, stream=0):
    rc = lib().ref_zero_block(kc.data_ptr(), vc.data_ptr(), block, num_layers, num_blocks,
                              block_elems, stream)
    assert rc == 0, rc
