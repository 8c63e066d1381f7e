"""Argument checks of pkv_resolve_and_cache_noalloc that return before any
device call, so they run without a GPU: fp8 pools are refused with their
own message, and strides are checked as pkv_reshape_and_cache_dev checks
them. The pointers passed are never dereferenced: every case fails first."""

import ctypes as C

import pytest

from pagedkv import _lib

DUMMY = 4096  # non-null stand-in address; no case reaches a device access


def call(cfg, pool=_lib.BF16, src=_lib.BF16, layer=-1, tokens=10, seqs=2, tok_stride=0,
         lay_stride=0):
    return _lib.lib.pkv_resolve_and_cache_noalloc(
        C.byref(cfg), pool, 0, 1, DUMMY, DUMMY, DUMMY, 4, DUMMY, DUMMY, seqs, tokens, DUMMY,
        layer, DUMMY, DUMMY, tok_stride, lay_stride, src, None, None)


def test_fp8_pool_is_refused_with_its_reason():
    cfg = _lib.Config(16, 16, 1, 8, 2, 1)
    assert call(cfg, pool=_lib.FP8_E4M3) == 9
    code, _, _, msg = _lib.last_error()
    assert code == 9 and "fp8" in msg and "pkv_resolve_and_cache_dev" in msg
    cfg2 = _lib.Config(16, 16, 1, 8, 2, 2)
    assert call(cfg2, src=_lib.FP8_E4M3) == 9 and "fp8" in _lib.last_error()[3]


def test_unknown_dtype_tag():
    cfg = _lib.Config(16, 16, 1, 8, 2, 2)
    assert call(cfg, pool=7) == 9 and _lib.last_error()[3] == "unknown dtype tag"


@pytest.mark.parametrize("tok_stride,lay_stride,expected", [
    (8, 79, (80, 79)),    # one element short of 10 rows of 8
    (12, 100, (120, 100)),
])
def test_short_layer_stride_is_shape_mismatch(tok_stride, lay_stride, expected):
    cfg = _lib.Config(16, 16, 1, 8, 2, 2)
    assert call(cfg, tok_stride=tok_stride, lay_stride=lay_stride) == 6
    code, a, b, msg = _lib.last_error()
    assert (code, a, b) == (6, *expected) and "layer stride" in msg


def test_short_token_stride_is_shape_mismatch():
    cfg = _lib.Config(16, 16, 1, 8, 2, 2)
    assert call(cfg, tok_stride=7) == 6
    assert _lib.last_error()[:3] == (6, 8, 7)


def test_sequence_limit_matches_the_regular_entry_points():
    cfg = _lib.Config(16, 16, 1, 8, 2, 2)
    assert call(cfg, seqs=56 * 1024 + 1, tokens=0) == 9
    assert "at most 57344 sequences" in _lib.last_error()[3]
