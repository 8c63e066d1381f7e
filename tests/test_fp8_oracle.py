"""The oracle's E4M3 format (oracle/pkv_oracle.c) pinned on the CPU.

fp8 pools have no counterpart in the reference (CpuBackend is f32 only,
crates/paged-kv-core/src/cpu.rs:22-25), so the oracle's encoder is pinned
against an independent implementation -- torch's float8_e4m3fn conversion,
round to nearest even -- on every value both define the same way (finite,
below 448 in magnitude), and against the saturation and subnormal cases
written out by hand from the OCP OFP8 E4M3 definition.
"""

import numpy as np
import pytest
import torch

from oracle import host_ref as H
from oracle.cpu import OracleBackend, e4m3_from_f32, e4m3_to_f32
from pagedkv import CacheConfig
from pagedkv.workloads import Stream


def test_every_bf16_value_encodes_as_torch_does():
    x = (np.arange(65536, dtype=np.uint32) << 16).view(np.float32)
    fin = np.isfinite(x) & (np.abs(x) < 448)
    want = torch.from_numpy(x[fin].copy()).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(e4m3_from_f32(x[fin]), want)


def test_random_f32_values_encode_as_torch_does():
    st = Stream(31)
    x = (st.normal(400_000) * np.exp(st.uniform(400_000, -14.0, 6.0))).astype(np.float32)
    x = x[np.abs(x) < 448]
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(e4m3_from_f32(x), want)


def test_every_code_widens_as_torch_does():
    codes = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    got = e4m3_to_f32(codes)
    nan = np.isnan(want)
    assert (np.isnan(got) == nan).all() and nan.sum() == 2  # S.1111.111
    np.testing.assert_array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))


@pytest.mark.parametrize("x,code", [
    (448.0, 0x7E), (-448.0, 0xFE), (449.0, 0x7E), (463.9, 0x7E), (464.0, 0x7E),
    (1e30, 0x7E), (np.inf, 0x7E), (-np.inf, 0xFE),      # satfinite
    (0.0, 0x00), (-0.0, 0x80),
    (2.0 ** -9, 0x01), (2.0 ** -10, 0x00), (-2.0 ** -10, 0x80),  # tie to even: 0
    (3 * 2.0 ** -10, 0x02),                              # 1.5 * 2^-9: tie to even 2
    (2.0 ** -6, 0x08), (7 * 2.0 ** -9, 0x07),             # smallest normal, largest subnormal
    (15 * 2.0 ** -10, 0x08),                             # 7.5 * 2^-9 rounds up into the normals
    (1.0, 0x38), (1.0625, 0x38), (1.1875, 0x3A), (240.0, 0x77), (256.0, 0x78),
])
def test_known_codes(x, code):
    assert int(e4m3_from_f32(np.array([x], np.float32))[0]) == code


def test_nan_stays_nan():
    q = e4m3_from_f32(np.array([np.nan, -np.nan], np.float32))
    assert ((q & 0x7F) == 0x7F).all()


def test_fp8_oracle_pool_quantises_per_layer_and_head():
    cfg = CacheConfig(8, 4, 3, 16, 2, 1)
    orc = OracleBackend(cfg)
    ks = np.array([[0.5, 2.0, 0.25], [1.0, 3.0, 0.1]], np.float32)
    vs = ks[::-1].copy()
    orc.set_fp8(ks, vs)
    e = cfg.entry_elems()
    st = Stream(4)
    k = (st.normal(e) * 4).astype(np.float32)
    v = (st.normal(e) * 4).astype(np.float32)
    orc.write_kv(1, (5, 3), k, v)
    pk, pv = orc.planes()
    head = np.arange(e) // cfg.head_dim
    want_k = e4m3_to_f32(e4m3_from_f32(k * (np.float32(1) / ks[1, head])))
    want_v = e4m3_to_f32(e4m3_from_f32(v * (np.float32(1) / vs[1, head])))
    np.testing.assert_array_equal(pk[1, 5, 3].view(np.uint32), want_k.view(np.uint32))
    np.testing.assert_array_equal(pv[1, 5, 3].view(np.uint32), want_v.view(np.uint32))
    rk, rv = orc.read_entry(1, (5, 3))
    np.testing.assert_array_equal(rk, want_k * ks[1, head])
    np.testing.assert_array_equal(rv, want_v * vs[1, head])
    with pytest.raises(H.RefError):
        orc.write_kv(2, (0, 0), k, v)  # layer check still first (cpu.rs:55-70)
