"""The C oracle against golden outputs of the reference's own CUDA kernels.

tests/golden/ref_kernels_golden.npz holds, per case of
tests/golden/ref_cases.py, a hash of every pool entry that the reference's
kernels (crates/paged-kv-cuda/kernels/kernels.cu, run on a B200 by
tests/golden/make_ref_golden.py) produced. Here the oracle replays the same
operations on the CPU and must reproduce every entry.
"""

import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))

from oracle.cpu import OracleBackend  # noqa: E402
from ref_cases import CASES, entry_hashes, ops  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden" / "ref_kernels_golden.npz"


@pytest.mark.parametrize("name", list(CASES))
def test_oracle_reproduces_the_reference_kernels(name):
    golden = np.load(GOLDEN)
    cfg, seq = ops(name)
    orc = OracleBackend(cfg)
    bs = cfg.block_size
    for op in seq:
        if op[0] == "write":
            _, layer, slots, k, v = op
            pairs = np.stack([slots // bs, slots % bs], 1).astype(np.uint64)
            orc.write_kv_batch_pairs(layer, np.ascontiguousarray(pairs), np.ascontiguousarray(k),
                                     np.ascontiguousarray(v))
        elif op[0] == "copy":
            orc.copy_blocks(op[1])
        else:
            orc.zero_block(op[1])
    got = entry_hashes(*orc.planes(), cfg)
    want = golden[name]
    assert got.shape == want.shape
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} entries differ, first (plane, layer, block, slot) = {bad[0]}"
    assert (want != 0).any()  # the case wrote something
