"""Writes tests/golden/ref_kernels_golden.npz: per-entry hashes of the pools
that the reference's own CUDA kernels (crates/paged-kv-cuda/kernels/kernels.cu,
built by oracle/ref.mk into oracle/_ref, launched with CudaBackend's shapes)
leave behind on the cases of ref_cases.py. Needs a GPU and the built
oracle/_ref library; run from the repository root:

    python tests/golden/make_ref_golden.py [output.npz]
"""

from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "paged-kv-cache_b200"))
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(__file__).resolve().parent))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from oracle import ref_kernels as ref  # noqa: E402
from ref_cases import CASES, entry_hashes, ops  # noqa: E402


def run_case(name):
    cfg, seq = ops(name)
    dev = torch.device("cuda:0")
    e, bs, nb, L = cfg.num_kv_heads * cfg.head_dim, cfg.block_size, cfg.num_blocks, cfg.num_layers
    kc = torch.zeros(L * nb * bs * e, dtype=torch.float32, device=dev)
    vc = torch.zeros_like(kc)
    for op in seq:
        if op[0] == "write":
            _, layer, slots, k, v = op
            ref.reshape_and_cache(torch.from_numpy(np.ascontiguousarray(k)).to(dev),
                                  torch.from_numpy(np.ascontiguousarray(v)).to(dev), kc, vc,
                                  torch.from_numpy(slots).to(dev), layer, nb, bs, e)
        elif op[0] == "copy":
            ref.copy_blocks(kc, vc, torch.from_numpy(op[1]).to(dev), L, nb, bs * e)
        else:
            ref.zero_block(kc, vc, op[1], L, nb, bs * e)
    torch.cuda.synchronize()
    return entry_hashes(kc.cpu().numpy(), vc.cpu().numpy(), cfg)


def main():
    out = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent / "ref_kernels_golden.npz"
    if not ref.available():
        raise SystemExit("oracle/_ref/libref_kernels.so is missing: build it with make -f oracle/ref.mk")
    arrays = {name: run_case(name) for name in CASES}
    np.savez_compressed(out, **arrays)
    print("wrote", out, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
