"""KV-head sharding of the pool across GPUs, and its verification.

Shard r of G owns the contiguous entry slice [r*E/G, (r+1)*E/G) of every
(layer, block, slot); each GPU writes only its slice, with the same slots
and block tables on every rank, so nothing crosses GPUs on the data path.
Verification exchanges only 64-bit digests: every rank digests its shard and
the rows it was given (element hashes over global indices), the ranks
all-gather the four numbers, and the shard digests must add up (mod 2^64) to
the digest of what was written. For small pools, gather_shards reassembles
the whole pool on rank 0 from the shards.
"""

from __future__ import annotations

_MASK = (1 << 64) - 1


def entry_slice(entry_elems: int, rank: int, world: int) -> tuple[int, int]:
    """(offset, width) of rank's slice of an entry."""
    if world < 1 or not 0 <= rank < world or entry_elems % world:
        raise ValueError(f"entry of {entry_elems} elements does not split into {world} shards")
    w = entry_elems // world
    return rank * w, w


def _signed(x: int) -> int:
    x &= _MASK
    return x - (1 << 64) if x >= 1 << 63 else x


def verify_over_group(pool: tuple[int, int], expected: tuple[int, int], device=None) -> dict:
    """All-gather (pool K, pool V, expected K, expected V) digests over the
    default process group (NCCL on GPUs, gloo on CPU) and check every shard
    and the sums."""
    import torch
    import torch.distributed as dist

    mine = torch.tensor([_signed(x) for x in (*pool, *expected)], dtype=torch.int64, device=device)
    if dist.is_available() and dist.is_initialized():
        world = dist.get_world_size()
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        how = f"all_gather over {dist.get_backend()} ({world} ranks)"
    else:
        gathered, how = [mine], "single rank"
    rows = [[int(v) & _MASK for v in g.tolist()] for g in gathered]
    per_rank = [r[0] == r[2] and r[1] == r[3] for r in rows]
    tot = [sum(r[i] for r in rows) & _MASK for i in range(4)]
    return {
        "ok": all(per_rank) and tot[0] == tot[2] and tot[1] == tot[3],
        "shards_ok": per_rank,
        "pool_digest_k": f"{tot[0]:016x}",
        "pool_digest_v": f"{tot[1]:016x}",
        "collective": how,
    }


def gather_shards(k_plane, v_plane, device=None):
    """The full pool reassembled on rank 0 from every rank's head shard.

    k_plane, v_plane: this rank's shard planes [L][NB][bs][E/G] (torch
    tensors; on the GPU for NCCL, on the CPU for gloo). Every rank sends its
    shard; rank 0 concatenates the slices along the entry axis in rank order
    and returns (K, V) [L][NB][bs][E]; other ranks return None. For pools
    that fit one rank's memory G times over: a check for tests and small
    configurations, beside the digest verification above."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return k_plane, v_plane
    world = dist.get_world_size()
    out = []
    for p in (k_plane, v_plane):
        src = p.contiguous()
        if device is not None:
            src = src.to(device)
        parts = [torch.empty_like(src) for _ in range(world)]
        dist.all_gather(parts, src)  # gather is not available on every backend
        out.append(torch.cat(parts, dim=-1) if dist.get_rank() == 0 else None)
    return tuple(out) if dist.get_rank() == 0 else None
