"""CacheConfig, PhysicalSlot and BlockId of paged-kv-core
(crates/paged-kv-core/src/config.rs:8-98, types.rs:10-43)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class CacheConfig:
    num_blocks: int
    block_size: int
    num_kv_heads: int
    head_dim: int
    num_layers: int
    dtype_bytes: int

    @staticmethod
    def llama_3_2_1b(num_blocks: int) -> "CacheConfig":  # config.rs:25-34
        return CacheConfig(num_blocks, 16, 8, 64, 16, 2)

    @staticmethod
    def tiny(num_blocks: int) -> "CacheConfig":  # config.rs:37-46
        return CacheConfig(num_blocks, 4, 2, 4, 2, 4)

    def entry_elems(self) -> int:  # config.rs:50-52
        return self.num_kv_heads * self.head_dim

    def block_elems(self) -> int:  # config.rs:56-58
        return self.block_size * self.entry_elems()

    def layer_elems(self) -> int:  # config.rs:62-64
        return self.num_blocks * self.block_elems()

    def total_elems(self) -> int:  # config.rs:68-70
        return 2 * self.num_layers * self.layer_elems()

    def total_bytes(self) -> int:  # config.rs:74-76
        return self.total_elems() * self.dtype_bytes

    def bytes_per_token(self) -> int:  # config.rs:83-85
        return 2 * self.num_layers * self.entry_elems() * self.dtype_bytes

    def blocks_for_tokens(self, num_tokens: int) -> int:  # config.rs:89-91
        return -(-num_tokens // self.block_size)

    def split_position(self, position: int) -> tuple[int, int]:  # config.rs:95-97
        return position // self.block_size, position % self.block_size


@dataclass(frozen=True)
class PhysicalSlot:  # types.rs:40-43
    block: int
    slot: int
