"""Host block-table model with the reference's semantics.

``PagedBlockTable`` keeps the behaviour of python_ref/latent_paged_attention/
block_table.py:14-61 (bump allocation of logical -> physical blocks, token
translation and its TypeError / ValueError / IndexError rules) and the Rust
``BlockTable`` of crates/plkv-core/src/lib.rs:1313-1414.  It also produces the
int32 device tables and slot numbers the CUDA append and decode consume.
"""

from __future__ import annotations

import math

import numpy as np


def _validate_positive_int(name: str, value: int) -> None:
    if not isinstance(value, int):
        raise TypeError(f"{name} must be an int, got {type(value).__name__}")
    if value <= 0:
        raise ValueError(f"{name} must be > 0, got {value}")


class PagedBlockTable:
    """Track logical token positions in fixed-size blocks (block_table.py:14-61)."""

    def __init__(self, block_size: int, first_physical_block: int = 0) -> None:
        _validate_positive_int("block_size", block_size)
        self.block_size = block_size
        self.logical_to_physical: list[int] = []
        self.next_physical_block = first_physical_block
        self.num_tokens = 0

    def allocate_token_positions(self, num_tokens: int) -> list[tuple[int, int, int]]:
        """Allocate positions; returns (token_pos, physical_block, offset) per token."""
        _validate_positive_int("num_tokens", num_tokens)
        allocated = []
        for _ in range(num_tokens):
            pos = self.num_tokens
            if pos // self.block_size == len(self.logical_to_physical):
                self.logical_to_physical.append(self.next_physical_block)
                self.next_physical_block += 1
            self.num_tokens += 1
            allocated.append((pos, *self.translate(pos)))
        return allocated

    def translate(self, token_pos: int) -> tuple[int, int]:
        """Token position -> (physical block, offset) (block_table.py:40-53)."""
        if not isinstance(token_pos, int):
            raise TypeError(f"token_pos must be an int, got {type(token_pos).__name__}")
        if token_pos < 0:
            raise ValueError(f"token_pos must be >= 0, got {token_pos}")
        if token_pos >= self.num_tokens:
            raise IndexError(f"token_pos {token_pos} is out of range for "
                             f"{self.num_tokens} allocated tokens")
        return self.logical_to_physical[token_pos // self.block_size], token_pos % self.block_size

    def slot(self, token_pos: int) -> int:
        """Flat slot number physical * block_size + offset of an allocated token."""
        physical, offset = self.translate(token_pos)
        return physical * self.block_size + offset

    @property
    def num_blocks(self) -> int:
        return len(self.logical_to_physical)

    def to_list(self) -> list[int]:
        return list(self.logical_to_physical)

    def to_numpy(self) -> list[int]:
        """Logical -> physical mapping in logical order (block_table.py:59-61)."""
        return list(self.logical_to_physical)


def logical_blocks_for_seq_len(seq_len: int, block_size: int) -> int:
    """block_table.py:64-68."""
    _validate_positive_int("seq_len", seq_len)
    _validate_positive_int("block_size", block_size)
    return math.ceil(seq_len / block_size)


def stack_tables(tables: list[list[int]], max_blocks: int | None = None) -> np.ndarray:
    """Per-sequence tables -> [batch, max_blocks] int32, padded with -1."""
    width = max_blocks if max_blocks is not None else max((len(t) for t in tables), default=1)
    out = np.full((len(tables), max(width, 1)), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        if len(t) > width:
            raise ValueError("table longer than max_blocks")
        out[i, :len(t)] = t
    return out
