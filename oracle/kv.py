"""Oracle paged KV cache: restates engine/kv.py:45-205 with numpy pools.

Test infrastructure only (see oracle/__init__.py).
"""

from __future__ import annotations

from typing import List

import numpy as np


class BlockExhaustedError(RuntimeError):
    pass


class BlockAllocator:
    """LIFO free list: list(range(cap)), pop() from the end (engine/kv.py:45-76)."""

    def __init__(self, capacity: int) -> None:
        if capacity < 1:
            raise ValueError("capacity_blocks must be >= 1")
        self.capacity = capacity
        self._free: List[int] = list(range(capacity))
        self._free_set = set(self._free)
        self._allocated = 0

    @property
    def num_allocated(self) -> int:
        return self._allocated

    def alloc(self) -> int:
        if not self._free:
            raise BlockExhaustedError(
                "paged KV block pool exhausted ({} blocks; raise max_num_blocks)".format(self.capacity)
            )
        block = self._free.pop()
        self._free_set.discard(block)
        self._allocated += 1
        return block

    def free(self, block: int) -> None:
        if block in self._free_set:  # idempotent (engine/kv.py:72-76)
            return
        self._free.append(block)
        self._free_set.add(block)
        self._allocated -= 1

    def free_list(self) -> List[int]:
        return list(self._free)


class PagedKVCache:
    """Pools (L, cap, bs, Hkv, d) float32 plus list-valued metadata (engine/kv.py:79-205)."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, capacity_blocks: int,
                 block_size: int, store: bool = True) -> None:
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.allocator = BlockAllocator(capacity_blocks)
        shape = (num_layers, capacity_blocks, block_size, num_kv_heads, head_dim)
        self.k = np.zeros(shape, dtype=np.float32) if store else None
        self.v = np.zeros(shape, dtype=np.float32) if store else None
        self.block_tables: List[List[int]] = []
        self.seq_lengths: List[int] = []

    def add_sequence(self, seq_id: int) -> None:
        while len(self.block_tables) <= seq_id:
            self.block_tables.append([])
            self.seq_lengths.append(0)

    @property
    def num_sequences(self) -> int:
        return len(self.seq_lengths)

    def _ensure_blocks_up_to(self, seq_id: int, max_block_index: int) -> None:
        table = self.block_tables[seq_id]
        while len(table) <= max_block_index:
            table.append(self.allocator.alloc())

    def slot(self, seq_id: int, token_pos: int) -> int:
        """Allocate-on-write and return phys*bs + offset (engine/kv.py:119-147)."""
        bi, off = divmod(token_pos, self.block_size)
        self._ensure_blocks_up_to(seq_id, bi)
        if self.seq_lengths[seq_id] <= token_pos:
            self.seq_lengths[seq_id] = token_pos + 1
        return self.block_tables[seq_id][bi] * self.block_size + off

    def write(self, layer: int, seq_id: int, token_pos: int, kvec: np.ndarray, vvec: np.ndarray) -> None:
        s = self.slot(seq_id, token_pos)
        phys, off = divmod(s, self.block_size)
        if self.k is not None:
            self.k[layer, phys, off] = kvec
            self.v[layer, phys, off] = vvec

    def reserve(self, seq_ids, starts, counts) -> List[int]:
        """The layer-0 write loop's allocations, sequence-major / token-minor."""
        out: List[int] = []
        for sid, st, c in zip(seq_ids, starts, counts):
            for j in range(int(c)):
                out.append(self.slot(int(sid), int(st) + j))
        return out

    def append(self, layer: int, slots, kvecs: np.ndarray, vvecs: np.ndarray) -> None:
        for t, s in enumerate(slots):
            if s < 0:
                continue
            phys, off = divmod(int(s), self.block_size)
            self.k[layer, phys, off] = kvecs[t]
            self.v[layer, phys, off] = vvecs[t]

    def truncate(self, seq_id: int, new_len: int) -> None:
        blocks_needed = 0 if new_len <= 0 else (new_len + self.block_size - 1) // self.block_size
        table = self.block_tables[seq_id]
        while len(table) > blocks_needed:
            self.allocator.free(table.pop())
        self.seq_lengths[seq_id] = max(0, new_len)

    def clear(self, seq_id: int) -> None:
        table = self.block_tables[seq_id] if seq_id < len(self.block_tables) else []
        for phys in table:
            self.allocator.free(phys)
        self.block_tables[seq_id] = []
        self.seq_lengths[seq_id] = 0

    def reset(self) -> None:
        for table in self.block_tables:
            for phys in table:
                self.allocator.free(phys)
        self.block_tables[:] = []
        self.seq_lengths[:] = []

    @property
    def num_allocated_blocks(self) -> int:
        return self.allocator.num_allocated

    @property
    def logical_tokens(self) -> int:
        return sum(self.seq_lengths)

    @property
    def block_utilization(self) -> float:
        if self.num_allocated_blocks == 0:
            return 0.0
        return float(self.logical_tokens) / float(self.num_allocated_blocks * self.block_size)

    def gather(self, layer: int, seq_id: int, length: int):
        """(K, V) of the first ``length`` positions, each (length, Hkv, d)."""
        bs = self.block_size
        nb = (length + bs - 1) // bs
        phys = self.block_tables[seq_id][:nb]
        k = self.k[layer][phys].reshape(-1, self.num_kv_heads, self.head_dim)[:length]
        v = self.v[layer][phys].reshape(-1, self.num_kv_heads, self.head_dim)[:length]
        return k, v
