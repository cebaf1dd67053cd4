"""Paged KV cache and physical block allocator, device-resident on B200.

Drop-in for the reference's ``engine/kv.py`` (sup-zzj/speculative-decoding-lab,
engine/kv.py:41-223): same class names, constructor arguments, methods,
properties, error types and messages, and the same pool layout

    K, V : (num_layers, capacity_blocks, block_size, num_kv_heads, head_dim)

What changes is where the metadata lives.  The free list (a LIFO stack whose
first pop returns ``capacity - 1``, engine/kv.py:52,68), the per-sequence
block tables and lengths are int32 arrays in HBM, mutated only by the
sm_100a kernels of ``libsdl_b200.so`` (reserve / append / release / commit),
so a whole decode or speculative round runs without host round trips.

The host keeps *shadows* of the counts (blocks per sequence, sequence
lengths, free blocks).  Every operation updates them with the same arithmetic
the kernels apply, so ``seq_lengths``, ``num_allocated_blocks``,
``block_utilization`` and the pre-launch ``BlockExhaustedError`` check never
synchronise.  Only ``block_tables`` (the physical ids) is read back from the
device, lazily, when a caller asks for it.

Differences from the reference, both on error paths only:
* an allocation that would exhaust the pool raises ``BlockExhaustedError``
  before anything is allocated (the reference pops blocks until it runs out
  and then raises, leaving a partially grown table);
* a sequence may hold at most ``max_blocks_per_seq`` blocks (a preallocated
  table width; default ``min(capacity, 65536 / block_size)``).
"""

from __future__ import annotations

import ctypes
from typing import Dict, List, Optional, Sequence

import torch

from . import _lib
from .utils import setup_logger

logger = setup_logger(__name__)


class BlockExhaustedError(RuntimeError):
    """Raised when the physical block pool is exhausted by an allocation."""


def _exhausted(capacity: int) -> BlockExhaustedError:
    return BlockExhaustedError(
        "paged KV block pool exhausted ({} blocks; raise max_num_blocks)".format(capacity)
    )


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


class BlockAllocator:
    """Device free list of physical block ids shared by every sequence.

    Mirrors engine/kv.py:45-76: ``alloc`` pops the most recently pushed id,
    ``free`` pushes and is idempotent for an id that is already free.
    """

    def __init__(self, capacity: int, device: torch.device, dtype: torch.dtype) -> None:
        if capacity < 1:
            raise ValueError("capacity_blocks must be >= 1")
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("BlockAllocator lives in HBM: device must be CUDA, got {}".format(device))
        self.capacity = int(capacity)
        self._device = device
        self._dtype = dtype
        self._free_stack = torch.empty(self.capacity, dtype=torch.int32, device=device)
        self._free_top = torch.empty(1, dtype=torch.int32, device=device)
        self._is_free = torch.empty(self.capacity, dtype=torch.uint8, device=device)
        self._err = torch.zeros(1, dtype=torch.int32, device=device)
        self._one = torch.empty(1, dtype=torch.int32, device=device)
        lib = _lib.load()
        _lib.check(
            lib.sdl_block_init(
                self._free_stack.data_ptr(), self._free_top.data_ptr(), self._is_free.data_ptr(),
                self.capacity, _lib.stream_handle(device),
            ),
            "sdl_block_init",
        )
        #: host shadow of the stack size (exact: updated by every operation)
        self._h_free = self.capacity

    @property
    def num_allocated(self) -> int:
        return self.capacity - self._h_free

    @property
    def num_free(self) -> int:
        return self._h_free

    def alloc(self) -> int:
        if self._h_free <= 0:
            raise _exhausted(self.capacity)
        _lib.check(
            _lib.load().sdl_block_alloc(
                self._free_stack.data_ptr(), self._free_top.data_ptr(), self._is_free.data_ptr(),
                self.capacity, 1, self._one.data_ptr(), self._err.data_ptr(),
                _lib.stream_handle(self._device),
            ),
            "sdl_block_alloc",
        )
        self._h_free -= 1
        return int(self._one.item())

    def free(self, block: int) -> None:
        block = int(block)
        if block < 0 or block >= self.capacity:
            raise IndexError("block id {} outside pool of {}".format(block, self.capacity))
        if bool(self._is_free[block].item()):
            return
        self._one.fill_(block)
        _lib.check(
            _lib.load().sdl_block_free(
                self._free_stack.data_ptr(), self._free_top.data_ptr(), self._is_free.data_ptr(),
                self.capacity, 1, self._one.data_ptr(), self._err.data_ptr(),
                _lib.stream_handle(self._device),
            ),
            "sdl_block_free",
        )
        self._h_free += 1

    def free_list(self) -> List[int]:
        """The device stack bottom-to-top (synchronises; for tests and debugging)."""
        top = int(self._free_top.item())
        return self._free_stack[:top].tolist()

    def resync(self) -> None:
        self._h_free = int(self._free_top.item())


class PagedKVCache:
    """Physical KV tensors plus the per-sequence metadata that maps to them."""

    def __init__(
        self,
        num_layers: int,
        num_kv_heads: int,
        head_dim: int,
        capacity_blocks: int,
        block_size: int,
        device: torch.device,
        dtype: torch.dtype,
        max_blocks_per_seq: Optional[int] = None,
        max_seqs: int = 64,
    ) -> None:
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("PagedKVCache lives in HBM: device must be CUDA, got {}".format(device))
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.num_layers = int(num_layers)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.block_size = int(block_size)
        self.device = device
        self.dtype = dtype
        _lib.dtype_code(dtype)
        self.allocator = BlockAllocator(capacity_blocks, device, dtype)
        self.capacity = self.allocator.capacity
        shape = (self.num_layers, self.capacity, self.block_size, self.num_kv_heads, self.head_dim)
        self._k = torch.zeros(shape, dtype=dtype, device=device)
        self._v = torch.zeros(shape, dtype=dtype, device=device)
        if max_blocks_per_seq is None:
            max_blocks_per_seq = min(self.capacity, max(1, _cdiv(65536, self.block_size)))
        self.width = int(max_blocks_per_seq)
        self._rows_cap = 0
        self._table = torch.empty(0, dtype=torch.int32, device=device)
        self._nb = torch.empty(0, dtype=torch.int32, device=device)
        self._len = torch.empty(0, dtype=torch.int32, device=device)
        self._grow_rows(max(1, int(max_seqs)))
        # host shadows
        self._h_nb: List[int] = []
        self._h_len: List[int] = []
        self._mirror: Optional[List[List[int]]] = None
        self._tmaps = None

    # ------------------------------------------------------------- plumbing
    def _grow_rows(self, rows: int) -> None:
        if rows <= self._rows_cap:
            return
        rows = max(rows, 2 * self._rows_cap)
        table = torch.full((rows, self.width), -1, dtype=torch.int32, device=self.device)
        nb = torch.zeros(rows, dtype=torch.int32, device=self.device)
        ln = torch.zeros(rows, dtype=torch.int32, device=self.device)
        if self._rows_cap:
            table[: self._rows_cap] = self._table
            nb[: self._rows_cap] = self._nb
            ln[: self._rows_cap] = self._len
        self._table, self._nb, self._len = table, nb, ln
        self._rows_cap = rows
        a = self.allocator
        self._meta = _lib.SdlKvMeta(
            self._table.data_ptr(), self._nb.data_ptr(), self._len.data_ptr(),
            a._free_stack.data_ptr(), a._free_top.data_ptr(), a._is_free.data_ptr(), a._err.data_ptr(),
            self.capacity, self.width, self._rows_cap, self.block_size,
        )

    @property
    def meta(self) -> _lib.SdlKvMeta:
        return self._meta

    @property
    def err_word(self) -> torch.Tensor:
        return self.allocator._err

    def _stream(self) -> int:
        return _lib.stream_handle(self.device)

    def tensor_maps(self):
        """128-byte TMA descriptors of the K and V pools (or None when the
        tensor-core attention path does not apply to this pool)."""
        if self._tmaps is None:
            ok = (
                self.dtype in (torch.bfloat16, torch.float16)
                and self.head_dim in (64, 128)
                and self.block_size == 16
                and self.num_layers * self.capacity * self.block_size < 2 ** 31
            )
            if not ok:
                self._tmaps = (None, None)
            else:
                lib = _lib.load()
                mk = ctypes.create_string_buffer(128)
                mv = ctypes.create_string_buffer(128)
                ntok = self.num_layers * self.capacity * self.block_size
                code = _lib.dtype_code(self.dtype)
                _lib.check(lib.sdl_make_kv_tensor_map(ctypes.addressof(mk), self._k.data_ptr(), code, ntok,
                                                      self.num_kv_heads, self.head_dim), "sdl_make_kv_tensor_map")
                _lib.check(lib.sdl_make_kv_tensor_map(ctypes.addressof(mv), self._v.data_ptr(), code, ntok,
                                                      self.num_kv_heads, self.head_dim), "sdl_make_kv_tensor_map")
                self._tmaps = (mk, mv)
        return self._tmaps

    # ------------------------------------------------------------- sequences
    def add_sequence(self, seq_id: int) -> None:
        """Register an empty sequence (no blocks, zero length)."""
        seq_id = int(seq_id)
        while len(self._h_len) <= seq_id:
            self._h_nb.append(0)
            self._h_len.append(0)
        self._grow_rows(len(self._h_len))
        self._mirror = None

    @property
    def num_sequences(self) -> int:
        return len(self._h_len)

    def seq_len(self, seq_id: int) -> int:
        return self._h_len[seq_id]

    def num_blocks_of(self, seq_id: int) -> int:
        return self._h_nb[seq_id]

    def resync(self) -> None:
        """Reload the host shadows (block counts, lengths, free count) from the
        device (synchronises).  For callers that ran device-side commits
        without mirroring them on the host."""
        n = len(self._h_len)
        self._h_nb = self._nb[:n].tolist()
        self._h_len = self._len[:n].tolist()
        self.allocator.resync()
        self._mirror = None

    # ------------------------------------------------------------ allocation
    def _plan_reserve(self, seq_ids: Sequence[int], starts: Sequence[int], counts: Sequence[int]) -> None:
        """Check capacity on the host and apply the reserve to the shadows."""
        bs = self.block_size
        need_total = 0
        plan = []
        for sid, st, c in zip(seq_ids, starts, counts):
            if sid < 0 or sid >= len(self._h_len):
                raise IndexError("sequence {} is not registered (add_sequence first)".format(sid))
            if st < 0:
                raise ValueError("negative token position {}".format(st))
            if c <= 0:
                continue
            nb_need = _cdiv(st + c, bs)
            new = nb_need - self._h_nb[sid]
            if new > 0:
                need_total += new
            plan.append((sid, nb_need, st + c))
        if need_total > self.allocator._h_free:
            raise _exhausted(self.capacity)
        for sid, nb_need, _ in plan:
            if nb_need > self.width:
                raise RuntimeError(
                    "sequence {} needs {} blocks > max_blocks_per_seq={}".format(sid, nb_need, self.width)
                )
        for sid, nb_need, end in plan:
            if nb_need > self._h_nb[sid]:
                self._h_nb[sid] = nb_need
            if self._h_len[sid] < end:
                self._h_len[sid] = end
        self.allocator._h_free -= need_total
        self._mirror = None

    def reserve(self, seq_ids: Sequence[int], starts: Sequence[int], counts: Sequence[int]) -> torch.Tensor:
        """Back positions ``[starts[i], starts[i]+counts[i])`` of each sequence.

        Allocation order equals the reference's per-token write loop at layer 0
        (sequence-major, token-minor).  Returns the int32 slot of every
        position (``phys * block_size + offset``), sequence-major.
        """
        seq_ids = [int(s) for s in seq_ids]
        starts = [int(s) for s in starts]
        counts = [int(c) for c in counts]
        n = len(seq_ids)
        if len(starts) != n or len(counts) != n:
            raise ValueError("seq_ids, starts and counts must have the same length")
        if len(set(seq_ids)) != n:
            raise ValueError("reserve: duplicate sequence ids in one call")
        self._plan_reserve(seq_ids, starts, counts)
        total = sum(c for c in counts if c > 0)
        slots = torch.empty(max(total, 1), dtype=torch.int32, device=self.device)
        if n == 0:
            return slots[:0]
        packed = _lib.i32(seq_ids + starts + counts, self.device)
        _lib.check(
            _lib.load().sdl_kv_reserve(
                ctypes.byref(self._meta), n, packed.data_ptr(), packed.data_ptr() + 4 * n,
                packed.data_ptr() + 8 * n, slots.data_ptr(), self._stream(),
            ),
            "sdl_kv_reserve",
        )
        return slots[:total]

    def append(self, layer: int, slots: torch.Tensor, kvecs: torch.Tensor, vvecs: torch.Tensor) -> None:
        """Write K/V rows ``(T, num_kv_heads, head_dim)`` of ``layer`` at ``slots``."""
        if not 0 <= layer < self.num_layers:
            raise IndexError("layer {} out of range".format(layer))
        T = int(slots.numel())
        if T == 0:
            return
        row = self.num_kv_heads * self.head_dim
        k = kvecs.reshape(T, row)
        v = vvecs.reshape(T, row)
        if k.dtype != self.dtype:
            k = k.to(self.dtype)
        if v.dtype != self.dtype:
            v = v.to(self.dtype)
        if k.stride(-1) != 1:
            k = k.contiguous()
        if v.stride(-1) != 1:
            v = v.contiguous()
        if k.stride(0) != v.stride(0):
            k, v = k.contiguous(), v.contiguous()
        _lib.require_cuda(k, "kvecs")
        _lib.check(
            _lib.load().sdl_kv_append(
                self._k.data_ptr(), self._v.data_ptr(), _lib.dtype_code(self.dtype), self.num_layers,
                self.capacity, self.block_size, row, int(layer), T, slots.data_ptr(), k.data_ptr(),
                v.data_ptr(), k.stride(0), self.err_word.data_ptr(), self._stream(),
            ),
            "sdl_kv_append",
        )

    # ------------------------------------------------------------ write path
    def write(
        self,
        layer: int,
        seq_id: int,
        token_pos: int,
        kvec: torch.Tensor,
        vvec: torch.Tensor,
    ) -> None:
        """Store the K/V vectors of one logical token position (engine/kv.py:125-147)."""
        slots = self.reserve([seq_id], [token_pos], [1])
        self.append(layer, slots, kvec.reshape(1, self.num_kv_heads, self.head_dim),
                    vvec.reshape(1, self.num_kv_heads, self.head_dim))

    # ------------------------------------------------------------ rollback
    def _shadow_release(self, sid: int, new_len: int, flags: int) -> None:
        bs = self.block_size
        nb = self._h_nb[sid]
        keep_b = nb
        do_trunc = bool(flags & _lib.REL_TRUNCATE) and (
            not (flags & _lib.REL_ONLY_IF_LONGER) or self._h_len[sid] > new_len
        )
        if do_trunc:
            kb = 0 if new_len <= 0 else _cdiv(new_len, bs)
            if kb < nb:
                keep_b = kb
        freed = nb - keep_b
        if do_trunc:
            self._h_nb[sid] = keep_b
            self._h_len[sid] = max(0, new_len)
        if flags & _lib.REL_CLEAR:
            freed += keep_b
            self._h_nb[sid] = 0
            self._h_len[sid] = 0
        self.allocator._h_free += freed

    def release(self, seq_ids: Sequence[int], new_lens: Sequence[int], flags: Sequence[int]) -> None:
        """Batched rewind/clear, processed in list order (kernel kv_release)."""
        seq_ids = [int(s) for s in seq_ids]
        new_lens = [int(x) for x in new_lens]
        flags = [int(f) for f in flags]
        n = len(seq_ids)
        if n == 0:
            return
        for sid in seq_ids:
            if sid < 0 or sid >= len(self._h_len):
                raise IndexError("sequence {} is not registered".format(sid))
        for sid, nl, f in zip(seq_ids, new_lens, flags):
            self._shadow_release(sid, nl, f)
        self._mirror = None
        packed = _lib.i32(seq_ids + new_lens + flags, self.device)
        _lib.check(
            _lib.load().sdl_kv_release(
                ctypes.byref(self._meta), n, packed.data_ptr(), packed.data_ptr() + 4 * n,
                packed.data_ptr() + 8 * n, self._stream(),
            ),
            "sdl_kv_release",
        )

    def truncate(self, seq_id: int, new_len: int) -> None:
        """Rewind sequence ``seq_id`` to ``new_len`` logical positions (engine/kv.py:150-162)."""
        self.release([seq_id], [new_len], [_lib.REL_TRUNCATE])

    def clear(self, seq_id: int) -> None:
        """Drop a finished sequence entirely, freeing all its blocks (engine/kv.py:164-171)."""
        if seq_id >= len(self._h_len):
            raise IndexError("list assignment index out of range")
        self.release([seq_id], [0], [_lib.REL_CLEAR])

    def reset(self) -> None:
        """Return the cache to a virgin state without reallocating the tensors."""
        n = len(self._h_len)
        if n:
            self.release(list(range(n)), [0] * n, [_lib.REL_CLEAR] * n)
        self._h_nb = []
        self._h_len = []
        self._mirror = None

    # ------------------------------------------------------------- mirrors
    @property
    def block_tables(self) -> List[List[int]]:
        """Per-sequence physical block lists, read back from HBM (synchronises)."""
        if self._mirror is None:
            n = len(self._h_len)
            if n == 0:
                self._mirror = []
            else:
                w = max(1, max(self._h_nb))
                rows = self._table[:n, :w].cpu().tolist()
                self._mirror = [rows[i][: self._h_nb[i]] for i in range(n)]
        return self._mirror

    @property
    def seq_lengths(self) -> List[int]:
        return self._h_len

    def device_state(self) -> Dict[str, object]:
        """Raw device metadata (synchronises) -- for parity tests."""
        n = len(self._h_len)
        return {
            "num_blocks": self._nb[:n].tolist(),
            "seq_lens": self._len[:n].tolist(),
            "free_list": self.allocator.free_list(),
        }

    def check_errors(self) -> None:
        """Raise on device-detected errors (synchronises)."""
        word = int(self.err_word.item())
        if word:
            self.err_word.zero_()
            if word & _lib.DEVERR_EXHAUSTED:
                raise _exhausted(self.capacity)
            raise RuntimeError("paged KV device error word 0x{:x}".format(word))

    # --------------------------------------------------------------- metrics
    @property
    def num_allocated_blocks(self) -> int:
        return self.allocator.num_allocated

    @property
    def logical_tokens(self) -> int:
        return sum(self._h_len)

    @property
    def block_utilization(self) -> float:
        """Fraction of allocated block *slots* actually holding a token."""
        if self.num_allocated_blocks == 0:
            return 0.0
        return float(self.logical_tokens) / float(self.num_allocated_blocks * self.block_size)

    @property
    def kv_memory_bytes(self) -> int:
        return 2 * self._k.numel() * self._k.element_size()

    # ------------------------------------------------------ read (for attention)
    def key_map(self, layer: int, phys: List[int]) -> torch.Tensor:
        """Gather the physical blocks of ``layer`` for a list of physical ids."""
        return self._k[layer][phys]

    def value_map(self, layer: int, phys: List[int]) -> torch.Tensor:
        return self._v[layer][phys]

    def kv_stats(self) -> Optional[Dict[str, float]]:
        if self.num_sequences == 0:
            return None
        return {
            "num_allocated_blocks": self.num_allocated_blocks,
            "logical_tokens": self.logical_tokens,
            "block_utilization": round(self.block_utilization, 4),
            "kv_memory_bytes": self.kv_memory_bytes,
            "max_seq_len": max(self.seq_lengths),
        }
