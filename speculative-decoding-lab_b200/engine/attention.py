"""Paged attention entry points backed by the sm_100a kernels.

Drop-in for the reference's ``engine/attention.py`` (engine/attention.py:32-215):
the same function names, arguments, shapes and semantics.  Instead of
gathering each sequence's pages into a dense tensor and calling SDPA per
sequence, every call is one launch of ``sdl_paged_attention`` over the whole
batch, reading K/V pages in place through the device block table:

* decode  -- row ``b`` attends its first ``seq_token_lengths[b]`` positions,
  unmasked (engine/attention.py:96-118);
* extend  -- chunk row ``j`` of sequence ``b`` attends positions
  ``0 .. start_positions[b] + j`` (engine/attention.py:170-215);
* prefill -- causal attention within a dense chunk, padded rows zeroed
  (engine/attention.py:121-167).

Softmax scale is ``1/sqrt(head_dim)`` (SDPA's default) and GQA maps q head
``h`` to kv head ``h // (Hq / Hkv)`` (engine/attention.py:32-38).
"""

from __future__ import annotations

import ctypes
import math
import threading
import weakref
from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from .kv import PagedKVCache


class AttnBatch:
    """Device-side description of one attention call's rows.

    ``rows`` are block-table rows (sequence ids), ``starts[b]`` the absolute
    position of chunk row 0 of entry ``b``; ``max_limit`` is a host upper
    bound of ``starts[b] + chunk`` used to size the launch grid.
    """

    __slots__ = ("rows", "starts", "max_limit", "valid_rows", "key_count")

    def __init__(self, rows: torch.Tensor, starts: torch.Tensor, max_limit: int,
                 valid_rows: Optional[torch.Tensor] = None, key_count: int = 0) -> None:
        self.rows = rows
        self.starts = starts
        self.max_limit = int(max_limit)
        self.valid_rows = valid_rows
        # host count of attended keys (sum of starts[b] + chunk), 0 = unknown:
        # sizes the split-K grid only, never changes the result
        self.key_count = int(key_count)

    @classmethod
    def from_lists(cls, device: torch.device, seq_ids: Sequence[int], starts: Sequence[int], chunk: int) -> "AttnBatch":
        seq_ids = [int(s) for s in seq_ids]
        starts = [int(s) for s in starts]
        n = len(seq_ids)
        packed = _lib.i32(seq_ids + starts, device)
        max_limit = (max(starts) + chunk) if n else chunk
        return cls(packed[:n], packed[n:], max_limit, key_count=sum(starts) + n * chunk)


def _args_common(q: torch.Tensor, out: torch.Tensor, Hkv: int, err: Optional[torch.Tensor]) -> _lib.SdlAttnArgs:
    a = _lib.SdlAttnArgs()
    a.q = q.data_ptr()
    a.q_sb, a.q_sj, a.q_sh = q.stride(0), q.stride(1), q.stride(2)
    a.out = out.data_ptr()
    a.o_sb, a.o_sj, a.o_sh = out.stride(0), out.stride(1), out.stride(2)
    a.out_dtype = _lib.dtype_code(out.dtype)
    a.dtype = _lib.dtype_code(q.dtype)
    a.B, a.chunk, a.Hq, a.head_dim = q.shape[0], q.shape[1], q.shape[2], q.shape[3]
    a.Hkv = Hkv
    a.scale = 1.0 / math.sqrt(q.shape[3])
    a.err = err.data_ptr() if err is not None else None
    return a


def _launch(a: _lib.SdlAttnArgs, device: torch.device, fn: str = "sdl_paged_attention") -> None:
    lib = _lib.load()
    need = lib.sdl_attention_workspace_bytes(a)
    if need:
        ws = _lib.Workspace.get(device, int(need))
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel() * 4
    _lib.check(getattr(lib, fn)(a, _lib.stream_handle(device)), fn)


def _paged_args(q, kv, layer, batch, out, force_generic=False, pages_per_split=0,
                kv_heads_per_cta=0, use_umma=0, cluster_merge=False, mma_layout=0) -> _lib.SdlAttnArgs:
    a = _args_common(q, out, kv.num_kv_heads, kv.err_word)
    a.k_pool, a.v_pool = kv._k.data_ptr(), kv._v.data_ptr()
    mk, mv = kv.tensor_maps()
    if mk is not None:
        a.tmap_k, a.tmap_v = ctypes.addressof(mk), ctypes.addressof(mv)
    a.block_table, a.width, a.capacity = kv._table.data_ptr(), kv.width, kv.capacity
    a.num_layers, a.layer, a.block_size = kv.num_layers, int(layer), kv.block_size
    a.rows = batch.rows.data_ptr()
    a.starts = batch.starts.data_ptr()
    a.valid_rows = batch.valid_rows.data_ptr() if batch.valid_rows is not None else None
    a.max_limit = batch.max_limit
    a.key_count = batch.key_count
    a.pages_per_split = int(pages_per_split)
    a.force_generic = 1 if force_generic else 0
    a.kv_heads_per_cta = int(kv_heads_per_cta)
    a.use_umma = int(use_umma)
    a.cluster_merge = 1 if cluster_merge else 0
    a.mma_layout = int(mma_layout)
    return a


def attention_launches(q: torch.Tensor, kv: PagedKVCache, batch: AttnBatch, use_umma: int = 0,
                       k_new: Optional[torch.Tensor] = None, v_new: Optional[torch.Tensor] = None,
                       mma_layout: int = 0, overlap_layers: bool = False) -> int:
    """Kernel launches one ``paged_attention`` call with these arguments
    makes: the attention launch, the split-K merge when the plan splits a
    row's pages across CTAs, and a positional append when ``k_new`` is given
    to a plan that does not write inside the attention kernel."""
    q4 = q if q.dim() == 4 else q.reshape(q.shape[0], 1, q.shape[-2], q.shape[-1])
    a = _paged_args(q4, kv, 0, batch, q4, use_umma=use_umma, mma_layout=mma_layout)
    keep = _set_new_rows(a, q4, kv, k_new, v_new)  # noqa: F841 (keeps copies alive)
    n = _lib.load().sdl_attention_launches(a)
    if n < 0:
        raise RuntimeError("sdl_attention_launches: " + _lib.last_error())
    return n


KERNEL_NAMES = ("generic", "mma", "tcgen05", "mma_rows", "mma_direct")


def attention_kernel(q: torch.Tensor, kv: PagedKVCache, batch: AttnBatch, use_umma: int = 0,
                     mma_layout: int = 0, overlap_layers: bool = False) -> str:
    """Which kernel ``paged_attention`` runs for these arguments: "generic"
    (CUDA cores), "mma" (mma.sync split-K, keys on the MMA M dimension),
    "mma_rows" (mma.sync split-K, query rows on M), "mma_direct" (keys on M,
    K/V loaded straight into registers; decode) or "tcgen05"
    (persistent)."""
    q4 = q if q.dim() == 4 else q.reshape(q.shape[0], 1, q.shape[-2], q.shape[-1])
    a = _paged_args(q4, kv, 0, batch, q4, use_umma=use_umma, mma_layout=mma_layout)
    n = _lib.load().sdl_attention_kernel(a)
    if n < 0:
        raise RuntimeError("sdl_attention_kernel: " + _lib.last_error())
    return KERNEL_NAMES[n]


def _set_new_rows(a: _lib.SdlAttnArgs, q4: torch.Tensor, kv: PagedKVCache, k_new: Optional[torch.Tensor],
                  v_new: Optional[torch.Tensor]):
    """Point ``a`` at the K/V rows to store before attending (fused append)."""
    if k_new is None:
        return None
    rows = q4.shape[0] * q4.shape[1]
    kn = k_new.reshape(rows, -1)
    vn = v_new.reshape(rows, -1)
    if kn.dtype != kv.dtype or vn.dtype != kv.dtype or kn.shape[1] != kv.num_kv_heads * kv.head_dim \
            or vn.shape != kn.shape:
        raise ValueError("k_new/v_new must be ({}, {}) rows of {}".format(rows, kv.num_kv_heads * kv.head_dim,
                                                                       kv.dtype))
    _lib.require_cuda(kn, "k_new")
    _lib.require_cuda(vn, "v_new")
    if kn.stride(1) != 1 or vn.stride(1) != 1 or kn.stride(0) != vn.stride(0):
        kn, vn = kn.contiguous(), vn.contiguous()
    a.k_new, a.v_new, a.new_row_stride = kn.data_ptr(), vn.data_ptr(), kn.stride(0)
    return kn, vn


class _ArgsEntry:
    """A filled argument struct for one (cache, batch, shapes, flags,
    thread) combination; calls that hit it only update the pointers that
    change from call to call (q, out, the new rows, the workspace) and the
    layer."""

    __slots__ = ("args", "need", "kv", "rope_fused")

    def __init__(self, args: _lib.SdlAttnArgs, need: int, kv: PagedKVCache, rope_fused: bool = False) -> None:
        self.args = args
        self.need = need
        self.kv = weakref.ref(kv)  # the struct points at the cache's tensor maps
        self.rope_fused = rope_fused  # the launch rotates q and k_new itself


_ARGS_CACHE = {}
_ARGS_CACHE_MAX = 64


def _new_rows_2d(q4: torch.Tensor, kv: PagedKVCache, k_new: torch.Tensor, v_new: torch.Tensor):
    """k_new / v_new as (rows, Hkv*d) views with unit column stride and a
    shared row stride (copied when they are not), checked against the pool."""
    rows = q4.shape[0] * q4.shape[1]
    kn = k_new if k_new.dim() == 2 else k_new.reshape(rows, -1)
    vn = v_new if v_new.dim() == 2 else v_new.reshape(rows, -1)
    if kn.dtype != kv.dtype or vn.dtype != kv.dtype or kn.shape != (rows, kv.num_kv_heads * kv.head_dim) \
            or vn.shape != kn.shape:
        raise ValueError("k_new/v_new must be ({}, {}) rows of {}".format(rows, kv.num_kv_heads * kv.head_dim,
                                                                       kv.dtype))
    _lib.require_cuda(kn, "k_new")
    _lib.require_cuda(vn, "v_new")
    if kn.stride(1) != 1 or vn.stride(1) != 1 or kn.stride(0) != vn.stride(0):
        kn, vn = kn.contiguous(), vn.contiguous()
    return kn, vn


def paged_attention(
    q: torch.Tensor,
    kv: PagedKVCache,
    layer: int,
    batch: AttnBatch,
    out: Optional[torch.Tensor] = None,
    out_dtype: Optional[torch.dtype] = None,
    force_generic: bool = False,
    pages_per_split: int = 0,
    kv_heads_per_cta: int = 0,
    use_umma: int = 0,
    k_new: Optional[torch.Tensor] = None,
    v_new: Optional[torch.Tensor] = None,
    cluster_merge: bool = False,
    mma_layout: int = 0,
    rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
    overlap_layers: bool = False,
) -> torch.Tensor:
    """Attention of ``q`` (B, chunk, Hq, d) against the pages of ``kv``.

    With ``k_new`` / ``v_new`` (B*chunk rows of Hkv*d, the pool's dtype) the
    call first stores them at positions ``starts[b] + j`` of layer ``layer``
    (the positions must already be reserved) -- the write-then-attend of a
    decoder layer in one launch on the tensor-core path.

    ``rope = (cos, sin)`` (one head_dim row per (b, j), e.g. ``(B, chunk, 1,
    d)``) applies the reference's rotate-half RoPE (engine/model.py:50-56) to
    ``q`` and ``k_new`` as part of the call, with the framework chain's
    roundings: the mma.sync kernels rotate q as they load it and k_new as
    they store it (no separate launch, q and k_new only read); other plans
    rotate ``q`` and ``k_new`` in place first.

    ``overlap_layers``: the caller launches attention over distinct layers
    back to back on the stream (an attention stack's decode step), so no
    kernel still running when this one starts writes this layer's older
    pages; the launch then overlaps its ramp with the previous layer's tail
    (sdl_attn_args.overlap_layers).  Leave it off when the previous kernel
    may have appended to this layer.

    ``pages_per_split`` / ``kv_heads_per_cta`` / ``use_umma`` /
    ``cluster_merge`` / ``mma_layout`` override the launch plan (pages per
    split-K CTA, kv heads sharing one CTA of the mma.sync kernel, 1 for the
    tcgen05 kernel, split partials merged on chip within a thread-block
    cluster instead of by a separate launch, 1 / 2 for the mma.sync kernel
    with keys / query rows on the MMA M dimension, 3 for keys on M with K/V
    loaded straight into registers); every plan gives the same
    result within rounding of the split merge.
    """
    _lib.require_cuda(q, "query")
    if q.dim() != 4 or q.shape[3] != kv.head_dim:
        raise ValueError("query must be (B, chunk, Hq, {}), got {}".format(kv.head_dim, tuple(q.shape)))
    if q.dtype != kv.dtype:
        q = q.to(kv.dtype)
    if q.stride(3) != 1:
        q = q.contiguous()
    if out is None:
        # rows past valid_rows are left unwritten by the kernels and read as zero
        alloc = torch.empty if batch.valid_rows is None else torch.zeros
        out = alloc(q.shape, dtype=out_dtype or q.dtype, device=q.device)
    if batch.max_limit > kv.width * kv.block_size:
        raise RuntimeError("attention span {} exceeds the block-table width".format(batch.max_limit))
    kn = vn = None
    if k_new is not None:
        kn, vn = _new_rows_2d(q, kv, k_new, v_new)
    rc = rs = None
    if rope is not None:
        if kn is None:
            raise ValueError("rope needs k_new (the rows it rotates before storing)")
        rc, rs = (t.reshape(-1, q.shape[3]) for t in rope)
        if rc.shape[0] != q.shape[0] * q.shape[1] or rs.shape[0] != rc.shape[0]:
            raise ValueError("rope: cos / sin need one row per (b, j) of q")
        rc = rc if (rc.dtype == q.dtype and rc.stride(-1) == 1) else rc.to(q.dtype).contiguous()
        rs = rs if (rs.dtype == q.dtype and rs.stride(-1) == 1) else rs.to(q.dtype).contiguous()
    vr = batch.valid_rows
    # Everything the launch plan and the struct's fixed fields depend on,
    # including the pointer alignments the plan tests.
    key = (id(kv), kv._table.data_ptr(), kv._k.data_ptr(), batch.rows.data_ptr(), batch.starts.data_ptr(),
           vr.data_ptr() if vr is not None else 0, batch.max_limit, batch.key_count, tuple(q.shape), q.stride(),
           q.dtype, q.data_ptr() % 16, out.stride(), out.dtype, force_generic, pages_per_split, kv_heads_per_cta,
           use_umma, cluster_merge, mma_layout,
           -1 if kn is None else (kn.stride(0), kn.data_ptr() % 16, vn.data_ptr() % 16),
           -1 if rc is None else (rc.stride(0), rc.data_ptr() % 16, rs.data_ptr() % 16), bool(overlap_layers),
           threading.get_ident())
    ent = _ARGS_CACHE.get(key)
    if ent is None or ent.kv() is not kv:
        a = _paged_args(q, kv, layer, batch, out, force_generic, pages_per_split, kv_heads_per_cta, use_umma,
                        cluster_merge, mma_layout)
        if kn is not None:
            a.k_new, a.v_new, a.new_row_stride = kn.data_ptr(), vn.data_ptr(), kn.stride(0)
        a.overlap_layers = 1 if overlap_layers else 0
        fused = False
        if rc is not None:
            a.rope_cos, a.rope_sin, a.rope_stride = rc.data_ptr(), rs.data_ptr(), rc.stride(0)
            fused = _lib.load().sdl_attention_fuses_rope(a) == 1
            if not fused:
                a.rope_cos = a.rope_sin = None
                a.rope_stride = 0
        need = int(_lib.load().sdl_attention_workspace_bytes(a))
        if len(_ARGS_CACHE) >= _ARGS_CACHE_MAX:
            _ARGS_CACHE.clear()
        ent = _ArgsEntry(a, need, kv, fused)
        _ARGS_CACHE[key] = ent
    a = ent.args
    a.q = q.data_ptr()
    a.out = out.data_ptr()
    a.layer = layer
    if rc is not None:
        if ent.rope_fused:
            a.rope_cos, a.rope_sin = rc.data_ptr(), rs.data_ptr()
        else:  # this plan's kernel cannot rotate inside the launch: rotate in place first
            from . import layer_ops
            layer_ops.rope_(q, rs.reshape(q.shape[0], q.shape[1], 1, -1), rc.reshape(q.shape[0], q.shape[1], 1, -1))
            layer_ops.rope_(kn.view(kn.shape[0], kv.num_kv_heads, kv.head_dim), rs, rc)
    if kn is not None:
        a.k_new, a.v_new = kn.data_ptr(), vn.data_ptr()
    dev = q.device
    if ent.need:
        ws = _lib.Workspace.get(dev, ent.need)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel() * 4
    _lib.check(_lib.load().sdl_paged_attention(a, _lib.stream_handle(dev)), "sdl_paged_attention")
    return out


def _expand_to_q_heads(kv: torch.Tensor, num_q_heads: int) -> torch.Tensor:
    """Broadcast ``(.., kv_heads, d)`` to ``(.., num_q_heads, d)`` for GQA."""
    kv_heads = kv.shape[-2]
    ratio = num_q_heads // kv_heads
    if ratio == 1:
        return kv
    return kv.repeat_interleave(ratio, dim=-2)


def gather_ctx(kv: PagedKVCache, layer: int, seq_id: int, length: int) -> torch.Tensor:
    """Return the stored K/V prefix of one sequence as ``(2, length, kv_heads, d)``.

    Reads the device block table directly (no host round trip).
    """
    if length <= 0:
        return torch.zeros((2, 0, kv.num_kv_heads, kv.head_dim), dtype=kv.dtype, device=kv.device)
    n_blocks = -(-length // kv.block_size)
    if n_blocks > kv.num_blocks_of(seq_id):
        raise IndexError("list index out of range")
    phys = kv._table[seq_id, :n_blocks].long()
    key = kv._k[layer][phys].reshape(-1, kv.num_kv_heads, kv.head_dim)[:length]
    value = kv._v[layer][phys].reshape(-1, kv.num_kv_heads, kv.head_dim)[:length]
    return torch.stack((key, value), dim=0)


def _dense_attention(q4: torch.Tensor, k: torch.Tensor, v: torch.Tensor, starts: List[int],
                     valid_rows: Optional[List[int]]) -> torch.Tensor:
    """Dense-K/V launch: q4 (B, chunk, Hq, d), k/v (B, kv_len, Hkv, d)."""
    _lib.require_cuda(q4, "query")
    B, chunk, Hq, d = q4.shape
    k = k.to(q4.dtype).contiguous()
    v = v.to(q4.dtype).contiguous()
    if q4.stride(3) != 1:
        q4 = q4.contiguous()
    out = torch.zeros(q4.shape, dtype=q4.dtype, device=q4.device)
    if B == 0:
        return out
    a = _args_common(q4, out, k.shape[2], None)
    a.k_dense, a.v_dense, a.kv_len = k.data_ptr(), v.data_ptr(), k.shape[1]
    packed = _lib.i32(list(starts) + (list(valid_rows) if valid_rows is not None else []), q4.device)
    a.starts = packed.data_ptr()
    a.valid_rows = packed.data_ptr() + 4 * B if valid_rows is not None else None
    a.max_limit = max(int(s) for s in starts) + chunk
    _launch(a, q4.device)
    return out


def full_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    num_q_heads: int,
) -> torch.Tensor:
    """Unmasked attention of ``query (Hq, d)`` over ``key/value (ctx, kv_heads, d)``."""
    ctx = key.shape[0]
    if ctx == 0:
        return torch.zeros_like(query)
    out = _dense_attention(query.reshape(1, 1, num_q_heads, -1), key.unsqueeze(0), value.unsqueeze(0),
                           [ctx - 1], None)
    return out[0, 0]


def paged_attention_decode(
    query_2d: torch.Tensor,
    kv: PagedKVCache,
    layer: int,
    seq_ids: Sequence[int],
    seq_token_lengths: Sequence[int],
    num_q_heads: int,
) -> torch.Tensor:
    """Attend one new query token per row against its full stored prefix.

    ``query_2d`` is ``(B, num_q_heads, d)``; returns ``(B, num_q_heads, d)``.
    """
    B = query_2d.shape[0]
    lengths = [int(x) for x in seq_token_lengths]
    batch = AttnBatch.from_lists(query_2d.device, seq_ids, [ln - 1 for ln in lengths], 1)
    out = paged_attention(query_2d.reshape(B, 1, num_q_heads, -1), kv, layer, batch)
    return out.reshape(B, num_q_heads, -1)


def paged_attention_prefill_chunk(
    query_3d: torch.Tensor,
    key_3d: torch.Tensor,
    value_3d: torch.Tensor,
    num_q_heads: int,
    chunk_query_lengths: Sequence[int],
) -> torch.Tensor:
    """Causal attention over a freshly prefilled prompt chunk (``query_start=0``).

    Returns ``(B, chunk_len, num_q_heads, d)`` with padded rows exactly zero.
    """
    B = query_3d.shape[0]
    lengths = [int(x) for x in chunk_query_lengths]
    return _dense_attention(query_3d, key_3d, value_3d, [0] * B, lengths)


def paged_attention_extend(
    query_3d: torch.Tensor,
    kv: PagedKVCache,
    layer: int,
    seq_ids: Sequence[int],
    start_positions: Sequence[int],
    num_q_heads: int,
) -> torch.Tensor:
    """Attend a chunk of fresh tokens against an existing prefix plus prior rows.

    ``query_3d`` is ``(B, chunk, num_q_heads, d)``; returns the same shape.
    """
    chunk = query_3d.shape[1]
    batch = AttnBatch.from_lists(query_3d.device, seq_ids, start_positions, chunk)
    return paged_attention(query_3d, kv, layer, batch)
