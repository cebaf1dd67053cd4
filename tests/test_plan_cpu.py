"""Launch-plan logic of the attention entry points, on the host (no GPU).

``sdl_attention_kernel`` / ``sdl_attention_launches`` /
``sdl_attention_workspace_bytes`` only read the scalar arguments and the
alignment of the pointers, so they run without a device: the pointers below
are aligned stand-ins that are never dereferenced.
"""

from __future__ import annotations

import ctypes

import pytest

from engine import _lib

KERNELS = {0: "generic", 1: "mma", 2: "tcgen05", 3: "mma_rows", 4: "mma_direct"}


def _args(B, chunk, Hq, Hkv, d, max_limit, dtype=_lib.SDL_BF16, **kw):
    a = _lib.SdlAttnArgs()
    a.q, a.out = 0x100000, 0x200000
    a.q_sb, a.q_sj, a.q_sh = chunk * Hq * d, Hq * d, d
    a.o_sb, a.o_sj, a.o_sh = chunk * Hq * d, Hq * d, d
    a.dtype = a.out_dtype = dtype
    a.k_pool, a.v_pool, a.block_table = 0x300000, 0x400000, 0x500000
    a.rows, a.starts = 0x600000, 0x700000
    a.width, a.capacity, a.num_layers, a.layer, a.block_size = 4096, 100000, 1, 0, 16
    a.B, a.chunk, a.Hq, a.Hkv, a.head_dim = B, chunk, Hq, Hkv, d
    a.max_limit = max_limit
    a.scale = d ** -0.5
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def _kernel(a):
    n = _lib.load().sdl_attention_kernel(ctypes.byref(a))
    assert n >= 0, _lib.last_error()
    return KERNELS[n]


@pytest.mark.parametrize("shape,flags,want", [
    ((64, 1, 12, 2, 128, 4096), {}, "mma"),                       # C2 decode: keys on M
    ((32, 6, 12, 2, 128, 2048), {}, "mma"),                       # C3 verify, 36 rows: keys on M
    ((32, 8, 12, 2, 128, 2048), {}, "mma_rows"),                  # 48 rows per kv head
    ((32, 5, 14, 2, 64, 2048), {}, "mma_rows"),                   # d 64, 35 rows
    ((16, 7, 16, 2, 128, 32768), {}, "tcgen05"),                  # C5 verify: long span
    ((16, 7, 16, 2, 128, 32768), {"key_count": 16 * 20000}, "tcgen05"),
    ((16, 5, 12, 2, 128, 32768), {"key_count": 16 * 20000}, "mma"),   # 30 rows: keys on M
    ((64, 5, 12, 2, 128, 4200), {"key_count": 64 * 700}, "mma_rows"),  # C4 verify: short mean span
    ((32, 6, 12, 2, 128, 2048), {"key_count": 32 * 1152}, "mma"),  # C3 verify: mean 1152 keys
    ((16, 7, 16, 2, 128, 32768), {"use_umma": -1}, "mma_rows"),   # mma.sync forced
    ((16, 7, 16, 2, 128, 32768), {"use_umma": -1, "mma_layout": 1}, "mma"),
    ((64, 1, 12, 2, 128, 4096), {"mma_layout": 2}, "mma_rows"),
    ((64, 1, 12, 2, 128, 4096), {"mma_layout": 3}, "mma_direct"),  # register-direct decode
    ((64, 1, 14, 2, 64, 4096), {"mma_layout": 3}, "mma_direct"),   # 7 columns, d 64
    ((64, 1, 14, 2, 64, 1500), {"key_count": 64 * 700}, "mma_direct"),  # 0.5B draft decode, short rows
    ((64, 1, 14, 2, 64, 3000), {"key_count": 64 * 2000}, "mma"),   # longer rows: the TMA kernel
    ((64, 1, 14, 2, 64, 1500), {}, "mma"),                         # no key count: the TMA kernel
    ((64, 1, 14, 2, 64, 1500), {"mma_layout": 1}, "mma"),
    ((64, 2, 14, 2, 64, 1500), {}, "mma"),                         # 14 columns
    ((32, 6, 12, 2, 128, 2048), {"mma_layout": 3}, "mma"),         # 36 columns: beyond one 8-column tile
    ((64, 1, 12, 2, 128, 4096), {"mma_layout": 3, "k_pool": 0x300008}, "mma"),  # pool not 16-byte aligned
    ((32, 8, 12, 2, 128, 2048), {"cluster_merge": 1}, "mma"),     # the cluster merge is keys-on-M only
    ((1, 512, 12, 2, 128, 512), {}, "mma_rows"),                  # prefill chunk
    ((8, 1, 4, 2, 16, 100), {"dtype": _lib.SDL_F32}, "generic"),  # fp32 pool
    ((32, 6, 12, 2, 128, 2048), {"force_generic": 1}, "generic"),
    # ragged rows of unknown lengths (a captured graph): register-direct only for
    # head_dim-64 decode of up to 128 sequences, no tcgen05 auto choice
    ((358, 5, 12, 2, 128, 4656), {"key_count": -1}, "mma_rows"),   # C4 verify, 30 rows
    ((358, 1, 14, 2, 64, 4656), {"key_count": -1}, "mma"),         # C4 draft decode
    ((160, 1, 14, 2, 64, 4656), {"key_count": -1}, "mma"),
    ((128, 1, 14, 2, 64, 4656), {"key_count": -1}, "mma_direct"),  # the drain's smaller batches
    ((96, 1, 14, 2, 64, 4656), {"key_count": -1}, "mma_direct"),
    ((64, 1, 14, 2, 64, 1500), {"key_count": -1}, "mma_direct"),
    ((1, 1, 14, 2, 64, 1024), {"key_count": -1}, "mma_direct"),
    ((64, 1, 14, 2, 64, 1500), {"key_count": -1, "mma_layout": 1}, "mma"),
    ((64, 1, 12, 2, 128, 4096), {"key_count": -1}, "mma"),         # head_dim 128: the TMA kernel
    ((64, 5, 14, 2, 64, 4656), {"key_count": -1}, "mma_rows"),     # 35-row draft blocks
    ((16, 7, 16, 2, 128, 32768), {"key_count": -1}, "mma_rows"),   # 56 rows: rows on M, not tcgen05
    ((16, 7, 16, 2, 128, 32768), {"key_count": -1, "use_umma": 1}, "tcgen05"),
])
def test_kernel_choice(shape, flags, want):
    assert _kernel(_args(*shape, **flags)) == want


def test_launch_counts_and_workspace():
    lib = _lib.load()
    # split decode rows: attention + merge, partials in the workspace
    a = _args(64, 1, 12, 2, 128, 4096)
    assert lib.sdl_attention_launches(ctypes.byref(a)) == 2
    assert lib.sdl_attention_workspace_bytes(ctypes.byref(a)) > 0
    # one page per split would need far more partial rows than 64 pages per split
    big = _args(64, 1, 12, 2, 128, 4096, pages_per_split=1)
    small = _args(64, 1, 12, 2, 128, 4096, pages_per_split=64)
    assert lib.sdl_attention_workspace_bytes(ctypes.byref(big)) > lib.sdl_attention_workspace_bytes(ctypes.byref(small))
    # one split per row: a single launch, no workspace
    one = _args(2000, 1, 12, 2, 128, 64)
    assert lib.sdl_attention_launches(ctypes.byref(one)) == 1
    assert lib.sdl_attention_workspace_bytes(ctypes.byref(one)) == 0
    # the rows-on-M kernel's splits are whole 32-key tiles: an odd request rounds up
    r1 = _args(32, 8, 12, 2, 128, 2048, pages_per_split=1)
    r2 = _args(32, 8, 12, 2, 128, 2048, pages_per_split=2)
    assert lib.sdl_attention_workspace_bytes(ctypes.byref(r1)) == lib.sdl_attention_workspace_bytes(ctypes.byref(r2))
    # a positional append launch is added only where the kernel does not store the rows itself
    fused = _args(64, 1, 12, 2, 128, 4096, k_new=0x800000, v_new=0x900000, new_row_stride=2 * 128)
    assert lib.sdl_attention_launches(ctypes.byref(fused)) == 2
    sep = _args(16, 7, 16, 2, 128, 32768, k_new=0x800000, v_new=0x900000, new_row_stride=2 * 128)
    assert lib.sdl_attention_launches(ctypes.byref(sep)) == 3  # append + tcgen05 + its merge


def test_invalid_arguments_are_refused():
    lib = _lib.load()
    a = _args(4, 1, 12, 5, 128, 100)  # Hq not a multiple of Hkv
    assert lib.sdl_attention_kernel(ctypes.byref(a)) == -1
    assert lib.sdl_attention_launches(ctypes.byref(a)) == -1
    assert lib.sdl_attention_workspace_bytes(ctypes.byref(a)) == 0


@pytest.mark.parametrize("shape,flags,want_kernel,fuses", [
    ((64, 1, 14, 2, 64, 4656), {"key_count": -1}, "mma_direct", 1),   # captured draft decode, small bucket
    ((358, 1, 14, 2, 64, 4656), {"key_count": -1}, "mma", 1),         # captured draft decode, large bucket
    ((358, 5, 12, 2, 128, 4656), {"key_count": -1}, "mma_rows", 1),   # captured verify
    ((16, 7, 16, 2, 128, 32768), {}, "tcgen05", 0),                   # tcgen05: q and k rotated first
    ((32, 6, 12, 2, 128, 2048), {"force_generic": 1}, "generic", 0),
])
def test_rope_fusion_follows_the_plan(shape, flags, want_kernel, fuses):
    """sdl_attention_fuses_rope (plan logic only, nothing launched): every
    mma.sync plan that stores the new rows itself, the register-direct one
    included, rotates q and k inside the launch; tcgen05 and CUDA-core plans
    do not."""
    lib = _lib.load()
    cs = dict(rope_cos=0xA00000, rope_sin=0xB00000, rope_stride=2 * shape[4])
    a = _args(*shape, k_new=0x800000, v_new=0x900000, new_row_stride=2 * shape[4], **cs, **flags)
    assert _kernel(a) == want_kernel
    assert lib.sdl_attention_fuses_rope(ctypes.byref(a)) == fuses



def _split_of(a):
    """(splits per row, pages per split) of a plan, from its workspace bytes."""
    lib = _lib.load()
    ws = lib.sdl_attention_workspace_bytes(ctypes.byref(a))
    return ws // (a.B * a.chunk * a.Hq * (a.head_dim + 2) * 4)


@pytest.mark.parametrize("B,chunk,Hq,d,span,base,bdiv", [
    (358, 5, 12, 128, 4656, 716, 16),    # verify rows on M: one CTA per (sequence, kv head)
    (1024, 5, 12, 128, 4656, 2048, 16),
    (64, 5, 12, 128, 4656, 128, 16),
    (16, 5, 12, 128, 4656, 32, 16),
    (358, 1, 14, 64, 4656, 358, 16),     # decode keys on M: both kv heads in one CTA
    (160, 1, 14, 64, 2048, 160, 16),
    (112, 1, 14, 64, 2048, 224, 8),
    (64, 1, 14, 64, 4656, 128, 8),       # register-direct decode: one CTA per (sequence, kv head)
    (64, 1, 14, 64, 2048, 128, 8),
    (96, 1, 14, 64, 2048, 192, 8),
    (96, 1, 14, 64, 4656, 192, 8),
    (16, 1, 14, 64, 32768, 32, 8),
    (16, 1, 14, 64, 1024, 32, 8),
])
def test_ragged_split_bounds(B, chunk, Hq, d, span, base, bdiv):
    """key_count < 0: splits of max(base/16, span pages/16) pages for decode
    (base/8 for the register-direct kernel) and max(base/16, span pages/32)
    for blocks, within 8..64; the grid still covers the span."""
    a = _args(B, chunk, Hq, 2, d, span, key_count=-1)
    max_pages = -(-span // 16)
    div = 32 if chunk > 1 else 16
    pps = min(64, max(8, max(base // bdiv, -(-max_pages // div))))
    pps = min(pps, max_pages)
    if chunk > 1:
        pps += pps % 2  # the rows-on-M kernel splits at whole 32-key tiles
    assert _split_of(a) == -(-max_pages // pps)
    assert _lib.load().sdl_attention_launches(ctypes.byref(a)) == 2


@pytest.mark.parametrize("R,span,want_splits", [(8, 4656, 1), (8, 1024, 1), (1, 4656, 7)])
def test_ragged_prefill_rows_split_only_to_fill_the_sms(R, span, want_splits):
    """Ragged prefill chunk rows (128 positions, 12 q / 2 kv heads: 12 row
    tiles per kv head) split only until every SM has a CTA: their partials
    outweigh the pages a split saves."""
    a = _args(R, 128, 12, 2, 128, span, key_count=-1)
    lib = _lib.load()
    ws = lib.sdl_attention_workspace_bytes(ctypes.byref(a))
    if want_splits == 1:
        assert ws == 0 and lib.sdl_attention_launches(ctypes.byref(a)) == 1
    else:
        assert _split_of(a) == want_splits
