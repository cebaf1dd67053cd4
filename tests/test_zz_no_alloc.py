"""The allocation-free attention entry point, called through the C ABI.

``sdl_paged_attention_noalloc`` serves callers that cannot allocate device
memory at call time (a runtime whose pool allocator owns all HBM, or an FFI
host that only owns the buffers it passes in): its split-K partials live in a
static device array instead of a caller workspace.  It must give the same
output as ``sdl_paged_attention`` with a workspace, on consecutive calls that
reuse the shared array, and refuse shapes whose scratch exceeds the array.

This file sorts last so that a stop-at-first-failure run has already run
every other test; it is also self-contained for a fresh process.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from engine import _lib
from engine.attention import AttnBatch, _paged_args, paged_attention
from engine.kv import PagedKVCache

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _case(seed: int, lens, chunk: int):
    """A paged bf16 cache with Qwen2.5-1.5B attention shapes and random K/V."""
    Hq, Hkv, d, bs = 12, 2, 128, 16
    rng = np.random.default_rng(seed)
    cap = sum(-(-(n + chunk) // bs) for n in lens) + 2
    kv = PagedKVCache(1, Hkv, d, cap, bs, DEV, torch.bfloat16)
    for sid, n in enumerate(lens):
        kv.add_sequence(sid)
        slots = kv.reserve([sid], [0], [n + chunk])
        k = torch.from_numpy(rng.standard_normal((n + chunk, Hkv, d)).astype(np.float32)).to(DEV, torch.bfloat16)
        v = torch.from_numpy(rng.standard_normal((n + chunk, Hkv, d)).astype(np.float32)).to(DEV, torch.bfloat16)
        kv.append(0, slots, k, v)
    q = torch.from_numpy(rng.standard_normal((len(lens), chunk, Hq, d)).astype(np.float32)).to(DEV, torch.bfloat16)
    return kv, q, AttnBatch.from_lists(DEV, list(range(len(lens))), lens, chunk)


def _noalloc(q, kv, batch, out_dtype=None, **kw):
    out = torch.zeros(q.shape, dtype=out_dtype or q.dtype, device=DEV)
    args = _paged_args(q, kv, 0, batch, out, **kw)
    lib = _lib.load()
    assert lib.sdl_attention_workspace_bytes(args) > 0, "case must exercise the split-K scratch"
    rc = lib.sdl_paged_attention_noalloc(ctypes.byref(args), _lib.stream_handle(DEV))
    _lib.check(rc, "sdl_paged_attention_noalloc")
    return out


def test_noalloc_matches_workspace_entry_point_on_consecutive_calls():
    for seed, lens, chunk in ((1, [3000, 17, 1200, 640], 1), (2, [2047, 900, 5], 6)):
        kv, q, batch = _case(seed, lens, chunk)
        want = paged_attention(q, kv, 0, batch)           # caller-provided workspace
        got = _noalloc(q, kv, batch)                      # static scratch, reused across calls
        torch.cuda.synchronize()
        # same plan and arithmetic: equal within the attention tolerance (in fact bit-equal)
        torch.testing.assert_close(got.float(), want.float(), rtol=2e-3, atol=2e-3)
        assert torch.equal(got, want)
        kv.check_errors()


def test_noalloc_shrinks_its_split_to_fit_the_array():
    """64 rows of a 7-row verify over 32k keys with 16 q heads: the
    automatic mma.sync plan's partials would exceed the array, so the
    allocation-free call takes larger splits until they fit; the result
    agrees with the workspace entry point within the attention tolerance."""
    lib = _lib.load()
    B, chunk, Hq, Hkv, d, bs, L = 64, 7, 16, 2, 128, 16, 32760
    cap = B * (-(-(L + chunk) // bs))
    kv = PagedKVCache(1, Hkv, d, cap, bs, DEV, torch.bfloat16, max_blocks_per_seq=-(-(L + chunk) // bs), max_seqs=B)
    sids = list(range(B))
    for sid in sids:
        kv.add_sequence(sid)
    kv.reserve(sids, [0] * B, [L + chunk] * B)
    g = torch.Generator(device=DEV)
    g.manual_seed(3)
    kv._k.normal_(generator=g)
    kv._v.normal_(generator=g)
    q = torch.randn((B, chunk, Hq, d), generator=g, device=DEV).to(torch.bfloat16)
    # no key count: the automatic split fills the GPU as if every row were
    # long, which needs more partials than the array holds
    full = AttnBatch.from_lists(DEV, sids, [L] * B, chunk)
    batch = AttnBatch(full.rows, full.starts, full.max_limit)
    args = _paged_args(q, kv, 0, batch, q, use_umma=-1)
    assert lib.sdl_attention_workspace_bytes(args) > lib.sdl_noalloc_scratch_bytes()
    for _ in range(2):
        got = _noalloc(q, kv, batch, out_dtype=torch.float32, use_umma=-1)
        want = paged_attention(q, kv, 0, batch, out_dtype=torch.float32, use_umma=-1)
        torch.cuda.synchronize()
        scale = want.abs().max().item()
        assert (got - want).abs().max().item() <= 2e-3 * scale
    kv.check_errors()


def test_noalloc_refuses_scratch_beyond_its_array():
    """A plan that cannot shrink (an explicit split size) and needs more
    scratch than the array is refused on the host, before any launch."""
    lib = _lib.load()
    kv = PagedKVCache(1, 2, 128, 8, 16, DEV, torch.bfloat16, max_blocks_per_seq=2100)
    q = torch.zeros((64, 7, 16, 128), device=DEV, dtype=torch.bfloat16)
    rows = torch.arange(64, dtype=torch.int32, device=DEV)
    starts = torch.zeros(64, dtype=torch.int32, device=DEV)
    batch = AttnBatch(rows, starts, 32768)
    # the mma.sync plan with 256-key splits: 64 rows x 128 splits of partials
    args = _paged_args(q, kv, 0, batch, q, use_umma=-1, pages_per_split=16)
    assert lib.sdl_attention_workspace_bytes(args) > lib.sdl_noalloc_scratch_bytes()
    rc = lib.sdl_paged_attention_noalloc(ctypes.byref(args), _lib.stream_handle(DEV))
    assert rc == 4  # SDL_ERR_WORKSPACE, refused on the host before any launch
    assert "static scratch" in _lib.last_error()
    assert int(kv.err_word.item()) == 0
