"""Paged attention kernels vs the reference fixtures and the fp64 oracle.

Tolerances (north star: 1e-5 relative in fp32, 2e-3 in bf16):
* fp32 pools (CUDA-core kernel): ``allclose(rtol=1e-5, atol=1e-5)``.
* bf16 pools (tensor-core kernels): ``conftest.check_attention_16bit`` --
  fp32 output within 2e-3 relative per element (elements at least 2 % of the
  call's largest output) and 2e-3 of the largest normwise; 16-bit output
  within one bf16 rounding of the exact value plus 2e-3 of the largest.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import check_attention_16bit, load_npz
from engine.attention import (
    AttnBatch,
    full_attention,
    gather_ctx,
    paged_attention,
    paged_attention_decode,
    paged_attention_extend,
    paged_attention_prefill_chunk,
)
from engine.kv import PagedKVCache
from oracle import attention as oatt
from oracle import kv as okv

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _build(lens_total, Hkv, d, bs, dtype, seed, extra_blocks=3, shuffle=True, layers=1, piece=None):
    """Device cache + oracle cache holding identical random K/V (written in
    interleaved pieces of 1 .. ``piece`` tokens, so block tables scatter)."""
    piece = piece or 3 * bs
    rng = np.random.default_rng(seed)
    cap = sum(-(-T // bs) for T in lens_total) + extra_blocks
    kv = PagedKVCache(layers, Hkv, d, cap, bs, DEV, dtype)
    ref = okv.PagedKVCache(layers, Hkv, d, cap, bs)
    B = len(lens_total)
    for sid in range(B):
        kv.add_sequence(sid)
        ref.add_sequence(sid)
    if shuffle:  # interleave the sequences' allocations so tables are scattered
        order = []
        pos = [0] * B
        while any(p < T for p, T in zip(pos, lens_total)):
            for sid in rng.permutation(B):
                if pos[sid] < lens_total[sid]:
                    n = int(min(lens_total[sid] - pos[sid], rng.integers(1, piece)))
                    order.append((int(sid), pos[sid], n))
                    pos[sid] += n
    else:
        order = [(sid, 0, T) for sid, T in enumerate(lens_total) if T > 0]
    for sid, st, n in order:
        slots = kv.reserve([sid], [st], [n])
        want = ref.reserve([sid], [st], [n])
        assert slots.tolist() == want
        for layer in range(layers):
            k = torch.from_numpy(rng.standard_normal((n, Hkv, d)).astype(np.float32)).to(DEV, dtype)
            v = torch.from_numpy(rng.standard_normal((n, Hkv, d)).astype(np.float32)).to(DEV, dtype)
            kv.append(layer, slots, k, v)
            ref.append(layer, want, k.float().cpu().numpy(), v.float().cpu().numpy())
    return kv, ref


def _check_bf16(out_bf16, out_f32, exact):
    """Normwise and per-element bounds (``conftest.check_attention_16bit``)."""
    check_attention_16bit(out_bf16, out_f32, exact)


# --------------------------------------------------------------- fixtures
def _golden_case(tag):
    a = load_npz("attention.npz")
    Hq, Hkv, d, bs, chunk, cap = (int(x) for x in a[tag + "_meta"])
    starts = a[tag + "_starts"].tolist()
    dtype = torch.bfloat16 if "bf16" in tag else torch.float32
    kv = PagedKVCache(1, Hkv, d, cap, bs, DEV, dtype)
    for sid, st in enumerate(starts):
        kv.add_sequence(sid)
        kv.reserve([sid], [0], [st + chunk])  # same order as the reference's writes
    tables = [[int(x) for x in row if x >= 0] for row in a[tag + "_tables"]]
    assert kv.block_tables == tables
    kv._k.copy_(torch.from_numpy(a[tag + "_k"]).to(DEV, dtype))
    kv._v.copy_(torch.from_numpy(a[tag + "_v"]).to(DEV, dtype))
    q = torch.from_numpy(a[tag + "_q"]).to(DEV, dtype)
    return kv, q, starts, chunk, Hq, a[tag + "_out"]


@pytest.mark.parametrize("tag", ["dec_f32_small", "dec_f32_d64", "ext_f32_d64"])
def test_fp32_attention_matches_reference_fixture(tag):
    kv, q, starts, chunk, Hq, ref = _golden_case(tag)
    if chunk == 1:
        out = paged_attention_decode(q[:, 0], kv, 0, list(range(len(starts))), [s + 1 for s in starts], Hq)[:, None]
    else:
        out = paged_attention_extend(q, kv, 0, list(range(len(starts))), starts, Hq)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("tag", ["dec_bf16_d128", "ext_bf16_d128", "dec_bf16_d64_r7"])
@pytest.mark.parametrize("layout", [0, 1, 2, 3])
def test_bf16_attention_matches_reference_fixture(tag, layout):
    """The reference's own outputs, on the automatic kernel and on every
    mma.sync layout (keys / query rows on the MMA M dimension, keys on M with
    register-direct loads)."""
    kv, q, starts, chunk, Hq, ref = _golden_case(tag)
    batch = AttnBatch.from_lists(DEV, list(range(len(starts))), starts, chunk)
    out = paged_attention(q, kv, 0, batch, mma_layout=layout)
    out32 = paged_attention(q, kv, 0, batch, out_dtype=torch.float32, mma_layout=layout)
    # exact value from the fp64 oracle on the same bf16 inputs
    a = load_npz("attention.npz")
    okvc = okv.PagedKVCache(1, kv.num_kv_heads, kv.head_dim, kv.capacity, kv.block_size)
    okvc.k[:] = a[tag + "_k"]
    okvc.v[:] = a[tag + "_v"]
    for sid, st in enumerate(starts):
        okvc.add_sequence(sid)
        okvc.block_tables[sid] = kv.block_tables[sid]
    exact = oatt.paged_attention_extend(a[tag + "_q"], okvc, 0, range(len(starts)), starts)
    _check_bf16(out.float().cpu().numpy(), out32.cpu().numpy(), exact)
    # and the reference's own bf16 result agrees to bf16 resolution
    assert np.abs(out.float().cpu().numpy() - ref).max() <= 2.0 ** -7 * np.abs(ref).max() + 1e-6


# ---------------------------------------------------------- random vs oracle
CASES = [
    # Hq, Hkv, d, chunk, lens (start positions), bs, dtype
    (12, 2, 128, 1, [1, 15, 16, 17, 300, 1029, 4095], 16, torch.bfloat16),     # C2 decode shape, split-K
    (12, 2, 128, 6, [0, 5, 250, 2047], 16, torch.bfloat16),                     # C3 verify (gamma=5)
    (16, 2, 128, 7, [100, 3000, 8191], 16, torch.bfloat16),                     # C5 verify (gamma=6, ratio 8)
    (14, 2, 64, 1, [2, 64, 777, 2100], 16, torch.bfloat16),                     # 0.5B draft (ratio 7, d 64)
    (14, 2, 64, 5, [0, 31, 1000], 16, torch.float16),                           # fp16, extend
    (4, 2, 64, 1, [0, 40, 333], 16, torch.bfloat16),                            # C1 shape (ratio 2)
    (8, 8, 128, 3, [10, 700], 16, torch.bfloat16),                              # MHA, Hkv 8
    (16, 2, 128, 8, [33, 1500], 16, torch.bfloat16),                            # 64 columns: 8 warps x 8
    (12, 2, 128, 11, [7, 640, 2000], 16, torch.bfloat16),                       # 66 columns: 16-column tiles
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("generic,umma,layout", [(False, 0, 0), (False, 1, 0), (False, -1, 1), (False, -1, 2),
                                                 (False, -1, 3), (True, 0, 0)])
def test_paged_attention_matches_oracle(case, generic, umma, layout):
    """Every kernel (tcgen05, mma.sync with keys or query rows on the MMA M
    dimension, CUDA-core) against the oracle."""
    Hq, Hkv, d, chunk, starts, bs, dtype = CASES[case]
    kv, ref = _build([s + chunk for s in starts], Hkv, d, bs, dtype, seed=100 + case)
    rng = np.random.default_rng(case)
    q = torch.from_numpy(rng.standard_normal((len(starts), chunk, Hq, d)).astype(np.float32)).to(DEV, dtype)
    batch = AttnBatch.from_lists(DEV, list(range(len(starts))), starts, chunk)
    kw = dict(force_generic=generic, use_umma=umma, mma_layout=layout)
    out = paged_attention(q, kv, 0, batch, **kw)
    out32 = paged_attention(q, kv, 0, batch, out_dtype=torch.float32, **kw)
    exact = oatt.paged_attention_extend(q.float().cpu().numpy(), ref, 0, range(len(starts)), starts)
    _check_bf16(out.float().cpu().numpy(), out32.cpu().numpy(), exact)
    kv.check_errors()


@pytest.mark.parametrize("pps", [1, 3, 0, 64, 12])
@pytest.mark.parametrize("heads_per_cta,umma,cluster,layout", [(0, -1, False, 1), (1, -1, False, 1),
                                                                (0, -1, True, 1), (1, -1, True, 1),
                                                                (0, 1, False, 0), (0, -1, False, 2),
                                                                (0, -1, False, 3), (2, -1, False, 3)])
def test_split_plans_agree(pps, heads_per_cta, umma, cluster, layout):
    """Every launch plan (pages per split-K CTA from 1, i.e. 150+ splits per
    row, to one split; one or two kv heads per CTA of the mma.sync kernel;
    split partials merged on chip inside a cluster (up to 16 splits) or by a
    separate launch; the tcgen05 kernel, whose 64-token tiles then end inside
    a split) gives the oracle's result for decode and verify rows."""
    kv, ref = _build([2500 + 6, 17 + 6, 900 + 6], 2, 128, 16, torch.bfloat16, seed=5)
    for chunk, starts in ((1, [2505, 22, 905]), (6, [2500, 17, 900])):
        q = torch.randn(3, chunk, 12, 128, device=DEV, dtype=torch.bfloat16)
        batch = AttnBatch.from_lists(DEV, [0, 1, 2], starts, chunk)
        out = paged_attention(q, kv, 0, batch, out_dtype=torch.float32, pages_per_split=pps,
                              kv_heads_per_cta=heads_per_cta, use_umma=umma, cluster_merge=cluster,
                              mma_layout=layout)
        exact = oatt.paged_attention_extend(q.float().cpu().numpy(), ref, 0, range(3), starts)
        check_attention_16bit(None, out.cpu().numpy(), exact)
    kv.check_errors()


@pytest.mark.parametrize("layout", [0, 1, 2, 3])
@pytest.mark.parametrize("chunk,Hq,d", [(5, 12, 128), (1, 14, 64)])
def test_ragged_plan_matches_oracle(chunk, Hq, d, layout):
    """The plan a captured model forward replays (key_count < 0: ragged rows
    of unknown lengths, grid sized by an 8192-key span bucket) on a skewed
    batch -- most rows short, a few near 4600 keys, split into up to 36
    CTAs each -- gives the oracle's result for C4's verify and draft decode
    shapes."""
    rng = np.random.default_rng(77)
    starts = [int(x) for x in np.minimum(np.floor(rng.lognormal(6, 0.8, 37)), 4096)] + [4600, 3100, 0]
    kv, ref = _build([s + chunk for s in starts], 2, d, 16, torch.bfloat16, seed=78)
    B = len(starts)
    q = torch.from_numpy(rng.standard_normal((B, chunk, Hq, d)).astype(np.float32)).to(DEV, torch.bfloat16)
    exact_batch = AttnBatch.from_lists(DEV, list(range(B)), starts, chunk)
    batch = AttnBatch(exact_batch.rows, exact_batch.starts, 8192, key_count=-1)
    out = paged_attention(q, kv, 0, batch, mma_layout=layout)
    out32 = paged_attention(q, kv, 0, batch, out_dtype=torch.float32, mma_layout=layout)
    exact = oatt.paged_attention_extend(q.float().cpu().numpy(), ref, 0, range(B), starts)
    _check_bf16(out.float().cpu().numpy(), out32.cpu().numpy(), exact)
    kv.check_errors()


@pytest.mark.parametrize("pps,chunk,cluster,layout", [(4, 1, False, 0), (0, 1, False, 0), (0, 6, True, 0),
                                                      (16, 6, True, 0), (0, 6, False, 0), (4, 6, False, 0),
                                                      (0, 6, False, 2), (4, 6, False, 2), (0, 1, False, 2),
                                                      (4, 1, False, 3), (0, 1, False, 3)])
def test_split_merge_is_deterministic(pps, chunk, cluster, layout):
    """The split-K merge (separate launch; on chip in a cluster) has a fixed
    reduction order: repeated calls give identical bits, on both mma.sync
    layouts."""
    kv, _ = _build([3000 + chunk, 1500 + chunk, 40 + chunk], 2, 128, 16, torch.bfloat16, seed=6)
    q = torch.randn(3, chunk, 12, 128, device=DEV, dtype=torch.bfloat16)
    batch = AttnBatch.from_lists(DEV, [0, 1, 2], [3000, 1500, 40], chunk)
    kw = dict(pages_per_split=pps, cluster_merge=cluster, mma_layout=layout)
    first = paged_attention(q, kv, 0, batch, **kw)
    for _ in range(5):
        assert torch.equal(paged_attention(q, kv, 0, batch, **kw), first)


def test_cluster_and_separate_merge_agree():
    """The on-chip cluster merge and the workspace merge launch combine the
    same partials: results agree to fp32 rounding, and the launch counts
    differ by the merge launch."""
    from engine.attention import attention_launches
    kv, ref = _build([4000 + 6, 2048 + 6, 31 + 6, 700 + 6], 2, 128, 16, torch.bfloat16, seed=8)
    starts = [4000, 2048, 31, 700]
    q = torch.randn(4, 6, 12, 128, device=DEV, dtype=torch.bfloat16)
    batch = AttnBatch.from_lists(DEV, [0, 1, 2, 3], starts, 6)
    on_chip = paged_attention(q, kv, 0, batch, out_dtype=torch.float32, cluster_merge=True)
    separate = paged_attention(q, kv, 0, batch, out_dtype=torch.float32)
    exact = oatt.paged_attention_extend(q.float().cpu().numpy(), ref, 0, range(4), starts)
    scale = np.abs(exact).max()
    assert np.abs(on_chip.cpu().numpy() - exact).max() <= 2e-3 * scale
    assert (on_chip - separate).abs().max().item() <= 1e-5 * scale
    assert attention_launches(q, kv, batch) == 2


def test_fp32_pools_use_exact_cuda_core_path():
    kv, ref = _build([9, 100, 1], 2, 16, 4, torch.float32, seed=9)
    q = torch.randn(3, 4, 4, 16, device=DEV)
    starts = [5, 96, 0]
    batch = AttnBatch.from_lists(DEV, [0, 1, 2], starts, 1)
    out = paged_attention(q[:, :1], kv, 0, batch)
    exact = oatt.paged_attention_extend(q[:, :1].cpu().numpy(), ref, 0, range(3), starts)
    np.testing.assert_allclose(out.cpu().numpy(), exact, rtol=1e-5, atol=1e-5)


def test_multi_layer_pool_reads_the_right_layer():
    kv, ref = _build([300, 45], 2, 128, 16, torch.bfloat16, seed=21, layers=3)
    q = torch.randn(2, 1, 12, 128, device=DEV, dtype=torch.bfloat16)
    for layer in range(3):
        out = paged_attention(q, kv, layer, AttnBatch.from_lists(DEV, [0, 1], [299, 44], 1), out_dtype=torch.float32)
        exact = oatt.paged_attention_extend(q.float().cpu().numpy(), ref, layer, range(2), [299, 44])
        assert np.abs(out.cpu().numpy() - exact).max() <= 2e-3 * np.abs(exact).max()


# ------------------------------------------------------ reference entry points
def test_decode_api_and_full_attention_match_oracle():
    kv, ref = _build([9, 10, 1, 7], 2, 8, 4, torch.float32, seed=3)
    q = torch.randn(4, 4, 8, device=DEV)
    lens = [9, 10, 1, 7]
    out = paged_attention_decode(q, kv, 0, [0, 1, 2, 3], lens, 4)
    exact = oatt.paged_attention_decode(q.cpu().numpy(), ref, 0, range(4), lens)
    np.testing.assert_allclose(out.cpu().numpy(), exact, rtol=1e-5, atol=1e-5)
    for sid in range(4):
        kvp = gather_ctx(kv, 0, sid, lens[sid])
        fo = full_attention(q[sid], kvp[0], kvp[1], 4)
        np.testing.assert_allclose(fo.cpu().numpy(), exact[sid], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("ctx", [1, 15, 16, 37, 1029])
@pytest.mark.parametrize("d", [64, 128])
def test_full_attention_dense_16bit_matches_fp32_torch(ctx, d):
    """Dense K/V of a length that is not a multiple of 16 (``full_attention``;
    at head_dim 64 the register-direct kernel, which must not load keys past
    the tensor's end) against plain fp32 torch attention with GQA 7:1."""
    g = torch.Generator().manual_seed(ctx * 7 + d)
    q = torch.randn(14, d, generator=g).to(DEV, torch.bfloat16)
    k = torch.randn(ctx, 2, d, generator=g).to(DEV, torch.bfloat16)
    v = torch.randn(ctx, 2, d, generator=g).to(DEV, torch.bfloat16)
    out = full_attention(q, k, v, 14).float()
    qf = q.float().view(2, 7, d)
    kf, vf = k.float().permute(1, 0, 2), v.float().permute(1, 0, 2)  # (2, ctx, d)
    p = torch.softmax(qf @ kf.transpose(1, 2) * d ** -0.5, dim=-1)
    ref = (p @ vf).reshape(14, d)
    assert torch.isfinite(out).all()
    assert (out - ref).abs().max().item() <= 2.0 ** -7 * ref.abs().max().item() + 2e-3


@pytest.mark.parametrize("dtype,d", [(torch.float32, 8), (torch.bfloat16, 128), (torch.bfloat16, 64)])
def test_prefill_chunk_matches_oracle_and_zeroes_padding(dtype, d):
    Hq, Hkv = (4, 2) if d == 8 else (12, 2)
    lens = [4, 6, 1] if d == 8 else [40, 77, 13]
    chunk = max(lens)
    q = torch.randn(3, chunk, Hq, d, device=DEV).to(dtype)
    k = torch.randn(3, chunk, Hkv, d, device=DEV).to(dtype)
    v = torch.randn(3, chunk, Hkv, d, device=DEV).to(dtype)
    out = paged_attention_prefill_chunk(q, k, v, Hq, lens)
    exact = oatt.paged_attention_prefill_chunk(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                               v.float().cpu().numpy(), lens)
    o = out.float().cpu().numpy()
    for b, ln in enumerate(lens):
        assert np.all(o[b, ln:] == 0.0)
    if dtype == torch.float32:
        np.testing.assert_allclose(o, exact, rtol=1e-5, atol=1e-5)
    else:
        assert np.all(np.abs(o - exact) <= 2.0 ** -8 * np.abs(exact) + 2e-3 * np.abs(exact).max())


def test_extend_matches_per_position_full_attention():
    """tests/test_paged_attention_extend.py restated: row j == full attention over start+j+1."""
    kv, ref = _build([12], 2, 16, 4, torch.float32, seed=12)
    q = torch.randn(1, 5, 4, 16, device=DEV)
    out = paged_attention_extend(q, kv, 0, [0], [7], 4)
    for j in range(5):
        kvp = gather_ctx(kv, 0, 0, 7 + j + 1)
        fo = full_attention(q[0, j], kvp[0], kvp[1], 4)
        torch.testing.assert_close(out[0, j], fo, rtol=1e-5, atol=1e-5)


# ------------------------------------------------------------ fused append
FUSED_CASES = [
    # Hq, Hkv, d, chunk, starts, valid rows, dtype, launch overrides
    (12, 2, 128, 1, [15, 16, 17, 1029, 4095], None, torch.bfloat16, {}),             # decode, page edges
    (12, 2, 128, 6, [0, 5, 250, 2047], None, torch.bfloat16, {}),                    # verify (gamma 5)
    (12, 2, 128, 6, [10, 300, 2047], None, torch.bfloat16, {"pages_per_split": 1}),  # new rows span 2 splits
    (12, 2, 128, 22, [3, 700], None, torch.bfloat16, {}),                            # 132 columns: 3 col tiles
    (14, 2, 64, 5, [0, 31, 1000], None, torch.float16, {"kv_heads_per_cta": 1}),     # fp16, d 64
    (12, 2, 128, 9, [0, 40, 91], [9, 3, 6], torch.bfloat16, {}),                      # ragged valid rows
    (12, 2, 128, 6, [5, 250], None, torch.bfloat16, {"use_umma": 1}),                # tcgen05: separate append
    (16, 2, 128, 7, [60, 4200], None, torch.bfloat16, {}),                           # auto tcgen05; rows cross a tile
    (12, 2, 128, 9, [0, 40, 91], [9, 3, 6], torch.bfloat16, {"use_umma": 1}),         # tcgen05, ragged valid rows
    (14, 2, 64, 5, [0, 31, 1000], None, torch.float16, {"use_umma": 1}),             # tcgen05, fp16, d 64
    (12, 2, 128, 6, [0, 5, 250, 2047], None, torch.bfloat16, {"mma_layout": 1}),     # keys-on-M kernel, verify
    (12, 2, 128, 22, [3, 700], None, torch.bfloat16, {"mma_layout": 1}),             # keys on M: 3 col tiles
    (12, 2, 128, 9, [0, 40, 91], [9, 3, 6], torch.bfloat16, {"mma_layout": 1}),       # keys on M, ragged rows
    (12, 2, 128, 24, [0, 37, 500], [24, 5, 17], torch.bfloat16, {"mma_layout": 2}),   # rows on M: 3 row tiles
    (12, 2, 128, 1, [15, 16, 1029], None, torch.bfloat16, {"mma_layout": 2}),        # rows on M, decode
    (12, 2, 128, 1, [15, 16, 17, 1029, 4095], None, torch.bfloat16, {"mma_layout": 3}),  # register-direct decode
    (14, 2, 64, 1, [0, 31, 1000], None, torch.float16, {"mma_layout": 3, "kv_heads_per_cta": 2}),  # fp16, d 64
    (8, 8, 128, 3, [14, 300], None, torch.bfloat16, {"mma_layout": 3, "pages_per_split": 1,
                                                      "kv_heads_per_cta": 4}),  # rows span 2 splits, 4 heads/CTA
    (4, 2, 64, 4, [0, 13, 90], [4, 1, 3], torch.bfloat16, {"mma_layout": 3}),        # register-direct, ragged rows
    (14, 2, 64, 1, [0, 15, 16, 700, 2047], None, torch.bfloat16, {"key_count": 2783}),  # 12-warp unsplit variant
    (14, 2, 64, 1, [3, 40, 1000], [1, 0, 1], torch.float16, {"key_count": 1045}),   # unsplit, an idle row
    (12, 2, 128, 6, [5, 250], None, torch.bfloat16, {"force_generic": True}),        # CUDA-core: separate append
    (4, 2, 16, 3, [0, 9, 33], None, torch.float32, {}),                              # fp32 pool: separate append
]


def _fused_pair(case, layers=2, layer=1, misalign=False):
    Hq, Hkv, d, chunk, starts, valid, dtype, kw = FUSED_CASES[case]
    kw = dict(kw)
    key_count = kw.pop("key_count", 0)
    B = len(starts)
    valid = valid or [chunk] * B
    bs = 4 if dtype == torch.float32 else 16
    pair = [_build(starts, Hkv, d, bs, dtype, seed=300 + case, extra_blocks=4 + chunk, layers=layers)[0]
            for _ in range(2)]
    slots = [kvc.reserve(list(range(B)), starts, valid) for kvc in pair]
    assert torch.equal(slots[0], slots[1])
    g = torch.Generator().manual_seed(case)
    q = torch.randn(B, chunk, Hq, d, generator=g).to(DEV, dtype)
    width = Hkv * d + (2 if misalign else 0)
    k_new = torch.randn(B * chunk, width, generator=g).to(DEV, dtype)[:, (2 if misalign else 0):]
    v_new = torch.randn(B * chunk, width, generator=g).to(DEV, dtype)[:, (2 if misalign else 0):]
    packed = _lib_i32(list(range(B)) + starts + valid)
    batch = AttnBatch(packed[:B], packed[B:2 * B], max(s + chunk for s in starts), packed[2 * B:], key_count)
    keep = torch.cat([torch.arange(b * chunk, b * chunk + valid[b]) for b in range(B)]).to(DEV)
    pair[0].append(layer, slots[0], k_new[keep].reshape(-1, Hkv, d), v_new[keep].reshape(-1, Hkv, d))
    sep = paged_attention(q, pair[0], layer, batch, **kw)
    fused = paged_attention(q, pair[1], layer, batch, k_new=k_new, v_new=v_new, **kw)
    torch.cuda.synchronize()
    return pair, sep, fused, valid


def _lib_i32(values):
    from engine import _lib
    return _lib.i32(values, DEV)


@pytest.mark.parametrize("case", range(len(FUSED_CASES)))
def test_fused_append_equals_append_then_attend(case):
    """``paged_attention(..., k_new, v_new)`` stores the new rows exactly where
    ``kv.append`` does (every layer's pool bit-identical afterwards) and
    returns the same bits as append-then-attend, on the path that writes
    inside the attention kernel and on those that launch a separate append."""
    pair, sep, fused, valid = _fused_pair(case)
    assert torch.equal(pair[0]._k, pair[1]._k)
    assert torch.equal(pair[0]._v, pair[1]._v)
    assert torch.equal(sep, fused)
    for kvc in pair:
        kvc.check_errors()


ROPE_CASES = [c for c in range(len(FUSED_CASES)) if FUSED_CASES[c][6] != torch.float32]


@pytest.mark.parametrize("case", ROPE_CASES)
def test_rope_in_launch_equals_rope_then_attend(case):
    """``paged_attention(..., rope=(cos, sin))`` on unrotated q / k_new gives
    the bits of RoPE first (the fused rope kernel, bit-exact to the
    reference's apply_rotary) and attention after: the same output and the
    same pool.  Plans whose kernel rotates inside the launch leave q and
    k_new untouched; the others rotate them in place first."""
    from engine import _lib as lib
    from engine import layer_ops
    from engine.model import make_rotary_cache

    Hq, Hkv, d, chunk, starts, valid, dtype, kw = FUSED_CASES[case]
    kw = dict(kw)
    key_count = kw.pop("key_count", 0)
    B = len(starts)
    valid = valid or [chunk] * B
    pair = [_build(starts, Hkv, d, 16, dtype, seed=400 + case, extra_blocks=4 + chunk, layers=2)[0]
            for _ in range(2)]
    for kvc in pair:
        kvc.reserve(list(range(B)), starts, valid)
    g = torch.Generator().manual_seed(1000 + case)
    q = torch.randn(B, chunk, Hq, d, generator=g).to(DEV, dtype)
    k_new = torch.randn(B * chunk, Hkv * d, generator=g).to(DEV, dtype)
    v_new = torch.randn(B * chunk, Hkv * d, generator=g).to(DEV, dtype)
    table = make_rotary_cache(d, 1e6, 8192, DEV).to(dtype)
    pos = torch.tensor([[s + j for j in range(chunk)] for s in starts], device=DEV)
    cos, sin = table[pos][:, :, 0, :], table[pos][:, :, 1, :]  # (B, chunk, d), rows 2d apart
    packed = _lib_i32(list(range(B)) + starts + valid)
    batch = AttnBatch(packed[:B], packed[B:2 * B], max(s + chunk for s in starts), packed[2 * B:], key_count)
    q_r = layer_ops.rope_(q.clone(), sin.unsqueeze(2), cos.unsqueeze(2))
    k_r = layer_ops.rope_(k_new.clone().view(B * chunk, Hkv, d), sin.reshape(-1, d), cos.reshape(-1, d))
    ref = paged_attention(q_r, pair[0], 1, batch, k_new=k_r.view(B * chunk, -1), v_new=v_new, **kw)
    q0, k0 = q.clone(), k_new.clone()
    got = paged_attention(q, pair[1], 1, batch, k_new=k_new, v_new=v_new, rope=(cos.unsqueeze(2), sin.unsqueeze(2)),
                          **kw)
    torch.cuda.synchronize()
    assert torch.equal(ref, got)
    assert torch.equal(pair[0]._k, pair[1]._k)
    assert torch.equal(pair[0]._v, pair[1]._v)
    if torch.equal(q, q0):  # rotated inside the launch: inputs only read
        assert torch.equal(k_new, k0)
    else:  # rotated in place first
        assert torch.equal(q, q_r) and torch.equal(k_new.view(B * chunk, Hkv, d), k_r)
    for kvc in pair:
        kvc.check_errors()


@pytest.mark.parametrize("chunk,Hq,d", [(1, 12, 128), (6, 12, 128), (1, 14, 64), (5, 12, 128)])
def test_overlap_layers_gives_the_same_bits(chunk, Hq, d):
    """Distinct layers launched back to back with overlap_layers (each launch
    lets the next become resident early and streams its older pages before
    waiting) store and return exactly what the plain launches do, for the
    keys-on-M and rows-on-M kernels with split merges."""
    starts = [5, 700, 1500, 2047, 31]
    layers = 4
    pair = [_build([s_ + chunk for s_ in starts], 2, d, 16, torch.bfloat16, seed=600 + chunk, layers=layers)[0]
            for _ in range(2)]
    g = torch.Generator().manual_seed(chunk * d)
    B = len(starts)
    q = torch.randn(layers, B, chunk, Hq, d, generator=g).to(DEV, torch.bfloat16)
    kn = torch.randn(layers, B * chunk, 2 * d, generator=g).to(DEV, torch.bfloat16)
    vn = torch.randn(layers, B * chunk, 2 * d, generator=g).to(DEV, torch.bfloat16)
    outs = []
    for kvc, ov in zip(pair, (False, True)):
        kvc.reserve(list(range(B)), starts, [chunk] * B)
        batch = AttnBatch.from_lists(DEV, list(range(B)), starts, chunk)
        o = torch.empty_like(q)
        for _ in range(2):  # the second pass stores the same rows again and reads them
            for layer in range(layers):
                paged_attention(q[layer], kvc, layer, batch, out=o[layer], k_new=kn[layer], v_new=vn[layer],
                                pages_per_split=8, overlap_layers=ov)
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(pair[0]._k, pair[1]._k) and torch.equal(pair[0]._v, pair[1]._v)
    for kvc in pair:
        kvc.check_errors()


def test_rope_fusion_query():
    """sdl_attention_fuses_rope: the mma.sync kernels that store the new rows
    themselves (TMA-fed or register-direct) rotate inside the launch;
    tcgen05 and CUDA-core plans do not (the Python call rotates in place
    first), and a call that asks a non-fusing plan for RoPE is refused."""
    import ctypes

    from engine import _lib as lib
    from engine.attention import _paged_args

    kv, _ = _build([100, 200], 2, 128, 16, torch.bfloat16, seed=9, layers=1)
    kn = torch.randn(10, 256, device=DEV, dtype=torch.bfloat16)
    cs = torch.randn(10, 128, device=DEV, dtype=torch.bfloat16)

    def args(chunk, **kw):
        q = torch.randn(2, chunk, 12, 128, device=DEV, dtype=torch.bfloat16)
        batch = AttnBatch.from_lists(DEV, [0, 1], [100, 200], chunk)
        a = _paged_args(q, kv, 0, batch, q, **kw)
        a.k_new, a.v_new, a.new_row_stride = kn.data_ptr(), kn.data_ptr(), 256
        a.rope_cos, a.rope_sin, a.rope_stride = cs.data_ptr(), cs.data_ptr(), 128
        return a, (q, batch)

    fuses = lambda a: lib.load().sdl_attention_fuses_rope(ctypes.byref(a))  # noqa: E731
    for layout in (0, 1, 2):  # verify block: rows or keys on M
        assert fuses(args(5, mma_layout=layout, use_umma=-1)[0]) == 1, layout
    assert fuses(args(1, mma_layout=1)[0]) == 1   # decode, keys on M
    assert fuses(args(1, mma_layout=3)[0]) == 1   # register-direct decode
    assert fuses(args(5, force_generic=True)[0]) == 0
    a, keep = args(5, use_umma=1)                  # tcgen05
    assert fuses(a) == 0
    assert lib.load().sdl_paged_attention(ctypes.byref(a), None) == 2  # SDL_ERR_UNSUPPORTED, nothing launched


def test_fused_append_unaligned_rows_fall_back_to_separate_append():
    """k_new rows that are 4- but not 16-byte aligned take the separate
    positional append and still match."""
    pair, sep, fused, _ = _fused_pair(1, misalign=True)
    assert torch.equal(pair[0]._k, pair[1]._k)
    assert torch.equal(pair[0]._v, pair[1]._v)
    assert torch.equal(sep, fused)


def test_fused_append_rejects_bad_rows():
    kv, _ = _build([40], 2, 128, 16, torch.bfloat16, seed=1)
    kv.reserve([0], [40], [1])
    q = torch.randn(1, 1, 12, 128, device=DEV, dtype=torch.bfloat16)
    batch = AttnBatch.from_lists(DEV, [0], [40], 1)
    with pytest.raises(ValueError):
        paged_attention(q, kv, 0, batch, k_new=torch.zeros(1, 255, device=DEV, dtype=torch.bfloat16),
                        v_new=torch.zeros(1, 255, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(ValueError):
        paged_attention(q, kv, 0, batch, k_new=torch.zeros(1, 256, device=DEV),
                        v_new=torch.zeros(1, 256, device=DEV))


def test_automatic_kernel_choice():
    """use_umma=0 picks the tcgen05 kernel for verify blocks of 48+ query
    rows per kv head over a mean span of 4096+ keys, the rows-on-M mma.sync
    kernel for shorter blocks of 48+ rows per kv head (16+ at head_dim 64;
    24+ at head_dim 128 over a mean span below 1024 keys), the keys-on-M one
    for decode and smaller blocks, and the CUDA-core kernel for fp32 pools;
    the explicit flags override it."""
    from engine.attention import attention_kernel
    kv, _ = _build([4200 + 7, 4100 + 7], 2, 128, 16, torch.bfloat16, seed=31)
    long_verify = AttnBatch.from_lists(DEV, [0, 1], [4200, 4100], 7)
    short_verify = AttnBatch.from_lists(DEV, [0, 1], [1000, 300], 7)
    q7 = torch.zeros(2, 7, 16, 128, device=DEV, dtype=torch.bfloat16)
    q1 = torch.zeros(2, 1, 16, 128, device=DEV, dtype=torch.bfloat16)
    assert attention_kernel(q7, kv, long_verify) == "tcgen05"
    assert attention_kernel(q7, kv, long_verify, use_umma=-1) == "mma_rows"   # 56 rows per kv head
    assert attention_kernel(q7, kv, short_verify) == "mma_rows"
    assert attention_kernel(q7, kv, short_verify, mma_layout=1) == "mma"
    assert attention_kernel(q7, kv, short_verify, use_umma=1) == "tcgen05"
    q6 = torch.zeros(2, 6, 12, 128, device=DEV, dtype=torch.bfloat16)            # 36 rows: keys on M
    assert attention_kernel(q6, kv, AttnBatch.from_lists(DEV, [0, 1], [1400, 1100], 6)) == "mma"
    assert attention_kernel(q6, kv, AttnBatch.from_lists(DEV, [0, 1], [1000, 300], 6)) == "mma_rows"  # short spans
    assert attention_kernel(q7, kv, AttnBatch.from_lists(DEV, [0, 1], [4200, 300], 7)) == "mma_rows"  # mean 2257
    assert attention_kernel(q1, kv, AttnBatch.from_lists(DEV, [0, 1], [4206, 306], 1)) == "mma"
    assert attention_kernel(q1, kv, AttnBatch.from_lists(DEV, [0, 1], [4206, 306], 1), mma_layout=2) == "mma_rows"
    kv32, _ = _build([40], 2, 16, 4, torch.float32, seed=32)
    assert attention_kernel(torch.zeros(1, 1, 4, 16, device=DEV), kv32, AttnBatch.from_lists(DEV, [0], [39], 1)) == "generic"
