"""Paged-KV storage on the GPU vs the reference fixtures and the oracle.

Bit-exact: block tables, free-list order, sequence lengths, slots, allocated
counts.  Covers the reference's own kv tests (tests/test_kv.py,
tests/test_spec_accept.py:76-98) through the drop-in API, plus the batched
kernels (reserve, release, spec commit) against the oracle's sequential
restatement.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_json
from engine import _lib
from engine.attention import gather_ctx
from engine.kv import BlockAllocator, BlockExhaustedError, PagedKVCache
from oracle import kv as okv

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _kv(block_size=4, capacity=8, layers=2, heads=2, d=8, dtype=torch.float32) -> PagedKVCache:
    return PagedKVCache(layers, heads, d, capacity, block_size, DEV, dtype)


def _vec(fill=1.0, d=8):
    return torch.full((2, d), fill, dtype=torch.float32, device=DEV)


def _assert_same_state(kv: PagedKVCache, ref: okv.PagedKVCache):
    assert kv.block_tables == ref.block_tables
    assert list(kv.seq_lengths) == ref.seq_lengths
    assert kv.num_allocated_blocks == ref.num_allocated_blocks
    dev = kv.device_state()
    assert dev["free_list"] == ref.allocator.free_list()
    assert dev["seq_lens"] == ref.seq_lengths
    assert dev["num_blocks"] == [len(t) for t in ref.block_tables]


# ------------------------------------------------------------ fixture replay
def test_kv_trace_replay_matches_reference():
    g = load_json("kv_trace.json")
    c = g["config"]
    kv = PagedKVCache(c["num_layers"], c["num_kv_heads"], c["head_dim"], c["capacity"], c["block_size"], DEV,
                      torch.float32)
    rng = np.random.default_rng(7)
    for step in g["ops"]:
        op = step["op"]
        if op[0] == "add":
            kv.add_sequence(op[1])
        elif op[0] == "write":
            vec = torch.from_numpy(rng.standard_normal((2, 8)).astype(np.float32)).to(DEV)
            kv.write(0, op[1], op[2], vec, vec)
        elif op[0] == "truncate":
            kv.truncate(op[1], op[2])
        elif op[0] == "clear":
            kv.clear(op[1])
        elif op[0] == "reset":
            kv.reset()
        st = step["state"]
        assert kv.block_tables == st["block_tables"], op
        assert list(kv.seq_lengths) == st["seq_lengths"], op
        assert kv.num_allocated_blocks == st["num_allocated"], op
        assert kv.allocator.free_list() == st["free_list"], op
    kv.check_errors()


def test_exhaustion_raises_reference_message_before_touching_state():
    g = load_json("kv_trace.json")
    kv = PagedKVCache(1, 1, 8, 3, 4, DEV, torch.float32)
    kv.add_sequence(0)
    for pos in range(12):
        kv.write(0, 0, pos, torch.zeros(1, 8, device=DEV), torch.zeros(1, 8, device=DEV))
    before = kv.block_tables
    with pytest.raises(BlockExhaustedError) as e:
        kv.write(0, 0, 12, torch.zeros(1, 8, device=DEV), torch.zeros(1, 8, device=DEV))
    assert str(e.value) == g["exhaustion_message"]
    assert kv.block_tables == before
    kv.check_errors()


# ------------------------------------------------ reference tests/test_kv.py
def test_allocator_alloc_free_roundtrip():
    a = BlockAllocator(capacity=4, device=DEV, dtype=torch.float32)
    blocks = [a.alloc() for _ in range(4)]
    assert blocks == [3, 2, 1, 0]
    assert a.num_allocated == 4
    a.free(blocks[0])
    a.free(blocks[1])
    assert a.num_allocated == 2
    blocks.extend([a.alloc(), a.alloc()])
    assert blocks[-2:] == [2, 3]
    assert a.num_allocated == 4


def test_allocator_exhaustion_raises_then_recovers():
    a = BlockAllocator(capacity=2, device=DEV, dtype=torch.float32)
    a.alloc()
    a.alloc()
    with pytest.raises(BlockExhaustedError):
        a.alloc()
    a.free(0)
    assert a.alloc() == 0


def test_allocator_free_twice_is_idempotent():
    a = BlockAllocator(capacity=3, device=DEV, dtype=torch.float32)
    b = a.alloc()
    a.free(b)
    a.free(b)
    assert a.num_allocated == 0
    assert a.free_list() == [0, 1, 2]


def test_capacity_must_be_positive():
    with pytest.raises(ValueError, match="capacity_blocks must be >= 1"):
        BlockAllocator(capacity=0, device=DEV, dtype=torch.float32)


def test_write_allocates_blocks_on_demand():
    kv = _kv()
    kv.add_sequence(0)
    kv.write(0, 0, 0, _vec(), _vec())
    assert kv.seq_lengths[0] == 1 and kv.num_allocated_blocks == 1
    kv.write(0, 0, 2, _vec(), _vec())
    assert kv.num_allocated_blocks == 1 and kv.seq_lengths[0] == 3
    kv.write(0, 0, 4, _vec(), _vec())
    assert kv.num_allocated_blocks == 2 and len(kv.block_tables[0]) == 2


def test_write_out_of_order_extends_length():
    kv = _kv()
    kv.add_sequence(0)
    kv.write(0, 0, 3, _vec(3.0), _vec(3.0))
    assert kv.seq_lengths[0] == 4 and kv.logical_tokens == 4


def test_gather_concatenates_blocks_in_order():
    kv = _kv()
    kv.add_sequence(0)
    for pos in range(9):
        kv.write(0, 0, pos, _vec(float(pos)), _vec(-float(pos)))
    stacked = gather_ctx(kv, 0, 0, 9)
    assert stacked.shape == (2, 9, 2, 8)
    assert torch.equal(stacked[0, 3], torch.full((2, 8), 3.0, device=DEV))
    assert torch.equal(stacked[1, 8], torch.full((2, 8), -8.0, device=DEV))


def test_truncate_rollback_frees_blocks_and_reuses_them():
    kv = _kv()
    kv.add_sequence(0)
    kv.add_sequence(1)
    for pos in range(10):
        kv.write(0, 0, pos, _vec(), _vec())
    before = kv.num_allocated_blocks
    kv.truncate(0, 3)
    assert kv.seq_lengths[0] == 3 and len(kv.block_tables[0]) == 1
    assert kv.num_allocated_blocks < before
    kv.write(0, 1, 4, _vec(), _vec())
    assert kv.seq_lengths[1] == 5 and len(kv.block_tables[1]) == 2


def test_truncate_rewound_sequence_writes_identically():
    kv = _kv()
    kv.add_sequence(0)
    for pos in range(8):
        kv.write(0, 0, pos, _vec(pos + 0.5), _vec())
    kv.truncate(0, 2)
    for pos in range(2, 8):
        kv.write(0, 0, pos, _vec(pos + 0.5), _vec())
    assert torch.equal(gather_ctx(kv, 0, 0, 8)[0][5], torch.full((2, 8), 5.5, device=DEV))


def test_clear_and_reset():
    kv = _kv()
    kv.add_sequence(0)
    kv.add_sequence(1)
    for pos in range(6):
        kv.write(0, 0, pos, _vec(), _vec())
    kv.write(0, 1, 1, _vec(), _vec())
    kv.clear(0)
    assert kv.block_tables[0] == [] and kv.seq_lengths[0] == 0
    assert kv.num_allocated_blocks == 1
    k_obj = kv._k
    kv.reset()
    assert kv.num_sequences == 0 and kv.num_allocated_blocks == 0 and kv._k is k_obj


def test_block_utilization_metric():
    kv = _kv()
    kv.add_sequence(0)
    kv.write(0, 0, 0, _vec(), _vec())
    assert kv.block_utilization == pytest.approx(0.25)
    kv.write(0, 0, 1, _vec(), _vec())
    assert kv.block_utilization == pytest.approx(0.5)


def test_truncate_releases_exactly_two_blocks():
    kv = _kv(capacity=32)
    kv.add_sequence(0)
    for pos in range(10):
        kv.write(0, 0, pos, torch.randn(2, 8, device=DEV), torch.randn(2, 8, device=DEV))
    full = kv.num_allocated_blocks
    kv.truncate(0, 4)
    assert kv.seq_lengths[0] == 4 and full - kv.num_allocated_blocks == 2 and kv.num_allocated_blocks == 1


# ------------------------------------------------------- batched kernels
def test_batched_reserve_append_and_release_match_oracle():
    rng = np.random.default_rng(3)
    bs, cap, L, H, d = 16, 400, 2, 2, 64
    kv = PagedKVCache(L, H, d, cap, bs, DEV, torch.bfloat16)
    ref = okv.PagedKVCache(L, H, d, cap, bs)
    lens = [0] * 24
    for sid in range(24):
        kv.add_sequence(sid)
        ref.add_sequence(sid)
    for rnd in range(40):
        n = int(rng.integers(1, 12))
        sids = sorted(rng.choice(24, size=n, replace=False).tolist())
        starts = [lens[s] for s in sids]
        counts = [int(rng.integers(0, 20)) for _ in sids]
        if sum(-(-(st + c) // bs) - len(ref.block_tables[s]) for s, st, c in zip(sids, starts, counts)
               if c > 0 and -(-(st + c) // bs) > len(ref.block_tables[s])) > len(ref.allocator._free):
            continue
        slots = kv.reserve(sids, starts, counts).tolist()
        want = ref.reserve(sids, starts, counts)
        assert slots == want
        T = len(want)
        if T:
            k = torch.randn(T, H, d, device=DEV, dtype=torch.bfloat16)
            v = torch.randn(T, H, d, device=DEV, dtype=torch.bfloat16)
            layer = rnd % L
            kv.append(layer, torch.tensor(slots, dtype=torch.int32, device=DEV), k, v)
            ref.append(layer, want, k.float().cpu().numpy(), v.float().cpu().numpy())
        for s, st, c in zip(sids, starts, counts):
            if c > 0:
                lens[s] = max(lens[s], st + c)
        # random rewinds / clears in one batched release (list order matters)
        m = int(rng.integers(0, 6))
        rel = rng.choice(24, size=m, replace=False).tolist()
        new_lens, flags = [], []
        for s in rel:
            kind = int(rng.integers(0, 3))
            if kind == 0:
                nl = int(rng.integers(0, lens[s] + 1))
                new_lens.append(nl)
                flags.append(_lib.REL_TRUNCATE)
                ref.truncate(s, nl)
                lens[s] = nl
            elif kind == 1:
                new_lens.append(0)
                flags.append(_lib.REL_CLEAR)
                ref.clear(s)
                lens[s] = 0
            else:
                nl = int(rng.integers(0, lens[s] + 1))
                new_lens.append(nl)
                flags.append(_lib.REL_TRUNCATE | _lib.REL_CLEAR)
                ref.truncate(s, nl)
                ref.clear(s)
                lens[s] = 0
        kv.release(rel, new_lens, flags)
        _assert_same_state(kv, ref)
    kv.check_errors()
    np.testing.assert_array_equal(kv._k.float().cpu().numpy(), ref.k)
    np.testing.assert_array_equal(kv._v.float().cpu().numpy(), ref.v)


def _oracle_commit(tk, dk, sids, n_out, tokens, remaining, eos, starts, prompt_len, gen_len):
    """engine/spec_scheduler.py:270-322 on oracle caches (allocation only)."""
    ks, flags, catch = [], [], []
    for b, sid in enumerate(sids):
        acc = list(tokens[b][: n_out[b]])
        if len(acc) > remaining[b]:
            acc = acc[: remaining[b]]
        eos_hit = False
        if eos >= 0:
            for i, t in enumerate(acc):
                if t == eos:
                    acc = acc[:i]
                    eos_hit = True
                    break
        k = len(acc)
        fin = eos_hit or k == 0 or k >= remaining[b]
        slot = -1
        if k > 0:
            keep = starts[b] + k
            tk.truncate(sid, keep)
            d_len = dk.seq_lengths[sid]
            if d_len > keep:
                dk.truncate(sid, keep)
            elif d_len < keep:
                slot = dk.slot(sid, d_len)
        if fin:
            tk.clear(sid)
            dk.clear(sid)
            slot = -1
        ks.append(k)
        flags.append(int(fin) | (int(eos_hit) << 1))
        catch.append(slot)
    return ks, flags, catch


def test_spec_commit_kernel_matches_reference_commit_order():
    import ctypes

    rng = np.random.default_rng(11)
    bs, cap, gamma = 4, 300, 3
    tk = PagedKVCache(1, 1, 8, cap, bs, DEV, torch.float32)
    dk = PagedKVCache(1, 1, 8, cap, bs, DEV, torch.float32)
    rt, rd = okv.PagedKVCache(1, 1, 8, cap, bs, store=False), okv.PagedKVCache(1, 1, 8, cap, bs, store=False)
    B = 10
    for sid in range(B):
        for c in (tk, dk, rt, rd):
            c.add_sequence(sid)
    plen = [int(rng.integers(3, 9)) for _ in range(B)]
    alive = list(range(B))
    gen = [1] * B
    tk.reserve(alive, [0] * B, [p for p in plen])
    dk.reserve(alive, [0] * B, [p for p in plen])
    rt.reserve(alive, [0] * B, plen)
    rd.reserve(alive, [0] * B, plen)
    for rnd in range(12):
        if not alive:
            break
        sids = list(alive)
        starts = [rt.seq_lengths[s] for s in sids]
        d0 = [rd.seq_lengths[s] for s in sids]
        for t in range(gamma):  # draft writes gamma positions, target gamma+1
            dk.reserve(sids, [d + t for d in d0], [1] * len(sids))
            rd.reserve(sids, [d + t for d in d0], [1] * len(sids))
        tk.reserve(sids, starts, [gamma + 1] * len(sids))
        rt.reserve(sids, starts, [gamma + 1] * len(sids))
        n = len(sids)
        n_out = [int(rng.integers(1, gamma + 2)) for _ in sids]
        toks = rng.integers(0, 6, size=(n, gamma + 1)).tolist()
        remaining = [int(rng.integers(1, 8)) for _ in sids]
        eos = 5
        want = _oracle_commit(rt, rd, sids, n_out, toks, remaining, eos, starts, plen, gen)
        packed = _lib.i32(sids + remaining + starts, DEV)
        tok_t = torch.tensor(toks, dtype=torch.int32, device=DEV)
        nout_t = torch.tensor(n_out, dtype=torch.int32, device=DEV)
        outs = torch.empty((3, n), dtype=torch.int32, device=DEV)
        _lib.check(_lib.load().sdl_spec_commit(
            ctypes.byref(tk.meta), ctypes.byref(dk.meta), n, packed.data_ptr(), nout_t.data_ptr(), tok_t.data_ptr(),
            gamma + 1, packed.data_ptr() + 4 * n, eos, packed.data_ptr() + 8 * n, outs[0].data_ptr(),
            outs[1].data_ptr(), outs[2].data_ptr(), _lib.stream_handle(DEV)), "commit")
        got = outs.tolist()
        assert got[0] == want[0] and got[1] == want[1] and got[2] == want[2]
        for c in (tk, dk):
            c.allocator.resync()
            c._mirror = None
        assert tk.device_state()["free_list"] == rt.allocator.free_list()
        assert dk.device_state()["free_list"] == rd.allocator.free_list()
        assert tk.device_state()["seq_lens"] == rt.seq_lengths
        assert dk.device_state()["seq_lens"] == rd.seq_lengths
        tk._h_len = list(rt.seq_lengths)
        tk._h_nb = [len(t) for t in rt.block_tables]
        dk._h_len = list(rd.seq_lengths)
        dk._h_nb = [len(t) for t in rd.block_tables]
        assert tk.block_tables == rt.block_tables and dk.block_tables == rd.block_tables
        alive = [s for s, f in zip(sids, want[1]) if not f & 1]
    tk.check_errors()
    dk.check_errors()
