"""One whole C3 verify step at the benchmark's own size against the oracle.

C3 (gamma = 5, batch 32, contexts U[256, 2048], Qwen2.5-1.5B attention shapes,
vocab 151,936, temperature 1.0, logits N(0, 2)) is the step ``bench.py
--workload c3`` times: reserve gamma+1 positions per sequence, 28 layers of
fused K/V append + verify attention, the logits-in rejection sampler and the
device commit that rewinds every block table to its accept length.  The
inputs below are built exactly as the benchmark builds them (same seeds, the
same random-permutation pool); the step runs through the same public calls,
and every stage is compared with the oracle:

* the slots of the reservation and the K/V rows the fused append stores (bit
  for bit) and all 28 layers' attention outputs (``check_attention_16bit``);
* accept lengths and tokens: ``oracle.sampler.batch_accept`` restating
  engine/spec_scheduler.py:46-88 on the same fp32 uniforms -- bit-exact;
* block tables, lengths and the free list after the commit: the oracle's
  ``truncate`` to ``start + accepted`` (engine/kv.py:150-162) in batch
  order -- bit-exact.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import check_attention_16bit
from engine import _lib
from engine.attention import AttnBatch, paged_attention
from engine.kv import PagedKVCache
from engine.workloads import C3, c2_layout
from oracle import attention as oatt
from oracle import kv as okv
from oracle import sampler as osamp
from specdec.sampler import UniformStream, probs_rows, sample_rows, spec_sample_logits

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("seed", [0, 1])
def test_c3_verify_step_matches_oracle_at_bench_size(seed):
    L, B, gam = 28, C3["batch"], C3["gamma"]
    chunk = gam + 1
    Hq, Hkv, d, bs, V, T = 12, 2, 128, 16, C3["vocab"], C3["temperature"]
    ctx, _, _ = c2_layout(seed, B, C3["ctx_lo"], C3["ctx_hi"], bs)
    cap = sum(-(-(x + chunk) // bs) for x in ctx) + B
    kv = PagedKVCache(L, Hkv, d, cap, bs, DEV, torch.bfloat16,
                      max_blocks_per_seq=-(-(C3["ctx_hi"] + chunk + 1) // bs), max_seqs=B)
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    perm = torch.randperm(cap, generator=g).to(torch.int32)
    kv.allocator._free_stack.copy_(perm)
    ref = okv.PagedKVCache(1, Hkv, d, cap, bs)
    ref.allocator._free = [int(x) for x in perm.tolist()]
    ref.allocator._free_set = set(ref.allocator._free)
    sids = list(range(B))
    for sid in sids:
        kv.add_sequence(sid)
        ref.add_sequence(sid)
    kv.reserve(sids, [0] * B, ctx)
    ref.reserve(sids, [0] * B, ctx)
    assert kv.block_tables == ref.block_tables
    gd = torch.Generator(device=DEV)
    gd.manual_seed(seed)
    kv._k.normal_(generator=gd)
    kv._v.normal_(generator=gd)
    q = torch.randn((L, B, chunk, Hq, d), generator=gd, device=DEV).to(torch.bfloat16)
    knew = torch.randn((L, B * chunk, Hkv, d), generator=gd, device=DEV).to(torch.bfloat16)
    vnew = torch.randn((L, B * chunk, Hkv, d), generator=gd, device=DEV).to(torch.bfloat16)
    p_logits = torch.randn((B, chunk, V), generator=gd, device=DEV) * C3["logit_std"]
    q_logits = torch.randn((B, gam, V), generator=gd, device=DEV) * C3["logit_std"]
    proposals = sample_rows(probs_rows(q_logits, T, False), UniformStream(DEV, seed=seed + 7)).view(B, gam)
    ustream = UniformStream(DEV, seed=seed + 11)
    uniforms = ustream.buffer[: 4 * B * chunk].cpu().numpy()
    k_before = kv._k.clone()
    v_before = kv._v.clone()

    # ---- the step, through the benchmark's calls
    slots = kv.reserve(sids, ctx, [chunk] * B)
    want_slots = ref.reserve(sids, ctx, [chunk] * B)
    assert slots.tolist() == want_slots
    batch = AttnBatch.from_lists(DEV, sids, ctx, chunk)
    out = torch.empty((L, B, chunk, Hq, d), device=DEV, dtype=torch.bfloat16)
    for layer in range(L):
        paged_attention(q[layer], kv, layer, batch, out=out[layer], k_new=knew[layer], v_new=vnew[layer])
    out32 = torch.empty((L, B, chunk, Hq, d), device=DEV, dtype=torch.float32)
    for layer in range(L):  # the rows are stored already: same K/V, fp32 output
        paged_attention(q[layer], kv, layer, batch, out=out32[layer])
    tokens = torch.empty((B, chunk), dtype=torch.int32, device=DEV)
    n_out = torch.empty(B, dtype=torch.int32, device=DEV)
    spec_sample_logits(p_logits, q_logits, T, proposals, ustream, err=kv.err_word, out=(tokens, n_out))
    packed = _lib.i32(sids + [1 << 30] * B + ctx, DEV)
    outs = torch.empty((3, B), dtype=torch.int32, device=DEV)
    _lib.check(_lib.load().sdl_spec_commit(
        ctypes.byref(kv.meta), None, B, packed.data_ptr(), n_out.data_ptr(), tokens.data_ptr(), chunk,
        packed.data_ptr() + 4 * B, -1, packed.data_ptr() + 8 * B, outs[0].data_ptr(), outs[1].data_ptr(),
        outs[2].data_ptr(), _lib.stream_handle(DEV)), "sdl_spec_commit")
    torch.cuda.synchronize(DEV)
    kv.check_errors()

    # ---- attention and the fused append, layer by layer
    slot_t = torch.tensor(want_slots, dtype=torch.long, device=DEV)
    untouched = torch.ones(cap * bs, dtype=torch.bool, device=DEV)
    untouched[slot_t] = False
    for layer in range(L):
        for pool, before, new in ((kv._k, k_before, knew), (kv._v, v_before, vnew)):
            flat = pool[layer].reshape(cap * bs, Hkv, d)
            assert torch.equal(flat[slot_t], new[layer])
            assert torch.equal(flat[untouched], before[layer].reshape(cap * bs, Hkv, d)[untouched])
        ref.k[0] = k_before[layer].float().cpu().numpy()
        ref.v[0] = v_before[layer].float().cpu().numpy()
        ref.append(0, want_slots, knew[layer].float().cpu().numpy(), vnew[layer].float().cpu().numpy())
        exact = oatt.paged_attention_extend(q[layer].float().cpu().numpy(), ref, 0, sids, ctx)
        check_attention_16bit(out[layer].float().cpu().numpy(), out32[layer].cpu().numpy(), exact)

    # ---- sampler: accept lengths and tokens
    pn = osamp.logits_to_probs(p_logits.cpu().numpy(), T)
    qn = osamp.logits_to_probs(q_logits.cpu().numpy(), T)
    props = proposals.cpu().tolist()
    want = osamp.batch_accept([pn[b] for b in range(B)], [[qn[b, j] for j in range(gam)] for b in range(B)],
                              props, osamp.UniformStream(uniforms))
    n = n_out.tolist()
    tk = tokens.tolist()
    assert [tk[b][: n[b]] for b in range(B)] == want
    assert outs[0].tolist() == n  # committed counts (no budget clip, no EOS)

    # ---- commit: rewind to start + accepted, pushes in batch order
    for b, sid in enumerate(sids):
        ref.truncate(sid, ctx[b] + len(want[b]))
    kv.resync()
    assert kv.block_tables == ref.block_tables
    assert kv.seq_lengths == ref.seq_lengths
    assert kv.allocator.free_list() == ref.allocator.free_list()
