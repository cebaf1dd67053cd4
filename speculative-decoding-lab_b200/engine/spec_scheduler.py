"""Speculative decoding fused into the continuous-batching engine, on B200.

Drop-in for the reference's ``engine/spec_scheduler.py``
(engine/spec_scheduler.py:41-322).  Cache invariant per model, unchanged:
``kv.seq_lengths[sid] == len(prompt) + len(generated) - 1``.

One round (``_spec_step``) is, on the device:

1. ``gamma`` batched draft decodes; each picks its proposals in-kernel
   (argmax, or temperature softmax + one uniform per sequence);
2. one batched target ``decode_block`` over ``[pending] + proposals``;
3. the fused rejection sampler (``sdl_spec_sample_logits``, straight from
   the target and draft logits): fp64 ``min(1, p/q)`` tests against the
   stream's uniforms in the reference's draw order, the residual ``(p - q)+``
   or bonus draw, accept lengths (with top-k / top-p filtering the
   probability rows are materialised and ``sdl_spec_sample`` runs instead);
4. ``sdl_spec_commit``: budget clip, EOS cut, rewind of the target cache to
   ``start + k`` and alignment of the draft cache (truncate, or reserve the
   single catch-up position), clears of finished sequences -- walked in batch
   order so both free lists see the reference's push/pop order.

The host then reads one packed int32 tensor (tokens, counts, flags, error
words) to update the Python ``Sequence`` records and runs the batched draft
catch-up decode for sequences that accepted everything plus the bonus.
"""

from __future__ import annotations

import ctypes
import time
from typing import Any, Callable, Dict, List, Optional, Sequence as Seq

import torch

from . import _lib
from .config import EngineConfig, SamplingConfig, WorkloadRequest
from .attention import AttnBatch
from .kv import PagedKVCache, _exhausted
from .scheduler import PagedScheduler, SchedulerResult, Sequence
from .utils import Stopwatch, setup_logger, sync_device
from specdec.sampler import (
    UniformStream,
    apply_top_k,
    apply_top_p,
    argmax_rows,
    probs_rows,
    sample_logits_rows,
    sample_rows,
    spec_sample,
    spec_sample_logits,
)

logger = setup_logger(__name__)


class _DraftLoop:
    """The gamma draft steps of a round as one CUDA graph, for one (batch
    bucket, draft key-span bucket): per step the reserve of one position per
    row (``sdl_kv_reserve`` on device rows / starts / counts), the draft
    forward, its LM head into step t's slice of the round buffer, the draw
    (``sdl_sample_logits_rows``, then the uniform counter advances by the
    batch size on the device) or the argmax, and the next step's input ids
    -- no host work between the steps.  (The reference captures one draft
    step, specdec/graph_draft.py:70-110.)

    Rows past the batch repeat row 0 with a count of 0 (nothing reserved);
    their ids are reset to row 0's after every step, so the K/V rows they
    store are row 0's own bytes.  Their draws read uniforms past the batch's,
    inside the stream storage's capacity, and are discarded."""

    EXTRA_FIELDS = 0  # per-row int32 fields staged between the ids and the batch size

    def __init__(self, sched: "SpeculativePagedScheduler", bucket: int, span: int, greedy: bool) -> None:
        draft, kv = sched.draft_model, sched.draft_kv
        dev = draft.device
        g = sched.gamma
        W = draft.lm_head.weight
        V = W.shape[0]
        self.bucket, self.span, self.greedy, self.gamma = bucket, span, greedy, g
        b = bucket
        self.n_off = (4 + self.EXTRA_FIELDS) * b  # meta: rows | d0 | counts | ids | extra fields | batch size
        self.meta_h = torch.zeros(self.n_off + 1, dtype=torch.int32).pin_memory()
        self.meta = torch.zeros(self.n_off + 1, dtype=torch.int32, device=dev)
        self.props = torch.zeros((g, b), dtype=torch.int32, device=dev)
        self.q = sched._loop_q_buffer(V, W.dtype, dev)  # (gamma, rows, V): the round buffer
        self.slots = torch.zeros(b, dtype=torch.int32, device=dev)
        self.draft, self.kv, self.W, self.V = draft, kv, W, V
        self.ws = None
        self.temp = float(sched.sampling.temperature)
        if not greedy:
            need = int(_lib.load().sdl_sampler_workspace_bytes(b, V))
            self.ws = _lib.Workspace.get(dev, need, tag="sampler")
            self.ubuf, self.ucnt = sched._u_storage
        self.graph = None
        self.calls = 0

    def _run(self) -> None:
        """The loop body (a method, not a closure: the loop holds its graph,
        and a reference cycle through it would let the garbage collector
        destroy a graph while another capture is open)."""
        lib, b, g, V, kv = _lib.load(), self.bucket, self.gamma, self.V, self.kv
        meta = self.meta
        rows, d0, counts = meta[:b], meta[b:2 * b], meta[2 * b:3 * b]
        keep = counts > 0
        n64 = meta[self.n_off:self.n_off + 1].to(torch.int64)
        cur = meta[3 * b:4 * b].to(torch.int64)
        for t in range(g):
            starts = d0 + t
            _lib.check(lib.sdl_kv_reserve(ctypes.byref(kv._meta), b, rows.data_ptr(), starts.data_ptr(),
                                          counts.data_ptr(), self.slots.data_ptr(), kv._stream()), "sdl_kv_reserve")
            batch = AttnBatch(rows, starts, self.span, key_count=-1)
            normed = self.draft._body(cur.view(b, 1), kv, batch, starts.to(torch.int64).unsqueeze(1))
            logits = self.q[t, :b]
            torch.matmul(normed, self.W.t(), out=logits.view(b, 1, V))
            if self.greedy:
                self.props[t].copy_(argmax_rows(logits))
            else:
                _lib.check(lib.sdl_sample_logits_rows(
                    logits.data_ptr(), _lib.dtype_code(logits.dtype), logits.stride(0), b, V, self.temp, 1e-12,
                    self.ubuf.data_ptr(), self.ubuf.numel(), self.ucnt.data_ptr(), 0, self.props[t].data_ptr(),
                    self.ws.data_ptr(), self.ws.numel() * 4, kv.err_word.data_ptr(), _lib.stream_handle(meta.device)),
                    "sdl_sample_logits_rows")
                self.ucnt.add_(n64)
            nxt = self.props[t].to(torch.int64)
            cur = torch.where(keep, nxt, nxt[:1])

    def capture(self, sids: List[int], d0: List[int], last: List[int]) -> None:
        """One eager pass over the staged scratch rows (it reserves their
        positions and, sampling, advances the uniform counter: the caller
        undoes both), then the capture."""
        self.stage(sids, d0, last)
        self._run()
        torch.cuda.synchronize(self.meta.device)
        self.graph = torch.cuda.CUDAGraph()
        c0 = _lib.calls()
        with _lib.no_gc(), torch.cuda.graph(self.graph, pool=self.draft._graph_pool()):
            self._run()
        self.calls = _lib.calls() - c0

    def stage(self, sids: List[int], d0: List[int], last: List[int]) -> None:
        """Fill the static inputs (one pinned host-to-device copy)."""
        b, B = self.bucket, len(sids)
        m = self.meta_h.numpy()
        m[0:B] = sids
        m[B:b] = sids[0]
        m[b:b + B] = d0
        m[b + B:2 * b] = d0[0]
        m[2 * b:2 * b + B] = 1
        m[2 * b + B:3 * b] = 0
        m[3 * b:3 * b + B] = last
        m[3 * b + B:4 * b] = last[0]
        m[self.n_off] = B
        self._stage_extra(m, B)
        self.meta.copy_(self.meta_h, non_blocking=True)

    def _stage_extra(self, m, B: int) -> None:
        """Fill the subclass's extra per-row fields of the pinned staging row."""

    def replay(self) -> None:
        self.graph.replay()
        _lib.count_calls(self.calls)


class _RoundGraph(_DraftLoop):
    """A whole speculative round as one CUDA graph, for one (batch bucket,
    key-span bucket of both caches): the captured draft loop, then the
    target's reserve of gamma+1 positions per row, its verify forward over
    [last token | proposals] with the head into the verify logits buffer,
    the rejection sampling (``sdl_spec_sample_logits_n``, or the argmax
    chain when greedy) and the device commit (``sdl_spec_commit_n``) -- both
    stop at the staged batch size, so padding rows consume no uniforms and
    commit nothing, and padding rows verify row 0's proposals, so what they
    store at row 0's positions is row 0's own K/V.  The host stages one
    pinned row, replays, and reads the packed results once, as the
    step-by-step round does."""

    EXTRA_FIELDS = 3  # target start, target count, remaining budget

    def __init__(self, sched: "SpeculativePagedScheduler", bucket: int, span: int, greedy: bool) -> None:
        super().__init__(sched, bucket, span, greedy)
        dev = self.meta.device
        b, g = bucket, sched.gamma
        self.target, self.tkv = sched.model, sched.kv
        self.Wt = sched.model.lm_head.weight
        self.eos = -1 if sched._eos is None else int(sched._eos)
        self.tslots = torch.zeros(b * (g + 1), dtype=torch.int32, device=dev)
        self.tokens = torch.zeros((b, g + 1), dtype=torch.int32, device=dev)
        self.n_out = torch.zeros(b, dtype=torch.int32, device=dev)
        self.outs = torch.zeros((3, b), dtype=torch.int32, device=dev)
        self.steps = torch.arange(g + 1, device=dev)
        if not greedy:
            V = self.Wt.shape[0]
            need = int(_lib.load().sdl_sampler_workspace_bytes(b * (2 * g + 1), V))
            self.sws = _lib.Workspace.get(dev, need, tag="sampler")

    def _stage_extra(self, m, B: int) -> None:
        b = self.bucket
        m[4 * b:4 * b + B] = self._tstart
        m[4 * b + B:5 * b] = self._tstart[0]
        m[5 * b:5 * b + B] = self.gamma + 1
        m[5 * b + B:6 * b] = 0
        m[6 * b:6 * b + B] = self._remaining
        m[6 * b + B:7 * b] = 0

    def stage_round(self, sids: List[int], d0: List[int], last: List[int], tstart: List[int],
                    remaining: List[int]) -> None:
        self._tstart, self._remaining = tstart, remaining
        self.stage(sids, d0, last)

    def _run(self) -> None:
        super()._run()  # the draft loop: proposals in self.props, draft logits in self.q
        lib, b, g, V = _lib.load(), self.bucket, self.gamma, self.Wt.shape[0]
        C = g + 1
        meta, dev = self.meta, self.meta.device
        rows, tstart, tcounts = meta[:b], meta[4 * b:5 * b], meta[5 * b:6 * b]
        remaining, nvalid = meta[6 * b:7 * b], meta[self.n_off:self.n_off + 1]
        # padding rows verify row 0's proposals (their own draws differ), so
        # the K/V rows they store at row 0's positions are row 0's bytes
        keep = meta[2 * b:3 * b] > 0
        props = torch.where(keep.unsqueeze(0), self.props, self.props[:, :1]).t().contiguous()  # (b, gamma)
        ids = torch.cat((meta[3 * b:4 * b].to(torch.int64).unsqueeze(1), props.to(torch.int64)), dim=1)
        tkv = self.tkv
        _lib.check(lib.sdl_kv_reserve(ctypes.byref(tkv._meta), b, rows.data_ptr(), tstart.data_ptr(),
                                      tcounts.data_ptr(), self.tslots.data_ptr(), tkv._stream()), "sdl_kv_reserve")
        batch = AttnBatch(rows, tstart, self.span, key_count=-1)
        positions = tstart.to(torch.int64).unsqueeze(1) + self.steps.unsqueeze(0)
        normed = self.target._body(ids, tkv, batch, positions)
        plog = self.target._graph_logits_buffer(C, b)
        torch.matmul(normed, self.Wt.t(), out=plog)
        st = _lib.stream_handle(dev)
        if self.greedy:
            p_arg = argmax_rows(plog.reshape(b * C, V)).reshape(b, C)
            tok, n_out = spec_sample(None, None, props, None, greedy=True, p_arg=p_arg)
            self.tokens.copy_(tok)
            self.n_out.copy_(n_out)
        else:
            R = self.q.shape[1]
            _lib.check(lib.sdl_spec_sample_logits_n(
                plog.data_ptr(), C * V, V, self.q.data_ptr(), V, R * V, _lib.dtype_code(plog.dtype), self.temp,
                1e-12, props.data_ptr(), b, g, V, self.ubuf.data_ptr(), self.ubuf.numel(), self.ucnt.data_ptr(), 0,
                self.tokens.data_ptr(), self.n_out.data_ptr(), self.sws.data_ptr(), self.sws.numel() * 4,
                tkv.err_word.data_ptr(), nvalid.data_ptr(), st), "sdl_spec_sample_logits_n")
        _lib.check(lib.sdl_spec_commit_n(
            ctypes.byref(tkv.meta), ctypes.byref(self.kv.meta), b, rows.data_ptr(), self.n_out.data_ptr(),
            self.tokens.data_ptr(), C, remaining.data_ptr(), self.eos, tstart.data_ptr(), self.outs[0].data_ptr(),
            self.outs[1].data_ptr(), self.outs[2].data_ptr(), nvalid.data_ptr(), st), "sdl_spec_commit_n")


def _draw_uniform(generator: torch.Generator) -> float:
    """Deterministic uniform coin (engine/spec_scheduler.py:41-43)."""
    return float(torch.rand(1, generator=generator).item())


def batch_accept(
    p_by_sid: Dict[int, torch.Tensor],
    q_by_sid: Dict[int, Seq[torch.Tensor]],
    proposals_by_sid: Dict[int, Seq[int]],
    generator: Any,
) -> Dict[int, List[int]]:
    """Accept/reject each sequence's draft block; return the committed tokens.

    Same contract as engine/spec_scheduler.py:46-88: sequences in dict order;
    scan proposals with ``u < min(1, p/q)``; on the first rejection draw from
    ``(p - q)+`` and stop; if all are accepted draw a bonus from ``p[gamma]``.
    One fused launch (``sdl_spec_sample``) for the whole batch.

    ``generator`` is a :class:`UniformStream` (uniforms consumed in the
    reference's order) or a ``torch.Generator`` (then ``B * (gamma + 1)``
    uniforms are pre-drawn from it, the most the round can use).
    """
    sids = list(p_by_sid.keys())
    if not sids:
        return {}
    p = torch.stack([p_by_sid[s].float() for s in sids]).contiguous()
    q = torch.stack([torch.stack([r.float() for r in q_by_sid[s]]) for s in sids]).contiguous()
    gamma = q.shape[1]
    props = _lib.to_device([list(proposals_by_sid[s]) for s in sids], torch.int32, p.device)
    if isinstance(generator, UniformStream):
        stream = generator
    else:
        u = torch.rand(len(sids) * (gamma + 1), generator=generator)
        stream = UniformStream(p.device, uniforms=u)
    tokens, n_out = spec_sample(p, q, props, stream, greedy=False)
    tok_h = tokens.tolist()
    n_h = n_out.tolist()
    return {sid: tok_h[b][: n_h[b]] for b, sid in enumerate(sids)}


class SpeculativePagedScheduler(PagedScheduler):
    """Continuous-batching scheduler with an integrated draft/verify round."""

    def __init__(self, model: Any, kv: PagedKVCache, draft_model: Any, draft_kv: PagedKVCache,
                 engine_cfg: EngineConfig, sampling: SamplingConfig, gamma: int,
                 uniforms: Optional[torch.Tensor] = None) -> None:
        super().__init__(model, kv, engine_cfg, sampling, uniforms=uniforms)
        self.draft_model = draft_model
        self.draft_kv = draft_kv
        self.gamma = int(gamma)
        if not 1 <= self.gamma <= 32:
            raise ValueError("gamma must be within [1, 32]")
        self._q_buf: Optional[torch.Tensor] = None
        # the draft's captured decodes end at the final norm and its LM head
        # writes each step's logits straight into the round's (gamma, rows, V)
        # buffer the rejection sampler reads, instead of a shared buffer
        # copied out after every step
        if hasattr(draft_model, "_graph_forward"):
            draft_model.graph_head = False
        # captured gamma-step draft loops (capture_graphs), keyed by (batch
        # bucket, key-span bucket); the round buffer and the uniform storage
        # they write and read live as long as the scheduler
        self.draft_loops = True
        # with draft_loops: capture whole rounds (draft loop, verify, sampling,
        # commit) rather than the draft phase alone
        self.round_graphs = True
        self._loops: Dict[Any, _DraftLoop] = {}
        self._loop_q: Optional[torch.Tensor] = None
        self._u_storage = None
        self.loop_replays = 0  # rounds whose draft phase was one loop replay
        self.round_replays = 0  # rounds that were one whole-round replay
        # optional observer of every round: called with (sequence ids, target
        # start positions, draft lengths) before the round's first launch
        self.round_hook: Optional[Callable[[List[int], List[int], List[int]], None]] = None
        # What a full KV pool does: "raise" (the reference: BlockExhaustedError,
        # engine/kv.py:61-66) or "recompute" -- admit only what fits, and
        # before a round that would not fit, park the most recently admitted
        # sequences (their blocks freed) and re-prefill them later.
        self.preemption = "raise"
        self.preemptions = 0  # sequences parked by the last run
        # prefill same-round arrivals together (16-bit models; see _flush_batched)
        self.batch_prefill = True

    # ------------------------------------------------------------ admission
    PREFILL_BATCH_TOKENS = 16384  # prompt tokens one batched prefill takes at most

    def _batch_prefill_ok(self) -> bool:
        """Same-round arrivals are prefilled together (``prefill_batch``) for
        16-bit models; fp32 models keep the reference's one-by-one prefill,
        whose reductions the parity runs pin."""
        if not self.batch_prefill:
            return False
        for m in (self.model, self.draft_model):
            emb = getattr(m, "embed_tokens", None)
            if not hasattr(m, "prefill_batch") or emb is None or emb.weight.dtype not in (torch.bfloat16,
                                                                                          torch.float16):
                return False
        return True

    def _flush_arrivals(self, arrivals: List[WorkloadRequest], when: int, result: SchedulerResult,
                        stream: Optional[UniformStream]) -> List[Sequence]:
        if len(arrivals) > 1 and self._batch_prefill_ok():
            return self._flush_batched(arrivals, when, result, stream)
        admitted: List[Sequence] = []
        for request in arrivals:
            seq = self._new_sequence(request, when)  # a CUDA tensor of ids is taken as is (prompts staged in HBM)
            seq.ttft_ms = self._prefill_spec_one(seq, result, stream)
            admitted.append(seq)
        result.sequences.extend(admitted)
        return admitted

    def _new_sequence(self, request: WorkloadRequest, when: int) -> Sequence:
        seq = Sequence(
            sid=self._next_sid,
            prompt_ids=(request.prompt if isinstance(request.prompt, torch.Tensor)
                        else self.model.encode(request.prompt)),
            max_new_tokens=request.max_new_tokens,
            arrive_time=request.arrive_time,
            admit_step=when,
        )
        self._next_sid += 1
        self.kv.add_sequence(seq.sid)
        self.draft_kv.add_sequence(seq.sid)
        return seq

    def _flush_batched(self, arrivals: List[WorkloadRequest], when: int, result: SchedulerResult,
                       stream: Optional[UniformStream]) -> List[Sequence]:
        """Admit several arrivals with one chunked prefill per model (groups of
        at most PREFILL_BATCH_TOKENS prompt tokens): the same positions,
        allocation order and first-token draws (one uniform per sequence, in
        arrival order) as admitting them one by one."""
        admitted: List[Sequence] = []
        group: List[Sequence] = []
        tokens = 0

        def flush() -> None:
            watch = Stopwatch()
            with watch:
                prompts = [s.prompt_ids for s in group]
                sids = [s.sid for s in group]
                logits = self.model.prefill_batch(prompts, self.kv, sids)
                toks = self._next_tokens(logits, stream)
                self.draft_model.prefill_batch(prompts, self.draft_kv, sids)
                first = toks.tolist()
            for s, t in zip(group, first):
                s.generated.append(int(t))
                s.prefilled = True
                s.ttft_ms = watch.elapsed_ms

        for request in arrivals:
            seq = self._new_sequence(request, when)
            n = len(seq.prompt_ids)
            if group and tokens + n > self.PREFILL_BATCH_TOKENS:
                flush()
                group, tokens = [], 0
            group.append(seq)
            tokens += n
            admitted.append(seq)
        if group:
            flush()
        result.sequences.extend(admitted)
        return admitted

    def _prefill_spec_one(self, seq: Sequence, result: SchedulerResult,
                          stream: Optional[UniformStream]) -> Optional[float]:
        watch = Stopwatch()
        with watch:
            if isinstance(seq.prompt_ids, torch.Tensor):  # prompt ids already in HBM
                ids = seq.prompt_ids.to(self.model.device, torch.long).reshape(1, -1)
            else:
                ids = _lib.to_device([list(seq.prompt_ids)], torch.long, self.model.device)
            logits = self.model.prefill(ids, self.kv, [seq.sid], [len(seq.prompt_ids)])
            tok = self._next_tokens(logits, stream)
            self.draft_model.prefill(ids, self.draft_kv, [seq.sid], [len(seq.prompt_ids)])
            seq.generated.append(int(tok[0].item()))
        seq.prefilled = True
        return watch.elapsed_ms

    # ------------------------------------------------------------ preemption
    def _blocks(self, kv: PagedKVCache, tokens: int) -> int:
        return -(-int(tokens) // kv.block_size)

    def _round_need(self, seqs: Seq[Sequence]) -> tuple:
        """Blocks a round of ``seqs`` can take from each pool at most: gamma+1
        target positions, gamma draft positions and the draft catch-up
        (from the caches' host shadows: no device access)."""
        g1 = self.gamma + 1
        bt, bd = self.kv.block_size, self.draft_kv.block_size
        lt, nbt = self.kv._h_len, self.kv._h_nb
        ld, nbd = self.draft_kv._h_len, self.draft_kv._h_nb
        nt = nd = 0
        for s in seqs:
            i = s.sid
            nt += max(0, -(-(lt[i] + g1) // bt) - nbt[i])
            nd += max(0, -(-(ld[i] + g1) // bd) - nbd[i])
        return nt, nd

    def _fits(self, need_t: int, need_d: int) -> bool:
        return need_t <= self.kv.allocator._h_free and need_d <= self.draft_kv.allocator._h_free

    def _context_need(self, tokens: int) -> tuple:
        """Blocks a sequence of ``tokens`` cached positions needs to join a round."""
        n = tokens + self.gamma + 1
        return self._blocks(self.kv, n), self._blocks(self.draft_kv, n)

    def _park(self, seq: Sequence) -> None:
        """Preempt ``seq``: free its blocks in both pools; it keeps its tokens."""
        self.kv.clear(seq.sid)
        self.draft_kv.clear(seq.sid)
        self.preemptions += 1

    def _recompute(self, seq: Sequence) -> None:
        """Re-prefill a parked sequence's prompt and generated tokens but the
        last (whose K/V a round writes), restoring the cache invariant
        ``seq_len == len(prompt) + len(generated) - 1``; nothing is sampled."""
        dev = self.model.device
        tail = _lib.to_device([list(seq.generated[:-1])], torch.long, dev)
        if isinstance(seq.prompt_ids, torch.Tensor):
            head = seq.prompt_ids.to(dev, torch.long).reshape(1, -1)
        else:
            head = _lib.to_device([list(seq.prompt_ids)], torch.long, dev)
        ids = torch.cat((head, tail), dim=1)
        n = ids.shape[1]
        self.model.prefill(ids, self.kv, [seq.sid], [n])
        self.draft_model.prefill(ids, self.draft_kv, [seq.sid], [n])

    def _admit_fitting(self, queue: List[WorkloadRequest], parked: List[Sequence], running: List[Sequence],
                       when: int, result: SchedulerResult, stream: Optional[UniformStream]) -> None:
        """Recompute policy: re-admit parked sequences, then queued arrivals,
        in order, while each fits beside the running round's needs."""
        # the pools' free counts drop by what a sequence holds once it is
        # in; its round need on top of that is what it has not reserved yet
        need_t, need_d = self._round_need(running)
        while parked:
            t, d = self._context_need(len(parked[0].prompt_ids) + len(parked[0].generated) - 1)
            if not self._fits(need_t + t, need_d + d):
                return
            seq = parked.pop(0)
            self._recompute(seq)
            rt, rd = self._round_need([seq])
            need_t, need_d = need_t + rt, need_d + rd
            running.append(seq)
        take: List[WorkloadRequest] = []
        while queue:
            t, d = self._context_need(len(queue[0].prompt))
            if not self._fits(need_t + t, need_d + d):
                break
            take.append(queue.pop(0))
            need_t, need_d = need_t + t, need_d + d  # its reservation plus its round need
        if take:
            running.extend(self._flush_arrivals(take, when, result, stream))

    def _make_room(self, running: List[Sequence], parked: List[Sequence]) -> List[Sequence]:
        """Recompute policy: park the most recently admitted sequences until
        the round fits both pools; returns the sequences that run."""
        running = list(running)
        need_t, need_d = self._round_need(running)
        while running and not self._fits(need_t, need_d):
            victim = max(running, key=lambda s: s.sid)
            vt, vd = self._round_need([victim])
            running.remove(victim)
            self._park(victim)  # frees what it held: the free counts grow
            need_t, need_d = need_t - vt, need_d - vd
            parked.append(victim)
            parked.sort(key=lambda s: s.sid)
        return running

    # ------------------------------------------------------------ start-up
    def _round_buffer(self, B: int, gamma: int, V: int, dtype: torch.dtype, device: torch.device,
                      t_slot: Optional[int] = None) -> torch.Tensor:
        """The round's draft rows, laid out ``(gamma, R, V)`` with R at least
        B and the draft's graph bucket of B: returns the ``(B, gamma, V)``
        view the samplers read, or with ``t_slot`` the contiguous ``(R, V)``
        slice of draft step ``t_slot`` (the draft's LM head output)."""
        bucket = getattr(self.draft_model, "_graph_bucket", lambda n: None)(B) or B
        rows = max(B, bucket)
        lq = self._loop_q
        if lq is not None and lq.shape[0] >= gamma and lq.shape[1] >= rows and lq.shape[2] == V and lq.dtype == dtype:
            buf = lq  # the captured loops' buffer serves the step-wise path too
            return buf[t_slot] if t_slot is not None else buf[:gamma, :B].permute(1, 0, 2)
        buf = self._q_buf
        if buf is None or buf.shape[0] < gamma or buf.shape[1] < rows or buf.shape[2] != V or buf.dtype != dtype:
            rows = max(rows, buf.shape[1] if buf is not None and buf.shape[2] == V else 0)
            self._q_buf = buf = torch.empty((gamma, rows, V), dtype=dtype, device=device)
        if t_slot is not None:
            return buf[t_slot]
        return buf[:gamma, :B].permute(1, 0, 2)

    # uniform storage of the captured loops: 2^20 valid uniforms plus room
    # for the draws of padding rows past them
    U_CAPACITY = 1 << 20
    U_MARGIN = 4096

    def _loop_q_buffer(self, V: int, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        """The round buffer the captured loops write: (gamma, largest graph
        bucket, V), allocated once (the graphs hold its address)."""
        rows = max(self.draft_model.GRAPH_BUCKETS)
        lq = self._loop_q
        if lq is None:
            self._loop_q = lq = torch.empty((self.gamma, rows, V), dtype=dtype, device=device)
        if lq.shape != (self.gamma, rows, V) or lq.dtype != dtype:
            raise RuntimeError("draft loop buffer shape changed")
        return lq

    def _make_stream(self, seed: int) -> Optional[UniformStream]:
        """As PagedScheduler's, placed in the captured loops' storage when
        there is one (and the stream fits it)."""
        if self.sampling.is_greedy or self._u_storage is None:
            return super()._make_stream(seed)
        buf, cnt = self._u_storage
        view = (buf[:self.U_CAPACITY], cnt)
        if self._uniforms is not None:
            if self._uniforms.numel() > self.U_CAPACITY:
                return super()._make_stream(seed)
            return UniformStream(self.model.device, uniforms=self._uniforms, storage=view)
        return UniformStream(self.model.device, seed=seed, storage=view)

    def _capture_draft_loops(self, sid: int) -> int:
        """Capture the draft loop for every batch bucket and key-span bucket
        of the draft's graphs (plain temperature or greedy sampling), on the
        scratch sequence ``sid``."""
        draft, kv = self.draft_model, self.draft_kv
        greedy = self.sampling.is_greedy
        W = getattr(getattr(draft, "lm_head", None), "weight", None)
        if (not self.draft_loops or not getattr(draft, "_graphs_enabled", False) or W is None
                or not hasattr(draft, "_body") or not (greedy or self._plain_temperature(W.shape[0]))):
            return 0
        dev = draft.device
        if self._u_storage is None:
            self._u_storage = (torch.zeros(self.U_CAPACITY + self.U_MARGIN, dtype=torch.float32, device=dev),
                               torch.zeros(1, dtype=torch.int64, device=dev))
        n, prev, g = 0, 0, self.gamma
        whole = self.round_graphs and hasattr(self.model, "_body") and \
            getattr(self.model, "_graphs_enabled", False) and \
            self.model.graph_spans(self.kv) == draft.graph_spans(kv)
        tkv = self.kv
        for span in draft.graph_spans(kv):
            need = max(prev + 1, int(0.55 * span), g + 2)
            prev = span
            for b in draft.GRAPH_BUCKETS:
                # the scratch pass reserves the draft's gamma positions and the
                # target's gamma + 1 (on the host shadows too) and, whole, commits
                kv.reserve([sid], [0], [need - g])
                kv._plan_reserve([sid], [need - g], [g])
                saved = self._u_storage[1].clone()
                if whole:
                    tkv.reserve([sid], [0], [need - g - 1])
                    tkv._plan_reserve([sid], [need - g - 1], [g + 1])
                    loop = _RoundGraph(self, b, span, greedy)
                    loop._tstart, loop._remaining = [need - g - 1], [1 << 20]
                else:
                    loop = _DraftLoop(self, b, span, greedy)
                loop.capture([sid], [need - g], [0])
                self._u_storage[1].copy_(saved)
                kv.clear(sid)
                if whole:
                    tkv.clear(sid)
                self._loops[(b, span, greedy, float(self.sampling.temperature))] = loop
                n += 1
        kv.check_errors()
        tkv.check_errors()
        return n

    def capture_graphs(self) -> int:
        """Capture every CUDA graph the models can replay in a run (draft
        decode, target verify of gamma+1 rows, both models' prefill, at every
        batch and key-span bucket) before serving, on a scratch sequence id.
        A no-op unless the models have CUDA graphs enabled.  Returns the
        number of graphs captured."""
        import gc

        gc.collect()  # dead objects that hold graphs go now, not inside a capture
        sid = self._next_sid
        self._next_sid += 1
        n = 0
        for model, kv, chunk in ((self.draft_model, self.draft_kv, 1), (self.model, self.kv, self.gamma + 1)):
            if not hasattr(model, "capture_graphs"):
                continue
            kv.add_sequence(sid)
            n += model.capture_graphs(kv, sid, chunk)
        if hasattr(self.draft_model, "capture_graphs"):
            n += self._capture_draft_loops(sid)
        return n

    # ------------------------------------------------------------ spec loop
    def run_spec_continuous(self, requests: Seq[WorkloadRequest], seed: int, measure: bool = True,
                            arrival_clock: str = "step") -> SchedulerResult:
        """Serve ``requests`` to completion (engine/spec_scheduler.py:166-222).

        ``arrival_clock="step"`` (the reference's): ``arrive_time`` counts
        scheduler rounds.  ``"wall"``: ``arrive_time`` is in seconds from the
        start of the run, and a request is admitted at the first round
        boundary at or after its arrival; with nothing to run the scheduler
        waits for the next arrival (that idle time is part of the makespan).
        """
        if arrival_clock not in ("step", "wall"):
            raise ValueError("arrival_clock must be 'step' or 'wall'")
        wall = arrival_clock == "wall"
        result = SchedulerResult(mode="spec-continuous", sampling=self.sampling.describe())
        stream = self._make_stream(seed)
        device = self.model.device
        arrivals = sorted(requests, key=lambda r: r.arrive_time)
        step = 0
        if measure:
            sync_device(device)
            torch.cuda.reset_peak_memory_stats(device)
        stopwatch = Stopwatch()
        with stopwatch:
            t0 = time.perf_counter()

            def clock():
                return (time.perf_counter() - t0) if wall else step

            recompute = self.preemption == "recompute"
            if self.preemption not in ("raise", "recompute"):
                raise ValueError("preemption must be 'raise' or 'recompute'")
            self.preemptions = 0
            queue: List[WorkloadRequest] = []  # arrived, not admitted (recompute policy)
            parked: List[Sequence] = []        # preempted, waiting to be recomputed

            active: List[Sequence] = []  # admitted and not finished (parked ones included)
            nxt = 0                       # arrivals[:nxt] have arrived

            def take_due(now_: float) -> List[WorkloadRequest]:
                nonlocal nxt
                k = nxt
                while k < len(arrivals) and arrivals[k].arrive_time <= now_:
                    k += 1
                due_ = arrivals[nxt:k]
                nxt = k
                return due_

            def live() -> List[Sequence]:
                active[:] = [s for s in active if not s.finished]
                if not parked:
                    return list(active)
                held = {s.sid for s in parked}
                return [s for s in active if s.sid not in held]

            def admit(due_now: List[WorkloadRequest]) -> None:
                n0 = len(result.sequences)
                if not recompute:
                    if due_now:
                        self._flush_arrivals(due_now, step, result, stream)
                else:
                    queue.extend(due_now)
                    self._admit_fitting(queue, parked, live(), step, result, stream)
                active.extend(result.sequences[n0:])

            admit(take_due(clock()))
            running = live()
            while running or nxt < len(arrivals) or queue or parked:
                running = live()
                if recompute and running:
                    running = self._make_room(running, parked)
                if running:
                    self._spec_step(running, result, stream)
                    result.total_forwards += 1
                elif queue or parked:
                    # nothing runs and the oldest waiting request still does not fit
                    raise _exhausted(self.kv.capacity)
                elif wall and nxt < len(arrivals):
                    time.sleep(max(0.0, arrivals[nxt].arrive_time - clock()))
                step += 1
                admit(take_due(clock()))
                running = live()
                result.batch_hist.append(len(running))
                result.block_util_hist.append(self.kv.block_utilization)
                if self.kv.num_allocated_blocks > result.kv_peak_blocks:
                    result.kv_peak_blocks = self.kv.num_allocated_blocks
                if self.draft_kv.num_allocated_blocks > result.draft_kv_peak_blocks:
                    result.draft_kv_peak_blocks = self.draft_kv.num_allocated_blocks
            result.steps = step
            if measure:
                sync_device(device)
        result.makespan_ms = stopwatch.elapsed_ms
        result.generated_tokens = sum(len(s.generated) for s in result.sequences)
        result.kv_peak_bytes = result.kv_peak_blocks * self._bytes_per_block()
        if result.tokens_per_round:
            result.mean_tokens_per_round = sum(result.tokens_per_round) / len(result.tokens_per_round)
            result.mean_acceptance = sum(result.tokens_per_round) / (len(result.tokens_per_round) * (self.gamma + 1))
        if measure:
            result.peak_memory_mb = round(torch.cuda.max_memory_allocated(device) / (1024.0 ** 2), 2)
        return result

    # ------------------------------------------------------------ one round
    def _draft_loop_for(self, B: int, d0: List[int], stream: Optional[UniformStream],
                        starts: List[int]) -> Optional[_DraftLoop]:
        """The captured round (or draft loop) for this round's batch and
        contexts, or None (not captured, a batch beyond the largest bucket,
        or a stream outside the captures' uniform storage)."""
        if not self._loops:
            return None
        draft = self.draft_model
        if stream is not None and (self._u_storage is None or
                                   stream.storage[0].data_ptr() != self._u_storage[0].data_ptr()):
            return None
        bucket = draft._graph_bucket(B)
        if bucket is None:
            return None
        need = max(max(d0) + self.gamma, max(starts) + self.gamma + 1)
        span = draft.span_bucket(self.draft_kv, need)
        return self._loops.get((bucket, span, self.sampling.is_greedy, float(self.sampling.temperature)))

    def _plain_temperature(self, vocab: int) -> bool:
        """True when sampling is softmax(logits / T) with no top-k / top-p."""
        s = self.sampling
        top_k = int(getattr(s, "top_k", 0) or 0)
        top_p = float(getattr(s, "top_p", 1.0))
        return (top_k <= 0 or top_k >= vocab) and (top_p >= 1.0 or top_p <= 0.0)

    def _probs_spec(self, logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """specdec logits_to_probs semantics (T floor 1e-12, optional top-k/top-p)."""
        s = self.sampling
        top_k = int(getattr(s, "top_k", 0) or 0)
        top_p = float(getattr(s, "top_p", 1.0))
        if self._plain_temperature(logits.shape[-1]):
            return probs_rows(logits, s.temperature, False, eps=1e-12, out=out)
        scaled = logits.float() / max(s.temperature, 1e-12)
        filtered = apply_top_p(apply_top_k(scaled, top_k), top_p)
        return probs_rows(filtered, 1.0, False, out=out)

    def _spec_step(self, running: Seq[Sequence], result: SchedulerResult, stream: Optional[UniformStream]) -> None:
        model, draft = self.model, self.draft_model
        device = model.device
        gamma = self.gamma
        chunk = gamma + 1
        greedy = self.sampling.is_greedy
        sids = [s.sid for s in running]
        B = len(running)
        starts = [self.kv.seq_len(sid) for sid in sids]
        d0 = [self.draft_kv.seq_len(sid) for sid in sids]
        if self.round_hook is not None:
            self.round_hook(sids, starts, d0)

        last = [s.generated[-1] for s in running]
        remaining = [s.max_new_tokens - len(s.generated) for s in running]
        loop = self._draft_loop_for(B, d0, stream, starts)
        if isinstance(loop, _RoundGraph):
            # the whole round is one graph replay; the host reads its packed results below
            self.draft_kv._plan_reserve(sids, d0, [gamma] * B)
            self.kv._plan_reserve(sids, starts, [chunk] * B)
            if not greedy:
                stream.reserve(gamma * B + B * chunk)
            loop.stage_round(sids, d0, last, starts, remaining)
            loop.replay()
            self.round_replays += 1
            result.draft_forward_calls += gamma
            draft.forward_calls = getattr(draft, "forward_calls", 0) + gamma
            model.forward_calls = getattr(model, "forward_calls", 0) + 1
            tokens, outs = loop.tokens[:B], loop.outs[:, :B]
        else:
            tokens, outs = self._round_steps(running, result, stream, loop, sids, starts, d0, last, remaining)
        self._finish_round(running, result, tokens, outs)

    def _round_steps(self, running, result, stream, loop, sids, starts, d0, last, remaining):
        """The round launch by launch (or with the captured draft loop):
        returns the sampled tokens and the commit's (k, flags, catch-up slot)."""
        model, draft = self.model, self.draft_model
        device = model.device
        gamma = self.gamma
        chunk = gamma + 1
        greedy = self.sampling.is_greedy
        B = len(running)

        # ---- 1. draft proposes gamma tokens per sequence
        q_probs = None
        if not greedy:
            stream.reserve(gamma * B)
        fused = False
        u_skip = gamma * B  # uniforms the draft draws read ahead of the accept walk
        V_d = getattr(getattr(draft, "lm_head", None), "weight", None)
        if loop is not None:
            # the whole draft phase is one graph replay: reserves, forwards,
            # heads into the round buffer, draws (advancing the counter)
            self.draft_kv._plan_reserve(sids, d0, [gamma] * B)
            loop.stage(sids, d0, last)
            loop.replay()
            self.loop_replays += 1
            result.draft_forward_calls += gamma
            draft.forward_calls = getattr(draft, "forward_calls", 0) + gamma
            proposals = loop.props[:, :B].t().contiguous()
            if not greedy:
                fused = True
                q_probs = loop.q[:, :B].permute(1, 0, 2)
                u_skip = 0
        else:
            proposals = torch.empty((B, gamma), dtype=torch.int32, device=device)
        cur = _lib.to_device(last, torch.long, device)
        # plain temperature: each draft step's logits land in step t's slice of
        # the round buffer, which the fused rejection sampler reads in place
        direct = (not greedy and V_d is not None and hasattr(draft, "_graph_forward")
                  and self._plain_temperature(V_d.shape[0]))
        for t in range(gamma if loop is None else 0):
            if direct:
                qb = self._round_buffer(B, gamma, V_d.shape[0], V_d.dtype, device, t_slot=t)
                q_logits = draft.decode(cur, self.draft_kv, sids, [d + t for d in d0], logits_out=qb)
            else:
                q_logits = draft.decode(cur, self.draft_kv, sids, [d + t for d in d0])
            result.draft_forward_calls += 1
            if greedy:
                prop_t = argmax_rows(q_logits)
            else:
                V = q_logits.shape[-1]
                fused = self._plain_temperature(V)
                # plain temperature keeps the draft logits (the fused sampler reads
                # them); filtering keeps the filtered probability rows instead
                dt = q_logits.dtype if fused else torch.float32
                q_probs = self._round_buffer(B, gamma, V, dt, device)
                if fused:
                    if not direct:
                        q_probs[:, t, :].copy_(q_logits.reshape(B, V))
                    prop_t = sample_logits_rows(q_probs[:, t, :], self.sampling.temperature, stream, offset=t * B,
                                                err=self.draft_kv.err_word, eps=1e-12)
                else:
                    self._probs_spec(q_logits, out=q_probs[:, t, :])
                    prop_t = sample_rows(q_probs[:, t, :], stream, offset=t * B, err=self.draft_kv.err_word)
            proposals[:, t] = prop_t
            cur = prop_t.long()

        # ---- 2. target verifies [pending] + proposals in one forward
        rows = torch.cat((_lib.to_device([[s.generated[-1]] for s in running], torch.long, device),
                          proposals.long()), dim=1)
        p_logits = model.decode_block(rows, self.kv, sids, starts)  # (B, chunk, V)

        # ---- 3. fused rejection sampling
        if greedy:
            p_arg = argmax_rows(p_logits.reshape(B * chunk, -1)).reshape(B, chunk)
            tokens, n_out = spec_sample(None, None, proposals, None, greedy=True, p_arg=p_arg)
        elif fused:
            pl = p_logits.reshape(B, chunk, -1)
            ql = q_probs
            if pl.dtype != ql.dtype:  # upcasts are exact, so the probabilities do not change
                pl, ql = pl.float(), ql.float()
            tokens, n_out = spec_sample_logits(pl, ql, self.sampling.temperature, proposals, stream,
                                               u_skip=u_skip, err=self.kv.err_word, eps=1e-12)
        else:
            p_probs = self._probs_spec(p_logits).reshape(B, chunk, -1)
            tokens, n_out = spec_sample(p_probs, q_probs, proposals, stream, greedy=False, u_skip=u_skip,
                                        err=self.kv.err_word)

        # ---- 4. device commit: clip, EOS cut, rewind, draft alignment, clears
        packed = _lib.i32(sids + remaining + starts, device)
        outs = torch.empty((3, B), dtype=torch.int32, device=device)
        eos = -1 if self._eos is None else int(self._eos)
        _lib.check(
            _lib.load().sdl_spec_commit(
                ctypes.byref(self.kv.meta), ctypes.byref(self.draft_kv.meta), B, packed.data_ptr(),
                n_out.data_ptr(), tokens.data_ptr(), chunk, packed.data_ptr() + 4 * B, eos,
                packed.data_ptr() + 8 * B, outs[0].data_ptr(), outs[1].data_ptr(), outs[2].data_ptr(),
                _lib.stream_handle(device),
            ),
            "sdl_spec_commit",
        )
        return tokens, outs

    def _finish_round(self, running, result, tokens, outs) -> None:
        """Read a round's packed results once and mirror them on the host
        (sequences, shadows), then run the draft catch-up."""
        draft = self.draft_model
        device = self.model.device
        chunk = self.gamma + 1
        B = len(running)
        host = torch.cat((tokens.reshape(-1), outs.reshape(-1), self.kv.err_word, self.draft_kv.err_word)).tolist()
        tok_h = host[: B * chunk]
        k_h = host[B * chunk: B * chunk + B]
        f_h = host[B * chunk + B: B * chunk + 2 * B]
        c_h = host[B * chunk + 2 * B: B * chunk + 3 * B]
        err_t, err_d = host[-2], host[-1]
        if err_t or err_d:
            self.kv.err_word.zero_()
            self.draft_kv.err_word.zero_()
            if (err_t | err_d) & _lib.DEVERR_EXHAUSTED:
                raise _exhausted(self.kv.capacity if err_t & _lib.DEVERR_EXHAUSTED else self.draft_kv.capacity)
            raise RuntimeError("device error during spec round: target 0x{:x} draft 0x{:x}".format(err_t, err_d))

        # ---- 5. host bookkeeping (mirrors engine/spec_scheduler.py:270-322)
        catch_sids: List[int] = []
        catch_pos: List[int] = []
        catch_tok: List[int] = []
        catch_slot: List[int] = []
        for b, s in enumerate(running):
            sid = s.sid
            k = k_h[b]
            fin = bool(f_h[b] & 1)
            result.tokens_per_round.append(k)
            if f_h[b] & 2:
                s.eos_hit = True
            if k == 0:
                s.finished = True
                s.finish_step = result.steps
            else:
                s.generated.extend(tok_h[b * chunk: b * chunk + k])
                if fin:
                    s.finished = True
                    s.finish_step = result.steps
                keep = len(s.prompt_ids) + len(s.generated) - 1
                self.kv._shadow_release(sid, keep, _lib.REL_TRUNCATE)
                d_len = self.draft_kv.seq_len(sid)
                if d_len > keep:
                    self.draft_kv._shadow_release(sid, keep, _lib.REL_TRUNCATE)
                elif d_len < keep:
                    self._shadow_extend_one(self.draft_kv, sid, d_len)
                    # the reference decodes (and counts) the catch-up token even
                    # when the sequence finishes this round; its K/V is discarded
                    result.draft_forward_calls += keep - d_len
                    if c_h[b] >= 0:
                        catch_sids.append(sid)
                        catch_pos.append(d_len)
                        catch_tok.append(s.generated[d_len - len(s.prompt_ids)])
                        catch_slot.append(c_h[b])
            if s.finished:
                self.kv._shadow_release(sid, 0, _lib.REL_CLEAR)
                self.draft_kv._shadow_release(sid, 0, _lib.REL_CLEAR)
        self.kv._mirror = None
        self.draft_kv._mirror = None

        # ---- 6. draft catch-up for fully accepted rounds (engine/spec_scheduler.py:308-319)
        if catch_sids:
            ids = _lib.to_device(catch_tok, torch.long, device)
            slots = _lib.i32(catch_slot, device)
            draft.decode(ids, self.draft_kv, catch_sids, catch_pos, slots=slots)

    @staticmethod
    def _shadow_extend_one(kv: PagedKVCache, sid: int, pos: int) -> None:
        need_b = pos // kv.block_size + 1
        if need_b > kv._h_nb[sid]:
            kv.allocator._h_free -= need_b - kv._h_nb[sid]
            kv._h_nb[sid] = need_b
        if kv._h_len[sid] <= pos:
            kv._h_len[sid] = pos + 1
