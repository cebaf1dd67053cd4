"""Oracle schedulers: restate engine/scheduler.py:157-284 (continuous) and
engine/spec_scheduler.py:110-322 (speculative) over the numpy model and cache.

Every stochastic draw takes the next value of one uniform stream, in the
reference's draw order.  Test infrastructure only (see oracle/__init__.py).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

from .kv import PagedKVCache
from .model import NumpyPagedLM
from .sampler import UniformStream, batch_accept, logits_to_probs, sample_index


@dataclass
class Req:
    prompt_ids: List[int]
    max_new_tokens: int
    arrive_time: int = 0


@dataclass
class Seq:
    sid: int
    prompt_ids: List[int]
    max_new_tokens: int
    arrive_time: int
    generated: List[int] = field(default_factory=list)
    finished: bool = False
    eos_hit: bool = False


@dataclass
class RunResult:
    sequences: List[Seq] = field(default_factory=list)
    steps: int = 0
    tokens_per_round: List[int] = field(default_factory=list)
    draft_forward_calls: int = 0
    kv_peak_blocks: int = 0
    draft_kv_peak_blocks: int = 0


def _pick(logits: np.ndarray, temperature: float, eps: float, stream: Optional[UniformStream]) -> int:
    """PagedScheduler._probs/_sample (engine/scheduler.py:227-239)."""
    if temperature <= 0.0:
        return int(np.argmax(logits))
    x = np.asarray(logits, np.float32) / np.float32(max(temperature, eps))
    e = np.exp(x - x.max()).astype(np.float32)
    p = (e / e.sum(dtype=np.float32)).astype(np.float32)
    return sample_index(p, stream.next())


def run_continuous(model: NumpyPagedLM, kv: PagedKVCache, requests: Sequence[Req], temperature: float,
                   stream: Optional[UniformStream] = None, eos: Optional[int] = None) -> RunResult:
    res = RunResult()
    arrivals = sorted(requests, key=lambda r: r.arrive_time)
    step = 0
    next_sid = 0

    def admit(due):
        nonlocal next_sid
        for r in due:
            s = Seq(next_sid, list(r.prompt_ids), r.max_new_tokens, r.arrive_time)
            next_sid += 1
            kv.add_sequence(s.sid)
            logits = model.prefill(s.prompt_ids, kv, s.sid)
            s.generated.append(_pick(logits, temperature, 1e-9, stream))
            res.sequences.append(s)

    admit([r for r in arrivals if r.arrive_time <= step])
    pending = [r for r in arrivals if r.arrive_time > step]
    running = [s for s in res.sequences if not s.finished]
    while running or pending:
        running = [s for s in res.sequences if not s.finished]
        if running:
            ids = np.array([[s.generated[-1]] for s in running])
            ctx = [kv.seq_lengths[s.sid] for s in running]
            logits = model.forward_rows(ids, kv, [s.sid for s in running], ctx)[:, 0]
            for b, s in enumerate(running):
                tok = _pick(logits[b], temperature, 1e-9, stream)
                if eos is not None and tok == eos:
                    s.eos_hit = s.finished = True
                else:
                    s.generated.append(tok)
                if len(s.generated) >= s.max_new_tokens:
                    s.finished = True
                if s.finished:
                    kv.clear(s.sid)
        step += 1
        due = [r for r in pending if r.arrive_time <= step]
        pending = [r for r in pending if r.arrive_time > step]
        if due:
            admit(due)
        running = [s for s in res.sequences if not s.finished]
        res.kv_peak_blocks = max(res.kv_peak_blocks, kv.num_allocated_blocks)
    res.steps = step
    return res


def run_spec_continuous(target: NumpyPagedLM, kv: PagedKVCache, draft: NumpyPagedLM, draft_kv: PagedKVCache,
                        requests: Sequence[Req], gamma: int, temperature: float,
                        stream: Optional[UniformStream] = None, eos: Optional[int] = None,
                        top_k: int = 0, top_p: float = 1.0, round_hook=None,
                        result: Optional[RunResult] = None) -> RunResult:
    """``result`` (optional) is filled in place, so a caller whose
    ``round_hook`` stops the run early by raising still sees the rounds done."""
    res = result if result is not None else RunResult()
    arrivals = sorted(requests, key=lambda r: r.arrive_time)
    step = 0
    next_sid = 0
    greedy = temperature <= 0.0

    def probs(logits):
        return logits_to_probs(logits, temperature, top_k, top_p)

    def draw(p):
        if greedy:
            return int(np.argmax(p))
        return sample_index(p, stream.next())

    def admit(due):
        nonlocal next_sid
        for r in due:
            s = Seq(next_sid, list(r.prompt_ids), r.max_new_tokens, r.arrive_time)
            next_sid += 1
            kv.add_sequence(s.sid)
            draft_kv.add_sequence(s.sid)
            logits = target.prefill(s.prompt_ids, kv, s.sid)
            s.generated.append(_pick(logits, temperature, 1e-9, stream))
            draft.prefill(s.prompt_ids, draft_kv, s.sid)
            res.sequences.append(s)

    def spec_step(running: List[Seq]):
        sids = [s.sid for s in running]
        B = len(running)
        proposals: Dict[int, List[int]] = {sid: [] for sid in sids}
        q_rows: Dict[int, List[np.ndarray]] = {sid: [] for sid in sids}
        cur = [s.generated[-1] for s in running]
        for _ in range(gamma):
            bctx = [draft_kv.seq_lengths[sid] for sid in sids]
            q_logits = draft.forward_rows(np.array(cur)[:, None], draft_kv, sids, bctx)[:, 0]
            res.draft_forward_calls += 1
            for b, s in enumerate(running):
                qp = probs(q_logits[b])
                q_rows[s.sid].append(qp)
                proposals[s.sid].append(draw(qp))
            cur = [proposals[s.sid][-1] for s in running]
        starts = [kv.seq_lengths[sid] for sid in sids]
        rows = np.array([[s.generated[-1]] + proposals[s.sid] for s in running])
        p_all = target.forward_rows(rows, kv, sids, starts)
        p_rows = [probs(p_all[b]) for b in range(B)]
        if greedy:
            accepted = []
            for b, s in enumerate(running):
                acc = []
                for j in range(gamma):
                    x = proposals[s.sid][j]
                    if int(np.argmax(p_rows[b][j])) == x:
                        acc.append(x)
                    else:
                        acc.append(int(np.argmax(p_rows[b][j])))
                        break
                else:
                    acc.append(int(np.argmax(p_rows[b][gamma])))
                accepted.append(acc)
        else:
            accepted = batch_accept(p_rows, [q_rows[s.sid] for s in running],
                                    [proposals[s.sid] for s in running], stream)
        for b, s in enumerate(running):
            sid = s.sid
            P = len(s.prompt_ids)
            acc = list(accepted[b])
            remaining = s.max_new_tokens - len(s.generated)
            if len(acc) > remaining:
                acc = acc[:remaining]
            if eos is not None:
                for i, tok in enumerate(acc):
                    if tok == eos:
                        acc = acc[:i]
                        s.eos_hit = s.finished = True
                        break
            k = len(acc)
            res.tokens_per_round.append(k)
            if k == 0:
                s.finished = True
            else:
                s.generated.extend(acc)
                if len(s.generated) >= s.max_new_tokens:
                    s.finished = True
                keep = P + len(s.generated) - 1
                kv.truncate(sid, keep)
                d_len = draft_kv.seq_lengths[sid]
                if d_len > keep:
                    draft_kv.truncate(sid, keep)
                elif d_len < keep:
                    p = d_len
                    while p < keep:
                        tok = s.generated[p - P]
                        draft.forward_rows(np.array([[tok]]), draft_kv, [sid], [draft_kv.seq_lengths[sid]])
                        res.draft_forward_calls += 1
                        p += 1
            if s.finished:
                kv.clear(sid)
                draft_kv.clear(sid)

    admit([r for r in arrivals if r.arrive_time <= step])
    pending = [r for r in arrivals if r.arrive_time > step]
    running = [s for s in res.sequences if not s.finished]
    while running or pending:
        running = [s for s in res.sequences if not s.finished]
        if running:
            spec_step(running)
            if round_hook is not None:
                round_hook()
        step += 1
        due = [r for r in pending if r.arrive_time <= step]
        pending = [r for r in pending if r.arrive_time > step]
        if due:
            admit(due)
        running = [s for s in res.sequences if not s.finished]
        res.kv_peak_blocks = max(res.kv_peak_blocks, kv.num_allocated_blocks)
        res.draft_kv_peak_blocks = max(res.draft_kv_peak_blocks, draft_kv.num_allocated_blocks)
    res.steps = step
    return res
