"""Continuous-batching scheduler and a static-batching baseline.

Drop-in for the reference's ``engine/scheduler.py`` (engine/scheduler.py:35-375):
same ``Sequence`` / ``SchedulerResult`` records and telemetry, same
``run_continuous`` / ``run_static`` step loops, admission order and
finish rules.  Per step the whole batch is decoded by one model forward
(batched reserve + per-layer append/attention kernels), the next tokens are
picked on the device (argmax kernel, or temperature softmax + the integer
inverse-CDF draw from a device ``UniformStream``), and a single host copy of
the token ids feeds the Python bookkeeping.  Finished sequences are released
by one batched kernel in batch order, which keeps the free-list order of the
reference's per-sequence ``kv.clear`` calls.

Stochastic draws: the reference draws with ``torch.multinomial`` from a CPU
generator seeded by ``seed``; here ``seed`` seeds the device uniform stream
(or ``uniforms=`` pins a pre-drawn stream, one uniform per draw in the
reference's draw order).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence as Seq

import torch

from . import _lib
from .config import EngineConfig, SamplingConfig, WorkloadRequest
from .kv import PagedKVCache
from .utils import Stopwatch, mean_std, setup_logger, sync_device
from specdec.sampler import UniformStream, argmax_rows, probs_rows, sample_logits_rows, sample_rows, sample_token

logger = setup_logger(__name__)


@dataclass
class Sequence:
    """One request plus its generation progress/telemetry."""

    sid: int
    prompt_ids: List[int]
    max_new_tokens: int
    arrive_time: int
    generated: List[int] = field(default_factory=list)
    prefilled: bool = False
    finished: bool = False
    finish_step: int = -1
    admit_step: int = -1
    ttft_ms: Optional[float] = None
    eos_hit: bool = False

    @property
    def done(self) -> bool:
        budget = 0 if self.finished else (self.max_new_tokens - len(self.generated))
        return budget <= 0


@dataclass
class SchedulerResult:
    """Aggregate telemetry for one scheduling run (engine/scheduler.py:57-133)."""

    mode: str = ""
    sequences: List[Sequence] = field(default_factory=list)
    steps: int = 0
    makespan_ms: float = 0.0
    generated_tokens: int = 0
    total_forwards: int = 0
    batch_hist: List[int] = field(default_factory=list)
    block_util_hist: List[float] = field(default_factory=list)
    kv_peak_blocks: int = 0
    kv_peak_bytes: int = 0
    peak_memory_mb: Optional[float] = None
    sampling: str = "greedy"
    draft_kv_peak_blocks: int = 0
    draft_forward_calls: int = 0
    tokens_per_round: List[int] = field(default_factory=list)
    mean_acceptance: Optional[float] = None
    mean_tokens_per_round: Optional[float] = None

    @property
    def throughput_tokens_per_s(self) -> Optional[float]:
        if self.makespan_ms <= 0:
            return None
        return self.generated_tokens / (self.makespan_ms / 1000.0)

    @property
    def avg_active_batch(self) -> float:
        return sum(self.batch_hist) / len(self.batch_hist) if self.batch_hist else 0.0

    @property
    def slot_utilization(self) -> float:
        peak = max(self.batch_hist) if self.batch_hist else 0.0
        if peak <= 0:
            return 0.0
        return self.generated_tokens / (self.steps * peak)

    def ttft_list(self) -> List[Optional[float]]:
        return [seq.ttft_ms for seq in self.sequences if seq.ttft_ms is not None]

    def to_dict(self) -> Dict[str, Any]:
        ttft = mean_std([v for v in self.ttft_list() if v is not None])
        return {
            "mode": self.mode,
            "sampling": self.sampling,
            "num_requests": len(self.sequences),
            "steps": self.steps,
            "makespan_ms": round(self.makespan_ms, 3),
            "generated_tokens": self.generated_tokens,
            "total_forwards": self.total_forwards,
            "throughput_tokens_per_s": (
                round(self.throughput_tokens_per_s, 3) if self.throughput_tokens_per_s is not None else None
            ),
            "avg_active_batch": round(self.avg_active_batch, 3),
            "slot_utilization": round(self.slot_utilization, 4),
            "ttft_ms_avg": ttft["mean"],
            "ttft_ms_p50": _p50(ttft),
            "kv_peak_blocks": self.kv_peak_blocks,
            "kv_peak_bytes": self.kv_peak_bytes,
            "peak_memory_mb": self.peak_memory_mb,
            "block_util_final": round(self.block_util_hist[-1], 4) if self.block_util_hist else None,
            "batch_hist": list(self.batch_hist),
            "block_util_hist": [round(v, 4) for v in self.block_util_hist],
        }


def _p50(stats: Dict[str, Optional[float]]) -> Optional[float]:
    return stats["mean"]


class PagedScheduler:
    """Drives ``model`` over ``kv`` to serve a list of requests under a policy."""

    def __init__(self, model: Any, kv: PagedKVCache, engine_cfg: EngineConfig, sampling: SamplingConfig,
                 uniforms: Optional[torch.Tensor] = None) -> None:
        self.model = model
        self.kv = kv
        self.engine_cfg = engine_cfg
        self.sampling = sampling
        self._eos = getattr(getattr(model, "tokenizer", None), "eos_token_id", None)
        self._next_sid = 0
        self._uniforms = uniforms

    # ------------------------------------------------------------- sampling
    def _make_stream(self, seed: int) -> Optional[UniformStream]:
        if self.sampling.is_greedy:
            return None
        if self._uniforms is not None:
            return UniformStream(self.model.device, uniforms=self._uniforms)
        return UniformStream(self.model.device, seed=seed)

    def _next_tokens(self, logits: torch.Tensor, stream: Optional[UniformStream]) -> torch.Tensor:
        """Device int32 next token per row (PagedScheduler._probs/_sample semantics)."""
        if self.sampling.is_greedy:
            return argmax_rows(logits)
        x = logits.reshape(-1, logits.shape[-1])
        rows = x.shape[0]
        stream.reserve(rows)
        toks = sample_logits_rows(x, self.sampling.temperature, stream, err=self.kv.err_word, eps=1e-9)
        stream.advance(rows)
        return toks

    def _probs(self, logits: torch.Tensor) -> torch.Tensor:
        """engine/scheduler.py:227-233: argmax index (greedy) or softmax(logits/max(T,1e-9))."""
        if self.sampling.is_greedy:
            return argmax_rows(logits.reshape(-1, logits.shape[-1])).long().reshape(logits.shape[:-1])
        return probs_rows(logits, self.sampling.temperature, False, eps=1e-9).reshape(logits.shape)

    def _sample(self, probs, generator) -> int:
        if self.sampling.is_greedy:
            return int(probs)
        return sample_token(probs, generator)

    # ------------------------------------------------------------ admission
    def _flush_arrivals(self, arrivals: List[WorkloadRequest], when: int, result: SchedulerResult,
                        stream: Optional[UniformStream]) -> List[Sequence]:
        admitted: List[Sequence] = []
        for request in arrivals:
            seq = Sequence(
                sid=self._next_sid,
                prompt_ids=self.model.encode(request.prompt),
                max_new_tokens=request.max_new_tokens,
                arrive_time=request.arrive_time,
                admit_step=when,
            )
            self._next_sid += 1
            self.kv.add_sequence(seq.sid)
            seq.ttft_ms = self._prefill_one(seq, result, stream)
            admitted.append(seq)
        result.sequences.extend(admitted)
        return admitted

    def _prefill_one(self, seq: Sequence, result: SchedulerResult, stream: Optional[UniformStream]) -> Optional[float]:
        watch = Stopwatch()
        with watch:
            ids = _lib.to_device([list(seq.prompt_ids)], torch.long, self.model.device)
            logits = self.model.prefill(ids, self.kv, [seq.sid], [len(seq.prompt_ids)])
            token = int(self._next_tokens(logits, stream)[0].item())
            seq.generated.append(token)
        seq.prefilled = True
        return watch.elapsed_ms

    # ------------------------------------------------------------ decode step
    def _decode_active(self, running: Seq[Sequence], result: SchedulerResult,
                       stream: Optional[UniformStream]) -> None:
        model = self.model
        ids = _lib.to_device([seq.generated[-1] for seq in running], torch.long, model.device)
        ctx = [self.kv.seq_len(seq.sid) for seq in running]
        logits = model.decode(ids, self.kv, [s.sid for s in running], ctx)
        tokens = self._next_tokens(logits, stream).tolist()
        finished: List[int] = []
        for b, seq in enumerate(running):
            token = tokens[b]
            if self._eos is not None and token == self._eos:
                seq.eos_hit = True
                seq.finished = True
                seq.finish_step = result.steps
            else:
                seq.generated.append(token)
            if len(seq.generated) >= seq.max_new_tokens:
                seq.finished = True
                seq.finish_step = result.steps
            if seq.finished:
                finished.append(seq.sid)
        if finished:
            self.kv.release(finished, [0] * len(finished), [_lib.REL_CLEAR] * len(finished))

    # -------------------------------------------------------------- policies
    def run_continuous(self, requests: Seq[WorkloadRequest], seed: int, measure: bool = True) -> SchedulerResult:
        result = SchedulerResult(mode="continuous", sampling=self.sampling.describe())
        stream = self._make_stream(seed)
        device = self.model.device
        arrivals = sorted(requests, key=lambda r: r.arrive_time)
        step = 0
        if measure:
            sync_device(device)
            torch.cuda.reset_peak_memory_stats(device)
        stopwatch = Stopwatch()
        with stopwatch:
            due = [r for r in arrivals if r.arrive_time <= step]
            pending = [r for r in arrivals if r.arrive_time > step]
            self._flush_arrivals(due, step, result, stream)
            running = [s for s in result.sequences if not s.finished]
            while running or pending:
                running = [s for s in result.sequences if not s.finished]
                if running:
                    self._decode_active(running, result, stream)
                    result.total_forwards += 1
                step += 1
                due = [r for r in pending if r.arrive_time <= step]
                pending = [r for r in pending if r.arrive_time > step]
                if due:
                    self._flush_arrivals(due, step, result, stream)
                running = [s for s in result.sequences if not s.finished]
                result.batch_hist.append(len(running))
                result.block_util_hist.append(self.kv.block_utilization)
                if self.kv.num_allocated_blocks > result.kv_peak_blocks:
                    result.kv_peak_blocks = self.kv.num_allocated_blocks
            result.steps = step
            if measure:
                sync_device(device)
        self.kv.check_errors()
        result.makespan_ms = stopwatch.elapsed_ms
        result.generated_tokens = sum(len(s.generated) for s in result.sequences)
        result.kv_peak_bytes = result.kv_peak_blocks * self._bytes_per_block()
        if measure:
            result.peak_memory_mb = round(torch.cuda.max_memory_allocated(device) / (1024.0 ** 2), 2)
        return result

    def run_static(self, requests: Seq[WorkloadRequest], seed: int, measure: bool = True) -> SchedulerResult:
        """Fixed-batch baseline: everything starts at step 0, idle slots until done."""
        result = SchedulerResult(mode="static", sampling=self.sampling.describe())
        stream = self._make_stream(seed)
        device = self.model.device
        if measure:
            sync_device(device)
            torch.cuda.reset_peak_memory_stats(device)
        stopwatch = Stopwatch()
        with stopwatch:
            self._flush_arrivals(list(requests), 0, result, stream)
            all_seqs = list(result.sequences)
            fixed = len(all_seqs)
            step = 0
            while any(not s.done for s in all_seqs):
                living = [b for b, s in enumerate(all_seqs) if not s.done]
                if living:
                    ids = _lib.to_device([s.generated[-1] if s.generated else 0 for s in all_seqs], torch.long,
                                         device)
                    ctx = [self.kv.seq_len(s.sid) for s in all_seqs]
                    logits = self.model.decode(ids, self.kv, [s.sid for s in all_seqs], ctx)
                    result.total_forwards += 1
                    rows = _lib.to_device(living, torch.long, device)
                    tokens = self._next_tokens(logits.index_select(0, rows), stream).tolist()
                    for token, b in zip(tokens, living):
                        s = all_seqs[b]
                        if self._eos is not None and token == self._eos:
                            s.eos_hit = True
                            s.finished = True
                        else:
                            s.generated.append(token)
                        if len(s.generated) >= s.max_new_tokens:
                            s.finished = True
                        s.finish_step = step
                step += 1
                result.steps = step
                result.batch_hist.append(fixed)
                result.block_util_hist.append(self.kv.block_utilization)
                if self.kv.num_allocated_blocks > result.kv_peak_blocks:
                    result.kv_peak_blocks = self.kv.num_allocated_blocks
            if measure:
                sync_device(device)
        self.kv.check_errors()
        result.makespan_ms = stopwatch.elapsed_ms
        result.generated_tokens = sum(len(s.generated) for s in result.sequences)
        result.kv_peak_bytes = result.kv_peak_blocks * self._bytes_per_block()
        if measure:
            result.peak_memory_mb = round(torch.cuda.max_memory_allocated(device) / (1024.0 ** 2), 2)
        return result

    def _bytes_per_block(self) -> int:
        """Bytes occupied by one physical block across all layers (K+V)."""
        return (
            2 * self.model.num_layers * self.engine_cfg.block_size * self.model.num_kv_heads
            * self.model.head_dim * self.model.dtype.itemsize
        )


def build_kv(model: Any, engine_cfg: EngineConfig, device: torch.device, **kwargs: Any) -> PagedKVCache:
    """Construct a sized paged cache from a model's shape and the engine config."""
    return PagedKVCache(
        num_layers=model.num_layers,
        num_kv_heads=model.num_kv_heads,
        head_dim=model.head_dim,
        capacity_blocks=engine_cfg.max_num_blocks,
        block_size=engine_cfg.block_size,
        device=device,
        dtype=model.dtype,
        **kwargs,
    )
