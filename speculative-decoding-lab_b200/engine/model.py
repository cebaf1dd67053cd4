"""Paged language-model interface and the deterministic toy implementation.

Drop-in for the reference's ``engine/model.py`` (engine/model.py:41-398).  The
"PagedLM" duck type the schedulers drive is unchanged:

* ``prefill(prompt_2d, kv, seq_ids, seq_lengths) -> (B, V)`` first-token logits;
* ``decode(input_ids, kv, seq_ids, ctx_lengths) -> (B, V)``;
* ``decode_block(input_ids_2d, kv, seq_ids, start_positions) -> (B, chunk, V)``.

The attention call sites are what change: each forward reserves the new
positions once (``PagedKVCache.reserve``: one kernel, reference allocation
order), and every layer does one batched K/V append and one paged-attention
launch instead of per-token ``kv.write`` loops and per-sequence SDPA.  The
write-then-attend order of engine/model.py:142-149 / 184-190 is kept: a token
attends its own freshly written K/V.

Module construction order (and so the torch RNG draws of the default
``nn.Linear`` / ``nn.Embedding`` initialisers under ``torch.manual_seed``) is
the reference's, so ``ToyPagedLM(ToyConfig(seed=s))`` has the reference's
weights bit-for-bit.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Union

import torch
from torch import nn

from .attention import AttnBatch, paged_attention
from .kv import PagedKVCache
from . import _lib, layer_ops
from .utils import setup_logger

logger = setup_logger(__name__)


# --------------------------------------------------------------------- rotary
def make_rotary_cache(head_dim: int, theta: float, max_len: int, device: torch.device) -> torch.Tensor:
    """RoPE ``cos``/``sin`` table ``(max_len, 2, head_dim)`` (rotate_half convention)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device="cpu") / head_dim))
    positions = torch.arange(max_len, dtype=torch.float32, device="cpu").unsqueeze(-1)
    freqs = positions * inv_freq.unsqueeze(0)
    emb = torch.cat((freqs, freqs), dim=-1)
    table = torch.stack((emb.cos(), emb.sin()), dim=1)
    return table.to(device)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1]
    return torch.cat((-x[..., d // 2:], x[..., : d // 2]), dim=-1)


def apply_rotary(x: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor) -> torch.Tensor:
    return x * cos + rotate_half(x) * sin


def apply_rotary_(x: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor) -> torch.Tensor:
    """``apply_rotary`` that may overwrite ``x`` (a fresh projection output):
    one fused in-place launch for 16-bit CUDA tensors with contiguous rows."""
    if layer_ops.fusable(x) and x.is_contiguous():
        return layer_ops.rope_(x, sin, cos)
    return apply_rotary(x, sin, cos)


# --------------------------------------------------------------------- norms
class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if layer_ops.fusable(x):  # one fused launch for 16-bit models
            return layer_ops.rmsnorm(x, self.weight, self.eps)
        input_dtype = x.dtype
        xf = x.float()
        rms = torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return ((xf / rms) * self.weight.float()).to(input_dtype)


class SwiGLU(nn.Module):
    def __init__(self, hidden: int, intermediate: int) -> None:
        super().__init__()
        self.gate = nn.Linear(hidden, intermediate, bias=False)
        self.up = nn.Linear(hidden, intermediate, bias=False)
        self.down = nn.Linear(intermediate, hidden, bias=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.down(torch.nn.functional.silu(self.gate(x)) * self.up(x))


# ------------------------------------------------------------ forward plans
class ForwardPlan:
    """Slots and attention rows of one forward, shared by every layer.

    ``slots`` has one int32 entry per (row, chunk position) in row-major order
    (-1 for padded prefill positions); ``batch`` describes the attention rows.
    """

    __slots__ = ("slots", "batch", "positions", "chunk", "append_first")

    def __init__(self, slots: torch.Tensor, batch: AttnBatch, positions: torch.Tensor, chunk: int,
                 append_first: bool = False) -> None:
        self.slots = slots
        self.batch = batch
        self.positions = positions
        self.chunk = chunk
        # rows of one sequence may read each other's new K/V (chunked
        # prefill): every layer stores all new rows before it attends
        self.append_first = append_first


def plan_decode(kv: PagedKVCache, seq_ids: Sequence[int], ctx_lengths: Sequence[int],
                slots: Optional[torch.Tensor] = None) -> ForwardPlan:
    """One new token per row at position ``ctx_lengths[b]``; it attends ``[0, ctx]``."""
    ctx = [int(c) for c in ctx_lengths]
    if slots is None:
        slots = kv.reserve(seq_ids, ctx, [1] * len(ctx))
    batch = AttnBatch.from_lists(kv.device, seq_ids, ctx, 1)
    return ForwardPlan(slots, batch, batch.starts.long().unsqueeze(1), 1)


def plan_block(kv: PagedKVCache, seq_ids: Sequence[int], start_positions: Sequence[int], chunk: int) -> ForwardPlan:
    """``chunk`` consecutive tokens per row from ``start_positions[b]``."""
    starts = [int(s) for s in start_positions]
    slots = kv.reserve(seq_ids, starts, [chunk] * len(starts))
    batch = AttnBatch.from_lists(kv.device, seq_ids, starts, chunk)
    pos = batch.starts.long().unsqueeze(1) + torch.arange(chunk, device=kv.device).unsqueeze(0)
    return ForwardPlan(slots, batch, pos, chunk)


def plan_prefill(kv: PagedKVCache, seq_ids: Sequence[int], seq_lengths: Sequence[int], chunk: int) -> ForwardPlan:
    """Ragged prompts (tail-padded to ``chunk``) written from position 0."""
    lengths = [int(x) for x in seq_lengths]
    B = len(lengths)
    slots = kv.reserve(seq_ids, [0] * B, lengths)
    if any(ln != chunk for ln in lengths):
        grid = torch.full((B * chunk,), -1, dtype=torch.int32, device=kv.device)
        lens_t = _lib.to_device(lengths, torch.long, kv.device)
        mask = (torch.arange(chunk, device=kv.device).unsqueeze(0) < lens_t.unsqueeze(1)).reshape(-1)
        grid[mask] = slots
        slots = grid
    packed = _lib.i32([int(s) for s in seq_ids] + [0] * B + lengths, kv.device)
    batch = AttnBatch(packed[:B], packed[B:2 * B], chunk, packed[2 * B:], key_count=sum(lengths))
    pos = torch.arange(chunk, device=kv.device).unsqueeze(0).expand(B, chunk)
    return ForwardPlan(slots, batch, pos, chunk)


def paged_attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv: PagedKVCache, layer: int,
                 plan: ForwardPlan, rope=None) -> torch.Tensor:
    """Store this layer's K/V at the plan's positions, then attend (write
    first) -- one fused call; the positions were reserved by the plan.
    ``rope = (cos, sin)``: q and k arrive unrotated and the call applies
    RoPE (inside the attention launch where its kernel can; not with
    ``append_first``, whose rows are stored before the call)."""
    B = q.shape[0]
    q4 = q.reshape(B, plan.chunk, q.shape[-2], q.shape[-1])
    if plan.append_first:
        if rope is not None:
            raise ValueError("paged_attend: rope with append_first (rotate q and k before the call)")
        kv.append(layer, plan.slots, k.reshape(B * plan.chunk, k.shape[-2], k.shape[-1]),
                  v.reshape(B * plan.chunk, v.shape[-2], v.shape[-1]))
        return paged_attention(q4, kv, layer, plan.batch)
    return paged_attention(q4, kv, layer, plan.batch, k_new=k.reshape(B * plan.chunk, -1),
                           v_new=v.reshape(B * plan.chunk, -1), rope=rope)


# ------------------------------------------------------------- decoder layer
class PagedDecoderLayer(nn.Module):
    """Decoder block with paged self-attention + SwiGLU MLP (engine/model.py:96-194)."""

    def __init__(self, hidden: int, num_q_heads: int, num_kv_heads: int, head_dim: int, intermediate: int) -> None:
        super().__init__()
        self.num_q_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.input_layernorm = RMSNorm(hidden)
        self.q = nn.Linear(hidden, num_q_heads * head_dim, bias=False)
        self.k = nn.Linear(hidden, num_kv_heads * head_dim, bias=False)
        self.v = nn.Linear(hidden, num_kv_heads * head_dim, bias=False)
        self.o = nn.Linear(num_q_heads * head_dim, hidden, bias=False)
        self.post_attention_layernorm = RMSNorm(hidden)
        self.mlp = SwiGLU(hidden, intermediate)

    def _qkv(self, x: torch.Tensor, lead: tuple):
        q = self.q(x).view(*lead, self.num_q_heads, self.head_dim)
        k = self.k(x).view(*lead, self.num_kv_heads, self.head_dim)
        v = self.v(x).view(*lead, self.num_kv_heads, self.head_dim)
        return q, k, v

    def forward_plan(self, hidden: torch.Tensor, kv: PagedKVCache, layer_index: int, plan: ForwardPlan,
                     cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """``hidden`` is ``(B, H)`` (chunk 1) or ``(B, chunk, H)``; cos/sin broadcast over heads."""
        lead = tuple(hidden.shape[:-1])
        residual = hidden
        x = self.input_layernorm(hidden)
        q_raw, k_raw, v_raw = self._qkv(x, lead)
        q = apply_rotary(q_raw, sin, cos)
        k = apply_rotary(k_raw, sin, cos)
        out = paged_attend(q, k, v_raw, kv, layer_index, plan)
        hidden = residual + self.o(out.reshape(*lead, -1))
        return hidden + self.mlp(self.post_attention_layernorm(hidden))

    def decode_step(self, hidden, kv, layer_index, seq_ids, ctx_lengths, cos, sin):
        plan = seq_ids if isinstance(seq_ids, ForwardPlan) else plan_decode(kv, seq_ids, ctx_lengths)
        return self.forward_plan(hidden, kv, layer_index, plan, cos, sin)

    def extend_block(self, hidden, kv, layer_index, seq_ids, start_positions, cos, sin):
        if isinstance(seq_ids, ForwardPlan):
            plan = seq_ids
        else:
            plan = plan_block(kv, seq_ids, start_positions, hidden.shape[1])
        return self.forward_plan(hidden, kv, layer_index, plan, cos[:, :, None, :], sin[:, :, None, :])


# ----------------------------------------------------------------- plain text
class ToyTokenizer:
    """Character-level tokenizer covering ``vocab_size`` symbols."""

    def __init__(self, vocab_size: int = 16) -> None:
        alphabet = "abcdefghijklmnopqrstuvwxyz"
        self.vocab_size = vocab_size
        self.itos = list(alphabet[:vocab_size])
        self.stoi = {ch: idx for idx, ch in enumerate(self.itos)}
        self.pad_token_id = 0
        self.eos_token_id = None

    def encode(self, text: Union[str, Sequence[int]]) -> List[int]:
        if not isinstance(text, str):
            return [int(t) for t in text]
        return [self.stoi[ch] for ch in text if ch in self.stoi]

    def decode(self, token_ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        return "".join(self.itos[int(i) % self.vocab_size] for i in token_ids)


class IdTokenizer:
    """Pass-through "tokenizer" for random-init models fed token-id prompts."""

    def __init__(self, vocab_size: int, eos_token_id: Optional[int] = None) -> None:
        self.vocab_size = vocab_size
        self.eos_token_id = eos_token_id
        self.pad_token_id = 0

    def encode(self, text: Union[str, Sequence[int]]) -> List[int]:
        if isinstance(text, str):
            return [int(t) % self.vocab_size for t in text.split()]
        return [int(t) for t in text]

    def decode(self, token_ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        return " ".join(str(int(t)) for t in token_ids)


# ----------------------------------------------------------------- toy model
@dataclass
class ToyConfig:
    vocab_size: int = 16
    hidden_size: int = 64
    num_layers: int = 2
    num_attention_heads: int = 4
    num_key_value_heads: int = 2
    head_dim: int = 16
    intermediate_size: int = 128
    max_position_embeddings: int = 256
    theta: float = 10000.0
    logit_scale: float = 6.0
    seed: int = 0


class _GraphedForward:
    """One captured paged forward (embedding to logits) for a fixed cache,
    rows per position (``chunk``) and padded batch size.

    Static device inputs (token ids, block-table rows, start positions) are
    refilled before each replay; rows beyond the real batch repeat row 0, so
    they store the same K/V bytes at the same positions and their logits are
    discarded.  Reservation of the positions and sampling stay outside the
    graph.
    """

    __slots__ = ("graph", "ids", "rows", "starts", "logits", "keep", "table_ptr", "calls")

    def __init__(self, graph, ids, rows, starts, logits, keep, table_ptr, calls=0) -> None:
        self.graph = graph
        self.calls = calls  # library entry calls captured (counted again at every replay)
        self.ids = ids
        self.rows = rows
        self.starts = starts
        self.logits = logits
        self.keep = keep  # every other tensor the captured kernels read (must outlive the graph)
        self.table_ptr = table_ptr  # the block table the graph reads; a grown (moved) table needs a new capture


class _GraphedPrefillRows:
    """One captured batched prefill of ``bucket`` 128-token chunk rows (the
    decoder layers and the final norm; the head runs on the selected last
    positions after the replay).  Static inputs: the chunk rows' token ids,
    the slot of every (row, position) (-1 past a chunk's end), and per row
    the sequence, start position and valid count; rows past the call's repeat
    row 0 with nothing valid, so they store nothing and attend nothing."""

    __slots__ = ("graph", "ids", "grid", "meta", "normed", "keep", "table_ptr", "calls")

    def __init__(self, graph, ids, grid, meta, normed, keep, table_ptr, calls=0) -> None:
        self.graph = graph
        self.ids = ids
        self.grid = grid
        self.meta = meta
        self.normed = normed
        self.keep = keep
        self.table_ptr = table_ptr
        self.calls = calls


class _GraphedPrefill:
    """One captured prefill of a single prompt, padded to a length bucket
    (``prefill_bucket_of``).  Static inputs (token ids, block-table row, prompt length,
    last position) are refilled before each replay; positions past the prompt
    are computed but never stored (the attention's valid-row count) and their
    hidden states are dropped."""

    __slots__ = ("graph", "ids", "meta", "logits", "keep", "table_ptr", "calls")

    def __init__(self, graph, ids, meta, logits, keep, table_ptr, calls=0) -> None:
        self.graph = graph
        self.calls = calls  # library entry calls captured (counted again at every replay)
        self.ids = ids
        self.meta = meta  # (block-table row, prompt length, last position) as device tensors
        self.logits = logits
        self.keep = keep  # every other tensor the captured kernels read (must outlive the graph)
        self.table_ptr = table_ptr


class PagedLMMixin:
    """prefill / decode / decode_block over a stack of layers with ``forward_plan``.

    ``enable_cuda_graphs()`` switches decode / decode_block to CUDA-graph
    replays of the whole forward (one capture per cache, chunk and batch
    bucket) -- the host issues a handful of copies and one replay instead of
    ~25 launches per layer.  The kernels are the same; a padded batch may
    change the GEMM library's and the split-K merge's reduction order, so
    logits agree with the eager path to rounding, not bit for bit.
    """

    GRAPH_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384, 448, 512,
                     640, 768, 896, 1024, 1280, 1536)

    def enable_cuda_graphs(self, enabled: bool = True) -> None:
        self._graphs_enabled = bool(enabled)
        if not enabled:
            self._graphs = {}

    def _graph_pool(self):
        """One memory pool shared by all of this model's live graphs: their
        intermediates are dead between replays, which never overlap (one
        stream), so later captures may reuse what earlier ones freed.  The
        pool is a live graph's (a pool whose graphs were all released cannot
        take new captures); with none alive, a fresh one."""
        for g in self.__dict__.get("_graphs", {}).values():
            return g.graph.pool()
        return torch.cuda.graph_pool_handle()

    def _graph_logits_buffer(self, chunk: int, bucket: int) -> torch.Tensor:
        """``(bucket, chunk, vocab)`` view of the one logits buffer the graphs
        of ``chunk`` rows per sequence share (sized for the largest bucket):
        a replay's logits are consumed before the next replay of this model."""
        bufs = self.__dict__.setdefault("_logits_bufs", {})
        buf = bufs.get(chunk)
        w = self.lm_head.weight
        if buf is None:
            buf = torch.empty((self.GRAPH_BUCKETS[-1], chunk, w.shape[0]), dtype=w.dtype, device=w.device)
            bufs[chunk] = buf
        return buf[:bucket]

    def _graph_bucket(self, batch: int) -> Optional[int]:
        if not getattr(self, "_graphs_enabled", False):
            return None
        for b in self.GRAPH_BUCKETS:
            if b >= batch:
                return b
        return None

    def _graph_forward(self, input_ids_2d: torch.Tensor, kv: PagedKVCache, seq_ids: Sequence[int],
                       starts: Sequence[int], bucket: int, logits_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Logits ``(B, chunk, V)`` of positions ``starts[b] + j`` (already
        reserved) through the captured forward for ``bucket`` rows.

        With ``graph_head`` False the graphs end at the final norm and the LM
        head runs after the replay, on all ``bucket`` rows (the shape the
        captured head would have), writing into ``logits_out`` (at least
        ``bucket`` rows of ``(chunk, V)``) when given: a caller that keeps
        several forwards' logits gets them without a copy.  With the head in
        the graph, ``logits_out`` receives a copy of the logits."""
        B, chunk = input_ids_2d.shape
        head = bool(getattr(self, "graph_head", True))
        graphs = self.__dict__.setdefault("_graphs", {})
        # key span bucket: the attention plan (split size, kernel choice) is
        # fixed at capture, so graphs are kept per power-of-two bound of the
        # rows' key span rather than per the whole table width
        span = self.span_bucket(kv, max(int(x) for x in starts) + chunk)
        key = (id(kv), chunk, bucket, span) if head else (id(kv), chunk, bucket, span, "headless")
        g = graphs.get(key)
        if g is not None and g.table_ptr != kv._table.data_ptr():
            # the cache grew its block table (more sequence rows): recapture
            del graphs[key]
            g = None
        meta = _lib.i32([int(x) for x in seq_ids] + [int(x) for x in starts], self.device)
        ids = input_ids_2d.to(self.device)

        def fill(dst_ids, dst_rows, dst_starts):
            dst_ids[:B].copy_(ids)
            dst_rows[:B].copy_(meta[:B])
            dst_starts[:B].copy_(meta[B:])
            if bucket > B:
                dst_ids[B:].copy_(ids[:1].expand(bucket - B, chunk))
                dst_rows[B:].copy_(meta[:1].expand(bucket - B))
                dst_starts[B:].copy_(meta[B:B + 1].expand(bucket - B))

        if g is None:
            s_ids = torch.zeros((bucket, chunk), dtype=torch.long, device=self.device)
            s_rows = torch.zeros(bucket, dtype=torch.int32, device=self.device)
            s_starts = torch.zeros(bucket, dtype=torch.int32, device=self.device)
            fill(s_ids, s_rows, s_starts)
            # replays run other lengths than this capture's: the attention
            # plans are the ones for ragged rows of unknown lengths
            # (key_count < 0), bounded by the bucket and the span
            batch = AttnBatch(s_rows, s_starts, span, key_count=-1)
            steps = torch.arange(chunk, device=self.device)

            shared_logits = self._graph_logits_buffer(chunk, bucket) if head else None

            def run() -> torch.Tensor:
                positions = s_starts.long().unsqueeze(1) + steps.unsqueeze(0)
                normed = self._body(s_ids, kv, batch, positions)
                if not head:
                    return normed  # the head runs after the replay
                # the head writes into the logits buffer every graph of this chunk shares
                return torch.matmul(normed, self.lm_head.weight.t(), out=shared_logits)

            # one eager pass sizes every workspace and stores this call's K/V;
            # the replay below stores the same bytes again
            run()
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            c0 = _lib.calls()
            with _lib.no_gc(), torch.cuda.graph(graph, pool=self._graph_pool()):
                logits = run()
            g = _GraphedForward(graph, s_ids, s_rows, s_starts, logits, (steps, batch, kv), kv._table.data_ptr(),
                                _lib.calls() - c0)
            graphs[key] = g
        else:
            fill(g.ids, g.rows, g.starts)
        g.graph.replay()
        _lib.count_calls(g.calls)
        if head:
            if logits_out is None:
                return g.logits[:B]
            dst = logits_out[:B].view(B, chunk, -1)
            dst.copy_(g.logits[:B])
            return dst
        V = self.lm_head.weight.shape[0]
        dst = logits_out if logits_out is not None else self._graph_logits_buffer(chunk, bucket)
        dst = dst[:bucket].view(bucket, chunk, V)
        torch.matmul(g.logits, self.lm_head.weight.t(), out=dst)
        return dst[:B]

    def _body(self, ids_2d: torch.Tensor, kv: PagedKVCache, batch: AttnBatch, positions: torch.Tensor) -> torch.Tensor:
        """Embedding, decoder layers and final norm of one forward over rows
        ``ids_2d`` (B, chunk) at ``positions`` (already reserved), from
        device tensors only, so a CUDA graph can capture it."""
        chunk = ids_2d.shape[1]
        plan = ForwardPlan(None, batch, positions, chunk)
        hidden = self.embed_tokens(ids_2d)
        cos, sin = self._rope(positions)
        hidden = self._run_layers(hidden, kv, plan, cos[:, :, None, :], sin[:, :, None, :])
        return self.norm(hidden)

    def max_positions(self) -> int:
        """Positions the rotary table covers (a forward may not reach past)."""
        return int(self._rope_table().shape[0])

    def _check_reach(self, need: int) -> None:
        """Raise on the host before a forward reaches position ``need - 1``
        past the rotary table (on the device that is an out-of-range gather)."""
        if need > self.max_positions():
            raise ValueError("position {} is past the rotary table ({} positions)".format(need - 1,
                                                                                         self.max_positions()))

    def _span_cap(self, kv: PagedKVCache) -> int:
        return min(kv.width * kv.block_size, self.max_positions())

    def span_bucket(self, kv: PagedKVCache, need: int) -> int:
        """The key-span bucket of a forward whose rows reach position
        ``need - 1``: a power of two from 1024, capped at the table width and
        the rotary table's length (a larger ``need`` raises)."""
        self._check_reach(need)
        span = 1024
        while span < need:
            span *= 2
        return min(span, self._span_cap(kv))

    def graph_spans(self, kv: PagedKVCache) -> List[int]:
        """The key-span buckets ``_graph_forward`` keys its graphs by for
        ``kv``: powers of two from 1024, the last one capped at the table's
        width in tokens and the rotary table's length."""
        cap = self._span_cap(kv)
        spans, s = [], 1024
        while True:
            spans.append(min(s, cap))
            if s >= cap:
                return spans
            s *= 2

    def capture_graphs(self, kv: PagedKVCache, sid: int, chunk: int, prefill: bool = True,
                       buckets: Optional[Sequence[int]] = None) -> int:
        """Capture, before serving, every forward graph a run can replay for
        ``kv``: ``chunk`` positions per row (1 = decode, gamma+1 = verify) at
        every batch bucket and key-span bucket, and with ``prefill`` every
        prompt-length bucket.  A serving process does this at start-up, so no
        capture (an eager pass plus a capture, tens of milliseconds) falls
        inside a run, whatever its requests.

        ``sid`` is a registered, empty block-table row used as scratch: its
        positions are reserved, written and released here.  Each span bucket
        is captured at a span just inside it (55 % of the bucket, and above
        the previous bucket), which sets the captured attention plans' split
        sizes.  Returns the number of graphs captured."""
        if not getattr(self, "_graphs_enabled", False):
            return 0
        graphs = self.__dict__.setdefault("_graphs", {})
        n0 = len(graphs)
        buckets = list(buckets) if buckets is not None else list(self.GRAPH_BUCKETS)
        ids = torch.zeros((1, chunk), dtype=torch.long, device=self.device)
        prev = 0
        for span in self.graph_spans(kv):
            need = max(prev + 1, int(0.55 * span), chunk)
            prev = span
            kv.reserve([sid], [0], [need])
            for b in buckets:
                self._graph_forward(ids, kv, [sid], [need - chunk], b)
            kv.clear(sid)
        if prefill:
            cb = self.PREFILL_MIN_BUCKET
            while self._prefill_bucket(kv, 1, cb, cb) == cb:
                self.prefill(torch.zeros((1, cb), dtype=torch.long, device=self.device), kv, [sid], [cb])
                kv.clear(sid)
                cb = self.prefill_bucket_of(cb + 1)
            if self._prefill_rows_bucket(kv, 1) is not None:
                # batched prefills: every row one full chunk of the scratch
                # sequence at position 0 (the rows store the same bytes)
                C = self.PREFILL_CHUNK
                slots = kv.reserve([sid], [0], [C])
                ids0 = torch.zeros((1, C), dtype=torch.long, device=self.device)
                for rb in self.PREFILL_ROW_BUCKETS:
                    self._graph_prefill_rows(kv, ids0.expand(rb, C), slots.repeat(rb), [sid] * rb, [0] * rb,
                                             [C] * rb, rb)
                kv.clear(sid)
        torch.cuda.synchronize(self.device)
        return len(graphs) - n0

    def _rope(self, positions: torch.Tensor):
        cs = self._rope_table()[positions]
        return cs[..., 0, :], cs[..., 1, :]

    def _run_layers(self, hidden: torch.Tensor, kv: PagedKVCache, plan: ForwardPlan,
                    cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        # A layer may hand on its residual stream as a pair (hidden, delta):
        # the next layer's input norm adds delta in the same launch.
        for index, layer in enumerate(self.layers):
            hidden = layer.forward_plan(hidden, kv, index, plan, cos, sin)
        if isinstance(hidden, tuple):
            hidden = hidden[0] + hidden[1]
        return hidden

    PREFILL_MIN_BUCKET = 64

    @classmethod
    def prefill_bucket_of(cls, n: int) -> int:
        """Padded length of a graphed prefill of ``n`` tokens: 64, then
        multiples of 128 up to 1024, of 256 up to 4096, then powers of two
        (the padded positions cost GEMM rows, so the steps stay fine where
        prompts are common)."""
        if n <= cls.PREFILL_MIN_BUCKET:
            return cls.PREFILL_MIN_BUCKET
        if n <= 1024:
            return -(-n // 128) * 128
        if n <= 4096:
            return -(-n // 256) * 256
        cb = 4096
        while cb < n:
            cb *= 2
        return cb

    def _prefill_bucket(self, kv: PagedKVCache, B: int, chunk: int, length: int) -> Optional[int]:
        """Length bucket of a graphed prefill, or None for the eager path:
        graphs on, one prompt without padding, a 16-bit model (fp32 models
        keep eager prefills, whose reductions the parity runs pin), and a
        bucket the block table and the rotary table both cover."""
        if not getattr(self, "_graphs_enabled", False) or B != 1 or chunk != length:
            return None
        if self.embed_tokens.weight.dtype not in (torch.bfloat16, torch.float16):
            return None
        cb = self.prefill_bucket_of(chunk)
        if cb > kv.width * kv.block_size or cb > self._rope_table().shape[0]:
            return None
        return cb

    def _graph_prefill(self, prompt_2d: torch.Tensor, kv: PagedKVCache, sid: int, length: int,
                       cb: int) -> torch.Tensor:
        """First-token logits ``(1, V)`` of one prompt (positions already
        reserved) through the captured prefill of bucket ``cb``."""
        graphs = self.__dict__.setdefault("_graphs", {})
        key = (id(kv), "prefill", cb)
        g = graphs.get(key)
        if g is not None and g.table_ptr != kv._table.data_ptr():
            del graphs[key]  # the block table grew (moved): recapture
            g = None
        meta = _lib.i32([int(sid), int(length), int(length) - 1], self.device)
        ids = prompt_2d.to(self.device)

        def fill(dst_ids, dst_meta):
            dst_ids[:, :length].copy_(ids)
            dst_ids[:, length:].zero_()
            dst_meta.copy_(meta)

        if g is None:
            s_ids = torch.zeros((1, cb), dtype=torch.long, device=self.device)
            s_meta = torch.zeros(3, dtype=torch.int32, device=self.device)
            fill(s_ids, s_meta)
            s_starts = torch.zeros(1, dtype=torch.int32, device=self.device)
            batch = AttnBatch(s_meta[0:1], s_starts, cb, s_meta[1:2], key_count=cb)
            positions = torch.arange(cb, device=self.device).unsqueeze(0)

            def run() -> torch.Tensor:
                plan = ForwardPlan(None, batch, positions, cb)
                hidden = self.embed_tokens(s_ids)
                cos, sin = self._rope(positions)
                hidden = self._run_layers(hidden, kv, plan, cos[:, :, None, :], sin[:, :, None, :])
                h_last = hidden.index_select(1, s_meta[2:3].long())[:, 0]
                return self._logits(h_last)

            # one eager pass sizes every workspace and stores this prompt's
            # K/V; the replay below stores the same bytes again
            run()
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            c0 = _lib.calls()
            with _lib.no_gc(), torch.cuda.graph(graph, pool=self._graph_pool()):
                logits = run()
            g = _GraphedPrefill(graph, s_ids, s_meta, logits, (s_starts, positions, batch, kv), kv._table.data_ptr(),
                                _lib.calls() - c0)
            graphs[key] = g
        else:
            fill(g.ids, g.meta)
        g.graph.replay()
        _lib.count_calls(g.calls)
        return g.logits

    def prefill(self, prompt_2d: torch.Tensor, kv: PagedKVCache, seq_ids: Sequence[int],
                seq_lengths: Sequence[int]) -> torch.Tensor:
        """Prefill ragged prompts; return first-token logits ``(B, V)``.

        With CUDA graphs enabled, a single unpadded prompt of a 16-bit model
        replays a captured prefill padded to a length bucket (``prefill_bucket_of``)."""
        self.forward_calls += 1
        B, chunk = prompt_2d.shape
        self._check_reach(chunk)
        cb = self._prefill_bucket(kv, B, chunk, int(seq_lengths[0]) if B == 1 else -1)
        if cb is not None:
            kv.reserve(seq_ids, [0], [chunk])
            return self._graph_prefill(prompt_2d, kv, seq_ids[0], chunk, cb)
        plan = plan_prefill(kv, seq_ids, seq_lengths, chunk)
        hidden = self.embed_tokens(prompt_2d.to(self.device))
        cos, sin = self._rope(plan.positions)
        hidden = self._run_layers(hidden, kv, plan, cos[:, :, None, :], sin[:, :, None, :])
        last = _lib.to_device([int(x) - 1 for x in seq_lengths], torch.long, self.device)
        h_last = hidden[torch.arange(B, device=self.device), last]
        return self._logits(h_last)

    PREFILL_CHUNK = 128

    def prefill_batch(self, prompts: Sequence, kv: PagedKVCache, seq_ids: Sequence[int]) -> torch.Tensor:
        """Prefill several prompts (lists of ids or 1-D id tensors) of
        registered, empty sequences in one forward; returns first-token
        logits ``(B, V)``.

        Every prompt is cut into PREFILL_CHUNK-token chunks and each chunk is
        one row of an extend-attention batch: row j of chunk c attends
        positions ``0 .. c*CHUNK + j`` of its own sequence, the earlier
        chunks' K/V coming from the pool -- so each layer stores all the new
        K/V rows (one append launch) before it attends.  The GEMMs run over
        the chunks, padded only in each prompt's last chunk.  Positions are
        reserved in the reference's order (sequence by sequence)."""
        self.forward_calls += 1
        C = self.PREFILL_CHUNK
        dev = self.device
        lens = [int(len(p)) for p in prompts]
        B = len(lens)
        self._check_reach(max(lens))
        slots = kv.reserve(seq_ids, [0] * B, lens)
        rows, starts, valid, src, idx = [], [], [], [], []
        off = 0
        last_row = []
        for i, L in enumerate(lens):
            for c0 in range(0, L, C):
                n = min(C, L - c0)
                rows.append(int(seq_ids[i]))
                starts.append(c0)
                valid.append(n)
                idx.append((off + c0, n))
            last_row.append((len(rows) - 1, valid[-1] - 1))
            off += L
        R = len(rows)
        rb = self._prefill_rows_bucket(kv, R)
        # token ids and the slot of every (row, position), -1 past a chunk's end
        pieces = [p.to(dev, torch.long).reshape(-1) if isinstance(p, torch.Tensor)
                  else _lib.to_device(list(p), torch.long, dev) for p in prompts]
        flat_ids = torch.cat(pieces) if B > 1 else pieces[0]
        gather = torch.full((R, C), -1, dtype=torch.long)
        for r, (o, n) in enumerate(idx):
            gather[r, :n] = torch.arange(o, o + n)
        gather = gather.to(dev, non_blocking=True)
        mask = gather >= 0
        safe = gather.clamp(min=0)
        ids = torch.where(mask, flat_ids[safe], torch.zeros_like(safe))
        grid = torch.where(mask, slots[safe].to(torch.int32), torch.full_like(safe, -1, dtype=torch.int32))
        if rb is not None:
            normed = self._graph_prefill_rows(kv, ids, grid.reshape(-1), rows, starts, valid, rb)
            sel = _lib.to_device([r * C + j for r, j in last_row], torch.long, dev)
            h_last = normed.reshape(rb * C, -1).index_select(0, sel)
            return torch.matmul(h_last, self.lm_head.weight.t())
        packed = _lib.i32(rows + starts + valid, dev)
        batch = AttnBatch(packed[:R], packed[R:2 * R], max(lens), packed[2 * R:],
                          key_count=sum(s_ + C for s_ in starts))
        positions = packed[R:2 * R].long().unsqueeze(1) + torch.arange(C, device=dev).unsqueeze(0)
        # a last chunk's padding positions may pass the rotary table: they are never stored or read
        positions = positions.clamp(max=self.max_positions() - 1)
        plan = ForwardPlan(grid.reshape(-1), batch, positions, C, append_first=True)
        hidden = self.embed_tokens(ids)
        cos, sin = self._rope(positions)
        hidden = self._run_layers(hidden, kv, plan, cos[:, :, None, :], sin[:, :, None, :])
        sel = _lib.to_device([r * C + j for r, j in last_row], torch.long, dev)
        h_last = hidden.reshape(R * C, -1).index_select(0, sel)
        return self._logits(h_last)

    # chunk-row buckets of graphed batched prefills: padding rows cost full
    # GEMM rows, so the steps stay within ~1/7 of the bucket
    PREFILL_ROW_BUCKETS = (1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 14, 16, 18, 20, 23, 26, 30, 34, 39, 44, 50, 57,
                           64, 73, 83, 95, 108, 128)

    def _prefill_rows_bucket(self, kv: PagedKVCache, R: int) -> Optional[int]:
        """Row bucket of a graphed batched prefill of ``R`` chunk rows, or
        None for the eager path (graphs off, an fp32 model -- whose
        reductions the parity runs pin -- or more rows than the largest
        bucket)."""
        if not getattr(self, "_graphs_enabled", False):
            return None
        if self.embed_tokens.weight.dtype not in (torch.bfloat16, torch.float16):
            return None
        for b in self.PREFILL_ROW_BUCKETS:
            if b >= R:
                return b
        return None

    def _graph_prefill_rows(self, kv: PagedKVCache, ids: torch.Tensor, grid: torch.Tensor, rows: List[int],
                            starts: List[int], valid: List[int], rb: int) -> torch.Tensor:
        """Normed hidden states ``(rb, C, H)`` of ``prefill_batch``'s chunk
        rows (positions already reserved) through the captured layers for
        ``rb`` rows; rows past ``len(rows)`` repeat row 0 with nothing valid.
        The attention plans are the ragged-rows ones over the table's whole
        reach, so one capture serves every prompt mix."""
        C = self.PREFILL_CHUNK
        R = len(rows)
        graphs = self.__dict__.setdefault("_graphs", {})
        key = (id(kv), "prefill_rows", rb)
        g = graphs.get(key)
        if g is not None and g.table_ptr != kv._table.data_ptr():
            del graphs[key]  # the block table grew (moved): recapture
            g = None
        pad = rb - R
        meta = _lib.i32(rows + [rows[0]] * pad + starts + [starts[0]] * pad + valid + [0] * pad, self.device)

        def fill(dst_ids, dst_grid, dst_meta):
            dst_ids[:R].copy_(ids)
            dst_grid[:R * C].copy_(grid)
            if pad:
                dst_ids[R:].zero_()
                dst_grid[R * C:].fill_(-1)
            dst_meta.copy_(meta.view(3, rb))

        if g is None:
            s_ids = torch.zeros((rb, C), dtype=torch.long, device=self.device)
            s_grid = torch.full((rb * C,), -1, dtype=torch.int32, device=self.device)
            s_meta = torch.zeros((3, rb), dtype=torch.int32, device=self.device)
            fill(s_ids, s_grid, s_meta)
            batch = AttnBatch(s_meta[0], s_meta[1], self._span_cap(kv), s_meta[2], key_count=-1)
            steps = torch.arange(C, device=self.device)
            top = self.max_positions() - 1

            def run() -> torch.Tensor:
                # a last chunk's padding positions may pass the rotary table:
                # they are never stored or read
                positions = (s_meta[1].long().unsqueeze(1) + steps.unsqueeze(0)).clamp(max=top)
                plan = ForwardPlan(s_grid, batch, positions, C, append_first=True)
                hidden = self.embed_tokens(s_ids)
                cos, sin = self._rope(positions)
                hidden = self._run_layers(hidden, kv, plan, cos[:, :, None, :], sin[:, :, None, :])
                return self.norm(hidden)

            # one eager pass sizes every workspace and stores this call's K/V;
            # the replay below stores the same bytes again
            run()
            torch.cuda.synchronize(self.device)
            graph = torch.cuda.CUDAGraph()
            c0 = _lib.calls()
            with _lib.no_gc(), torch.cuda.graph(graph, pool=self._graph_pool()):
                normed = run()
            g = _GraphedPrefillRows(graph, s_ids, s_grid, s_meta, normed, (steps, batch, kv),
                                    kv._table.data_ptr(), _lib.calls() - c0)
            graphs[key] = g
        else:
            fill(g.ids, g.grid, g.meta)
        g.graph.replay()
        _lib.count_calls(g.calls)
        return g.normed

    def decode(self, input_ids: torch.Tensor, kv: PagedKVCache, seq_ids: Sequence[int],
               ctx_lengths: Sequence[int], slots: Optional[torch.Tensor] = None,
               logits_out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One token per row at position ``ctx_lengths[b]``; returns ``(B, V)``.

        ``slots`` (optional) are positions already reserved by a commit kernel.
        ``logits_out`` (optional, contiguous ``(R, V)`` with R at least B and at
        least the graph bucket of B) receives the logits, which are then
        returned as its first B rows.
        """
        self.forward_calls += 1
        B = len(seq_ids)
        if B:
            self._check_reach(max(int(c) for c in ctx_lengths) + 1)
        bucket = self._graph_bucket(B)
        if logits_out is not None and (logits_out.shape[0] < max(B, bucket or 0) or not logits_out.is_contiguous()):
            raise ValueError("logits_out needs max(B, graph bucket) contiguous rows")
        if bucket is not None:
            ctx = [int(c) for c in ctx_lengths]
            if slots is None:
                kv.reserve(seq_ids, ctx, [1] * len(ctx))
            return self._graph_forward(input_ids.reshape(-1, 1), kv, seq_ids, ctx, bucket, logits_out)[:, 0]
        plan = plan_decode(kv, seq_ids, ctx_lengths, slots)
        hidden = self.embed_tokens(input_ids.to(self.device).reshape(-1))
        cos, sin = self._rope(plan.positions[:, 0])
        hidden = self._run_layers(hidden, kv, plan, cos.unsqueeze(1), sin.unsqueeze(1))
        logits = self._logits(hidden)
        if logits_out is None:
            return logits
        logits_out[:B].copy_(logits)
        return logits_out[:B]

    def decode_block(self, input_ids_2d: torch.Tensor, kv: PagedKVCache, seq_ids: Sequence[int],
                     start_positions: Sequence[int]) -> torch.Tensor:
        """``chunk`` consecutive tokens per row; returns ``(B, chunk, V)``."""
        self.forward_calls += 1
        B, chunk = input_ids_2d.shape
        if B:
            self._check_reach(max(int(x) for x in start_positions) + chunk)
        bucket = self._graph_bucket(B)
        if bucket is not None:
            starts = [int(x) for x in start_positions]
            kv.reserve(seq_ids, starts, [chunk] * B)
            return self._graph_forward(input_ids_2d, kv, seq_ids, starts, bucket)
        plan = plan_block(kv, seq_ids, start_positions, chunk)
        hidden = self.embed_tokens(input_ids_2d.to(self.device))
        cos, sin = self._rope(plan.positions)
        hidden = self._run_layers(hidden, kv, plan, cos[:, :, None, :], sin[:, :, None, :])
        return self._logits(hidden)


class ToyPagedLM(PagedLMMixin, nn.Module):
    """Deterministic, memory-lean transformer consuming ``PagedKVCache``."""

    def __init__(self, cfg: ToyConfig, device: torch.device) -> None:
        super().__init__()
        torch.manual_seed(cfg.seed)
        self.cfg = cfg
        self.tokenizer = ToyTokenizer(cfg.vocab_size)
        self.device = torch.device(device)
        self.num_layers = cfg.num_layers
        self.num_q_heads = cfg.num_attention_heads
        self.num_kv_heads = cfg.num_key_value_heads
        self.head_dim = cfg.head_dim
        self._cos_sin = make_rotary_cache(cfg.head_dim, cfg.theta, cfg.max_position_embeddings, self.device)
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(
            [
                PagedDecoderLayer(cfg.hidden_size, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim,
                                  cfg.intermediate_size)
                for _ in range(cfg.num_layers)
            ]
        )
        self.norm = RMSNorm(cfg.hidden_size)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        if cfg.logit_scale != 1.0:
            with torch.no_grad():
                self.lm_head.weight.mul_(cfg.logit_scale)
        self.config = cfg
        self.forward_calls = 0
        self.to(device=self.device)
        self.requires_grad_(False)

    def _rope_table(self) -> torch.Tensor:
        return self._cos_sin

    def _logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.lm_head(self.norm(hidden))

    @property
    def vocab_size(self) -> int:
        return self.cfg.vocab_size

    @property
    def dtype(self) -> torch.dtype:
        return next(self.parameters()).dtype

    def encode(self, text) -> List[int]:
        return self.tokenizer.encode(text)

    def decode_text(self, token_ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        return self.tokenizer.decode(token_ids, skip_special_tokens)

    def reset_counters(self) -> None:
        self.forward_calls = 0
