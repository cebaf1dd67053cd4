"""Logit post-processing, token sampling and distribution distances on B200.

Drop-in for the reference's ``specdec/sampler.py`` (specdec/sampler.py:16-154):
same names and semantics, with the per-row work done by sm_100a kernels:

* ``logits_to_probs`` -- greedy one-hot at the first argmax, else
  ``softmax(logits / max(T, 1e-12))`` in fp32 (specdec/sampler.py:19-36);
* ``sample_token`` -- one draw with the exact integer inverse-CDF rule
  (``sdl_sample_rows``) from a uniform, instead of ``torch.multinomial`` on a
  CPU copy (specdec/sampler.py:59-69);
* the fused rejection sampler (``spec_sample``) behind
  ``engine.spec_scheduler.batch_accept``.

Uniforms come from a :class:`UniformStream`: fp32 values in HBM read through a
device counter, so a whole speculative round draws without host syncs.  The
stream order is the reference's draw order (draft proposals step-major then
sequence-major, then per sequence its accept tests and one final draw), so a
stream pre-drawn once and fed to both this engine and the reference (with its
``_draw_uniform`` / ``sample_token`` reading the same stream) yields identical
tokens.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple, Union

import torch

from engine import _lib

from .config import SamplingConfig

_EPS = 1e-12


class UniformStream:
    """fp32 uniforms in HBM with a device-side read counter.

    ``seed`` draws them on the device in chunks (deterministic for a given
    seed and consumption); ``uniforms`` pins a pre-drawn stream (parity
    harnesses).  ``storage = (buffer, counter)`` places the stream in
    caller-owned device tensors (fp32 of some capacity, int64 of one entry)
    that outlive it: a CUDA graph captured over those addresses reads every
    later stream built on the same storage.  Refills then happen in place,
    and ``capacity`` may exceed the valid length (``len``), so a captured
    launch whose padding rows read past the valid uniforms stays in bounds.
    """

    def __init__(self, device: torch.device, seed: Optional[int] = None,
                 uniforms: Optional[torch.Tensor] = None, chunk: int = 1 << 20,
                 storage: Optional[Tuple[torch.Tensor, torch.Tensor]] = None) -> None:
        device = torch.device(device)
        if device.type != "cuda":
            raise RuntimeError("UniformStream lives in HBM: device must be CUDA")
        self.device = device
        self._chunk = int(chunk)
        self._gen = None
        if uniforms is not None:
            u = uniforms.detach().to(device=device, dtype=torch.float32).reshape(-1)
        else:
            self._gen = torch.Generator(device=device)
            self._gen.manual_seed(int(0 if seed is None else seed))
        if storage is not None:
            buf, counter = storage
            if buf.dtype != torch.float32 or counter.dtype != torch.int64 or buf.device != device:
                raise ValueError("storage must be (fp32 buffer, int64 counter) on the stream's device")
            n = u.numel() if uniforms is not None else min(self._chunk, buf.numel())
            if n > buf.numel():
                raise ValueError("uniform storage holds {} values, the stream needs {}".format(buf.numel(), n))
            if uniforms is not None:
                buf[:n].copy_(u)
            else:
                buf[:n].copy_(torch.rand(n, generator=self._gen, device=device, dtype=torch.float32))
            buf[n:].zero_()
            counter.zero_()
            self._buf, self.counter, self._len, self._fixed = buf, counter, n, True
        else:
            if uniforms is not None:
                self._buf = u.contiguous()
            else:
                self._buf = torch.rand(self._chunk, generator=self._gen, device=device, dtype=torch.float32)
            self.counter = torch.zeros(1, dtype=torch.int64, device=device)
            self._len, self._fixed = self._buf.numel(), False
        self._hi = 0  # host upper bound of the counter

    @property
    def buffer(self) -> torch.Tensor:
        """The valid uniforms (a view starting at the storage's address)."""
        return self._buf[:self._len]

    @property
    def storage(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """The whole buffer (its capacity) and the counter."""
        return self._buf, self.counter

    def __len__(self) -> int:
        return self._len

    def reserve(self, n: int) -> None:
        """Make sure ``n`` more uniforms can be read; refills when needed."""
        if self._hi + n <= self._len:
            self._hi += n
            return
        c = int(self.counter.item())
        self._hi = c
        if c + n > self._len:
            if self._gen is None:
                raise RuntimeError("uniform stream exhausted ({} consumed, {} more needed)".format(c, n))
            tail = self._buf[c:self._len].clone()
            k = tail.numel()
            if self._fixed:
                # in place: captured graphs hold the storage's address
                fill = self._buf.numel() - k
                if fill < n:
                    raise RuntimeError("uniform storage of {} values cannot hold {} more".format(self._buf.numel(), n))
                fill = min(fill, max(self._chunk, n))
                self._buf[:k].copy_(tail)
                self._buf[k:k + fill].copy_(torch.rand(fill, generator=self._gen, device=self.device,
                                                       dtype=torch.float32))
                self._len = k + fill
            else:
                fresh = torch.rand(max(self._chunk, n), generator=self._gen, device=self.device, dtype=torch.float32)
                self._buf = torch.cat((tail, fresh))
                self._len = self._buf.numel()
            self.counter.zero_()
            self._hi = 0
        self._hi += n

    def consumed(self) -> int:
        return int(self.counter.item())

    def advance(self, n: int) -> None:
        _lib.check(_lib.load().sdl_counter_add(self.counter.data_ptr(), int(n), _lib.stream_handle(self.device)),
                   "sdl_counter_add")


# ------------------------------------------------------------ device kernels
def _rows2d(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    return x2


def probs_rows(logits: torch.Tensor, temperature: float, greedy: bool, eps: float = _EPS,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32 probabilities of every row of ``logits`` (one kernel launch)."""
    _lib.require_cuda(logits, "logits")
    x = _rows2d(logits)
    rows, V = x.shape
    if out is None:
        out = torch.empty((rows, V), dtype=torch.float32, device=x.device)
    _lib.check(
        _lib.load().sdl_logits_to_probs(
            x.data_ptr(), _lib.dtype_code(x.dtype), x.stride(0), rows, V, float(temperature), float(eps),
            1 if greedy else 0, out.data_ptr(), out.stride(0), _lib.stream_handle(x.device),
        ),
        "sdl_logits_to_probs",
    )
    return out


def argmax_rows(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """First-index argmax of every row (int32)."""
    _lib.require_cuda(logits, "logits")
    x = _rows2d(logits)
    rows, V = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=x.device)
    _lib.check(
        _lib.load().sdl_argmax_rows(x.data_ptr(), _lib.dtype_code(x.dtype), x.stride(0), rows, V, out.data_ptr(),
                                    _lib.stream_handle(x.device)),
        "sdl_argmax_rows",
    )
    return out


def sample_rows(weights: torch.Tensor, stream: UniformStream, offset: int = 0,
                out: Optional[torch.Tensor] = None, err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One draw per row; row ``r`` reads uniform ``counter + offset + r``.

    Does not advance the counter (callers advance once per batch of draws).
    """
    _lib.require_cuda(weights, "weights")
    w = _rows2d(weights)
    if w.dtype != torch.float32:
        w = w.float()
    rows, V = w.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=w.device)
    _lib.check(
        _lib.load().sdl_sample_rows(
            w.data_ptr(), w.stride(0), rows, V, stream.buffer.data_ptr(), stream.buffer.numel(),
            stream.counter.data_ptr(), int(offset), out.data_ptr(), err.data_ptr() if err is not None else None,
            _lib.stream_handle(w.device),
        ),
        "sdl_sample_rows",
    )
    return out


def spec_sample(
    p: Optional[torch.Tensor],
    q: Optional[torch.Tensor],
    proposals: torch.Tensor,
    stream: Optional[UniformStream],
    greedy: bool,
    p_arg: Optional[torch.Tensor] = None,
    u_skip: int = 0,
    err: Optional[torch.Tensor] = None,
    out: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Fused rejection sampling of a batch of draft blocks (sdl_spec_sample).

    ``p`` (B, gamma+1, V) target probs, ``q`` (B, gamma, V) draft probs,
    ``proposals`` (B, gamma) int32; greedy mode takes ``p_arg`` (B, gamma+1)
    target argmaxes instead of ``p``/``q``.  Returns ``tokens`` (B, gamma+1)
    int32 and ``n_out`` (B,) int32 (accepted + 1).
    """
    _lib.require_cuda(proposals, "proposals")
    device = proposals.device
    B, gamma = proposals.shape
    prop = proposals.to(torch.int32).contiguous()
    if out is None:
        tokens = torch.empty((B, gamma + 1), dtype=torch.int32, device=device)
        n_out = torch.empty(B, dtype=torch.int32, device=device)
        scratch = torch.empty(max(2 * B, 1), dtype=torch.int32, device=device)
    else:
        tokens, n_out, scratch = out
    if greedy:
        if p_arg is None:
            raise ValueError("greedy spec_sample needs p_arg")
        pa = p_arg.to(torch.int32).contiguous()
        pp = qq = None
        V = 1
        p_sb = p_sj = q_sb = q_sj = 0
    else:
        if p.dtype != torch.float32 or q.dtype != torch.float32:
            raise TypeError("spec_sample expects fp32 probabilities")
        pa = None
        pp, qq = p, q
        if pp.stride(-1) != 1:
            pp = pp.contiguous()
        if qq.stride(-1) != 1:
            qq = qq.contiguous()
        V = pp.shape[-1]
        p_sb, p_sj, q_sb, q_sj = pp.stride(0), pp.stride(1), qq.stride(0), qq.stride(1)
    if stream is not None:
        stream.reserve(u_skip + B * (gamma + 1))
    _lib.check(
        _lib.load().sdl_spec_sample(
            _lib.ptr(pp), p_sb, p_sj, _lib.ptr(qq), q_sb, q_sj, _lib.ptr(pa), prop.data_ptr(), B, gamma, V,
            1 if greedy else 0,
            stream.buffer.data_ptr() if stream is not None else None,
            stream.buffer.numel() if stream is not None else 0,
            stream.counter.data_ptr() if stream is not None else None,
            int(u_skip), tokens.data_ptr(), n_out.data_ptr(), scratch.data_ptr(),
            err.data_ptr() if err is not None else None, _lib.stream_handle(device),
        ),
        "sdl_spec_sample",
    )
    return tokens, n_out


def _sampler_ws(device: torch.device, rows: int, vocab: int) -> torch.Tensor:
    need = int(_lib.load().sdl_sampler_workspace_bytes(int(rows), int(vocab)))
    return _lib.Workspace.get(device, need, tag="sampler")


def sample_logits_rows(logits: torch.Tensor, temperature: float, stream: UniformStream, offset: int = 0,
                       out: Optional[torch.Tensor] = None, err: Optional[torch.Tensor] = None,
                       eps: float = _EPS) -> torch.Tensor:
    """One draw per row of ``softmax(logits / T)`` without writing the
    probabilities; bit-equal to ``sample_rows(probs_rows(logits, T))``.

    Row ``r`` reads uniform ``counter + offset + r``; the counter is not
    advanced.
    """
    _lib.require_cuda(logits, "logits")
    x = _rows2d(logits)
    rows, V = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.int32, device=x.device)
    ws = _sampler_ws(x.device, rows, V)
    _lib.check(
        _lib.load().sdl_sample_logits_rows(
            x.data_ptr(), _lib.dtype_code(x.dtype), x.stride(0), rows, V, float(temperature), float(eps),
            stream.buffer.data_ptr(), stream.buffer.numel(), stream.counter.data_ptr(), int(offset), out.data_ptr(),
            ws.data_ptr(), ws.numel() * 4, err.data_ptr() if err is not None else None,
            _lib.stream_handle(x.device),
        ),
        "sdl_sample_logits_rows",
    )
    return out


def spec_sample_logits(
    p_logits: torch.Tensor,
    q_logits: torch.Tensor,
    temperature: float,
    proposals: torch.Tensor,
    stream: UniformStream,
    u_skip: int = 0,
    err: Optional[torch.Tensor] = None,
    out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
    eps: float = _EPS,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Fused rejection sampling straight from logits (sdl_spec_sample_logits).

    ``p_logits`` (B, gamma+1, V) target logits, ``q_logits`` (B, gamma, V)
    draft logits of the same dtype, ``proposals`` (B, gamma).  Returns
    ``tokens`` (B, gamma+1) and ``n_out`` (B,), bit-equal to
    ``spec_sample(probs_rows(p), probs_rows(q), ...)``.
    """
    _lib.require_cuda(p_logits, "p_logits")
    device = p_logits.device
    B, gamma = proposals.shape
    if p_logits.dtype != q_logits.dtype:
        raise TypeError("p_logits and q_logits must share a dtype")
    pl, ql = p_logits, q_logits
    if pl.stride(-1) != 1:
        pl = pl.contiguous()
    if ql.stride(-1) != 1:
        ql = ql.contiguous()
    V = pl.shape[-1]
    prop = proposals if (proposals.dtype == torch.int32 and proposals.is_contiguous()) else \
        proposals.to(torch.int32).contiguous()
    if out is None:
        tokens = torch.empty((B, gamma + 1), dtype=torch.int32, device=device)
        n_out = torch.empty(B, dtype=torch.int32, device=device)
    else:
        tokens, n_out = out
    ws = _sampler_ws(device, B * (2 * gamma + 1), V)
    stream.reserve(u_skip + B * (gamma + 1))
    _lib.check(
        _lib.load().sdl_spec_sample_logits(
            pl.data_ptr(), pl.stride(0), pl.stride(1), ql.data_ptr(), ql.stride(0), ql.stride(1),
            _lib.dtype_code(pl.dtype), float(temperature), float(eps), prop.data_ptr(), B, gamma, V,
            stream.buffer.data_ptr(), stream.buffer.numel(), stream.counter.data_ptr(), int(u_skip),
            tokens.data_ptr(), n_out.data_ptr(), ws.data_ptr(), ws.numel() * 4,
            err.data_ptr() if err is not None else None, _lib.stream_handle(device),
        ),
        "sdl_spec_sample_logits",
    )
    return tokens, n_out


# ------------------------------------------------------- reference-shaped API
def logits_to_probs(logits: torch.Tensor, sampling: SamplingConfig) -> torch.Tensor:
    """Convert raw logits of shape (..., vocab) into a probability distribution."""
    greedy = sampling.is_greedy
    top_k = int(getattr(sampling, "top_k", 0) or 0)
    top_p = float(getattr(sampling, "top_p", 1.0))
    shape = logits.shape
    if greedy or (top_k <= 0 or top_k >= shape[-1]) and (top_p >= 1.0 or top_p <= 0.0):
        return probs_rows(logits, sampling.temperature if not greedy else 1.0, greedy).reshape(shape)
    scaled = logits.float() / max(sampling.temperature, _EPS)
    filtered = apply_top_k(scaled, top_k)
    filtered = apply_top_p(filtered, top_p)
    return probs_rows(filtered, 1.0, False).reshape(shape)


def apply_top_k(logits: torch.Tensor, top_k: int) -> torch.Tensor:
    """Mask every logit outside the top-k to -inf (kept logits pass through)."""
    if top_k <= 0 or top_k >= logits.shape[-1]:
        return logits
    kth_value = torch.topk(logits, top_k, dim=-1).values[..., -1, None]
    return torch.where(logits < kth_value, torch.full_like(logits, float("-inf")), logits)


def apply_top_p(logits: torch.Tensor, top_p: float) -> torch.Tensor:
    """Nucleus filtering: keep the smallest set whose cumulative mass exceeds ``top_p``."""
    if top_p >= 1.0 or top_p <= 0.0:
        return logits
    sorted_logits, sorted_index = torch.sort(logits, descending=True, dim=-1)
    sm = torch.softmax(sorted_logits, dim=-1)
    mask = torch.cumsum(sm, dim=-1) - sm >= top_p
    sorted_logits = sorted_logits.masked_fill(mask, float("-inf"))
    return sorted_logits.scatter(-1, sorted_index, sorted_logits)


GeneratorLike = Union[None, torch.Generator, UniformStream]


def sample_token(probs: torch.Tensor, generator: GeneratorLike = None) -> int:
    """Draw a single token id from a probability vector (synchronises).

    With a :class:`UniformStream` the draw consumes its next uniform; with a
    ``torch.Generator`` (or None) one fp32 uniform is drawn from it.
    """
    _lib.require_cuda(probs, "probs")
    flat = probs.detach().reshape(1, -1).float()
    if isinstance(generator, UniformStream):
        generator.reserve(1)
        tok = sample_rows(flat, generator)
        generator.advance(1)
        return int(tok.item())
    u = torch.rand(1, generator=generator) if generator is not None else torch.rand(1)
    one = UniformStream(flat.device, uniforms=u)
    return int(sample_rows(flat, one).item())


def residual_distribution(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """Normalised positive part of ``p - q``, used when a draft token is rejected."""
    residual = torch.clamp(p - q, min=0.0)
    total = residual.sum()
    if float(total) <= _EPS:
        return p / p.sum().clamp_min(_EPS)
    return residual / total


def acceptance_probability(p: torch.Tensor, q: torch.Tensor, token_id: int) -> float:
    """``min(1, p(x) / q(x))`` for the proposed token (fp64 on the host)."""
    q_prob = float(q[token_id].item())
    p_prob = float(p[token_id].item())
    if q_prob <= _EPS:
        return 1.0 if p_prob > _EPS else 0.0
    return float(min(1.0, p_prob / q_prob))


def build_generator(seed: int, device: Optional[torch.device] = None) -> torch.Generator:
    """Deterministic CPU generator (workload synthesis, host-side draws)."""
    generator = torch.Generator(device="cpu")
    generator.manual_seed(int(seed))
    return generator


def kl_divergence(p: torch.Tensor, q: torch.Tensor, eps: float = 1e-12) -> float:
    """KL(p || q) in nats, evaluated on the support of ``p``."""
    p = p.double().reshape(-1)
    q = q.double().reshape(-1)
    support = p > 0
    if support.sum() == 0:
        return 0.0
    ps = p[support]
    qs = torch.clamp(q[support], min=eps)
    return float(torch.sum(ps * torch.log(ps / qs)).item())


def total_variation(p: torch.Tensor, q: torch.Tensor) -> float:
    """``0.5 * sum |p - q|`` in [0, 1]."""
    return float(0.5 * torch.abs(p.double().reshape(-1) - q.double().reshape(-1)).sum().item())


def js_divergence(p: torch.Tensor, q: torch.Tensor) -> float:
    p = p.double().reshape(-1)
    q = q.double().reshape(-1)
    m = 0.5 * (p + q)
    return 0.5 * kl_divergence(p, m) + 0.5 * kl_divergence(q, m)


def empirical_distribution(token_ids, vocab_size: int, device: torch.device) -> torch.Tensor:
    counts = torch.zeros(vocab_size, dtype=torch.float64, device=device)
    for token_id in token_ids:
        counts[token_id] += 1.0
    total = counts.sum()
    return counts if total == 0 else counts / total


def assert_shared_vocab(draft_logits: torch.Tensor, target_logits: torch.Tensor) -> None:
    if draft_logits.shape[-1] != target_logits.shape[-1]:
        raise ValueError(
            "draft/target vocab mismatch: {} vs {}. Pick two models that share a "
            "tokenizer (e.g. Qwen2.5-0.5B and Qwen2.5-1.5B).".format(draft_logits.shape[-1], target_logits.shape[-1])
        )


def top_tokens(probs: torch.Tensor, k: int = 5) -> Tuple[torch.Tensor, torch.Tensor]:
    values, indices = torch.topk(probs.reshape(-1).float(), min(k, probs.numel()))
    return indices, values
