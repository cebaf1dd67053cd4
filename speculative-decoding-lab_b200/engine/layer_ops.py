"""Fused elementwise ops of a decoder layer for 16-bit models on CUDA.

``rmsnorm`` / ``add_rmsnorm`` / ``rope_`` / ``silu_mul`` each replace a chain
of small framework kernels of engine/model.py and engine/qwen.py with one
launch of ``csrc/layer_ops.cu`` and round where the chain rounds (RMSNorm's
mean may differ in the last fp32 bit: its sum order is the kernel's).
``fusable(x)`` says whether a tensor takes this path; fp32 models keep the
framework ops.
"""

from __future__ import annotations

from typing import Tuple

import torch

from . import _lib


def fusable(x: torch.Tensor) -> bool:
    return x.is_cuda and x.dtype in (torch.bfloat16, torch.float16)


def _rows(x: torch.Tensor) -> torch.Tensor:
    x2 = x.reshape(-1, x.shape[-1])
    return x2 if x2.stride(-1) == 1 else x2.contiguous()


def add_rmsnorm(x: torch.Tensor, delta, weight: torch.Tensor, eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """``h = x + delta`` (when ``delta`` is given) and ``rmsnorm(h)``; returns ``(h, normed)``."""
    xr = _rows(x)
    out = torch.empty(xr.shape, dtype=x.dtype, device=x.device)
    if delta is not None:
        dr = _rows(delta)
        h = torch.empty_like(out)
        args = (dr.data_ptr(), dr.stride(0), h.data_ptr(), h.stride(0))
    else:
        h = None
        args = (None, 0, None, 0)
    w = weight if weight.dtype == x.dtype else weight.to(x.dtype)
    _lib.check(
        _lib.load().sdl_rmsnorm(xr.data_ptr(), xr.stride(0), *args, w.data_ptr(), out.data_ptr(), out.stride(0),
                                xr.shape[0], xr.shape[1], float(eps), _lib.dtype_code(x.dtype),
                                _lib.stream_handle(x.device)),
        "sdl_rmsnorm",
    )
    normed = out.reshape(x.shape)
    return (h.reshape(x.shape) if h is not None else x), normed


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return add_rmsnorm(x, None, weight, eps)[1]


def rope_(x: torch.Tensor, sin: torch.Tensor, cos: torch.Tensor) -> torch.Tensor:
    """In-place ``x * cos + rotate_half(x) * sin`` for ``x`` of shape
    ``(..., heads, d)`` with contiguous rows; ``cos`` / ``sin`` hold one
    ``d``-row per leading position of ``x`` (broadcast over heads)."""
    d = x.shape[-1]
    heads = x.shape[-2]
    xr = x.reshape(-1, heads * d)
    if xr.stride(-1) != 1 or (xr.data_ptr() != x.data_ptr()):
        raise ValueError("rope_: rows of x must be contiguous")
    c = cos.reshape(-1, d)
    s = sin.reshape(-1, d)
    if c.shape[0] != xr.shape[0] or s.shape[0] != xr.shape[0] or c.stride(-1) != 1 or s.stride(-1) != 1:
        raise ValueError("rope_: cos/sin must hold one row per position of x")
    c = c if c.dtype == x.dtype else c.to(x.dtype)
    s = s if s.dtype == x.dtype else s.to(x.dtype)
    _lib.check(
        _lib.load().sdl_rope(xr.data_ptr(), xr.stride(0), xr.shape[0], heads, d, c.data_ptr(), c.stride(0),
                             s.data_ptr(), s.stride(0), _lib.dtype_code(x.dtype), _lib.stream_handle(x.device)),
        "sdl_rope",
    )
    return x


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` with the framework's two roundings."""
    g = gate.contiguous()
    u = up.contiguous()
    out = torch.empty_like(g)
    _lib.check(
        _lib.load().sdl_silu_mul(g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(), _lib.dtype_code(g.dtype),
                                 _lib.stream_handle(g.device)),
        "sdl_silu_mul",
    )
    return out


def swiglu(gate_up: torch.Tensor, inter: int) -> torch.Tensor:
    """``silu(gate) * up`` on rows ``[gate | up]`` of one fused projection
    (``inter`` columns each), with ``silu_mul``'s two roundings."""
    x = gate_up.reshape(-1, gate_up.shape[-1])
    if x.stride(-1) != 1:
        x = x.contiguous()
    out = torch.empty((x.shape[0], inter), dtype=x.dtype, device=x.device)
    _lib.check(
        _lib.load().sdl_swiglu(x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), x.shape[0], int(inter),
                               _lib.dtype_code(x.dtype), _lib.stream_handle(x.device)),
        "sdl_swiglu",
    )
    return out.reshape(*gate_up.shape[:-1], inter)

