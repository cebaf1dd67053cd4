"""Fused decoder-layer ops (csrc/layer_ops.cu) vs the framework op chains
they replace (engine/model.py RMSNorm / apply_rotary, engine/qwen.py SwiGLU).

RoPE and the SwiGLU gate round exactly where the chains round: bit-exact.
RMSNorm's mean is a fixed-order block sum, so an element may differ from the
chain by one 16-bit ulp; almost all are identical.
"""

from __future__ import annotations

import pytest
import torch

from engine import layer_ops
from engine.model import apply_rotary, make_rotary_cache

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
DTYPES = [torch.bfloat16, torch.float16]


def _ulps(a, b, dtype):
    ia = a.view(torch.int16).int()
    ib = b.view(torch.int16).int()
    return (ia - ib).abs()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("heads,d", [(12, 128), (2, 64), (14, 64)])
def test_rope_is_bit_exact(dtype, heads, d):
    g = torch.Generator(device=DEV).manual_seed(heads * d)
    table = make_rotary_cache(d, 1e6, 8192, DEV).to(dtype)
    pos = torch.randint(0, 8192, (5, 3), generator=g, device=DEV)
    cs = table[pos]
    cos, sin = cs[..., 0, :][:, :, None, :], cs[..., 1, :][:, :, None, :]
    x = (torch.randn((5, 3, heads, d), generator=g, device=DEV) * 3).to(dtype)
    want = apply_rotary(x, sin, cos)
    got = layer_ops.rope_(x.clone(), sin, cos)
    assert torch.equal(got, want)


@pytest.mark.parametrize("dtype", DTYPES)
def test_silu_mul_is_bit_exact(dtype):
    g = torch.Generator(device=DEV).manual_seed(3)
    gate = (torch.randn((64, 8960), generator=g, device=DEV) * 4).to(dtype)
    up = torch.randn((64, 8960), generator=g, device=DEV).to(dtype)
    want = torch.nn.functional.silu(gate) * up
    assert torch.equal(layer_ops.silu_mul(gate, up), want)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("dim", [200, 256, 896, 1025, 1536, 2048, 4096, 4097, 5000])
def test_rmsnorm_matches_the_chain(dtype, dim):
    g = torch.Generator(device=DEV).manual_seed(dim)
    x = (torch.randn((67, dim), generator=g, device=DEV) * 2).to(dtype)
    delta = torch.randn((67, dim), generator=g, device=DEV).to(dtype)
    w = (1 + 0.1 * torch.randn(dim, generator=g, device=DEV)).to(dtype)
    eps = 1e-6

    def chain(v):
        vf = v.float()
        return ((vf / torch.sqrt(vf.pow(2).mean(-1, keepdim=True) + eps)) * w.float()).to(dtype)

    got = layer_ops.rmsnorm(x, w, eps)
    u = _ulps(got, chain(x), dtype)
    assert u.max().item() <= 1 and (u == 0).float().mean().item() > 0.99
    h, normed = layer_ops.add_rmsnorm(x, delta, w, eps)
    assert torch.equal(h, x + delta)
    u = _ulps(normed, chain(x + delta), dtype)
    assert u.max().item() <= 1 and (u == 0).float().mean().item() > 0.99


@pytest.mark.parametrize("dtype", DTYPES)
def test_swiglu_on_fused_rows_equals_silu_mul(dtype):
    """The gate over rows [gate | up] of one fused projection gives silu_mul's
    bits on the two halves."""
    g = torch.Generator(device=DEV).manual_seed(3)
    for inter in (4864, 77):  # even: column pairs; odd: one column per thread
        gu = (torch.randn((37, 2 * inter), generator=g, device=DEV) * 3).to(dtype)
        want = layer_ops.silu_mul(gu[:, :inter], gu[:, inter:])
        assert torch.equal(layer_ops.swiglu(gu, inter), want)

