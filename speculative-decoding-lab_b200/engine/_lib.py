"""ctypes binding of the sm_100a C-ABI library (``lib/libsdl_b200.so``).

There is no CPU or PyTorch fallback: every entry point below requires the
library and CUDA tensors, and raises when either is missing.  Signatures
mirror ``include/sdl_b200.h``.
"""

from __future__ import annotations

import contextlib
import ctypes
import gc
import os
from typing import Optional

import torch

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_ROOT, "lib", "libsdl_b200.so")

c_int = ctypes.c_int32
c_i64 = ctypes.c_int64
c_size = ctypes.c_size_t
c_float = ctypes.c_float
c_void = ctypes.c_void_p
c_char_p = ctypes.c_char_p

SDL_F32, SDL_BF16, SDL_F16 = 0, 1, 2

DEVERR_EXHAUSTED = 1
DEVERR_TABLE_OVERFLOW = 2
DEVERR_BAD_INDEX = 4
DEVERR_TIMEOUT = 8
DEVERR_BAD_SLOT = 16
DEVERR_BAD_SAMPLE = 32
DEVERR_UNIFORMS = 64

REL_TRUNCATE = 1
REL_ONLY_IF_LONGER = 2
REL_CLEAR = 4

#: Every symbol ``include/sdl_b200.h`` declares (checked by the CPU test suite).
EXPORTED_SYMBOLS = (
    "sdl_version",
    "sdl_last_error",
    "sdl_block_init",
    "sdl_block_alloc",
    "sdl_block_free",
    "sdl_kv_reserve",
    "sdl_kv_append",
    "sdl_kv_release",
    "sdl_kv_truncate",
    "sdl_spec_commit",
    "sdl_spec_commit_n",
    "sdl_make_kv_tensor_map",
    "sdl_attention_workspace_bytes",
    "sdl_attention_launches",
    "sdl_attention_kernel",
    "sdl_attention_fuses_rope",
    "sdl_paged_attention",
    "sdl_paged_attention_noalloc",
    "sdl_noalloc_scratch_bytes",
    "sdl_paged_decode",
    "sdl_paged_verify",
    "sdl_prefill_chunk",
    "sdl_logits_to_probs",
    "sdl_argmax_rows",
    "sdl_sample_rows",
    "sdl_counter_add",
    "sdl_spec_sample",
    "sdl_spec_sample_scratch_bytes",
    "sdl_sampler_workspace_bytes",
    "sdl_sample_logits_rows",
    "sdl_spec_sample_logits",
    "sdl_spec_sample_logits_n",
    "sdl_set_spec_sampler_mode",
    "sdl_get_error",
    "sdl_rmsnorm",
    "sdl_rope",
    "sdl_silu_mul",
    "sdl_swiglu",
)


class SdlKvMeta(ctypes.Structure):
    _fields_ = [
        ("block_table", c_void),
        ("num_blocks", c_void),
        ("seq_lens", c_void),
        ("free_stack", c_void),
        ("free_top", c_void),
        ("is_free", c_void),
        ("err", c_void),
        ("capacity", c_int),
        ("width", c_int),
        ("max_rows", c_int),
        ("block_size", c_int),
    ]


class SdlAttnArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void),
        ("q_sb", c_i64), ("q_sj", c_i64), ("q_sh", c_i64),
        ("out", c_void),
        ("o_sb", c_i64), ("o_sj", c_i64), ("o_sh", c_i64),
        ("out_dtype", c_int),
        ("dtype", c_int),
        ("k_pool", c_void),
        ("v_pool", c_void),
        ("tmap_k", c_void),
        ("tmap_v", c_void),
        ("block_table", c_void), ("width", c_int), ("capacity", c_int),
        ("num_layers", c_int), ("layer", c_int), ("block_size", c_int),
        ("rows", c_void),
        ("k_dense", c_void), ("v_dense", c_void), ("kv_len", c_int),
        ("starts", c_void),
        ("valid_rows", c_void),
        ("B", c_int), ("chunk", c_int), ("Hq", c_int), ("Hkv", c_int), ("head_dim", c_int),
        ("max_limit", c_int),
        ("scale", c_float),
        ("workspace", c_void),
        ("workspace_bytes", c_size),
        ("pages_per_split", c_int),
        ("force_generic", c_int),
        ("kv_heads_per_cta", c_int),
        ("use_umma", c_int),
        ("cluster_merge", c_int),
        ("key_count", c_i64),
        ("mma_layout", c_int),
        ("k_new", c_void),
        ("v_new", c_void),
        ("new_row_stride", c_i64),
        ("err", c_void),
        ("rope_cos", c_void),
        ("rope_sin", c_void),
        ("rope_stride", c_i64),
        ("overlap_layers", c_int),
    ]


_P = ctypes.POINTER
_SIGS = {
    "sdl_version": (c_char_p, []),
    "sdl_last_error": (c_char_p, []),
    "sdl_block_init": (c_int, [c_void, c_void, c_void, c_int, c_void]),
    "sdl_block_alloc": (c_int, [c_void, c_void, c_void, c_int, c_int, c_void, c_void, c_void]),
    "sdl_block_free": (c_int, [c_void, c_void, c_void, c_int, c_int, c_void, c_void, c_void]),
    "sdl_kv_reserve": (c_int, [_P(SdlKvMeta), c_int, c_void, c_void, c_void, c_void, c_void]),
    "sdl_kv_append": (c_int, [c_void, c_void, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void,
                              c_void, c_void, c_i64, c_void, c_void]),
    "sdl_kv_release": (c_int, [_P(SdlKvMeta), c_int, c_void, c_void, c_void, c_void]),
    "sdl_kv_truncate": (c_int, [_P(SdlKvMeta), c_int, c_void, c_void, c_void]),
    "sdl_spec_commit": (c_int, [_P(SdlKvMeta), _P(SdlKvMeta), c_int, c_void, c_void, c_void, c_int, c_void,
                                c_int, c_void, c_void, c_void, c_void, c_void]),
    "sdl_spec_commit_n": (c_int, [_P(SdlKvMeta), _P(SdlKvMeta), c_int, c_void, c_void, c_void, c_int, c_void,
                                  c_int, c_void, c_void, c_void, c_void, c_void, c_void]),
    "sdl_make_kv_tensor_map": (c_int, [c_void, c_void, c_int, c_i64, c_int, c_int]),
    "sdl_attention_workspace_bytes": (c_size, [_P(SdlAttnArgs)]),
    "sdl_attention_launches": (c_int, [_P(SdlAttnArgs)]),
    "sdl_attention_kernel": (c_int, [_P(SdlAttnArgs)]),
    "sdl_attention_fuses_rope": (c_int, [_P(SdlAttnArgs)]),
    "sdl_paged_attention": (c_int, [_P(SdlAttnArgs), c_void]),
    "sdl_paged_attention_noalloc": (c_int, [_P(SdlAttnArgs), c_void]),
    "sdl_noalloc_scratch_bytes": (c_size, []),
    "sdl_paged_decode": (c_int, [_P(SdlAttnArgs), c_void]),
    "sdl_paged_verify": (c_int, [_P(SdlAttnArgs), c_void]),
    "sdl_prefill_chunk": (c_int, [_P(SdlAttnArgs), c_void]),
    "sdl_logits_to_probs": (c_int, [c_void, c_int, c_i64, c_int, c_int, c_float, c_float, c_int, c_void,
                                    c_i64, c_void]),
    "sdl_argmax_rows": (c_int, [c_void, c_int, c_i64, c_int, c_int, c_void, c_void]),
    "sdl_sample_rows": (c_int, [c_void, c_i64, c_int, c_int, c_void, c_i64, c_void, c_i64, c_void, c_void,
                                c_void]),
    "sdl_counter_add": (c_int, [c_void, c_i64, c_void]),
    "sdl_spec_sample": (c_int, [c_void, c_i64, c_i64, c_void, c_i64, c_i64, c_void, c_void, c_int, c_int,
                                c_int, c_int, c_void, c_i64, c_void, c_i64, c_void, c_void, c_void, c_void,
                                c_void]),
    "sdl_spec_sample_scratch_bytes": (c_size, [c_int]),
    "sdl_sampler_workspace_bytes": (c_size, [c_int, c_int]),
    "sdl_sample_logits_rows": (c_int, [c_void, c_int, c_i64, c_int, c_int, c_float, c_float, c_void, c_i64, c_void,
                                       c_i64, c_void, c_void, c_size, c_void, c_void]),
    "sdl_spec_sample_logits": (c_int, [c_void, c_i64, c_i64, c_void, c_i64, c_i64, c_int, c_float, c_float, c_void,
                                       c_int, c_int, c_int, c_void, c_i64, c_void, c_i64, c_void, c_void, c_void,
                                       c_size, c_void, c_void]),
    "sdl_spec_sample_logits_n": (c_int, [c_void, c_i64, c_i64, c_void, c_i64, c_i64, c_int, c_float, c_float,
                                         c_void, c_int, c_int, c_int, c_void, c_i64, c_void, c_i64, c_void, c_void,
                                         c_void, c_size, c_void, c_void, c_void]),
    "sdl_set_spec_sampler_mode": (c_int, [c_int]),
    "sdl_get_error": (c_int, [c_void, c_void, c_int, c_void]),
    "sdl_rmsnorm": (c_int, [c_void, c_i64, c_void, c_i64, c_void, c_i64, c_void, c_void, c_i64, c_int, c_int, c_float,
                            c_int, c_void]),
    "sdl_rope": (c_int, [c_void, c_i64, c_int, c_int, c_int, c_void, c_i64, c_void, c_i64, c_int, c_void]),
    "sdl_silu_mul": (c_int, [c_void, c_void, c_void, c_i64, c_int, c_void]),
    "sdl_swiglu": (c_int, [c_void, c_i64, c_void, c_i64, c_int, c_int, c_int, c_void]),
}

_LIB: Optional[ctypes.CDLL] = None


def load() -> ctypes.CDLL:
    """Load (once) and type the library; raise when it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                "sdl_b200 CUDA library missing at {}; build it with "
                "`python speculative-decoding-lab_b200/build_lib.py`".format(LIB_PATH)
            )
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def last_error() -> str:
    msg = load().sdl_last_error()
    return msg.decode() if msg else ""


# Entry calls into the library made from this process (each launches one or
# more of its kernels); CUDA-graph replays add the calls their capture made.
_CALLS = [0]


def calls() -> int:
    """Library entry calls so far (``check`` counts every one)."""
    return _CALLS[0]


def count_calls(n: int) -> None:
    """Add ``n`` calls replayed inside a CUDA graph."""
    _CALLS[0] += int(n)


def check(rc: int, what: str) -> None:
    _CALLS[0] += 1
    if rc != 0:
        raise RuntimeError("{} failed (status {}): {}".format(what, rc, last_error()))


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_handle(device: Optional[torch.device] = None) -> int:
    """cudaStream_t of the current stream of ``device`` (as an int)."""
    if _raw_stream is not None and device is not None and device.index is not None:
        return _raw_stream(device.index)
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        raise RuntimeError(
            "{} must be a CUDA tensor: the B200 path has no CPU fallback".format(name)
        )


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return SDL_F32
    if dtype == torch.bfloat16:
        return SDL_BF16
    if dtype == torch.float16:
        return SDL_F16
    raise TypeError("unsupported dtype {} (float32, bfloat16, float16)".format(dtype))


def to_device(values, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """Host values -> CUDA tensor without waiting for the stream: built on
    the host and copied with ``non_blocking`` (the copy is queued behind the
    stream's work), where ``torch.tensor(values, device=...)`` would wait for
    every queued kernel first."""
    return torch.tensor(values, dtype=dtype).to(device, non_blocking=True)


def i32(values, device: torch.device) -> torch.Tensor:
    """Host list -> contiguous int32 CUDA tensor (one H2D copy)."""
    if isinstance(values, torch.Tensor):
        return values.to(device=device, dtype=torch.int32).contiguous()
    return torch.tensor(list(values), dtype=torch.int32).to(device, non_blocking=True)


@contextlib.contextmanager
def no_gc():
    """Keep Python's cyclic garbage collector from running inside a CUDA
    graph capture: collecting an unreachable object that holds a captured
    graph would destroy that graph mid-capture and invalidate the capture."""
    was = gc.isenabled()
    gc.disable()
    try:
        yield
    finally:
        if was:
            gc.enable()


class Workspace:
    """Per-device growable fp32 scratch (split-K attention partials under the
    default tag, sampler statistics under ``"sampler"``).

    Buffers start zeroed: a sampler workspace begins with the fused
    sampler's control block, which must be zero before its first use.  A
    buffer that is outgrown is kept alive rather than freed: CUDA graphs
    captured earlier still hold its address.
    """

    _bufs = {}
    _retired = []

    @classmethod
    def get(cls, device: torch.device, nbytes: int, tag: str = "attention") -> torch.Tensor:
        key = (device.type, device.index if device.index is not None else torch.cuda.current_device(), tag)
        buf = cls._bufs.get(key)
        need = max(4, (nbytes + 3) // 4)
        if buf is None or buf.numel() < need:
            if buf is not None:
                cls._retired.append(buf)
            buf = torch.zeros(int(need * 1.25) + 1024, dtype=torch.float32, device=device)
            cls._bufs[key] = buf
        return buf
