"""The C-ABI library builds, loads and exports every symbol the header declares
(CPU only: no kernel is launched)."""

from __future__ import annotations

import ctypes
import os
import re

from conftest import PKG, ROOT


def _header_symbols():
    with open(os.path.join(ROOT, "include", "sdl_b200.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(sdl_[a-z0-9_]+)\s*\(", text)))


def test_library_builds_and_exports_every_header_symbol():
    import build_lib  # speculative-decoding-lab_b200/build_lib.py

    path = build_lib.build()
    lib = ctypes.CDLL(path)
    declared = _header_symbols()
    assert len(declared) >= 20
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing


def test_binding_declares_every_header_symbol():
    from engine import _lib

    assert sorted(_lib.EXPORTED_SYMBOLS) == _header_symbols()
    lib = _lib.load()
    assert lib.sdl_version().startswith(b"sdl_b200")


def test_library_is_sm100a_only():
    """The fatbinary carries sm_100a code (cuobjdump-free check: nvcc flags)."""
    import build_lib

    assert "arch=compute_100a,code=sm_100a" in " ".join(build_lib.ARCH_FLAGS)


def test_kernels_refuse_cpu_tensors():
    import pytest
    import torch

    from engine import _lib

    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.require_cuda(torch.zeros(1), "x")
    from engine.kv import PagedKVCache

    with pytest.raises(RuntimeError, match="CUDA"):
        PagedKVCache(1, 1, 8, 4, 4, torch.device("cpu"), torch.float32)


def test_ctypes_structs_match_the_header_layout(tmp_path):
    """Every field of the ctypes mirrors of ``sdl_attn_args`` and
    ``sdl_kv_meta`` sits at the header's offset (gcc's offsetof), and the
    structs have the header's size, so a field added on one side only fails
    here instead of shifting every later argument."""
    import shutil
    import subprocess

    import pytest

    from engine import _lib

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    structs = {"sdl_attn_args": _lib.SdlAttnArgs, "sdl_kv_meta": _lib.SdlKvMeta}
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "sdl_b200.h"', "int main(void) {"]
    for cname, cls in structs.items():
        lines.append('printf("{0} sizeof %zu\\n", sizeof({0}));'.format(cname))
        for fname, _ in cls._fields_:
            lines.append('printf("{0} {1} %zu\\n", offsetof({0}, {1}));'.format(cname, fname))
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-std=c11", "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
                    str(src), "-o", str(exe)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    got = {}
    for line in out:
        if line.strip():
            cname, fname, val = line.split()
            got[(cname, fname)] = int(val)
    for cname, cls in structs.items():
        assert got[(cname, "sizeof")] == ctypes.sizeof(cls), cname
        for fname, _ in cls._fields_:
            assert got[(cname, fname)] == getattr(cls, fname).offset, (cname, fname)



def test_c4_wall_clock_stream_draws_like_the_step_stream():
    """The wall-clock C4 stream draws prompts and output lengths in the same
    order as the step-clock one; arrivals are Poisson gaps in seconds (mean
    1/rate); slices cover the stream in order, each rebased to start at 0."""
    import numpy as np

    from engine import workloads

    a = workloads.c4_requests(3, 200, 1.0)
    b = workloads.c4_requests_wall(3, 200, 64.0)
    assert [x[0] for x in a] == [x[0] for x in b] and [x[1] for x in a] == [x[1] for x in b]
    t = np.array([x[2] for x in b])
    assert t[0] == 0.0 and np.all(np.diff(t) >= 0)
    assert 0.5 / 64 < np.diff(t).mean() < 2.0 / 64
    parts = workloads.c4_slices(b, 7)
    assert sum(len(p) for p in parts) == 200 and all(p[0][2] == 0.0 for p in parts)
    assert [x[0] for p in parts for x in p] == [x[0] for x in b]


def test_prefill_buckets_are_fine_where_prompts_are_common():
    """Graphed prefills pad a prompt to 64, a multiple of 128 up to 1024, of
    256 up to 4096, then a power of two; every bucket holds its prompt."""
    from engine.model import PagedLMMixin

    f = PagedLMMixin.prefill_bucket_of
    assert [f(n) for n in (1, 64, 65, 128, 129, 556, 1024, 1025, 4096, 4097, 9000)] == \
        [64, 64, 128, 128, 256, 640, 1024, 1280, 4096, 8192, 16384]
    assert all(f(n) >= n and f(f(n)) == f(n) for n in range(1, 5000, 7))
