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

