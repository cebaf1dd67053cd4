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
